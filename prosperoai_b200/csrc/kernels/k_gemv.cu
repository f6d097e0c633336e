// Fused dequantise-and-dot GEMV on the int8 tensor cores.
//
// Each consumer warp owns one 16-row tile of W and walks K in units (4
// blocks of Q4_0/Q8_0, one Q4_K super-block). For every 32-weight block it
// issues one m16n8k32 int8 MMA: A = the tile's 16 x 32 quant codes,
// unpacked from the packed bytes with two LOP3s per word (Q4_0/Q4_K
// nibbles) or used as-is (Q8_0); B = x in 24-bit fixed point, three int8
// digit columns per vector (two vectors per MMA). The integer products are
// exact; each lane folds its two accumulator columns into one integer,
// converts it once, and applies the block's scales in fp32:
//   sum_j w_j x_j = d * (s_b * sum_j q_j X_j  - 8 s_b sum_j X_j)   (Q4_0)
//                 = d * s_b * sum_j q_j X_j                         (Q8_0)
//                 = d sc_s * s_b sum q X - dmin m_s * s_b sum X     (Q4_K)
// so the per-weight work is the unpack plus 1/16 of an MMA, instead of an
// unpack, convert and FMA per weight on the CUDA cores.
//
// Memory pipeline (warp-specialised): the CTA's 8 consumer warps own the 8
// tiles of a 128-row group, and in the unit-major packed layout the group's
// tiles of one K unit are one contiguous run of bytes. One producer thread
// streams those runs (two bulk asynchronous copies per unit: codes and
// headers; cp.async.bulk, completion on an mbarrier per stage, no
// multicast) into a 4-stage ring shared by the consumers, which only
// unpack, multiply and accumulate from shared memory. Work is split
// stream-K style: the (group, unit) pairs are numbered group-major and CTA
// i takes the i-th contiguous share, so every CTA streams the same number
// of bytes. x (digits and scales) is staged in shared memory: all of it
// once per CTA when the CTA reuses it across groups, else per sub-item in
// three rotating slots filled one sub-item ahead. Under programmatic
// dependent launch the producer fills the ring before it waits for the
// previous kernel: weights never depend on it.
//
// Split-K is deterministic: a CTA that holds part of a group parks its
// partial row sums in scratch, and at the end of its range the last part
// of a tile to arrive (atomic ticket per tile) adds them in CTA order.
// Epilogues: plain store, residual add (the executor's following
// PAI_OP_ADD, adapters/llama/llama.c:747-749,793-795), and SiLU(gate)*up
// (llama.c:774-781); for the latter the last tile of each 64-row group
// (ticket per group) also re-quantises the group's 32 outputs for the down
// projection. Every mbarrier wait is bounded; on timeout the kernel raises
// the context's error flag (reported as PAI_ERR_TIMEOUT), waits (bounded)
// for its copies in flight and stops.
// Reference result: dequant_block rows (adapters/llama/gguf.c:680-693,
// 750-761, 852-882) dotted as in pai_ref_gemv_f32 (cpu/reference/ref_ops.c:92-106).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "../b200_internal.h"
#include "b200_device.cuh"
#include "gemv_unit.cuh"

namespace {

using namespace gemv;

constexpr int kStages = 4;                   // depth of the CTA's weight ring
constexpr int kXSlots = 3;                   // staged-x slots (current, next, one being released)
// CTA shape: CONS consumer warps (one 16-row tile each; a group is CONS
// tiles) + one producer warp, one CTA per SM. Batch <= 2 with 8 consumers
// keeps its shared memory to 110 KB so that, under programmatic dependent
// launch, the next kernel's CTA fits beside it and its producer prefills
// that kernel's weights while this one streams. Large batch-1/2 matrices
// (>= kWideRows rows) run 16 consumers: the consumers bound the stream
// there (about 0.7 us of issue per 18 KB stage with 8 of them), and twice
// the warps hide their latencies (the 66 MB gate/up matrix: 23.7 -> 18.4
// us per launch under programmatic dependent launch).
constexpr uint32_t kWideRows = 16384;
template <int NT, int CONS>
constexpr int kThreadsT = (CONS + 1) * 32;
template <int NT, int CONS>
constexpr size_t kSmemCap = (NT == 1 && CONS == 8) ? 110 * 1024 : 220 * 1024;  // dynamic shared memory per CTA

struct GemvP {
  const uint8_t *qs, *sc;
  b200_xq_t xq;  // input activations (xnorm: only batch, k and quads are used)
  const float *res;
  float *y;
  float *partial;        // [segment][batch][npad] split-K partial sums
  uint32_t *tile_cnt;    // split-K tickets, one per tile, left at zero
  uint32_t *grp_cnt;     // SILU_GLU re-quantisation tickets, one per 64-row group
  uint32_t *err;         // host-mapped error word (timeouts)
  uint64_t wait_ns;      // the context's limit on every wait
  b200_xq_t xo;          // SILU_GLU: re-quantised output (limbs == nullptr: none)
  uint32_t n, nout, units, ntiles, ngroups, upc, batch, npad;
  uint32_t resident;     // 1: all of x staged once per CTA (slot 0)
  uint32_t xslot_bytes;  // bytes of one staged-x slot
  int epi;
  // xnorm: x arrives in fp32 and each CTA applies RMSNorm (gamma, eps) and
  // quantises it into its resident x slot itself (no xq input, no norm kernel)
  int xnorm;
  const float *xf, *gamma;
  float eps;
};

// Work walk shared by the producer and the consumers of a CTA. The flat
// index pos = group * units + unit runs over all (8-tile group, K unit)
// pairs; CTA i owns [i*T/G, (i+1)*T/G) (stream-K), cut into sub-items that
// stay inside one group and hold at most `upc` units (one staged-x slot).
struct Sub {
  uint32_t g, u0, u1;
  bool first, last;  // starts / ends this CTA's segment of group g
};

// The CTA whose share holds flat position x: the largest i with
// floor(i*total/grid) <= x.
__device__ __forceinline__ uint32_t cta_of(uint64_t x, uint64_t total, uint32_t grid) {
  return (uint32_t)(((x + 1) * grid - 1) / total);
}

__device__ __forceinline__ Sub sub_at(const GemvP &p, uint64_t pos, uint64_t r0, uint64_t r1) {
  Sub s;
  s.g = (uint32_t)(pos / p.units);
  s.u0 = (uint32_t)(pos - (uint64_t)s.g * p.units);
  const uint64_t seg_end = min(r1, (uint64_t)(s.g + 1) * p.units);
  s.u1 = (uint32_t)min((uint64_t)s.u0 + p.upc, seg_end - (uint64_t)s.g * p.units);
  s.first = (pos == r0) || s.u0 == 0;
  s.last = (uint64_t)s.g * p.units + s.u1 == seg_end;
  return s;
}

// SiLU*up outputs wait for re-quantisation until all 4 tiles of their
// 64-row group are written (ticket per group); tickets are batched so one
// fence covers several.
struct Requant {
  uint32_t q[4];
  int n = 0;
  __device__ void flush(const GemvP &p, int lane) {
    if (n == 0) return;
    __threadfence();
    __syncwarp();
    for (int i = 0; i < n; i++) {
      uint32_t ticket = 0;
      if (lane == 0) ticket = atomicAdd(&p.grp_cnt[q[i]], 1u);
      ticket = __shfl_sync(0xffffffffu, ticket, 0);
      if (ticket == 3) {  // the last of the group's 4 tiles quantises outputs 32q..32q+31
        __threadfence();
        for (uint32_t vec = 0; vec < p.batch; vec++)
          xq_store_block(p.xo, vec, q[i], __ldcg(&p.y[(size_t)vec * p.nout + q[i] * 32 + lane]));
        if (lane == 0) p.grp_cnt[q[i]] = 0;
      }
    }
    n = 0;
  }
  __device__ void add(const GemvP &p, int lane, uint32_t group) {
    if (n == 4) flush(p, lane);
    q[n++] = group;
  }
};

// Final row sums of a tile (holder lanes: rows r and r+8 of vector
// 2nt + vsel) -> y through the epilogue.
template <int NT>
__device__ void finish_tile(const GemvP &p, uint32_t tile, int lane, const float (&ya)[NT], const float (&yb)[NT],
                            Requant &pend) {
  const uint32_t r = lane >> 2, vsel = (lane & 3) >> 1;
  const bool holder = (lane & 1) == 0;
  if (p.epi == B200_EPI_SILU_GLU) {
    // rows r (gate) and r+8 (up) of the tile are in the same lane
    const uint32_t o = tile * 8 + r;
    if (holder) {
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        const uint32_t vec = 2 * nt + vsel;
        if (vec < p.batch && o < p.nout) {
          const float gate = ya[nt], up = yb[nt];
          p.y[(size_t)vec * p.nout + o] = __fmul_rn(__fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate))), up);
        }
      }
    }
    if (p.xo.limbs) pend.add(p, lane, tile / 4);
    return;
  }
  if (!holder) return;
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const uint32_t vec = 2 * nt + vsel;
    if (vec >= p.batch) continue;
    const uint32_t row = tile * 16 + r;
    float a = ya[nt], b = yb[nt];
    if (p.epi == B200_EPI_RESIDUAL) {
      if (row < p.n) a = __fadd_rn(p.res[(size_t)vec * p.n + row], a);
      if (row + 8 < p.n) b = __fadd_rn(p.res[(size_t)vec * p.n + row + 8], b);
    }
    if (row < p.n) p.y[(size_t)vec * p.n + row] = a;
    if (row + 8 < p.n) p.y[(size_t)vec * p.n + row + 8] = b;
  }
}

// Take the split-K tickets of this warp's parked tiles; the last part of
// a tile to arrive adds all parts in CTA order and finishes the tile.
template <int NT>
__device__ void settle_splits(const GemvP &p, uint32_t (&tiles)[2], uint32_t (&nsegs)[2], int &n, int lane,
                              Requant &pend) {
  if (n == 0) return;
  const uint32_t r = lane >> 2, vsel = (lane & 3) >> 1;
  const bool holder = (lane & 1) == 0;
  __threadfence();
  __syncwarp();
  for (int i = 0; i < n; i++) {
    const uint32_t tile = tiles[i], nseg = nsegs[i];
    uint32_t ticket = 0;
    if (lane == 0) ticket = atomicAdd(&p.tile_cnt[tile], 1u);
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket != nseg - 1) continue;  // another part finishes this tile
    __threadfence();
    float ya[NT], yb[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      const uint32_t vec = 2 * nt + vsel;
      float a = 0.f, b = 0.f;
      if (holder && vec < p.batch) {
        // parts in CTA order, eight loads in flight at a time
        const float *pp = p.partial + (size_t)vec * p.npad + (size_t)tile * 16 + r;
        const size_t stride = (size_t)p.batch * p.npad;
        for (uint32_t q0 = 0; q0 < nseg; q0 += 8) {
          float ta[8], tb[8];
#pragma unroll
          for (int m = 0; m < 8; m++) {
            if (q0 + m < nseg) {
              ta[m] = __ldcg(pp + (q0 + m) * stride);
              tb[m] = __ldcg(pp + (q0 + m) * stride + 8);
            }
          }
#pragma unroll
          for (int m = 0; m < 8; m++) {
            if (q0 + m < nseg) {
              a += ta[m];
              b += tb[m];
            }
          }
        }
      }
      ya[nt] = a;
      yb[nt] = b;
    }
    if (lane == 0) p.tile_cnt[tile] = 0;
    finish_tile<NT>(p, tile, lane, ya, yb, pend);
  }
  n = 0;
}

// RMSNorm of x[batch][k] (pai_ref_rmsnorm_gamma_f32, ref_ops.c:196-216:
// the sum of squares in double, scale = 1/sqrtf(mean + eps), then
// (x*gamma)*scale with single roundings) computed by the 8 consumer warps
// of a CTA, quantised straight into the CTA's resident x slot. Warp c owns
// blocks c, c+8, c+16, ... (lane = element); each pass loads kPB of them at
// once and quantises them unrolled, so loads and warp reductions overlap
// instead of paying one L2 round trip per block.
constexpr int kPB = 16;
template <int NT, int CONS>
__device__ void norm_prologue(const GemvP &p, const XS &slot, int c, int lane, double (&red)[CONS][8]) {
  constexpr int kCons = CONS;
  const uint32_t nthr = kCons * 32, nblk = slot.quads * 4, kk = (uint32_t)p.xq.k;
  for (uint32_t vec = 0; vec < p.batch; vec++) {
    const float *xr = p.xf + (size_t)vec * kk;
    double acc = 0.0;
    for (uint32_t b0 = 0; b0 < nblk; b0 += kPB * kCons) {
      float xv[kPB];
#pragma unroll
      for (int m = 0; m < kPB; m++) {
        const uint32_t i = (b0 + m * kCons + c) * 32 + lane;
        xv[m] = i < kk ? xr[i] : 0.0f;
      }
#pragma unroll
      for (int m = 0; m < kPB; m++) acc = __dadd_rn(acc, __dmul_rn((double)xv[m], (double)xv[m]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) red[c][vec] = acc;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
  b200_xq_t v;
  v.limbs = const_cast<uint8_t *>(slot.limbs);
  v.sb = const_cast<float *>(slot.sb);
  v.sx = const_cast<float *>(slot.sx);
  v.batch = p.batch;
  v.k = kk;
  v.quads = slot.quads;
  for (uint32_t vec = 0; vec < p.batch; vec++) {
    double t = 0.0;
    for (int w = 0; w < kCons; w++) t += red[w][vec];
    const float ms = (float)__ddiv_rn(t, (double)kk);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
    const float *xr = p.xf + (size_t)vec * kk;
    for (uint32_t b0 = 0; b0 < nblk; b0 += kPB * kCons) {
      float xv[kPB];
#pragma unroll
      for (int m = 0; m < kPB; m++) {
        const uint32_t i = (b0 + m * kCons + c) * 32 + lane;
        xv[m] = i < kk ? __fmul_rn(__fmul_rn(xr[i], p.gamma[i]), scale) : 0.0f;
      }
#pragma unroll
      for (int m = 0; m < kPB; m++) {
        const uint32_t b = b0 + m * kCons + c;
        if (b < nblk) xq_store_block(v, vec, b, xv[m]);
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
}

template <uint32_t T, int NT, int CONS>
__global__ void __launch_bounds__(kThreadsT<NT, CONS>, 1) k_gemv(GemvP p) {
  constexpr int kCons = CONS;
  using Un = Unit<T>;
  constexpr int U = Un::U, XPU = Un::XPU;
  constexpr uint32_t GQ = kCons * Un::QB, GS = kCons * Un::SB;  // bytes of one unit of a group
  constexpr uint32_t STAGE = U * (GQ + GS);
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ __align__(8) uint64_t xfull[kXSlots], xempty[kXSlots];
  __shared__ double red[kCons][8];  // xnorm: per-warp sums of squares per vector

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t total = (uint64_t)p.ngroups * p.units;
  const uint64_t r0 = (uint64_t)blockIdx.x * total / gridDim.x;
  const uint64_t r1 = (uint64_t)(blockIdx.x + 1) * total / gridDim.x;
  uint8_t *ring = smem;                            // [kStages][STAGE]
  uint8_t *xbuf = smem + (size_t)kStages * STAGE;  // [kXSlots][xslot_bytes]
  const uint32_t xq_slot = p.upc * XPU;            // x-quads one slot holds
  auto slot_view = [&](int xs) {
    XS v;
    uint8_t *b = xbuf + (size_t)xs * p.xslot_bytes;
    v.limbs = b;
    v.sb = reinterpret_cast<const float *>(b + (size_t)NT * xq_slot * 1024);
    v.sx = v.sb + (size_t)p.batch * xq_slot * 4;
    v.quads = xq_slot;
    v.batch = p.batch;
    return v;
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCons);
    }
    for (int x = 0; x < kXSlots; x++) {
      mbar_init(&xfull[x], 1);
      mbar_init(&xempty[x], kCons);
    }
    fence_mbar_init();
    pdl_trigger();
  }
  __syncthreads();

  if (warp == 0) {
    // ---- producer (one thread): stage x, stream the weights of each sub-item ----
    if (lane != 0) return;
    bool ok = true;
    uint32_t xuse[kXSlots];
    for (int x = 0; x < kXSlots; x++) xuse[x] = 0;
    // x of quads [u0*XPU, u1*XPU) into slot xs, after the consumers released it
    auto stage_x = [&](int xs, uint32_t u0, uint32_t u1) {
      if (xuse[xs] > 0 && !mbar_wait(&xempty[xs], (xuse[xs] - 1) & 1u, p.wait_ns)) {
        ok = false;
        return;
      }
      xuse[xs]++;
      XS v = slot_view(xs);
      const uint32_t qx0 = u0 * XPU, nq = (u1 - u0) * XPU;
      fence_proxy_async();
      mbar_expect_tx(&xfull[xs], NT * nq * 1024 + 2 * p.batch * nq * 16);
      for (int nt = 0; nt < NT; nt++)
        bulk_g2s(const_cast<uint8_t *>(v.limbs) + (size_t)nt * xq_slot * 1024,
                 p.xq.limbs + ((size_t)nt * p.xq.quads + qx0) * 1024, nq * 1024, &xfull[xs]);
      for (uint32_t vec = 0; vec < p.batch; vec++) {
        bulk_g2s(const_cast<float *>(v.sb) + (size_t)vec * xq_slot * 4, p.xq.sb + ((size_t)vec * p.xq.quads + qx0) * 4,
                 nq * 16, &xfull[xs]);
        bulk_g2s(const_cast<float *>(v.sx) + (size_t)vec * xq_slot * 4, p.xq.sx + ((size_t)vec * p.xq.quads + qx0) * 4,
                 nq * 16, &xfull[xs]);
      }
    };
    // Weight walker: sub-item wi (w, at flat position wpos), next unit wu.
    uint32_t fill = 0, wi = 0;
    uint64_t wpos = r0;
    Sub w = sub_at(p, r0, r0, r1);
    uint32_t wu = w.u0;
    // Fill one ring stage at the weight walker; false once all are issued.
    auto fill_stage = [&]() -> bool {
      if (wpos >= r1) return false;
      const uint32_t ua = wu, ub = min(w.u1, ua + U), slot = fill % kStages;
      if (fill >= (uint32_t)kStages && !mbar_wait(&empty[slot], ((fill / kStages) - 1) & 1u, p.wait_ns)) {
        ok = false;
        return false;
      }
      const uint32_t nv = min((uint32_t)kCons, p.ntiles - w.g * kCons);  // tiles present in the group
      const size_t tile0 = (size_t)w.g * kCons;
      uint8_t *dst = ring + (size_t)slot * STAGE;
      mbar_expect_tx(&full[slot], (ub - ua) * nv * (Un::QB + Un::SB));
      for (uint32_t u = ua; u < ub; u++) {  // unit-major: the group's tiles of one unit are contiguous
        const size_t t0 = (size_t)u * p.ntiles + tile0;
        bulk_g2s(dst + (u - ua) * GQ, p.qs + t0 * Un::QB, nv * Un::QB, &full[slot]);
        bulk_g2s(dst + U * GQ + (u - ua) * GS, p.sc + t0 * Un::SB, nv * Un::SB, &full[slot]);
      }
      fill++;
      wu = ub;
      if (wu >= w.u1) {
        wpos += w.u1 - w.u0;
        wi++;
        if (wpos < r1) {
          w = sub_at(p, wpos, r0, r1);
          wu = w.u0;
        }
      }
      return true;
    };
    // The weights do not depend on the previous kernel: fill the ring
    // before waiting for it.
    for (int i = 0; i < kStages && fill_stage(); i++) {
    }
    pdl_wait();
    if (p.resident && !p.xnorm && ok) stage_x(0, 0, p.units);
    uint64_t xpos = r0;  // x walker: next sub-item whose x is staged (index xi)
    uint32_t xi = 0;
    while (ok) {
      // x stays one sub-item ahead of the weights
      while (!p.resident && ok && xpos < r1 && xi <= wi + 1) {
        const Sub sx = sub_at(p, xpos, r0, r1);
        stage_x((int)(xi % kXSlots), sx.u0, sx.u1);
        xpos += sx.u1 - sx.u0;
        xi++;
      }
      if (!ok || !fill_stage()) break;
    }
    if (!ok) {
      // A wait ran out: raise the error, let this CTA's copies land
      // (bounded), and stop; the consumers time out on their own waits.
      atomicExch(p.err, 1u);
      for (uint32_t f = fill > (uint32_t)kStages ? fill - kStages : 0; f < fill; f++)
        mbar_wait(&full[f % kStages], (f / kStages) & 1u, p.wait_ns);
      for (int x = 0; x < kXSlots; x++)
        if (xuse[x]) mbar_wait(&xfull[x], (xuse[x] - 1) & 1u, p.wait_ns);
    }
    return;
  }

  // ---- consumers: warp c owns tile c of every group ----
  pdl_wait();  // before the prologue reads x and the epilogue writes y and scratch
  const int c = warp - 1;
  const uint32_t r = lane >> 2;
  const bool holder = (lane & 1) == 0;  // c = 0 (even vector of the pair) or c = 2 (odd)
  const uint32_t vsel = (lane & 3) >> 1;
  uint32_t seq = 0, xuse = 0;
  int xs = 0;
  float yr[NT], yr8[NT];
  uint32_t split_tile[2], split_n[2];
  int nsplit = 0;
  Requant pend;
  if (p.xnorm) {
    norm_prologue<NT, CONS>(p, slot_view(0), c, lane, red);
  } else if (p.resident && !mbar_wait(&xfull[0], 0, p.wait_ns)) {
    if (lane == 0) atomicExch(p.err, 1u);
    return;
  }
  for (uint64_t pos = r0; pos < r1;) {
    const Sub s = sub_at(p, pos, r0, r1);
    pos += s.u1 - s.u0;
    if (!p.resident && !mbar_wait(&xfull[xs], (xuse / kXSlots) & 1u, p.wait_ns)) {
      if (lane == 0) atomicExch(p.err, 1u);
      return;
    }
    const XS v = slot_view(p.resident ? 0 : xs);
    const uint32_t xu0 = p.resident ? 0 : s.u0;  // unit held at the slot's start
    const uint32_t tile = s.g * kCons + c;
    const bool active = tile < p.ntiles;
    if (s.first) {
#pragma unroll
      for (int nt = 0; nt < NT; nt++) yr[nt] = yr8[nt] = 0.f;
    }
    for (uint32_t ua = s.u0; ua < s.u1; ua += U) {
      const uint32_t slot = seq % kStages, par = (seq / kStages) & 1u;
      if (!mbar_wait(&full[slot], par, p.wait_ns)) {
        if (lane == 0) atomicExch(p.err, 1u);
        return;
      }
      if (active) {
        const uint8_t *st = ring + (size_t)slot * STAGE;
#pragma unroll
        for (int uu = 0; uu < U; uu++) {
          const uint32_t u = ua + uu;
          if (u < s.u1)
            Un::template compute<NT>(st + uu * GQ + c * Un::QB, st + U * GQ + uu * GS + c * Un::SB, v,
                                     (u - xu0) * XPU, lane, yr, yr8);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      seq++;
    }
    if (!p.resident) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&xempty[xs]);  // this warp is done with the x slot
      xs = (xs + 1) % kXSlots;
      xuse++;
    }
    if (!s.last || !active) continue;

    // ---- segment finished ----
    const uint32_t cta_lo = cta_of((uint64_t)s.g * p.units, total, gridDim.x);
    const uint32_t nseg = cta_of((uint64_t)(s.g + 1) * p.units - 1, total, gridDim.x) - cta_lo + 1;
    float ya[NT], yb[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {  // lane pairs (c, c^1) hold the two halves of one sum
      ya[nt] = yr[nt] + __shfl_xor_sync(0xffffffffu, yr[nt], 1);
      yb[nt] = yr8[nt] + __shfl_xor_sync(0xffffffffu, yr8[nt], 1);
    }
    if (nseg == 1) {
      finish_tile<NT>(p, tile, lane, ya, yb, pend);
      continue;
    }
    // part of a split tile: park the partial sums; the ticket is taken at
    // the end, so the fence it needs does not stall the ring
    const uint32_t split = blockIdx.x - cta_lo;
    if (holder) {
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        const uint32_t vec = 2 * nt + vsel;
        if (vec < p.batch) {
          float *pp = p.partial + ((size_t)split * p.batch + vec) * p.npad + (size_t)tile * 16 + r;
          pp[0] = ya[nt];
          pp[8] = yb[nt];
        }
      }
    }
    if (nsplit == 2) settle_splits<NT>(p, split_tile, split_n, nsplit, lane, pend);  // only first and last split
    split_tile[nsplit] = tile;
    split_n[nsplit++] = nseg;
  }
  settle_splits<NT>(p, split_tile, split_n, nsplit, lane, pend);
  pend.flush(p, lane);
}

int sm_count(pai_b200_ctx_t *ctx) {
  static std::atomic<int> cached[64];
  int dev = b200_ctx_device(ctx);
  if (dev >= 0 && dev < 64) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c) return c;
  }
  int v = 148;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev].store(v, std::memory_order_relaxed);
  return v;
}

template <uint32_t T, int NT, int CONS>
pai_status_t launch_t(pai_b200_ctx_t *ctx, GemvP p) {
  auto kern = k_gemv<T, NT, CONS>;
  using Un = Unit<T>;
  constexpr int kCons = CONS;
  const size_t ring = (size_t)kStages * Un::U * kCons * (Un::QB + Un::SB);
  p.ngroups = (p.ntiles + kCons - 1) / kCons;
  const uint64_t total = (uint64_t)p.ngroups * p.units;
  const uint32_t grid = (uint32_t)std::min<uint64_t>(total, (uint64_t)sm_count(ctx));
  // x staging: all of x once per CTA when it fits beside the ring (one
  // bulk copy up front keeps the producer free to stream weights; staging
  // x per sub-item made the producer wait on x slots: the 66 MB gate/up
  // matrix went from 23.7 to 21.3 us per launch this way); else three
  // slots of up to `upc` units, refilled one sub-item ahead.
  const size_t per_unit_x = (size_t)Un::XPU * (NT * 1024 + 2 * p.batch * 16);
  const size_t room = kSmemCap<NT, CONS> - ring;
  const bool fits = p.units * per_unit_x + 256 <= room;
  if (p.xnorm && !fits)
    return b200_fail(PAI_ERR_UNSUPPORTED, "gemv: x of %u units does not fit for the fused norm", p.units);
  if (fits) {
    p.resident = 1;
    p.upc = p.units;
  } else {
    p.resident = 0;
    p.upc = (uint32_t)std::max<size_t>(Un::U, (room / kXSlots - 256) / per_unit_x);
  }
  const size_t xq_slot = (size_t)p.upc * Un::XPU;
  p.xslot_bytes = (uint32_t)b200_align256(NT * xq_slot * 1024 + 2 * (size_t)p.batch * xq_slot * 16);
  const size_t smem = ring + (p.resident ? 1 : kXSlots) * (size_t)p.xslot_bytes;
  if (smem > kSmemCap<NT, CONS>) return b200_fail(PAI_ERR_UNSUPPORTED, "gemv: %zu B of shared memory", smem);
  // Function attributes are set once per device (the largest size seen),
  // not per launch: they cost host time on the decode path.
  static SmemOptIn opt;
  pai_status_t st = b200_cuda(opt.ensure(b200_ctx_device(ctx), smem,
                                         [&](size_t b) {
                                           cudaError_t e = cudaFuncSetAttribute(
                                               kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)b);
                                           if (e == cudaSuccess)
                                             e = cudaFuncSetAttribute(
                                                 kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
                                           return e;
                                         }),
                              "k_gemv smem attribute");
  if (st) return st;
  // Most segments a group can be cut into: a CTA's share is at least
  // floor(total / grid) units, so a group of `units` meets at most
  // ceil(units / share) + 1 CTAs.
  const uint64_t share = total / grid;
  const uint32_t maxseg = (uint32_t)std::min<uint64_t>(grid, (p.units + share - 1) / share + 1);
  const uint32_t ngroups4 = (p.ntiles + 3) / 4;
  float *partial = nullptr;
  uint32_t *cnt = nullptr;
  st = b200_ctx_scratch(ctx, maxseg > 1 ? (uint64_t)maxseg * p.batch * p.npad : 0, p.ntiles + ngroups4, &partial,
                        &cnt);
  if (st) return st;
  p.partial = partial;
  p.tile_cnt = cnt;
  p.grp_cnt = cnt + p.ntiles;
  p.err = b200_ctx_errflag(ctx);
  p.wait_ns = b200_ctx_wait_ns(ctx);
  b200_launch(ctx, kern, dim3(grid), dim3(kThreadsT<NT, CONS>), smem, p);
  return b200_launched(ctx, 1, "k_gemv");
}

template <uint32_t T>
pai_status_t launch_b(pai_b200_ctx_t *ctx, const GemvP &p) {
  switch ((p.batch + 1) / 2) {
    case 1: return p.n >= kWideRows ? launch_t<T, 1, 16>(ctx, p) : launch_t<T, 1, 8>(ctx, p);
    case 2: return launch_t<T, 2, 8>(ctx, p);
    case 3: return launch_t<T, 3, 8>(ctx, p);
    default: return launch_t<T, 4, 8>(ctx, p);
  }
}

// Quantise x[batch][k] into xq: one warp per 32-element block, including
// the zero padding blocks of the last x-quad (whose scales must read 0).
__global__ void __launch_bounds__(256) k_xprep(const float *__restrict__ x, uint64_t k, b200_xq_t xq) {
  const uint32_t vec = blockIdx.y;
  const uint64_t b = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (b >= xq.quads * 4) return;
  const float v = b * 32 < k ? x[(size_t)vec * k + b * 32 + (threadIdx.x & 31)] : 0.0f;
  xq_store_block(xq, vec, (uint32_t)b, v);
}

// Shared argument checks and parameter set-up of both GEMV launchers; x is
// either xq (staged by the producer) or fp32 x with RMSNorm applied in the
// kernel (xf != nullptr).
pai_status_t gemv_launch(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch, uint64_t n, uint64_t k, const void *w,
                         const b200_xq_t *xq, const float *xf, const float *gamma, float eps, const float *residual,
                         float *y, int epi, const b200_xq_t *xq_out) {
  if (!ctx || !w || (!xq && !(xf && gamma)) || !y) return b200_fail(PAI_ERR_INVALID_ARG, "gemv: NULL pointer");
  if (!b200_type_ok(type)) return b200_fail(PAI_ERR_UNSUPPORTED, "gemv: block type %u", type);
  if (n == 0 || k == 0 || k % b200_blk_elems(type))
    return b200_fail(PAI_ERR_MISMATCH, "gemv: k=%llu is not a whole number of %u-element blocks",
                     (unsigned long long)k, b200_blk_elems(type));
  if (batch == 0 || batch > 8) return b200_fail(PAI_ERR_UNSUPPORTED, "gemv: batch %u (1..8)", batch);
  if (n > 0x7FFFFFF0ull || k > 0x7FFFFFFFull) return b200_fail(PAI_ERR_UNSUPPORTED, "gemv: shape too large");
  if (xq && (xq->batch < batch || xq->k < k)) return b200_fail(PAI_ERR_MISMATCH, "gemv: activation buffer too small");
  if (epi == B200_EPI_RESIDUAL && !residual) return b200_fail(PAI_ERR_INVALID_ARG, "gemv: NULL residual");
  if (epi == B200_EPI_SILU_GLU && (n % 64 || (xq_out && (xq_out->batch < batch || xq_out->k < n / 2))))
    return b200_fail(PAI_ERR_MISMATCH, "gemv: gate/up rows must come in 64-row groups");
  if ((uintptr_t)w & 255) return b200_fail(PAI_ERR_INVALID_ARG, "gemv: weights not 256-byte aligned");
  GemvP p{};
  p.qs = (const uint8_t *)w;
  p.sc = p.qs + b200_sc_offset(type, n, k);
  if (xq) {
    p.xq = *xq;
  } else {
    p.xnorm = 1;
    p.xf = xf;
    p.gamma = gamma;
    p.eps = eps == 0.0f ? 1e-5f : eps;
    p.xq.batch = batch;
    p.xq.k = k;
    p.xq.quads = b200_xq_quads(k);
  }
  p.res = residual;
  p.y = y;
  if (epi == B200_EPI_SILU_GLU && xq_out) p.xo = *xq_out;
  p.n = (uint32_t)n;
  p.nout = (uint32_t)(n / 2);
  p.units = (uint32_t)b200_units(type, k);
  p.ntiles = (uint32_t)b200_ntiles(n);
  p.npad = p.ntiles * 16;
  p.batch = batch;
  p.epi = epi;
  switch (type) {
    case PAI_B200_Q4_0: return launch_b<PAI_B200_Q4_0>(ctx, p);
    case PAI_B200_Q8_0: return launch_b<PAI_B200_Q8_0>(ctx, p);
    default: return launch_b<PAI_B200_Q4_K>(ctx, p);
  }
}

}  // namespace

extern "C" pai_status_t b200_launch_xprep(pai_b200_ctx_t *ctx, uint32_t batch, uint64_t k, const float *x,
                                          const b200_xq_t *xq) {
  const uint64_t nb = xq->quads * 4;
  k_xprep<<<dim3((unsigned)((nb + 7) / 8), batch), 256, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(x, k, *xq);
  return b200_launched(ctx, 1, "k_xprep");
}

extern "C" pai_status_t b200_launch_gemv(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch, uint64_t n,
                                         uint64_t k, const void *w, const b200_xq_t *xq, const float *residual,
                                         float *y, int epi, const b200_xq_t *xq_out) {
  if (!xq) return b200_fail(PAI_ERR_INVALID_ARG, "gemv: NULL activations");
  return gemv_launch(ctx, type, batch, n, k, w, xq, nullptr, nullptr, 0.0f, residual, y, epi, xq_out);
}

extern "C" pai_status_t b200_launch_gemv_norm(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch, uint64_t n,
                                              uint64_t k, const void *w, const float *x, const float *gamma,
                                              float eps, const float *residual, float *y, int epi,
                                              const b200_xq_t *xq_out) {
  return gemv_launch(ctx, type, batch, n, k, w, nullptr, x, gamma, eps, residual, y, epi, xq_out);
}

// Public GEMV: x arrives in fp32, is quantised into the context's
// activation scratch, then multiplied.
static pai_status_t gemv_public(pai_b200_ctx_t *ctx, uint32_t type, uint64_t batch, uint64_t n, uint64_t k,
                                const void *w, const float *x, const float *residual, float *y) {
  if (!ctx || !x) return b200_fail(PAI_ERR_INVALID_ARG, "gemv: NULL pointer");
  if (batch == 0 || batch > 8)
    return b200_fail(PAI_ERR_UNSUPPORTED, "gemv: batch %llu (1..8)", (unsigned long long)batch);
  if (!b200_type_ok(type) || k == 0 || k % b200_blk_elems(type))
    return b200_fail(b200_type_ok(type) ? PAI_ERR_MISMATCH : PAI_ERR_UNSUPPORTED, "gemv: type %u with k=%llu", type,
                     (unsigned long long)k);
  void *buf = nullptr;
  pai_status_t st = b200_ctx_xq(ctx, b200_xq_bytes((uint32_t)batch, k), &buf);
  if (st) return st;
  b200_xq_t xq = b200_xq_view(buf, (uint32_t)batch, k);
  st = b200_launch_xprep(ctx, (uint32_t)batch, k, x, &xq);
  if (st) return st;
  return b200_launch_gemv(ctx, type, (uint32_t)batch, n, k, w, &xq, residual, y,
                          residual ? B200_EPI_RESIDUAL : B200_EPI_STORE, nullptr);
}

extern "C" pai_status_t pai_b200_gemv_f32(pai_b200_ctx_t *ctx, uint32_t type, uint64_t batch, uint64_t n,
                                          uint64_t k, const void *w, const float *x, const float *residual,
                                          float *y) {
  return gemv_public(ctx, type, batch, n, k, w, x, residual, y);
}
extern "C" pai_status_t pai_b200_gemv_q8_0_f32(pai_b200_ctx_t *ctx, uint64_t n, uint64_t k, const void *w,
                                               const float *x, float *y) {
  return gemv_public(ctx, PAI_B200_Q8_0, 1, n, k, w, x, nullptr, y);
}
extern "C" pai_status_t pai_b200_gemv_q4_0_f32(pai_b200_ctx_t *ctx, uint64_t n, uint64_t k, const void *w,
                                               const float *x, float *y) {
  return gemv_public(ctx, PAI_B200_Q4_0, 1, n, k, w, x, nullptr, y);
}
extern "C" pai_status_t pai_b200_gemv_q4_k_f32(pai_b200_ctx_t *ctx, uint64_t n, uint64_t k, const void *w,
                                               const float *x, float *y) {
  return gemv_public(ctx, PAI_B200_Q4_K, 1, n, k, w, x, nullptr, y);
}

extern "C" uint64_t pai_b200_xq_bytes(uint64_t batch, uint64_t k) {
  return (batch == 0 || batch > 8 || k == 0) ? 0 : b200_xq_bytes((uint32_t)batch, k);
}

extern "C" pai_status_t pai_b200_prepare_x_f32(pai_b200_ctx_t *ctx, uint64_t batch, uint64_t k, const float *x,
                                               void *xq) {
  if (!ctx || !x || !xq) return b200_fail(PAI_ERR_INVALID_ARG, "prepare_x: NULL pointer");
  if (batch == 0 || batch > 8)
    return b200_fail(PAI_ERR_UNSUPPORTED, "prepare_x: batch %llu (1..8)", (unsigned long long)batch);
  if (k == 0 || k % 32)
    return b200_fail(PAI_ERR_MISMATCH, "prepare_x: k=%llu is not a multiple of 32", (unsigned long long)k);
  if ((uintptr_t)xq & 255) return b200_fail(PAI_ERR_INVALID_ARG, "prepare_x: buffer not 256-byte aligned");
  const b200_xq_t v = b200_xq_view(xq, (uint32_t)batch, k);
  return b200_launch_xprep(ctx, (uint32_t)batch, k, x, &v);
}

extern "C" pai_status_t pai_b200_gemv_prepared_f32(pai_b200_ctx_t *ctx, uint32_t type, uint64_t batch, uint64_t n,
                                                   uint64_t k, const void *w, const void *xq, const float *residual,
                                                   float *y) {
  if (!ctx || !xq) return b200_fail(PAI_ERR_INVALID_ARG, "gemv_prepared: NULL pointer");
  if (batch == 0 || batch > 8)
    return b200_fail(PAI_ERR_UNSUPPORTED, "gemv_prepared: batch %llu (1..8)", (unsigned long long)batch);
  if (!b200_type_ok(type) || k == 0 || k % b200_blk_elems(type))
    return b200_fail(b200_type_ok(type) ? PAI_ERR_MISMATCH : PAI_ERR_UNSUPPORTED, "gemv_prepared: type %u with k=%llu",
                     type, (unsigned long long)k);
  const b200_xq_t v = b200_xq_view(const_cast<void *>(xq), (uint32_t)batch, k);
  return b200_launch_gemv(ctx, type, (uint32_t)batch, n, k, w, &v, residual, y,
                          residual ? B200_EPI_RESIDUAL : B200_EPI_STORE, nullptr);
}

extern "C" pai_status_t pai_b200_gemv_rmsnorm_f32(pai_b200_ctx_t *ctx, uint32_t type, uint64_t batch, uint64_t n,
                                                  uint64_t k, const void *w, const float *x, const float *gamma,
                                                  float eps, const float *residual, float *y) {
  if (!ctx || !x || !gamma) return b200_fail(PAI_ERR_INVALID_ARG, "gemv_rmsnorm: NULL pointer");
  return b200_launch_gemv_norm(ctx, type, (uint32_t)batch, n, k, w, x, gamma, eps, residual, y,
                               residual ? B200_EPI_RESIDUAL : B200_EPI_STORE, nullptr);
}
