// Persistent decode step: one cooperative launch runs the layers of a
// greedy decode step of the LLaMA-shaped model -- embedding row, every layer
// (RMSNorm, the fused q|k|v GEMV, RoPE + K/V append + attention over the fp16
// cache, the o GEMV with the residual add, RMSNorm, the gate|up GEMV with
// SiLU*up, the down GEMV with the residual add; adapters/llama/llama.c:
// 669-797) and the final RMSNorm -- as a list of phases over one CTA per SM.
// The lm head (a matrix of the embedding's block type) and the greedy pick
// follow as the regular GEMV and argmax launches (k_gemv.cu, k_ops.cu).
//
// Why one kernel: a decode step at batch 1 is ~230 small dependent
// operations. As separate launches each GEMV pays a ramp to first data, a
// tail and a launch gap that do not shrink with its size (about 10 us per
// matrix on B200, against 1.5-10 us of streaming at HBM speed). Here:
//
//  * One producer thread per CTA streams the packed weights of every GEMV
//    phase of the step, in phase order, with bulk asynchronous copies
//    (cp.async.bulk, mbarrier completion, no multicast) into a 4-stage
//    shared-memory ring. Weights never depend on activations, so the
//    producer does not wait for phases to finish: while the consumers sit at
//    a grid barrier or compute attention, the next matrix is already landing
//    in shared memory. The HBM stream runs across phase boundaries.
//  * CONS consumer warps run the phases in order. Between dependent phases
//    they meet at a grid barrier (one arrival counter in global memory,
//    bounded spin, release/acquire at GPU scope). The producer never joins
//    a barrier.
//  * GEMV phases reuse the fused dequantise-and-dot arithmetic of k_gemv.cu
//    (gemv_unit.cuh): warp c owns tile c of each CONS-tile row group, the
//    (group, K unit) pairs are split stream-K over the CTAs, split tiles are
//    summed by their last contributor (tickets), and the epilogues store,
//    add the residual, or apply SiLU*up and re-quantise for the down GEMV.
//    The activation operand of each phase is staged into shared memory by
//    the consumers after the barrier: for a normed input every CTA computes
//    the row's RMSNorm scale itself (same order in every CTA, so the same
//    bits) and quantises only the K units its range uses.
//  * Attention items are (sequence, kv head, position chunk): q and k are
//    rotated at the position, the CTA whose chunk holds the position appends
//    k and v to the cache, scores and exp-weighted V run over the chunk in
//    rounds of kAttnSub positions with a running max, and the last chunk of
//    a (sequence, kv head) to finish merges the chunks and quantises the
//    output for the o GEMV.
//  * The final RMSNorm phase quantises the last hidden state into the lm
//    head's operand, a slice of blocks per CTA.
//  * The kernel is compiled per block type of the layer matrices
//    (k_decode_q4_0.cu, ...): one GEMV path per kernel keeps the consumers
//    within 128 registers without spills.
//
// All data written inside the launch and read by another CTA is read with
// ld.global.cg (L2): L1 is not coherent across SMs. Every wait is bounded by
// %globaltimer; on timeout the kernel raises the context's error word and a
// device abort word that ends the other CTAs' waits, and every consumer
// thread leaves through the same barrier points, so no named barrier is
// left short of arrivals.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <new>

#include "../b200_internal.h"
#include "b200_device.cuh"
#include "gemv_unit.cuh"

namespace b200dec {

using namespace gemv;

constexpr int kStages = 4;
// bytes of one ring stage: the largest of U units x CONS tiles x (codes +
// headers) over the block types (Q4_0: 2 x 1152, Q8_0: 2176, Q4_K: 2304)
template <int CONS>
constexpr uint32_t kStageBytes = CONS * 2304u;
constexpr uint32_t kHD = 128;
constexpr uint32_t kAttnSub = 256;  // positions per running-softmax round of an attention item

// Device form of a phase: b200_phase_t plus the shape of its work split.
struct DPh {
  uint32_t kind, type, epi, xsrc;
  const uint8_t *qs, *sc;
  uint32_t n, k, nout, units, ntiles, ngroups, npad, maxseg;
  const float *xf, *gamma;
  b200_xq_t xq;
  const float *res;
  float *y;
  b200_xq_t xo;
  uint32_t layer, xi;  // attention: cache layer; EPI_PUSH / XCHG: index of the row exchange in the step
};

struct KP {
  const DPh *__restrict__ ph;
  uint32_t nph, batch;
  float eps;
  // embedding
  uint32_t etype, n_embd;
  const uint8_t *emb_qs, *emb_sc;
  uint64_t emb_ntiles;
  const int32_t *tok_in;
  float *x;
  // attention
  uint32_t h, hk, per_head;
  int32_t *pos;
  uint64_t cap, seq_stride, layer_stride;
  __half *kc, *vc;
  const float *cos_t, *sin_t;
  const float *qkv;
  float *att;
  b200_xq_t xq_att;
  float inv_scale;
  // scratch
  float *partial;      // split-K partial sums [split][batch][npad]
  uint32_t *tile_cnt;  // split-K tickets (left at zero)
  uint32_t *grp_cnt;   // SiLU*up re-quantisation tickets (left at zero)
  float *apart;        // attention chunk partials [batch][h][per_head][kHD + 2]
  uint32_t *attn_cnt;  // attention merge tickets [batch][hk] (left at zero)
  uint32_t *bar;       // [0] barrier arrivals, [1] exits, [2] abort
  uint32_t *err;       // the context's host-mapped error word
  uint64_t wait_ns;
  // tensor parallelism: every rank's landing buffer as mapped here
  uint8_t *land[B200_TP_MAX_RANKS];
  uint32_t rank, nranks;
  uint32_t xrows;  // floats per landing slot (batch x n_embd)
  uint32_t nx;     // row exchanges per step
};

__device__ __forceinline__ uint64_t *land_words(uint8_t *b) { return reinterpret_cast<uint64_t *>(b); }
__device__ __forceinline__ float *land_rows(const KP &p, uint32_t r, uint32_t parity, uint32_t src) {
  return reinterpret_cast<float *>(p.land[r] + B200_LAND_HDR) + ((size_t)parity * p.nranks + src) * p.xrows;
}
__device__ __forceinline__ uint64_t ld_acquire_sys64(const uint64_t *q) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(q) : "memory");
  return v;
}

__device__ __forceinline__ void cbar(int nthr) { asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory"); }

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void raise_abort(const KP &p) {
  atomicExch(p.bar + 2, 1u);
  atomicExch(p.err, 1u);
}

// Grid barrier of the consumer threads of every CTA. The CTA's consumers
// first meet at named barrier 1; one thread publishes the CTA's writes
// (fence), arrives, and waits (bounded; an abort raised elsewhere ends the
// wait) until all CTAs arrived at this barrier. Returns the same answer to
// every consumer thread of the CTA.
__device__ inline bool grid_sync(const KP &p, uint32_t &epoch, int ctid, int nthr, volatile int *sflag) {
  cbar(nthr);
  if (ctid == 0) {
    epoch++;
    bool ok = true;
    __threadfence();
    atomicAdd(p.bar, 1u);
    const uint32_t target = epoch * gridDim.x;
    uint64_t t0 = 0;
    for (uint32_t it = 0;; it++) {
      if (ld_acquire_gpu(p.bar) >= target) break;
      if ((it & 63u) == 0) {
        if (*(volatile uint32_t *)(p.bar + 2)) {
          ok = false;
          break;
        }
        const uint64_t now = globaltimer_ns();
        if (it == 0) {
          t0 = now;
        } else if (now - t0 > p.wait_ns) {
          raise_abort(p);
          ok = false;
          break;
        }
      }
    }
    __threadfence();
    *sflag = ok ? 1 : 0;
  }
  cbar(nthr);
  return *sflag != 0;
}

// ---- GEMV phases ------------------------------------------------------------------------

// CTAs a GEMV phase's work is split over: every CTA when the phase has at
// least one (group, unit) pair per CTA, else one pair each for the first
// `total` CTAs (the rest idle). No CTA inside the split has an empty range,
// so the CTAs that meet a row group are consecutive owners of its pairs.
__device__ __forceinline__ uint32_t work_grid(const DPh &ph) {
  return (uint32_t)min((uint64_t)gridDim.x, (uint64_t)ph.ngroups * ph.units);
}

__device__ __forceinline__ void phase_range(const DPh &ph, uint64_t &r0, uint64_t &r1) {
  const uint64_t total = (uint64_t)ph.ngroups * ph.units;
  const uint32_t gw = work_grid(ph);
  if (blockIdx.x >= gw) {
    r0 = r1 = total;
    return;
  }
  r0 = (uint64_t)blockIdx.x * total / gw;
  r1 = (uint64_t)(blockIdx.x + 1) * total / gw;
}

// A piece of a CTA's range inside one row group: units [u0, u1) of group g.
struct Sub {
  uint32_t g, u0, u1;
  bool first, last;  // starts / ends this CTA's segment of group g
};

__device__ __forceinline__ Sub sub_at(const DPh &ph, uint64_t pos, uint64_t r0, uint64_t r1) {
  Sub s;
  s.g = (uint32_t)(pos / ph.units);
  s.u0 = (uint32_t)(pos - (uint64_t)s.g * ph.units);
  const uint64_t seg_end = min(r1, (uint64_t)(s.g + 1) * ph.units);
  s.u1 = (uint32_t)(seg_end - (uint64_t)s.g * ph.units);
  s.first = (pos == r0) || s.u0 == 0;
  s.last = true;  // a sub-item always runs to the end of the CTA's segment of its group
  return s;
}

__device__ __forceinline__ uint32_t cta_of(uint64_t x, uint64_t total, uint32_t grid) {
  return (uint32_t)(((x + 1) * grid - 1) / total);
}

// Producer: stream the weights of the CTA's range of one GEMV phase into the
// ring, one stage per U units of a sub-item. Returns false when a wait for
// a free stage ran out.
template <uint32_t T, int CONS>
__device__ bool produce(const KP &p, const DPh &ph, uint8_t *ring, uint64_t *full, uint64_t *empty,
                        uint32_t &fill) {
  using Un = Unit<T>;
  constexpr int U = Un::U;
  constexpr uint32_t GQ = CONS * Un::QB, GS = CONS * Un::SB;
  uint64_t r0, r1;
  phase_range(ph, r0, r1);
  for (uint64_t pos = r0; pos < r1;) {
    const Sub s = sub_at(ph, pos, r0, r1);
    pos += s.u1 - s.u0;
    const uint32_t nv = min((uint32_t)CONS, ph.ntiles - s.g * CONS);  // tiles present in the group
    const size_t tile0 = (size_t)s.g * CONS;
    for (uint32_t ua = s.u0; ua < s.u1; ua += U) {
      const uint32_t ub = min(s.u1, ua + U), slot = fill % kStages;
      if (fill >= (uint32_t)kStages && !mbar_wait(&empty[slot], ((fill / kStages) - 1) & 1u, p.wait_ns)) return false;
      uint8_t *dst = ring + (size_t)slot * kStageBytes<CONS>;
      mbar_expect_tx(&full[slot], (ub - ua) * nv * (Un::QB + Un::SB));
      for (uint32_t u = ua; u < ub; u++) {  // unit-major: the group's tiles of one unit are contiguous
        const size_t t0 = (size_t)u * ph.ntiles + tile0;
        bulk_g2s(dst + (u - ua) * GQ, ph.qs + t0 * Un::QB, nv * Un::QB, &full[slot]);
        bulk_g2s(dst + U * GQ + (u - ua) * GS, ph.sc + t0 * Un::SB, nv * Un::SB, &full[slot]);
      }
      fill++;
    }
  }
  return true;
}

// Shared-memory view of the staged activation operand of the CTA's range:
// entry e holds the XPU x-quads of one K unit; with a range of at least a
// whole group every unit has its own entry (entry = unit), otherwise entry e
// belongs to flat position r0 + e.
struct XArea {
  XS xs;
  uint32_t nent;
  bool resident;
};

template <int NT, int XPU>
__device__ __forceinline__ XArea x_area(const KP &p, const DPh &ph, uint8_t *area, uint64_t r0, uint64_t r1) {
  XArea a;
  const uint64_t L = r1 - r0;
  a.resident = L >= ph.units;
  a.nent = a.resident ? ph.units : (uint32_t)L;
  const uint32_t nq = a.nent * XPU;
  a.xs.limbs = area;
  a.xs.sb = reinterpret_cast<const float *>(area + (size_t)NT * nq * 1024);
  a.xs.sx = a.xs.sb + (size_t)p.batch * nq * 4;
  a.xs.quads = nq;
  a.xs.batch = p.batch;
  return a;
}

__device__ __forceinline__ uint32_t entry_unit(const DPh &ph, const XArea &a, uint64_t r0, uint32_t e) {
  return a.resident ? e : (uint32_t)((r0 + e) % ph.units);
}

// Copy the quantised input of the entries from global memory (written by an
// earlier phase of this launch: read through L2).
template <int NT, int XPU>
__device__ void stage_xq(const DPh &ph, const XArea &a, uint64_t r0, uint32_t batch, int ctid, int nthr) {
  const uint32_t nq = a.nent * XPU, per = NT * XPU * 64;  // uint4 per entry (digits)
  uint4 *dl = reinterpret_cast<uint4 *>(const_cast<uint8_t *>(a.xs.limbs));
  const uint4 *sl = reinterpret_cast<const uint4 *>(ph.xq.limbs);
  for (uint32_t i = ctid; i < a.nent * per; i += nthr) {
    const uint32_t e = i / per, r = i % per, nt = r / (XPU * 64), o = r % (XPU * 64);
    const uint32_t u = entry_unit(ph, a, r0, e);
    dl[(((size_t)nt * nq + (size_t)e * XPU) * 1024) / 16 + o] =
        __ldcg(sl + (((size_t)nt * ph.xq.quads + (size_t)u * XPU) * 1024) / 16 + o);
  }
  float4 *db = reinterpret_cast<float4 *>(const_cast<float *>(a.xs.sb));
  float4 *dx = reinterpret_cast<float4 *>(const_cast<float *>(a.xs.sx));
  const float4 *sb = reinterpret_cast<const float4 *>(ph.xq.sb);
  const float4 *sx = reinterpret_cast<const float4 *>(ph.xq.sx);
  for (uint32_t i = ctid; i < a.nent * batch * XPU; i += nthr) {
    const uint32_t e = i / (batch * XPU), r = i % (batch * XPU), vec = r / XPU, q = r % XPU;
    const uint32_t u = entry_unit(ph, a, r0, e);
    const size_t s = (size_t)vec * ph.xq.quads + (size_t)u * XPU + q, d = (size_t)vec * nq + (size_t)e * XPU + q;
    db[d] = __ldcg(sb + s);
    dx[d] = __ldcg(sx + s);
  }
}

// RMSNorm of the fp32 rows (pai_ref_rmsnorm_gamma_f32's operations: sum of
// squares in double, scale = 1/sqrtf(mean + eps), (x*gamma)*scale), then
// quantised into the entries. Every CTA sums the whole row in the same order
// (warp c: blocks c, c+CONS, ...; a fixed shuffle tree; warps in order), so
// every CTA gets the same scale. With at most kNormRegs blocks per warp and
// a resident range, the values loaded for the sum are reused for the
// quantisation.
constexpr int kNormRegs = 8;
template <int NT, int XPU, int CONS>
__device__ void stage_norm(const KP &p, const DPh &ph, const XArea &a, uint64_t r0, int c, int lane, int nthr,
                           double (*red)[8]) {
  const uint32_t k = ph.k, nblk = k / 32, nbq = a.xs.quads * 4;  // blocks of x; blocks of whole x-quads
  const bool regs = a.resident && p.batch <= 2 && nbq <= (uint32_t)CONS * kNormRegs;
  float keep[2][kNormRegs];
  for (uint32_t vec = 0; vec < p.batch; vec++) {
    const float *xr = ph.xf + (size_t)vec * k;
    double acc = 0.0;
    for (uint32_t b0 = c; b0 < nblk; b0 += CONS * kNormRegs) {
      float v[kNormRegs];
#pragma unroll
      for (int m = 0; m < kNormRegs; m++) {
        const uint32_t b = b0 + m * CONS;
        v[m] = b < nblk ? __ldcg(xr + (size_t)b * 32 + lane) : 0.0f;
      }
#pragma unroll
      for (int m = 0; m < kNormRegs; m++) {
        acc = __dadd_rn(acc, __dmul_rn((double)v[m], (double)v[m]));
        if (vec < 2) keep[vec][m] = v[m];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) red[c][vec] = acc;
  }
  cbar(nthr);
  b200_xq_t v;
  v.limbs = const_cast<uint8_t *>(a.xs.limbs);
  v.sb = const_cast<float *>(a.xs.sb);
  v.sx = const_cast<float *>(a.xs.sx);
  v.batch = p.batch;
  v.k = k;
  v.quads = a.xs.quads;
  const uint32_t bpe = XPU * 4;  // 32-element blocks per entry
  for (uint32_t vec = 0; vec < p.batch; vec++) {
    double t = 0.0;
    for (int w = 0; w < CONS; w++) t += red[w][vec];
    const float ms = (float)__ddiv_rn(t, (double)k);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
    const float *xr = ph.xf + (size_t)vec * k;
    if (regs) {
      // resident: entry = unit, slot block j = source block j; warp c owns
      // blocks c, c+CONS, ... as in the sum above (blocks past k, padding
      // of the last x-quad, are written as zeros)
#pragma unroll
      for (int m = 0; m < kNormRegs; m++) {
        const uint32_t b = c + m * CONS;
        if (b < nbq) {
          const uint32_t i = b * 32 + lane;
          const float xv = b < nblk ? __fmul_rn(__fmul_rn(keep[vec][m], __ldg(ph.gamma + i)), scale) : 0.0f;
          xq_store_block(v, vec, b, xv);
        }
      }
    } else {
      const uint32_t nb = a.nent * bpe;
      for (uint32_t j0 = c; j0 < nb; j0 += CONS * kNormRegs) {
        float xv[kNormRegs];
#pragma unroll
        for (int m = 0; m < kNormRegs; m++) {
          const uint32_t j = j0 + m * CONS;
          xv[m] = 0.0f;
          if (j < nb) {
            const uint32_t e = j / bpe, src = entry_unit(ph, a, r0, e) * bpe + j % bpe;
            const uint32_t i = src * 32 + lane;
            if (i < k) xv[m] = __fmul_rn(__fmul_rn(__ldcg(xr + i), __ldg(ph.gamma + i)), scale);
          }
        }
#pragma unroll
        for (int m = 0; m < kNormRegs; m++) {
          const uint32_t j = j0 + m * CONS;
          if (j < nb) xq_store_block(v, vec, j, xv[m]);
        }
      }
    }
  }
}

// SiLU*up outputs wait for re-quantisation until all 4 tiles of their
// 64-row group are written (ticket per group); tickets are batched so one
// fence covers several.
struct Requant {
  uint32_t q[4];
  int n = 0;
  __device__ void flush(const DPh &ph, uint32_t batch, uint32_t *grp_cnt, int lane) {
    if (n == 0) return;
    __threadfence();
    __syncwarp();
    for (int i = 0; i < n; i++) {
      uint32_t ticket = 0;
      if (lane == 0) ticket = atomicAdd(&grp_cnt[q[i]], 1u);
      ticket = __shfl_sync(0xffffffffu, ticket, 0);
      if (ticket == 3) {  // the last of the group's 4 tiles quantises outputs 32q..32q+31
        __threadfence();
        for (uint32_t vec = 0; vec < batch; vec++)
          xq_store_block(ph.xo, vec, q[i], __ldcg(&ph.y[(size_t)vec * ph.nout + q[i] * 32 + lane]));
        if (lane == 0) grp_cnt[q[i]] = 0;
      }
    }
    n = 0;
  }
  __device__ void add(const DPh &ph, uint32_t batch, uint32_t *grp_cnt, int lane, uint32_t group) {
    if (n == 4) flush(ph, batch, grp_cnt, lane);
    q[n++] = group;
  }
};

// Final row sums of a tile (holder lanes: rows r and r+8 of vector
// 2nt + vsel) through the phase's epilogue.
template <int NT>
__device__ void finish_tile(const DPh &ph, const KP &p, uint32_t tile, int lane, const float (&ya)[NT],
                            const float (&yb)[NT], Requant &pend, uint32_t parity) {
  const uint32_t r = lane >> 2, vsel = (lane & 3) >> 1;
  const bool holder = (lane & 1) == 0;
  if (ph.epi == B200_EPI_PUSH) {
    // row-parallel partial sums of this rank into slot [parity][rank] of
    // every rank's landing buffer (plain peer stores over NVLink)
    if (!holder) return;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      const uint32_t vec = 2 * nt + vsel;
      if (vec >= p.batch) continue;
      const uint32_t row = tile * 16 + r;
      for (uint32_t q = 0; q < p.nranks; q++) {
        float *dst = land_rows(p, q, parity, p.rank) + (size_t)vec * ph.n;
        if (row < ph.n) dst[row] = ya[nt];
        if (row + 8 < ph.n) dst[row + 8] = yb[nt];
      }
    }
    return;
  }
  if (ph.epi == B200_EPI_SILU_GLU) {
    const uint32_t o = tile * 8 + r;  // rows r (gate) and r+8 (up) of the tile are in the same lane
    if (holder) {
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        const uint32_t vec = 2 * nt + vsel;
        if (vec < p.batch && o < ph.nout) {
          const float gate = ya[nt], up = yb[nt];
          ph.y[(size_t)vec * ph.nout + o] = __fmul_rn(__fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate))), up);
        }
      }
    }
    if (ph.xo.limbs) pend.add(ph, p.batch, p.grp_cnt, lane, tile / 4);
    return;
  }
  if (!holder) return;
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const uint32_t vec = 2 * nt + vsel;
    if (vec >= p.batch) continue;
    const uint32_t row = tile * 16 + r;
    float a = ya[nt], b = yb[nt];
    if (ph.epi == B200_EPI_RESIDUAL) {
      if (row < ph.n) a = __fadd_rn(__ldcg(ph.res + (size_t)vec * ph.n + row), a);
      if (row + 8 < ph.n) b = __fadd_rn(__ldcg(ph.res + (size_t)vec * ph.n + row + 8), b);
    }
    if (row < ph.n) ph.y[(size_t)vec * ph.n + row] = a;
    if (row + 8 < ph.n) ph.y[(size_t)vec * ph.n + row + 8] = b;
  }
}

// Take the split-K tickets of this warp's parked tiles; the last part of a
// tile to arrive adds all parts in CTA order and finishes the tile.
template <int NT>
__device__ void settle_splits(const DPh &ph, const KP &p, uint32_t (&tiles)[2], uint32_t (&nsegs)[2], int &n,
                              int lane, Requant &pend, uint32_t parity) {
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
        const float *pp = p.partial + (size_t)vec * ph.npad + (size_t)tile * 16 + r;
        const size_t stride = (size_t)p.batch * ph.npad;
        for (uint32_t q0 = 0; q0 < nseg; q0 += 8) {  // parts in CTA order, eight loads in flight
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
    finish_tile<NT>(ph, p, tile, lane, ya, yb, pend, parity);
  }
  n = 0;
}

// Consumer side of one GEMV phase. `failed` (shared) records a ring wait
// that ran out; the loop structure is the same either way, so every thread
// reaches the same barriers.
template <uint32_t T, int NT, int CONS>
__device__ void consume(const KP &p, const DPh &ph, uint8_t *ring, uint64_t *full, uint64_t *empty, uint32_t &seq,
                        uint8_t *area, double (*red)[8], int c, int lane, int ctid, int nthr, volatile int *failed,
                        uint64_t xbase) {
  const uint32_t parity = (uint32_t)((xbase + ph.xi) & 1u);
  using Un = Unit<T>;
  constexpr int U = Un::U, XPU = Un::XPU;
  constexpr uint32_t GQ = CONS * Un::QB, GS = CONS * Un::SB;
  uint64_t r0, r1;
  phase_range(ph, r0, r1);
  if (r0 >= r1) return;
  const XArea a = x_area<NT, XPU>(p, ph, area, r0, r1);
  if (ph.xsrc == B200_X_NORM)
    stage_norm<NT, XPU, CONS>(p, ph, a, r0, c, lane, nthr, red);
  else
    stage_xq<NT, XPU>(ph, a, r0, p.batch, ctid, nthr);
  cbar(nthr);
  const uint64_t total = (uint64_t)ph.ngroups * ph.units;
  const uint32_t r = lane >> 2, vsel = (lane & 3) >> 1;
  const bool holder = (lane & 1) == 0;
  float yr[NT], yr8[NT];
  uint32_t split_tile[2], split_n[2];
  int nsplit = 0;
  Requant pend;
  bool bad = false;
  for (uint64_t pos = r0; pos < r1;) {
    const Sub s = sub_at(ph, pos, r0, r1);
    const uint32_t eoff = (uint32_t)(pos - r0);  // entry of unit s.u0 when not resident
    pos += s.u1 - s.u0;
    const uint32_t tile = s.g * CONS + c;
    const bool active = tile < ph.ntiles;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) yr[nt] = yr8[nt] = 0.f;
    for (uint32_t ua = s.u0; ua < s.u1; ua += U) {
      const uint32_t slot = seq % kStages, par = (seq / kStages) & 1u;
      if (!bad) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&full[slot], par, p.wait_ns);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) {
          bad = true;
          if (lane == 0) *failed = 1;
        }
      }
      if (active && !bad) {
        const uint8_t *st = ring + (size_t)slot * kStageBytes<CONS>;
#pragma unroll
        for (int uu = 0; uu < U; uu++) {
          const uint32_t u = ua + uu;
          if (u < s.u1) {
            const uint32_t e = a.resident ? u : eoff + (u - s.u0);
            Un::template compute<NT>(st + uu * GQ + c * Un::QB, st + U * GQ + uu * GS + c * Un::SB, a.xs, e * XPU,
                                     lane, yr, yr8);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      seq++;
    }
    if (!active || bad) continue;
    // ---- this CTA's segment of group g is done ----
    const uint32_t gw = work_grid(ph);
    const uint32_t cta_lo = cta_of((uint64_t)s.g * ph.units, total, gw);
    const uint32_t nseg = cta_of((uint64_t)(s.g + 1) * ph.units - 1, total, gw) - cta_lo + 1;
    float ya[NT], yb[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {  // lane pairs (c, c^1) hold the two halves of one sum
      ya[nt] = yr[nt] + __shfl_xor_sync(0xffffffffu, yr[nt], 1);
      yb[nt] = yr8[nt] + __shfl_xor_sync(0xffffffffu, yr8[nt], 1);
    }
    if (nseg == 1) {
      finish_tile<NT>(ph, p, tile, lane, ya, yb, pend, parity);
      continue;
    }
    const uint32_t split = blockIdx.x - cta_lo;
    if (holder) {
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        const uint32_t vec = 2 * nt + vsel;
        if (vec < p.batch) {
          float *pp = p.partial + ((size_t)split * p.batch + vec) * ph.npad + (size_t)tile * 16 + r;
          pp[0] = ya[nt];
          pp[8] = yb[nt];
        }
      }
    }
    if (nsplit == 2) settle_splits<NT>(ph, p, split_tile, split_n, nsplit, lane, pend, parity);
    split_tile[nsplit] = tile;
    split_n[nsplit++] = nseg;
  }
  if (!bad) {
    settle_splits<NT>(ph, p, split_tile, split_n, nsplit, lane, pend, parity);
    pend.flush(ph, p.batch, p.grp_cnt, lane);
  }
}

// ---- attention phase ----------------------------------------------------------------------

// Attention over the cache of layer ph.layer for every (sequence, kv head,
// chunk) item this CTA owns; G query heads share a kv head. Shared memory
// (area): q [G][128], scores [G][kAttnSub], the partial V sums of the
// thread groups [nthr/64][G][128] and the running statistics [G][4].
// Not inlined: the attention variants keep their own register allocation,
// so their arrays (q, scores and sums of up to 8 heads) do not push the
// GEMV consumer loop into spills.
template <int G, int CONS>
__device__ __noinline__ void attention(const KP &p, const DPh &ph, uint8_t *area, int warp, int lane, int ctid, int nthr,
                          volatile uint32_t *sticket) {
  constexpr int W = CONS;
  const uint32_t nsub = nthr / 64;  // whole groups of 64 threads (2 dims each) share the positions
  float *qs = reinterpret_cast<float *>(area);
  float *sc = qs + G * kHD;
  float *red = sc + G * kAttnSub;
  float *stat = red + (size_t)nsub * G * kHD;
  const uint32_t npos = (uint32_t)__ldcg(p.pos) + 1u, pos = npos - 1;
  const uint32_t chunk = max(32u, ((npos + p.per_head - 1) / p.per_head + 31u) / 32u * 32u);
  const uint32_t nch = (npos + chunk - 1) / chunk;
  const uint32_t nitems = p.batch * p.hk * nch;
  const uint32_t r2 = kHD / 2;
  const size_t lofs = (size_t)ph.layer * p.layer_stride;
  for (uint32_t item = blockIdx.x; item < nitems; item += gridDim.x) {
    const uint32_t b = item / (p.hk * nch), rem = item % (p.hk * nch), kvh = rem / nch, ch = rem % nch;
    const uint32_t start = ch * chunk, len = min(chunk, npos - start), h0 = kvh * G;
    const float *row = p.qkv + (size_t)b * (p.h + 2 * p.hk) * kHD;
    // q of the G heads rotated at the position (pai_ref_rope_f32 on the q part
    // of the projection row, llama.c:713-724)
    for (uint32_t i = ctid; i < G * r2; i += nthr) {
      const uint32_t g = i / r2, j = i % r2;
      const float *xr = row + (size_t)(h0 + g) * kHD;
      float o0, o1;
      rope_pair(__ldcg(xr + j), __ldcg(xr + j + r2), __ldg(p.cos_t + (size_t)pos * r2 + j),
                __ldg(p.sin_t + (size_t)pos * r2 + j), o0, o1);
      qs[g * kHD + j] = o0;
      qs[g * kHD + j + r2] = o1;
    }
    const size_t kvbase = lofs + (size_t)b * p.seq_stride + (size_t)kvh * p.cap * kHD;
    if (start + len == npos) {  // this chunk holds the position: append the rotated k and v (fp16)
      const size_t at = kvbase + (size_t)pos * kHD;
      if (ctid < (int)r2) {
        const float *kr = row + (size_t)(p.h + kvh) * kHD;
        float o0, o1;
        rope_pair(__ldcg(kr + ctid), __ldcg(kr + ctid + r2), __ldg(p.cos_t + (size_t)pos * r2 + ctid),
                  __ldg(p.sin_t + (size_t)pos * r2 + ctid), o0, o1);
        p.kc[at + ctid] = __float2half_rn(o0);
        p.kc[at + ctid + r2] = __float2half_rn(o1);
      } else if (ctid < (int)(r2 + kHD)) {
        const uint32_t d = ctid - r2;
        p.vc[at + d] = __float2half_rn(__ldcg(row + (size_t)(p.h + p.hk + kvh) * kHD + d));
      }
    }
    if (ctid < G) {
      stat[ctid * 4 + 0] = -INFINITY;  // running max
      stat[ctid * 4 + 1] = 0.0f;       // running sum
    }
    cbar(nthr);
    float qr[G][4];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
      for (int e = 0; e < 4; e++) qr[g][e] = qs[g * kHD + 4 * lane + e];
    const __half *kb = p.kc + kvbase + (size_t)start * kHD;
    const __half *vb = p.vc + kvbase + (size_t)start * kHD;
    const uint32_t dp = ctid & 63, sub = ctid >> 6;
    const bool pv = sub < nsub;  // threads past the last whole group of 64 sit out the V sums
    float acc[G][2];
#pragma unroll
    for (int g = 0; g < G; g++) acc[g][0] = acc[g][1] = 0.f;
    for (uint32_t s0 = 0; s0 < len; s0 += kAttnSub) {
      const uint32_t cnt = min(kAttnSub, len - s0);
      // scores: warp w takes positions w, w+W, ...; four per round in flight
      for (uint32_t i0 = warp; i0 < cnt; i0 += 4 * W) {
        float part[4][G];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const uint32_t i = i0 + u * W;
          float2 k01 = make_float2(0.f, 0.f), k23 = k01;
          if (i < cnt) {
            const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(kb + (size_t)(s0 + i) * kHD + 4 * lane));
            k01 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
            k23 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
          }
#pragma unroll
          for (int g = 0; g < G; g++) {
            float sv = qr[g][0] * k01.x;
            sv = fmaf(qr[g][1], k01.y, sv);
            sv = fmaf(qr[g][2], k23.x, sv);
            sv = fmaf(qr[g][3], k23.y, sv);
            part[u][g] = sv;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int u = 0; u < 4; u++)
#pragma unroll
            for (int g = 0; g < G; g++) part[u][g] += __shfl_xor_sync(0xffffffffu, part[u][g], o);
        if (lane == 0) {
#pragma unroll
          for (int u = 0; u < 4; u++)
            if (i0 + u * W < cnt) {
#pragma unroll
              for (int g = 0; g < G; g++) sc[g * kAttnSub + i0 + u * W] = part[u][g] * p.inv_scale;
            }
        }
      }
      cbar(nthr);
      // running softmax statistics; warp g takes head g
      if (warp < G) {
        float *sg = sc + warp * kAttnSub;
        float m = -INFINITY;
        for (uint32_t i = lane; i < cnt; i += 32) m = fmaxf(m, sg[i]);
        m = warp_max(m);
        const float m_old = stat[warp * 4 + 0], m_new = fmaxf(m_old, m);
        float l = 0.f;
        for (uint32_t i = lane; i < cnt; i += 32) {
          const float e = expf(sg[i] - m_new);
          sg[i] = e;
          l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
          const float alpha = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
          stat[warp * 4 + 0] = m_new;
          stat[warp * 4 + 1] = fmaf(stat[warp * 4 + 1], alpha, l);
          stat[warp * 4 + 2] = alpha;
        }
      }
      cbar(nthr);
      // exp-weighted V: thread covers dims 2dp, 2dp+1 over every nsub-th position
#pragma unroll
      for (int g = 0; g < G; g++) {
        const float al = stat[g * 4 + 2];
        acc[g][0] *= al;
        acc[g][1] *= al;
      }
      for (uint32_t i = sub; pv && i < cnt; i += nsub) {
        const uint32_t raw = __ldcg(reinterpret_cast<const unsigned int *>(vb + (size_t)(s0 + i) * kHD + 2 * dp));
        const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&raw));
#pragma unroll
        for (int g = 0; g < G; g++) {
          const float e = sc[g * kAttnSub + i];
          acc[g][0] = fmaf(e, v.x, acc[g][0]);
          acc[g][1] = fmaf(e, v.y, acc[g][1]);
        }
      }
      cbar(nthr);  // the scores are rewritten by the next round
    }
    if (pv) {
#pragma unroll
      for (int g = 0; g < G; g++) {
        red[((size_t)sub * G + g) * kHD + 2 * dp] = acc[g][0];
        red[((size_t)sub * G + g) * kHD + 2 * dp + 1] = acc[g][1];
      }
    }
    cbar(nthr);
    for (uint32_t i = ctid; i < G * kHD; i += nthr) {
      const uint32_t g = i / kHD, d = i % kHD;
      float o = 0.f;
      for (uint32_t s2 = 0; s2 < nsub; s2++) o += red[((size_t)s2 * G + g) * kHD + d];
      float *slot = p.apart + (((size_t)b * p.h + h0 + g) * p.per_head + ch) * (kHD + 2);
      slot[d] = o;
      if (d == 0) {
        slot[kHD] = stat[g * 4 + 0];
        slot[kHD + 1] = stat[g * 4 + 1];
      }
    }
    __threadfence();
    cbar(nthr);
    if (ctid == 0) *sticket = atomicAdd(&p.attn_cnt[b * p.hk + kvh], 1u);
    cbar(nthr);
    if (*sticket == nch - 1) {
      // the last chunk to finish merges all chunks of this (sequence, kv head);
      // threads of one warp hold 32 consecutive dimensions of one head
      __threadfence();
      for (uint32_t i = ctid; i < G * kHD; i += nthr) {
        const uint32_t g = i / kHD, d = i % kHD;
        const float *base = p.apart + (((size_t)b * p.h + h0 + g) * p.per_head) * (kHD + 2);
        float M = -INFINITY;
        for (uint32_t s2 = 0; s2 < nch; s2++) M = fmaxf(M, __ldcg(base + (size_t)s2 * (kHD + 2) + kHD));
        float L = 0.f, o = 0.f;
        for (uint32_t s0 = 0; s0 < nch; s0 += 8) {
          float mv[8], lv[8], ov[8];
#pragma unroll
          for (int m = 0; m < 8; m++) {
            if (s0 + m < nch) {
              const float *sl = base + (size_t)(s0 + m) * (kHD + 2);
              mv[m] = __ldcg(sl + kHD);
              lv[m] = __ldcg(sl + kHD + 1);
              ov[m] = __ldcg(sl + d);
            }
          }
#pragma unroll
          for (int m = 0; m < 8; m++) {
            if (s0 + m < nch) {
              const float w = expf(mv[m] - M);
              L = fmaf(lv[m], w, L);
              o = fmaf(ov[m], w, o);
            }
          }
        }
        const float v = o / L;
        p.att[((size_t)b * p.h + h0 + g) * kHD + d] = v;
        // head h0+g covers x blocks 4(h0+g) .. 4(h0+g)+3 of the o projection's input
        xq_store_block(p.xq_att, b, (h0 + g) * 4 + d / 32, v);
      }
      if (ctid == 0) p.attn_cnt[b * p.hk + kvh] = 0;
    }
    cbar(nthr);  // shared memory is reused by the next item
  }
}

// ---- embedding and the final norm --------------------------------------------------

__device__ inline void embed(const KP &p, int ctid, int nthr) {
  const uint32_t el = b200_blk_elems(p.etype), nb = p.n_embd / el;
  const uint32_t total = p.batch * nb;
  for (uint32_t i = blockIdx.x * nthr + ctid; i < total; i += gridDim.x * nthr) {
    const uint32_t b = i / nb, blk = i % nb;
    const uint64_t r = (uint32_t)__ldcg(p.tok_in + b);
    dequant_block_dev(p.etype, p.emb_ntiles, p.emb_qs, p.emb_sc, r, blk, p.x + (size_t)b * p.n_embd + (size_t)blk * el);
  }
}

// Final RMSNorm of the hidden state into the lm head's operand (ph.xo):
// every CTA computes the row's scale as stage_norm does, then quantises its
// slice of the 32-element blocks.
template <int CONS>
__device__ void norm_out(const KP &p, const DPh &ph, int c, int lane, int nthr, double (*red)[8]) {
  const uint32_t k = ph.k, nblk = k / 32;
  for (uint32_t vec = 0; vec < p.batch; vec++) {
    const float *xr = ph.xf + (size_t)vec * k;
    double acc = 0.0;
    for (uint32_t b0 = c; b0 < nblk; b0 += CONS * kNormRegs) {
      float v[kNormRegs];
#pragma unroll
      for (int m = 0; m < kNormRegs; m++) {
        const uint32_t b = b0 + m * CONS;
        v[m] = b < nblk ? __ldcg(xr + (size_t)b * 32 + lane) : 0.0f;
      }
#pragma unroll
      for (int m = 0; m < kNormRegs; m++) acc = __dadd_rn(acc, __dmul_rn((double)v[m], (double)v[m]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) red[c][vec] = acc;
  }
  cbar(nthr);
  const uint32_t nq = (uint32_t)ph.xo.quads * 4, per = (nq + gridDim.x - 1) / gridDim.x;
  const uint32_t b0 = min(nq, blockIdx.x * per), b1 = min(nq, b0 + per);
  for (uint32_t vec = 0; vec < p.batch; vec++) {
    double t = 0.0;
    for (int w = 0; w < CONS; w++) t += red[w][vec];
    const float ms = (float)__ddiv_rn(t, (double)k);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
    const float *xr = ph.xf + (size_t)vec * k;
    for (uint32_t b = b0 + c; b < b1; b += CONS) {
      const uint32_t i = b * 32 + lane;
      const float v = i < k ? __fmul_rn(__fmul_rn(__ldcg(xr + i), __ldg(ph.gamma + i)), scale) : 0.0f;
      xq_store_block(ph.xo, vec, b, v);
    }
  }
}

// ---- tensor-parallel row exchange ----------------------------------------------------

// After a row-parallel GEMV phase (B200_EPI_PUSH): every CTA of every rank
// adds one arrival to every rank's counter once its pushes are out, waits
// (bounded) until all ranks' CTAs arrived at this exchange, then adds the
// ranks' partial rows of its slice, in rank order, to x (the residual add of
// llama.c:747-749, 793-795). Every rank computes the same bits. The arrival
// takes the place of a grid barrier: it also proves this rank's CTAs are done.
__device__ inline bool exchange(const KP &p, const DPh &ph, uint64_t xbase, int ctid, int nthr, volatile int *sflag) {
  cbar(nthr);  // this CTA's pushes are issued
  const uint64_t e = xbase + ph.xi;
  if (ctid == 0) {
    bool ok = true;
    __threadfence_system();
    for (uint32_t q = 0; q < p.nranks; q++)
      atomicAdd_system(reinterpret_cast<unsigned long long *>(land_words(p.land[q])), 1ull);
    const uint64_t target = (e + 1) * (uint64_t)gridDim.x * p.nranks;
    const uint64_t *cnt = land_words(p.land[p.rank]);
    uint64_t t0 = 0;
    for (uint32_t it = 0;; it++) {
      if (ld_acquire_sys64(cnt) >= target) break;
      if ((it & 63u) == 0) {
        if (*(volatile uint32_t *)(p.bar + 2)) {
          ok = false;
          break;
        }
        const uint64_t now = globaltimer_ns();
        if (it == 0) {
          t0 = now;
        } else if (now - t0 > p.wait_ns) {
          raise_abort(p);
          ok = false;
          break;
        }
      }
    }
    *sflag = ok ? 1 : 0;
  }
  cbar(nthr);
  if (!*sflag) return false;
  const uint32_t parity = (uint32_t)(e & 1u);
  const uint32_t n4 = p.xrows / 4, per = (n4 + gridDim.x - 1) / gridDim.x;
  const uint32_t g0 = min(n4, blockIdx.x * per), g1 = min(n4, g0 + per);
  for (uint32_t g = g0 + ctid; g < g1; g += nthr) {
    float4 sum = __ldcg(reinterpret_cast<const float4 *>(land_rows(p, p.rank, parity, 0)) + g);
    for (uint32_t q = 1; q < p.nranks; q++) {  // rank order: the same sum on every rank
      const float4 v = __ldcg(reinterpret_cast<const float4 *>(land_rows(p, p.rank, parity, q)) + g);
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
    }
    float4 *xp = reinterpret_cast<float4 *>(ph.y) + g;
    float4 xv = __ldcg(xp);
    xv.x += sum.x;
    xv.y += sum.y;
    xv.z += sum.z;
    xv.w += sum.w;
    *xp = xv;
  }
  return true;
}

// ---- the kernel ---------------------------------------------------------------------

template <uint32_t T, int NT, int CONS>
__global__ void __launch_bounds__((CONS + 1) * 32, 1) k_decode(const __grid_constant__ KP p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ double red[CONS][8];
  __shared__ int sflag, sfailed;
  __shared__ uint32_t sticket;
  uint8_t *ring = smem;
  uint8_t *area = smem + (size_t)kStages * kStageBytes<CONS>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CONS);
    }
    fence_mbar_init();
    sfailed = 0;
  }
  __syncthreads();

  if (warp == 0) {
    // ---- producer: every GEMV phase's weights, in phase order ----
    if (lane != 0) return;
    uint32_t fill = 0;
    bool ok = true;
    for (uint32_t i = 0; i < p.nph && ok; i++) {
      const DPh &ph = p.ph[i];
      if (ph.kind == B200_PH_GEMV) ok = produce<T, CONS>(p, ph, ring, full, empty, fill);
    }
    if (!ok) {
      // a wait for a free stage ran out: raise the error and let the copies
      // already issued land (bounded) before this thread leaves
      raise_abort(p);
      for (uint32_t f = fill > (uint32_t)kStages ? fill - kStages : 0; f < fill; f++)
        mbar_wait(&full[f % kStages], (f / kStages) & 1u, p.wait_ns);
    }
    return;
  }

  // ---- consumers ----
  const int c = warp - 1, ctid = threadIdx.x - 32, nthr = CONS * 32;
  uint32_t seq = 0, epoch = 0;
  // row exchanges this rank completed in earlier steps (written by the
  // previous launch's last CTA)
  const uint64_t xbase = p.nranks > 1 ? *(volatile uint64_t *)(land_words(p.land[p.rank]) + 1) : 0;
  bool ok = true;
  for (uint32_t i = 0; i < p.nph && ok; i++) {
    const DPh &ph = p.ph[i];
    if (ph.kind == B200_PH_XCHG) {  // its arrival counter also serves as the barrier
      ok = exchange(p, ph, xbase, ctid, nthr, &sflag);
      continue;
    }
    if (i > 0 && !grid_sync(p, epoch, ctid, nthr, &sflag)) {
      ok = false;
      break;
    }
    switch (ph.kind) {
      case B200_PH_EMBED: embed(p, ctid, nthr); break;
      case B200_PH_GEMV:
        consume<T, NT, CONS>(p, ph, ring, full, empty, seq, area, red, c, lane, ctid, nthr, &sfailed, xbase);
        cbar(nthr);
        if (sfailed) {
          if (ctid == 0) raise_abort(p);
          ok = false;
        }
        break;
      case B200_PH_ATTN:
        switch (p.h / p.hk) {
          case 1: attention<1, CONS>(p, ph, area, c, lane, ctid, nthr, &sticket); break;
          case 2: attention<2, CONS>(p, ph, area, c, lane, ctid, nthr, &sticket); break;
          case 4: attention<4, CONS>(p, ph, area, c, lane, ctid, nthr, &sticket); break;
          default: attention<8, CONS>(p, ph, area, c, lane, ctid, nthr, &sticket); break;
        }
        break;
      default: norm_out<CONS>(p, ph, c, lane, nthr, red); break;
    }
  }
  // Leave: the last CTA out resets the barrier words for the next launch
  // (every CTA counted here has passed every barrier of this launch).
  cbar(nthr);
  if (ctid == 0) {
    __threadfence();
    const uint32_t out = atomicAdd(p.bar + 1, 1u);
    if (out == gridDim.x - 1 && !*(volatile uint32_t *)(p.bar + 2)) {
      p.bar[0] = 0;
      p.bar[1] = 0;
      if (p.nranks > 1) land_words(p.land[p.rank])[1] = xbase + p.nx;  // read by the next launch
    }
  }
}


// Host side of one kernel instantiation (defined per block type in
// k_decode_<type>.cu).
struct Plan {
  int device;
  int nt, cons;
  uint32_t type;
  uint32_t grid;
  size_t smem;
  DPh *dph;
  void *scratch;
  KP kp;
};

template <uint32_t T>
pai_status_t attrs(Plan *pl);
template <uint32_t T>
pai_status_t launch(pai_b200_ctx_t *ctx, Plan *pl);
template <>
pai_status_t attrs<PAI_B200_Q4_0>(Plan *pl);
template <>
pai_status_t attrs<PAI_B200_Q8_0>(Plan *pl);
template <>
pai_status_t attrs<PAI_B200_Q4_K>(Plan *pl);
template <>
pai_status_t launch<PAI_B200_Q4_0>(pai_b200_ctx_t *ctx, Plan *pl);
template <>
pai_status_t launch<PAI_B200_Q8_0>(pai_b200_ctx_t *ctx, Plan *pl);
template <>
pai_status_t launch<PAI_B200_Q4_K>(pai_b200_ctx_t *ctx, Plan *pl);

template <uint32_t T, int NT, int CONS>
pai_status_t attrs_k(Plan *pl) {
  auto kern = k_decode<T, NT, CONS>;
  pai_status_t st = b200_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl->smem),
                              "k_decode smem attribute");
  if (st) return st;
  int per_sm = 0;
  st = b200_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (CONS + 1) * 32, pl->smem),
                 "k_decode occupancy");
  if (st) return st;
  if (per_sm < 1) return b200_fail(PAI_ERR_UNSUPPORTED, "decode: %zu B of shared memory do not fit an SM", pl->smem);
  return PAI_OK;
}

template <uint32_t T, int NT, int CONS>
pai_status_t launch_k(pai_b200_ctx_t *ctx, Plan *pl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl->grid);
  cfg.blockDim = dim3((CONS + 1) * 32);
  cfg.dynamicSmemBytes = pl->smem;
  cfg.stream = (cudaStream_t)b200_ctx_stream(ctx);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barriers need it
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return b200_cuda(cudaLaunchKernelEx(&cfg, k_decode<T, NT, CONS>, pl->kp), "k_decode launch");
}

// Consumer warps per CTA for `nt` vector pairs: 15 (512 threads, 128
// registers each) for one pair, 8 (288 threads) for more.
constexpr int cons_for(int nt) { return nt == 1 ? 15 : 8; }

#define B200_DECODE_INSTANTIATE(T)                                       \
  template <>                                                            \
  pai_status_t attrs<T>(Plan * pl) {                                     \
    switch (pl->nt) {                                                    \
      case 1: return attrs_k<T, 1, cons_for(1)>(pl);                     \
      case 2: return attrs_k<T, 2, cons_for(2)>(pl);                     \
      default: return attrs_k<T, 4, cons_for(4)>(pl);                    \
    }                                                                    \
  }                                                                      \
  template <>                                                            \
  pai_status_t launch<T>(pai_b200_ctx_t * ctx, Plan * pl) {              \
    switch (pl->nt) {                                                    \
      case 1: return launch_k<T, 1, cons_for(1)>(ctx, pl);               \
      case 2: return launch_k<T, 2, cons_for(2)>(ctx, pl);               \
      default: return launch_k<T, 4, cons_for(4)>(ctx, pl);              \
    }                                                                    \
  }

}  // namespace b200dec
