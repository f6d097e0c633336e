// Persistent decode step: one cooperative launch runs the layers of a greedy
// decode step of the LLaMA-shaped model over one CTA per SM -- the embedding
// row and every layer in the op order of adapters/llama/llama.c:669-797
// (RMSNorm, q|k|v, RoPE + K/V append + attention over the fp16 cache, o, the
// residual add, RMSNorm, gate|up, SiLU*up, down, the residual add) -- and
// leaves RMSNorm(x) * output_norm quantised for the lm head, which follows as
// the regular GEMV and argmax launches (k_gemv.cu, k_ops.cu).
//
// Why one kernel: a decode step at batch 1 is ~230 small dependent
// operations; as separate launches every GEMV pays a ramp to first data, a
// tail and a launch gap that do not shrink with its size.
//
//  * One producer thread per CTA streams the packed weights of the four
//    matrices of every layer, in order, with bulk asynchronous copies
//    (cp.async.bulk, mbarrier completion, no multicast) into a 4-stage
//    shared-memory ring. Weights never depend on activations: the producer
//    does not wait for phases, so the next matrix is already landing while
//    the consumers reduce, attend or sit at a barrier.
//  * CONS consumer warps run a fixed sequence of phases per layer and meet at
//    a grid barrier (one arrival counter, bounded spin, release/acquire at GPU
//    scope) between them; the producer never joins one.
//  * GEMV phases use the fused dequantise-and-dot arithmetic of k_gemv.cu
//    (gemv_unit.cuh): warp c owns tile c of each CONS-tile row group and the
//    (group, K unit) pairs are split stream-K over the CTAs. A CTA's segment
//    of a group is written as partial row sums ([split][batch][row]); there
//    are no tickets: whoever reads the rows next adds the group's partials in
//    split order (the same bits wherever they are read):
//      - the attention phase adds the q|k|v partials of the rows it uses;
//      - the down GEMV's staging adds the gate|up partials, applies SiLU*up
//        and quantises h for its K units;
//      - a reduce phase after o and after down adds the partials and the
//        residual (llama.c:747-749, 793-795), writes x, the sum of squares of
//        every 32-row block, and x * gamma of the next RMSNorm quantised once
//        ("unscaled": the digits of a block do not depend on the norm's
//        scale, only its block scale does).
//    A normed GEMV input is then staged by adding the block sums of squares
//    (the same order in every CTA: the same scale, pai_ref_rmsnorm_gamma_f32's
//    sqrt(mean + eps)) and copying the quantised blocks with their scales
//    multiplied by it: one round of loads.
//  * Attention: (sequence, kv head) pairs get per_head CTAs each, a CTA
//    covers a contiguous range of positions, its warps take chunks of 32
//    (scores with the G query heads of the kv head, a running max, exp-
//    weighted V), the CTA merges its warps in shared memory and writes one
//    partial (o, max, sum) per head. The o GEMV's staging merges the CTAs'
//    partials of the heads in its K units and quantises them.
//  * Under tensor parallelism the reduce phases exchange: each CTA reduces a
//    slice of rows of this rank's o/down partial sums, stores them into every
//    rank's landing buffer (plain peer stores over NVLink), stamps its
//    arrival into every rank's header, waits (bounded) for the same CTA of
//    every rank, and adds the ranks' rows in rank order: every rank computes
//    the same bits.
//
// All data written inside the launch and read by another CTA is read with
// ld.global.cg (L2): L1 is not coherent across SMs. Every wait is bounded by
// %globaltimer; on timeout the kernel raises the context's error word and a
// device abort word that ends the other CTAs' waits, and every consumer
// thread leaves through the same barrier points.
//
// The kernel is compiled per block type of the layer matrices
// (k_decode_q4_0.cu, ...): one GEMV path per kernel keeps the consumers
// within their register budget.
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
enum { M_QKV = 0, M_O = 1, M_GU = 2, M_DOWN = 3 };

// Shape and work split of one layer-matrix kind (the same for every layer).
struct Shape {
  uint32_t n, k, units, ntiles, ngroups, npad, gw, maxseg, cons;
  uint64_t sc_off;  // byte offset of the header plane in the packed matrix
};

struct Layer {
  const uint8_t *w[4];  // packed q|k|v, o, gate|up, down
  const float *attn_norm, *ffn_norm;
};

struct KP {
  const Layer *__restrict__ layers;
  Shape sh[4];
  uint32_t n_layer, batch;
  float eps;
  // embedding
  uint32_t etype, n_embd;
  const uint8_t *emb_qs, *emb_sc;
  uint64_t emb_ntiles;
  const int32_t *tok_in;
  // attention
  uint32_t h, hk, per_head;
  int32_t *pos;
  uint64_t cap, seq_stride, layer_stride;
  __half *kc, *vc;
  const float *cos_t, *sin_t;
  float inv_scale;
  // state
  float *x;          // hidden state [batch][n_embd]
  b200_xq_t xqn;     // x * gamma of the next RMSNorm, quantised unscaled
  double *ssq;       // [batch][n_embd / 32] sums of squares of x per block
  b200_xq_t xq_out;  // RMSNorm(x) * out_norm for the lm head
  const float *out_norm;
  float *part[2];  // split-K partials: q|k|v and gate|up in [0], o and down in [1]
  float *apart;    // attention CTA partials [batch][h][per_head][kHD + 2]
  uint32_t *bar;   // [0] barrier arrivals, [1] exits, [2] abort
  uint32_t *err;   // the context's host-mapped error word
  uint64_t wait_ns;
  // tensor parallelism: every rank's landing buffer as mapped here
  uint8_t *land[B200_TP_MAX_RANKS];
  uint32_t rank, nranks;
};

__device__ __forceinline__ void cbar(int nthr) { asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory"); }

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_acquire_sys64(const uint64_t *q) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(q) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys64(uint64_t *q, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(q), "l"(v) : "memory");
}

__device__ __forceinline__ void raise_abort(const KP &p) {
  atomicExch(p.bar + 2, 1u);
  atomicExch(p.err, 1u);
}

// Grid barrier of the consumer threads of every CTA. The CTA's consumers
// first meet at named barrier 1; one thread publishes the CTA's writes
// (fence), arrives, and waits (bounded; an abort raised elsewhere ends the
// wait) until all CTAs arrived. Returns the same answer to every consumer
// thread of the CTA.
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

// ---- the work split of a GEMV phase and its partial sums --------------------------------

// CTAs a GEMV phase's work is split over: every CTA when the phase has at
// least one (group, unit) pair per CTA, else one pair each for the first
// `total` CTAs. No CTA inside the split has an empty range, so the CTAs that
// meet a row group are consecutive owners of its pairs.
__device__ __forceinline__ uint32_t cta_of(uint64_t x, uint64_t total, uint32_t grid) {
  return (uint32_t)(((x + 1) * grid - 1) / total);
}

__device__ __forceinline__ void phase_range(const Shape &sh, uint64_t &r0, uint64_t &r1) {
  const uint64_t total = (uint64_t)sh.ngroups * sh.units;
  if (blockIdx.x >= sh.gw) {
    r0 = r1 = total;
    return;
  }
  r0 = (uint64_t)blockIdx.x * total / sh.gw;
  r1 = (uint64_t)(blockIdx.x + 1) * total / sh.gw;
}

// First CTA of row group g's split and the number of CTAs it is split over.
__device__ __forceinline__ void group_split(const Shape &sh, uint32_t g, uint32_t &lo, uint32_t &nseg) {
  const uint64_t total = (uint64_t)sh.ngroups * sh.units;
  lo = cta_of((uint64_t)g * sh.units, total, sh.gw);
  nseg = cta_of((uint64_t)(g + 1) * sh.units - 1, total, sh.gw) - lo + 1;
}

// Row `row` of vector b: the group's partial sums added in split order.
__device__ __forceinline__ float row_sum(const float *part, const Shape &sh, uint32_t batch, uint32_t b,
                                         uint32_t row) {
  uint32_t lo, nseg;
  group_split(sh, row / 16 / sh.cons, lo, nseg);
  const float *q = part + (size_t)b * sh.npad + row;
  const size_t stride = (size_t)batch * sh.npad;
  float s = __ldcg(q);
  for (uint32_t i = 1; i < nseg; i++) s += __ldcg(q + i * stride);
  return s;
}

// A piece of a CTA's range inside one row group: units [u0, u1) of group g.
struct Sub {
  uint32_t g, u0, u1;
};

__device__ __forceinline__ Sub sub_at(const Shape &sh, uint64_t pos, uint64_t r1) {
  Sub s;
  s.g = (uint32_t)(pos / sh.units);
  s.u0 = (uint32_t)(pos - (uint64_t)s.g * sh.units);
  const uint64_t seg_end = min(r1, (uint64_t)(s.g + 1) * sh.units);
  s.u1 = (uint32_t)(seg_end - (uint64_t)s.g * sh.units);
  return s;
}

// Producer: stream the weights of the CTA's range of one GEMV phase into the
// ring, one stage per U units of a sub-item. Returns false when a wait for
// a free stage ran out.
template <uint32_t T, int CONS>
__device__ bool produce(const KP &p, const Shape &sh, const uint8_t *w, uint8_t *ring, uint64_t *full,
                        uint64_t *empty, uint32_t &fill) {
  using Un = Unit<T>;
  constexpr int U = Un::U;
  constexpr uint32_t GQ = CONS * Un::QB, GS = CONS * Un::SB;
  const uint8_t *qs = w, *sc = w + sh.sc_off;
  uint64_t r0, r1;
  phase_range(sh, r0, r1);
  for (uint64_t pos = r0; pos < r1;) {
    const Sub s = sub_at(sh, pos, r1);
    pos += s.u1 - s.u0;
    const uint32_t nv = min((uint32_t)CONS, sh.ntiles - s.g * CONS);  // tiles present in the group
    const size_t tile0 = (size_t)s.g * CONS;
    for (uint32_t ua = s.u0; ua < s.u1; ua += U) {
      const uint32_t ub = min(s.u1, ua + U), slot = fill % kStages;
      if (fill >= (uint32_t)kStages && !mbar_wait(&empty[slot], ((fill / kStages) - 1) & 1u, p.wait_ns)) return false;
      uint8_t *dst = ring + (size_t)slot * kStageBytes<CONS>;
      mbar_expect_tx(&full[slot], (ub - ua) * nv * (Un::QB + Un::SB));
      for (uint32_t u = ua; u < ub; u++) {  // unit-major: the group's tiles of one unit are contiguous
        const size_t t0 = (size_t)u * sh.ntiles + tile0;
        bulk_g2s(dst + (u - ua) * GQ, qs + t0 * Un::QB, nv * Un::QB, &full[slot]);
        bulk_g2s(dst + U * GQ + (u - ua) * GS, sc + t0 * Un::SB, nv * Un::SB, &full[slot]);
      }
      fill++;
    }
  }
  return true;
}

// ---- staging the activation operand of a GEMV phase --------------------------------------

// Shared-memory view of the staged operand of the CTA's range: entry e holds
// the XPU x-quads of one K unit; with a range of at least a whole group
// every unit has its own entry (entry = unit), otherwise entry e belongs to
// flat position r0 + e.
struct XArea {
  XS xs;
  uint32_t nent;
  bool resident;
};

template <int NT, int XPU>
__device__ __forceinline__ XArea x_area(const KP &p, const Shape &sh, uint8_t *area, uint64_t r0, uint64_t r1) {
  XArea a;
  const uint64_t L = r1 - r0;
  a.resident = L >= sh.units;
  a.nent = a.resident ? sh.units : (uint32_t)L;
  const uint32_t nq = a.nent * XPU;
  a.xs.limbs = area;
  a.xs.sb = reinterpret_cast<const float *>(area + (size_t)NT * nq * 1024);
  a.xs.sx = a.xs.sb + (size_t)p.batch * nq * 4;
  a.xs.quads = nq;
  a.xs.batch = p.batch;
  return a;
}

// Bytes of the staged operand for `nent` entries (x_area's layout).
__host__ __device__ constexpr size_t x_area_bytes(uint32_t nt, uint32_t batch, uint32_t xpu, uint64_t nent) {
  return (size_t)nt * nent * xpu * 1024 + 2 * (size_t)batch * nent * xpu * 16;
}

__device__ __forceinline__ uint32_t entry_unit(const Shape &sh, const XArea &a, uint64_t r0, uint32_t e) {
  return a.resident ? e : (uint32_t)((r0 + e) % sh.units);
}

__device__ __forceinline__ b200_xq_t slot_view(const KP &p, const XArea &a, uint32_t k) {
  b200_xq_t v;
  v.limbs = const_cast<uint8_t *>(a.xs.limbs);
  v.sb = const_cast<float *>(a.xs.sb);
  v.sx = const_cast<float *>(a.xs.sx);
  v.batch = p.batch;
  v.k = k;
  v.quads = a.xs.quads;
  return v;
}

// RMSNorm scale of vector b from the block sums of squares, computed by one
// warp in a fixed order (every CTA and warp gets the same bits):
// 1/sqrtf((float)(sum / k) + eps), pai_ref_rmsnorm_gamma_f32's operations.
__device__ __forceinline__ float norm_scale(const KP &p, uint32_t b, int lane) {
  const uint32_t nb = p.n_embd / 32;
  const double *s = p.ssq + (size_t)b * nb;
  double acc = 0.0;
  for (uint32_t i = lane; i < nb; i += 32) acc = __dadd_rn(acc, __ldcg(s + i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  const float ms = (float)__ddiv_rn(acc, (double)p.n_embd);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
}

// Normed input: the unscaled quantised x * gamma (xqn) of the entries' units
// with their block scales multiplied by the norm scale.
template <int NT, int XPU, int CONS>
__device__ void stage_normq(const KP &p, const Shape &sh, const XArea &a, uint64_t r0, int c, int lane, int ctid,
                            int nthr, float *scales) {
  if (c == 0)
    for (uint32_t b = 0; b < p.batch; b++) {
      const float s = norm_scale(p, b, lane);
      if (lane == 0) scales[b] = s;
    }
  const uint32_t nq = a.nent * XPU, per = NT * XPU * 64;  // uint4 per entry (digits)
  uint4 *dl = reinterpret_cast<uint4 *>(const_cast<uint8_t *>(a.xs.limbs));
  const uint4 *sl = reinterpret_cast<const uint4 *>(p.xqn.limbs);
  for (uint32_t i = ctid; i < a.nent * per; i += nthr) {
    const uint32_t e = i / per, r = i % per, nt = r / (XPU * 64), o = r % (XPU * 64);
    const uint32_t u = entry_unit(sh, a, r0, e);
    dl[(((size_t)nt * nq + (size_t)e * XPU) * 1024) / 16 + o] =
        __ldcg(sl + (((size_t)nt * p.xqn.quads + (size_t)u * XPU) * 1024) / 16 + o);
  }
  cbar(nthr);  // the scales are in shared memory
  float4 *db = reinterpret_cast<float4 *>(const_cast<float *>(a.xs.sb));
  float4 *dx = reinterpret_cast<float4 *>(const_cast<float *>(a.xs.sx));
  const float4 *sb = reinterpret_cast<const float4 *>(p.xqn.sb);
  const float4 *sx = reinterpret_cast<const float4 *>(p.xqn.sx);
  for (uint32_t i = ctid; i < a.nent * p.batch * XPU; i += nthr) {
    const uint32_t e = i / (p.batch * XPU), r = i % (p.batch * XPU), vec = r / XPU, q = r % XPU;
    const uint32_t u = entry_unit(sh, a, r0, e);
    const size_t s = (size_t)vec * p.xqn.quads + (size_t)u * XPU + q, d = (size_t)vec * nq + (size_t)e * XPU + q;
    const float f = scales[vec];
    float4 b4 = __ldcg(sb + s), x4 = __ldcg(sx + s);
    b4.x = __fmul_rn(b4.x, f), b4.y = __fmul_rn(b4.y, f), b4.z = __fmul_rn(b4.z, f), b4.w = __fmul_rn(b4.w, f);
    x4.x = __fmul_rn(x4.x, f), x4.y = __fmul_rn(x4.y, f), x4.z = __fmul_rn(x4.z, f), x4.w = __fmul_rn(x4.w, f);
    db[d] = b4;
    dx[d] = x4;
  }
}

// o's input: the attention output of the heads in the entries' units,
// merged from the attention CTAs' partials (fixed order) and quantised.
// One warp per (vector, head): lane l holds dims 4l..4l+3; the 128 values
// go through the warp's shared scratch to quantise lane = element.
template <int NT, int XPU, int CONS>
__device__ void stage_att(const KP &p, const Shape &sh, const XArea &a, uint64_t r0, int c, int lane,
                          float *scratch) {
  b200_xq_t v = slot_view(p, a, sh.k);
  float *ws = scratch + c * kHD;
  const uint32_t heads = a.nent * XPU, ph = p.per_head;
  for (uint32_t j = c; j < heads * p.batch; j += CONS) {
    const uint32_t b = j / heads, eh = j % heads, e = eh / XPU;
    const uint32_t hh = entry_unit(sh, a, r0, e) * XPU + eh % XPU;  // head of this rank
    const float *base = p.apart + (((size_t)b * p.h + hh) * ph) * (kHD + 2);
    float M = -INFINITY;
    for (uint32_t s0 = 0; s0 < ph; s0 += 8) {
      float mv[8], lv[8];
#pragma unroll
      for (int m = 0; m < 8; m++) {
        mv[m] = s0 + m < ph ? __ldcg(base + (size_t)(s0 + m) * (kHD + 2) + kHD) : -INFINITY;
        lv[m] = s0 + m < ph ? __ldcg(base + (size_t)(s0 + m) * (kHD + 2) + kHD + 1) : 0.0f;
      }
#pragma unroll
      for (int m = 0; m < 8; m++)
        if (lv[m] > 0.0f) M = fmaxf(M, mv[m]);
    }
    float L = 0.f, o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    for (uint32_t s0 = 0; s0 < ph; s0 += 8) {
      float mv[8], lv[8];
      float4 ov[8];
#pragma unroll
      for (int m = 0; m < 8; m++) {
        const float *sl = base + (size_t)(s0 + m) * (kHD + 2);
        const bool in = s0 + m < ph;
        mv[m] = in ? __ldcg(sl + kHD) : -INFINITY;
        lv[m] = in ? __ldcg(sl + kHD + 1) : 0.0f;
        if (in) {
          ov[m].x = __ldcg(sl + 4 * lane), ov[m].y = __ldcg(sl + 4 * lane + 1);
          ov[m].z = __ldcg(sl + 4 * lane + 2), ov[m].w = __ldcg(sl + 4 * lane + 3);
        } else {
          ov[m] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int m = 0; m < 8; m++) {
        if (lv[m] > 0.0f) {
          const float w = expf(mv[m] - M);
          L = fmaf(lv[m], w, L);
          o0 = fmaf(ov[m].x, w, o0), o1 = fmaf(ov[m].y, w, o1);
          o2 = fmaf(ov[m].z, w, o2), o3 = fmaf(ov[m].w, w, o3);
        }
      }
    }
    __syncwarp();
    ws[4 * lane] = o0 / L, ws[4 * lane + 1] = o1 / L, ws[4 * lane + 2] = o2 / L, ws[4 * lane + 3] = o3 / L;
    __syncwarp();
    // head hh is x blocks 4 hh .. 4 hh + 3; in the entry they are blocks
    // 4 (e XPU + eh % XPU) .. of the slot
    const uint32_t blk0 = (e * XPU + eh % XPU) * 4;
#pragma unroll
    for (int q = 0; q < 4; q++) xq_store_block(v, b, blk0 + q, ws[32 * q + lane]);
  }
}

// down's input: h = silu(gate) * up for the entries' units, from the
// gate|up partial sums (gate|up tile t holds gate rows 8t.. then the
// matching up rows), quantised. One warp per (vector, 32-element block).
template <int NT, int XPU, int CONS>
__device__ void stage_silu(const KP &p, const Shape &sh, const XArea &a, uint64_t r0, int c, int lane) {
  b200_xq_t v = slot_view(p, a, sh.k);
  const Shape &gu = p.sh[M_GU];
  const float *part = p.part[0];
  const uint32_t bpe = XPU * 4, nb = a.nent * bpe;
  for (uint32_t j = c; j < nb * p.batch; j += CONS) {
    const uint32_t b = j / nb, jb = j % nb, e = jb / bpe;
    const uint32_t o = (entry_unit(sh, a, r0, e) * bpe + jb % bpe) * 32 + lane;  // output of the gate/up pair
    float h = 0.0f;
    if (o < sh.k) {
      const uint32_t grow = (o / 8) * 16 + o % 8;
      const float gate = row_sum(part, gu, p.batch, b, grow), up = row_sum(part, gu, p.batch, b, grow + 8);
      h = __fmul_rn(__fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate))), up);  // llama.c:774-781
    }
    xq_store_block(v, b, jb, h);
  }
}

// ---- GEMV phases ------------------------------------------------------------------------

enum { X_NORMQ = 0, X_ATT = 1, X_SILU = 2 };

// Consumer side of one GEMV phase: stage the operand, run the ring, write
// the CTA's segments as partial row sums. `failed` (shared) records a ring
// wait that ran out; the loop structure is the same either way, so every
// thread reaches the same barriers.
template <uint32_t T, int NT, int CONS>
__device__ void consume(const KP &p, const Shape &sh, int xsrc, float *part, uint8_t *ring, uint64_t *full,
                        uint64_t *empty, uint32_t &seq, uint8_t *area, float *scratch, float *scales, int c,
                        int lane, int ctid, int nthr, volatile int *failed) {
  using Un = Unit<T>;
  constexpr int U = Un::U, XPU = Un::XPU;
  constexpr uint32_t GQ = CONS * Un::QB, GS = CONS * Un::SB;
  uint64_t r0, r1;
  phase_range(sh, r0, r1);
  if (r0 >= r1) return;
  const XArea a = x_area<NT, XPU>(p, sh, area, r0, r1);
  if (xsrc == X_NORMQ)
    stage_normq<NT, XPU, CONS>(p, sh, a, r0, c, lane, ctid, nthr, scales);
  else if (xsrc == X_ATT)
    stage_att<NT, XPU, CONS>(p, sh, a, r0, c, lane, scratch);
  else
    stage_silu<NT, XPU, CONS>(p, sh, a, r0, c, lane);
  cbar(nthr);
  const uint64_t total = (uint64_t)sh.ngroups * sh.units;
  const uint32_t r = lane >> 2, vsel = (lane & 3) >> 1;
  const bool holder = (lane & 1) == 0;
  float yr[NT], yr8[NT];
  bool bad = false;
  for (uint64_t pos = r0; pos < r1;) {
    const Sub s = sub_at(sh, pos, r1);
    const uint32_t eoff = (uint32_t)(pos - r0);  // entry of unit s.u0 when not resident
    pos += s.u1 - s.u0;
    const uint32_t tile = s.g * CONS + c;
    const bool active = tile < sh.ntiles;
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
    // this CTA's segment of group g: its partial row sums
    uint32_t lo, nseg;
    group_split(sh, s.g, lo, nseg);
    (void)total;
    const uint32_t split = blockIdx.x - lo;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {  // lane pairs (c, c^1) hold the two halves of one sum
      const float ya = yr[nt] + __shfl_xor_sync(0xffffffffu, yr[nt], 1);
      const float yb = yr8[nt] + __shfl_xor_sync(0xffffffffu, yr8[nt], 1);
      const uint32_t vec = 2 * nt + vsel;
      if (holder && vec < p.batch) {
        float *pp = part + ((size_t)split * p.batch + vec) * sh.npad + (size_t)tile * 16 + r;
        pp[0] = ya;
        pp[8] = yb;
      }
    }
  }
}

// ---- reduce phases: residual add, block sums of squares, the next norm's operand -----------

// x block (32 rows) of vector b: v = x + sum; writes x, the block's sum of
// squares (fixed shuffle order) and v * gamma quantised (unscaled). One warp.
__device__ __forceinline__ void finish_block(const KP &p, uint32_t b, uint32_t blk, float v, const float *gamma,
                                             int lane) {
  const uint32_t row = blk * 32 + lane;
  p.x[(size_t)b * p.n_embd + row] = v;
  double sq = __dmul_rn((double)v, (double)v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq = __dadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
  if (lane == 0) p.ssq[(size_t)b * (p.n_embd / 32) + blk] = sq;
  xq_store_block(p.xqn, b, blk, __fmul_rn(v, __ldg(gamma + row)));
}

// One GPU: x += the o or down GEMV's row sums (the residual adds of
// llama.c:747-749, 793-795); warp per 32-row block.
template <int CONS>
__device__ void reduce_rows(const KP &p, const Shape &sh, const float *gamma, int c, int lane) {
  const uint32_t nb = p.n_embd / 32;
  for (uint32_t wb = blockIdx.x * CONS + c; wb < p.batch * nb; wb += gridDim.x * CONS) {
    const uint32_t b = wb / nb, blk = wb % nb, row = blk * 32 + lane;
    const float v = __fadd_rn(__ldcg(p.x + (size_t)b * p.n_embd + row), row_sum(p.part[1], sh, p.batch, b, row));
    finish_block(p, b, blk, v, gamma, lane);
  }
}

__device__ __forceinline__ uint64_t *land_words(uint8_t *b) { return reinterpret_cast<uint64_t *>(b); }
__device__ __forceinline__ float *land_rows(const KP &p, uint32_t r, uint32_t parity, uint32_t src) {
  return reinterpret_cast<float *>(p.land[r] + B200_LAND_HDR) + ((size_t)parity * p.nranks + src) * p.batch * p.n_embd;
}

// Tensor parallelism: the same as reduce_rows with the sum over ranks. This
// CTA's blocks of this rank's row sums go into slot [parity][rank] of every
// rank's landing buffer; then the CTA stamps epoch e into flag [rank][cta] of
// every rank, waits (bounded) for flag [r][cta] >= e of every rank (the same
// CTA index of every rank handled the same blocks), and adds the ranks' rows
// in rank order to x.
template <int CONS>
__device__ bool exchange_rows(const KP &p, const Shape &sh, const float *gamma, uint64_t e, int c, int lane, int ctid,
                              int nthr, volatile int *sflag) {
  const uint32_t nb = p.n_embd / 32, parity = (uint32_t)(e & 1u);
  for (uint32_t wb = blockIdx.x * CONS + c; wb < p.batch * nb; wb += gridDim.x * CONS) {
    const uint32_t b = wb / nb, blk = wb % nb, row = blk * 32 + lane;
    const float v = row_sum(p.part[1], sh, p.batch, b, row);
    for (uint32_t q = 0; q < p.nranks; q++) land_rows(p, q, parity, p.rank)[(size_t)b * p.n_embd + row] = v;
  }
  cbar(nthr);  // this CTA's stores are issued
  if (ctid == 0) {
    bool ok = true;
    __threadfence_system();
    for (uint32_t q = 0; q < p.nranks; q++)
      st_release_sys64(reinterpret_cast<uint64_t *>(p.land[q] + B200_LAND_FLAGS) +
                           (size_t)p.rank * B200_LAND_MAX_CTAS + blockIdx.x,
                       e + 1);
    const uint64_t *fl = reinterpret_cast<const uint64_t *>(p.land[p.rank] + B200_LAND_FLAGS);
    for (uint32_t q = 0; q < p.nranks && ok; q++) {
      uint64_t t0 = 0;
      for (uint32_t it = 0;; it++) {
        if (ld_acquire_sys64(fl + (size_t)q * B200_LAND_MAX_CTAS + blockIdx.x) >= e + 1) break;
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
    }
    *sflag = ok ? 1 : 0;
  }
  cbar(nthr);
  if (!*sflag) return false;
  for (uint32_t wb = blockIdx.x * CONS + c; wb < p.batch * nb; wb += gridDim.x * CONS) {
    const uint32_t b = wb / nb, blk = wb % nb, row = blk * 32 + lane;
    const size_t at = (size_t)b * p.n_embd + row;
    float s = __ldcg(land_rows(p, p.rank, parity, 0) + at);
    for (uint32_t q = 1; q < p.nranks; q++) s += __ldcg(land_rows(p, p.rank, parity, q) + at);  // rank order
    finish_block(p, b, blk, __fadd_rn(__ldcg(p.x + at), s), gamma, lane);
  }
  return true;
}

// ---- attention ---------------------------------------------------------------------------

// RoPE (pai_ref_rope_f32's pairs (i, i + 64)) of the 4 dims 4l..4l+3 a lane
// holds: its partner dims sit in lane l ^ 16.
__device__ __forceinline__ void rope4(float (&x)[4], const KP &p, uint32_t pos, int lane) {
  float y[4];
#pragma unroll
  for (int e = 0; e < 4; e++) y[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
  const uint32_t r2 = kHD / 2;
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const uint32_t i = (4 * lane + e) % r2;
    const float c = __ldg(p.cos_t + (size_t)pos * r2 + i), s = __ldg(p.sin_t + (size_t)pos * r2 + i);
    float o0, o1;
    if (lane < 16) {
      rope_pair(x[e], y[e], c, s, o0, o1);
      x[e] = o0;
    } else {
      rope_pair(y[e], x[e], c, s, o0, o1);
      x[e] = o1;
    }
  }
}

// Attention over layer `layer`'s cache (the last row of pai_ref_attention_f32,
// cpu/reference/ref_ops.c:307-349, on the cache contents: scores scaled by
// 1/sqrtf(hd) after the dot, softmax with the maximum subtracted, sum of
// p_i v_i). Not inlined: its arrays keep their own register allocation.
template <int G, int CONS>
__device__ __noinline__ void attention(const KP &p, uint32_t layer, int warp, int lane, int ctid, int nthr,
                                       float *sm) {
  const Shape &sq = p.sh[M_QKV];
  const float *part = p.part[0];
  const uint32_t npos = (uint32_t)__ldcg(p.pos) + 1u, pos = npos - 1, ph = p.per_head;
  const uint32_t cpos = max(32u, ((npos + ph - 1) / ph + 31u) / 32u * 32u);  // positions per CTA
  const uint32_t nitems = p.batch * p.hk * ph;
  const size_t lofs = (size_t)layer * p.layer_stride;
  for (uint32_t item = blockIdx.x; item < nitems; item += gridDim.x) {
    const uint32_t b = item / (p.hk * ph), kvh = (item / ph) % p.hk, j = item % ph, h0 = kvh * G;
    const uint32_t p0 = j * cpos, p1 = min(npos, p0 + cpos);
    float m[G], l[G], o[G][4];
#pragma unroll
    for (int g = 0; g < G; g++) {
      m[g] = -INFINITY, l[g] = 0.f;
#pragma unroll
      for (int e = 0; e < 4; e++) o[g][e] = 0.f;
    }
    if (p0 + 32 * warp < p1) {
      // q of the G heads (the partial sums of their rows), rotated at the position
      float q[G][4];
#pragma unroll
      for (int g = 0; g < G; g++) {
#pragma unroll
        for (int e = 0; e < 4; e++) q[g][e] = row_sum(part, sq, p.batch, b, (h0 + g) * kHD + 4 * lane + e);
        rope4(q[g], p, pos, lane);
      }
      const size_t kvbase = lofs + (size_t)b * p.seq_stride + (size_t)kvh * p.cap * kHD;
      for (uint32_t c0 = p0 + 32 * warp; c0 < p1; c0 += 32 * CONS) {
        const uint32_t cnt = min(32u, p1 - c0);
        if (c0 <= pos && pos < c0 + cnt) {
          // this chunk holds the position: append the rotated k and v (fp16);
          // lane l writes dims 4l..4l+3, the words it reads back below
          float kk[4], vv[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            kk[e] = row_sum(part, sq, p.batch, b, (p.h + kvh) * kHD + 4 * lane + e);
            vv[e] = row_sum(part, sq, p.batch, b, (p.h + p.hk + kvh) * kHD + 4 * lane + e);
          }
          rope4(kk, p, pos, lane);
          const size_t at = kvbase + (size_t)pos * kHD + 4 * lane;
          __half2 k01 = __floats2half2_rn(kk[0], kk[1]), k23 = __floats2half2_rn(kk[2], kk[3]);
          __half2 v01 = __floats2half2_rn(vv[0], vv[1]), v23 = __floats2half2_rn(vv[2], vv[3]);
          uint2 kw, vw;
          kw.x = *reinterpret_cast<uint32_t *>(&k01), kw.y = *reinterpret_cast<uint32_t *>(&k23);
          vw.x = *reinterpret_cast<uint32_t *>(&v01), vw.y = *reinterpret_cast<uint32_t *>(&v23);
          *reinterpret_cast<uint2 *>(p.kc + at) = kw;
          *reinterpret_cast<uint2 *>(p.vc + at) = vw;
        }
        // scores of the chunk: lane i keeps position c0 + i
        float s_mine[G];
#pragma unroll
        for (int g = 0; g < G; g++) s_mine[g] = -INFINITY;
        for (uint32_t i0 = 0; i0 < cnt; i0 += 4) {
          float d[4][G];
#pragma unroll
          for (int u = 0; u < 4; u++) {
            float2 k01 = make_float2(0.f, 0.f), k23 = k01;
            if (i0 + u < cnt) {
              const uint2 raw =
                  __ldcg(reinterpret_cast<const uint2 *>(p.kc + kvbase + (size_t)(c0 + i0 + u) * kHD + 4 * lane));
              k01 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
              k23 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
            }
#pragma unroll
            for (int g = 0; g < G; g++) {
              float sv = q[g][0] * k01.x;
              sv = fmaf(q[g][1], k01.y, sv);
              sv = fmaf(q[g][2], k23.x, sv);
              sv = fmaf(q[g][3], k23.y, sv);
              d[u][g] = sv;
            }
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int u = 0; u < 4; u++)
#pragma unroll
              for (int g = 0; g < G; g++) d[u][g] += __shfl_xor_sync(0xffffffffu, d[u][g], off);
#pragma unroll
          for (int u = 0; u < 4; u++)
            if ((uint32_t)lane == i0 + u && i0 + u < cnt) {
#pragma unroll
              for (int g = 0; g < G; g++) s_mine[g] = d[u][g] * p.inv_scale;
            }
        }
        // running softmax statistics
        float e_mine[G];
#pragma unroll
        for (int g = 0; g < G; g++) {
          const float m_new = fmaxf(m[g], warp_max(s_mine[g]));
          const float alpha = m[g] == -INFINITY ? 0.0f : expf(m[g] - m_new);
          e_mine[g] = (uint32_t)lane < cnt ? expf(s_mine[g] - m_new) : 0.0f;
          l[g] = fmaf(l[g], alpha, warp_sum(e_mine[g]));
          m[g] = m_new;
#pragma unroll
          for (int e = 0; e < 4; e++) o[g][e] *= alpha;
        }
        // exp-weighted V: position i's weight broadcast from lane i
        for (uint32_t i = 0; i < cnt; i++) {
          const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(p.vc + kvbase + (size_t)(c0 + i) * kHD + 4 * lane));
          const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
          const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
#pragma unroll
          for (int g = 0; g < G; g++) {
            const float w = __shfl_sync(0xffffffffu, e_mine[g], i);
            o[g][0] = fmaf(w, v01.x, o[g][0]);
            o[g][1] = fmaf(w, v01.y, o[g][1]);
            o[g][2] = fmaf(w, v23.x, o[g][2]);
            o[g][3] = fmaf(w, v23.y, o[g][3]);
          }
        }
      }
    }
    // the CTA's warps merged in shared memory: sm[warp][g][kHD + 2]
#pragma unroll
    for (int g = 0; g < G; g++) {
      float *w = sm + ((size_t)warp * G + g) * (kHD + 2);
#pragma unroll
      for (int e = 0; e < 4; e++) w[4 * lane + e] = o[g][e];
      if (lane == 0) w[kHD] = m[g], w[kHD + 1] = l[g];
    }
    cbar(nthr);
    for (uint32_t i = ctid; i < G * kHD; i += nthr) {
      const uint32_t g = i / kHD, dd = i % kHD;
      float M = -INFINITY;
      for (int w = 0; w < CONS; w++) {
        const float *ws = sm + ((size_t)w * G + g) * (kHD + 2);
        if (ws[kHD + 1] > 0.0f) M = fmaxf(M, ws[kHD]);
      }
      float L = 0.f, od = 0.f;
      for (int w = 0; w < CONS; w++) {
        const float *ws = sm + ((size_t)w * G + g) * (kHD + 2);
        if (ws[kHD + 1] > 0.0f) {
          const float wt = expf(ws[kHD] - M);
          L = fmaf(ws[kHD + 1], wt, L);
          od = fmaf(ws[dd], wt, od);
        }
      }
      float *dst = p.apart + (((size_t)b * p.h + h0 + g) * ph + j) * (kHD + 2);
      dst[dd] = od;
      if (dd == 0) dst[kHD] = M, dst[kHD + 1] = L;
    }
    cbar(nthr);  // shared memory is reused by the next item
  }
}

// ---- embedding, final norm ---------------------------------------------------------------

// Element e of row r of the packed embedding table (gguf.c's dequant_block
// arithmetic, as dequant_block_dev).
__device__ __forceinline__ float emb_elem(const KP &p, uint64_t r, uint32_t e) {
  const uint32_t t = p.etype, el = b200_blk_elems(t), b = e / el, j = e % el;
  const uint8_t *h = p.emb_sc + pk_hdr_off(t, p.emb_ntiles, r, b);
  const float d = f16_bits_to_f32((uint16_t)(h[0] | (h[1] << 8)));
  if (t == PAI_B200_Q4_0) {
    const uint8_t v = p.emb_qs[pk_qs_off(t, p.emb_ntiles, r, b, j % 16)];
    return __fmul_rn((float)((int)(j < 16 ? (v & 15) : (v >> 4)) - 8), d);
  }
  if (t == PAI_B200_Q8_0) return __fmul_rn((float)(int8_t)p.emb_qs[pk_qs_off(t, p.emb_ntiles, r, b, j)], d);
  const float dmin = f16_bits_to_f32((uint16_t)(h[2] | (h[3] << 8)));
  const uint32_t c = j / 64, hi = (j % 64) / 32, l = j % 32;
  uint8_t s, mn;
  k4_scale_min(2 * c + hi, h + 4, &s, &mn);
  const uint8_t v = p.emb_qs[pk_qs_off(t, p.emb_ntiles, r, b, 32 * c + l)];
  return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), (float)(hi ? (v >> 4) : (v & 15))), __fmul_rn(dmin, (float)mn));
}

// x[b] = row tok_in[b] of the embedding (llama.c:510-522), with its block
// sums of squares and x * attn_norm[0] quantised; warp per 32-element block.
template <int CONS>
__device__ void embed(const KP &p, int c, int lane) {
  const uint32_t nb = p.n_embd / 32;
  const float *gamma = p.layers[0].attn_norm;
  for (uint32_t wb = blockIdx.x * CONS + c; wb < p.batch * nb; wb += gridDim.x * CONS) {
    const uint32_t b = wb / nb, blk = wb % nb;
    const uint64_t r = (uint32_t)__ldcg(p.tok_in + b);
    finish_block(p, b, blk, emb_elem(p, r, blk * 32 + lane), gamma, lane);
  }
}

// The lm head's operand: xqn (x * output_norm, quantised unscaled by the last
// reduce phase) with its block scales multiplied by the norm scale.
template <int CONS>
__device__ void final_norm(const KP &p, int c, int lane, int ctid, int nthr, float *scales) {
  if (c == 0)
    for (uint32_t b = 0; b < p.batch; b++) {
      const float s = norm_scale(p, b, lane);
      if (lane == 0) scales[b] = s;
    }
  cbar(nthr);
  const uint32_t quads = (uint32_t)p.xqn.quads;
  const uint32_t limb16 = (uint32_t)(b200_xq_limb_bytes(p.batch, p.n_embd) / 16);
  for (uint32_t i = blockIdx.x * nthr + ctid; i < limb16; i += gridDim.x * nthr)
    reinterpret_cast<uint4 *>(p.xq_out.limbs)[i] = __ldcg(reinterpret_cast<const uint4 *>(p.xqn.limbs) + i);
  for (uint32_t i = blockIdx.x * nthr + ctid; i < p.batch * quads * 4; i += gridDim.x * nthr) {
    const float f = scales[i / (quads * 4)];
    p.xq_out.sb[i] = __fmul_rn(__ldcg(p.xqn.sb + i), f);
    p.xq_out.sx[i] = __fmul_rn(__ldcg(p.xqn.sx + i), f);
  }
}

// ---- the kernel -------------------------------------------------------------------------

template <uint32_t T, int NT, int CONS>
__global__ void __launch_bounds__((CONS + 1) * 32, 1) k_decode(const __grid_constant__ KP p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ int sflag, sfailed;
  __shared__ float scales[8];
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
    // ---- producer: the four matrices of every layer, in order ----
    if (lane != 0) return;
    uint32_t fill = 0;
    bool ok = true;
    for (uint32_t l = 0; l < p.n_layer && ok; l++)
      for (int k = 0; k < 4 && ok; k++) ok = produce<T, CONS>(p, p.sh[k], p.layers[l].w[k], ring, full, empty, fill);
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
  // the x staging area comes first; per-warp scratch (128 floats) after it
  float *scratch = reinterpret_cast<float *>(area + ((x_area_bytes(NT, p.batch, Unit<T>::XPU, p.sh[M_O].units) + 127) &
                                                     ~(size_t)127));
  uint32_t seq = 0, epoch = 0;
  // row exchanges this rank completed in earlier steps (written by the
  // previous launch's last CTA)
  const uint64_t xbase = p.nranks > 1 ? *(volatile uint64_t *)(land_words(p.land[p.rank]) + 1) : 0;
  bool ok = true;
  auto gemv = [&](int k, int xsrc, int pi) {
    consume<T, NT, CONS>(p, p.sh[k], xsrc, p.part[pi], ring, full, empty, seq, area, scratch, scales, c, lane, ctid,
                         nthr, &sfailed);
    cbar(nthr);
    if (sfailed) {
      if (ctid == 0) raise_abort(p);
      ok = false;
    }
  };
  auto sync = [&]() {
    if (ok && !grid_sync(p, epoch, ctid, nthr, &sflag)) ok = false;
    return ok;
  };
  embed<CONS>(p, c, lane);
  for (uint32_t l = 0; l < p.n_layer && ok; l++) {
    const Layer &L = p.layers[l];
    const float *g_next = l + 1 < p.n_layer ? p.layers[l + 1].attn_norm : p.out_norm;
    if (!sync()) break;
    gemv(M_QKV, X_NORMQ, 0);
    if (!sync()) break;
    switch (p.h / p.hk) {
      case 1: attention<1, CONS>(p, l, c, lane, ctid, nthr, reinterpret_cast<float *>(area)); break;
      case 2: attention<2, CONS>(p, l, c, lane, ctid, nthr, reinterpret_cast<float *>(area)); break;
      case 4: attention<4, CONS>(p, l, c, lane, ctid, nthr, reinterpret_cast<float *>(area)); break;
      default: attention<8, CONS>(p, l, c, lane, ctid, nthr, reinterpret_cast<float *>(area)); break;
    }
    if (!sync()) break;
    gemv(M_O, X_ATT, 1);
    if (!sync()) break;
    if (p.nranks > 1)
      ok = exchange_rows<CONS>(p, p.sh[M_O], L.ffn_norm, xbase + 2ull * l, c, lane, ctid, nthr, &sflag);
    else
      reduce_rows<CONS>(p, p.sh[M_O], L.ffn_norm, c, lane);
    if (!sync()) break;
    gemv(M_GU, X_NORMQ, 0);
    if (!sync()) break;
    gemv(M_DOWN, X_SILU, 1);
    if (!sync()) break;
    if (p.nranks > 1)
      ok = exchange_rows<CONS>(p, p.sh[M_DOWN], g_next, xbase + 2ull * l + 1, c, lane, ctid, nthr, &sflag);
    else
      reduce_rows<CONS>(p, p.sh[M_DOWN], g_next, c, lane);
  }
  if (ok && sync()) final_norm<CONS>(p, c, lane, ctid, nthr, scales);
  // Leave: the last CTA out resets the barrier words for the next launch
  // (every CTA counted here has passed every barrier of this launch).
  cbar(nthr);
  if (ctid == 0) {
    __threadfence();
    const uint32_t out = atomicAdd(p.bar + 1, 1u);
    if (out == gridDim.x - 1 && !*(volatile uint32_t *)(p.bar + 2)) {
      p.bar[0] = 0;
      p.bar[1] = 0;
      if (p.nranks > 1) land_words(p.land[p.rank])[1] = xbase + 2ull * p.n_layer;  // read by the next launch
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
  Layer *layers;
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
