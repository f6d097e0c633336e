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
// Tiles per consumer warp and K units per ring stage: with two or more
// vector pairs, Q4_0 gives each warp two tiles (one unit per stage), so a
// warp reads a stage's activations -- four times the weights' bytes at
// batch 8 -- once for both (measured: 8 % off the batch-8 step). At batch
// 1-2 the larger row groups would double the splits the residual phases add
// up, which costs more than it saves; Q8_0 and Q4_K keep one tile (a
// two-tile stage would not fit the ring).
template <uint32_t T, int NT>
constexpr int kTPW = (T == PAI_B200_Q4_0 && NT > 1) ? 2 : 1;
template <uint32_t T, int NT>
constexpr int kUPS = kTPW<T, NT> == 2 ? 1 : gemv::Unit<T>::U;
// bytes of one ring stage: the largest of units x tiles x (codes + headers)
// over the block types (Q4_0: 1 x 2 CONS x 1152, Q8_0: CONS x 2176, Q4_K:
// CONS x 2304)
template <int CONS>
constexpr uint32_t kStageBytes = CONS * 2304u;
constexpr uint32_t kHD = 128;
constexpr uint32_t kAS = kHD + 4;  // attention partial: o[kHD], max, sum, 2 pad (16-byte rows)
constexpr uint32_t kMaxSlots = 16;  // attention CTAs per (sequence, kv head) at most
enum { M_QKV = 0, M_O = 1, M_GU = 2, M_DOWN = 3 };

// Shape and work split of one layer-matrix kind (the same for every layer).
struct Shape {
  uint32_t n, k, units, ntiles, ngroups, npad, gw, maxseg;
  uint32_t gt;      // 16-row tiles per row group (consumer warps x tiles per warp)
  uint32_t tab;     // first entry of this shape's groups in the split-count table
  uint64_t sc_off;  // byte offset of the header plane in the packed matrix
};

// Split counts (CTAs per row group) of the four shapes' groups, filled by
// every CTA at the start of the launch: readers of partial sums look the
// count up instead of recomputing the split.
constexpr uint32_t kTab = 2048;
static __shared__ uint8_t s_nseg[kTab];

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
  b200_xq_t xqa, xqh;  // batches of 3+: attention output and silu(gate) * up, quantised once
  double *ssq;       // [batch][n_embd / 32] sums of squares of x per block
  b200_xq_t xq_out;  // RMSNorm(x) * out_norm for the lm head
  const float *out_norm;
  float *part[2];  // split-K partials: q|k|v and gate|up in [0], o and down in [1]
  float *apart;    // attention CTA partials [batch][h][per_head][kAS]
  uint32_t *bar;   // [0] barrier arrivals, [1] exits, [2] abort
  uint32_t *err;   // the context's host-mapped error word
  uint32_t scratch_off;  // per-warp staging scratch: byte offset in the staging area
  uint64_t wait_ns;
  // tensor parallelism: every rank's landing buffer as mapped here
  uint8_t *land[B200_TP_MAX_RANKS];
  uint32_t rank, nranks;
};

// The launch's parameters and position count, copied into shared memory
// at the start: the phases compiled out of line reach them through a
// reference, and a reference to a __grid_constant__ parameter reads through
// the memory system, one dependent round trip per first access.
static __shared__ KP s_kp;
static __shared__ uint32_t s_npos;  // positions of the cache including this step's

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
// wait) until all CTAs arrived. Returns the same answer to every consumer
// thread of the CTA.
__device__ inline bool grid_sync(const KP &p, uint32_t &epoch, int ctid, int nthr, volatile int *sflag) {
  cbar(nthr);
  if (ctid == 0) {
    epoch++;
    bool ok = true;
    // publish the CTA's writes (ordered before this thread by the named
    // barrier) at GPU scope, then arrive without waiting for a reply
    asm volatile("fence.acq_rel.gpu;\n red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
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
    *sflag = ok ? 1 : 0;  // the acquire load that saw the count orders the reads after it
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

// Row `row` of vector b is the sum of its group's partials in split order.
// row_load issues the loads of the first CH parts (predicated, no branch: the
// loads of several rows go out together); row_finish adds them in order and
// loads any further parts.
struct RowRef {
  const float *q;
  uint32_t nseg;
};
template <int CH, int CONS>
__device__ __forceinline__ RowRef row_load(const float *part, const Shape &sh, uint32_t batch, uint32_t b,
                                           uint32_t row, float (&v)[CH]) {
  RowRef r;
  r.nseg = s_nseg[sh.tab + row / (16u * sh.gt)];
  r.q = part + (size_t)b * sh.npad + row;
  const size_t stride = (size_t)batch * sh.npad;
#pragma unroll
  for (int i = 0; i < CH; i++) v[i] = (uint32_t)i < r.nseg ? __ldcg(r.q + i * stride) : 0.0f;
  return r;
}
template <int CH>
__device__ __forceinline__ float row_finish(const RowRef &r, const float (&v)[CH], uint32_t batch, uint32_t npad) {
  float s = v[0];
#pragma unroll
  for (int i = 1; i < CH; i++)
    if ((uint32_t)i < r.nseg) s += v[i];
  for (uint32_t i = CH; i < r.nseg; i++) s += __ldcg(r.q + (size_t)i * batch * npad);
  return s;
}
template <int CH, int CONS>
__device__ __forceinline__ float row_sum(const float *part, const Shape &sh, uint32_t batch, uint32_t b,
                                         uint32_t row) {
  float v[CH];
  const RowRef r = row_load<CH, CONS>(part, sh, batch, b, row, v);
  return row_finish<CH>(r, v, batch, sh.npad);
}

// This CTA's (group, unit) range [r0, r1) of one shape, the group of r0 and
// the CTA's split index in that group (it is split 0 of every later group
// it touches), computed once per launch (64-bit arithmetic).
struct Range {
  uint32_t r0, r1, g0, split0;
};
static __shared__ Range s_rng[4];

__device__ inline Range make_range(const Shape &sh) {
  uint64_t r0, r1;
  phase_range(sh, r0, r1);
  Range r;
  r.r0 = (uint32_t)r0;
  r.r1 = (uint32_t)r1;
  r.g0 = r0 < r1 ? (uint32_t)(r0 / sh.units) : 0u;
  uint32_t lo = blockIdx.x, nseg;
  if (r0 < r1) group_split(sh, r.g0, lo, nseg);
  r.split0 = blockIdx.x - lo;
  return r;
}

// Fill s_nseg (consumer threads; a named barrier follows before any use).
__device__ inline void fill_split_table(const KP &p, int ctid, int nthr) {
#pragma unroll
  for (int k = 0; k < 4; k++)
    for (uint32_t g = ctid; g < p.sh[k].ngroups; g += nthr) {
      uint32_t lo, nseg;
      group_split(p.sh[k], g, lo, nseg);
      s_nseg[p.sh[k].tab + g] = (uint8_t)nseg;
    }
}

// A piece of a CTA's range inside one row group: units [u0, u1) of group g.
struct Sub {
  uint32_t g, u0, u1;
};

__device__ __forceinline__ Sub sub_at(const Shape &sh, uint32_t pos, uint32_t r1) {
  Sub s;
  s.g = pos / sh.units;
  s.u0 = pos - s.g * sh.units;
  s.u1 = min(r1, (s.g + 1) * sh.units) - s.g * sh.units;
  return s;
}

// Q4_0, two consecutive 16-row tiles of one K unit (codes at qs and
// qs + 1024, headers at sc and sc + 128; the layout of gemv_unit.cuh's
// Unit<Q4_0>): the activation digits and their scale products are loaded and
// formed once and used for both tiles. Per tile the arithmetic is
// Unit<Q4_0>::compute's, in the same order.
template <int NT>
__device__ __forceinline__ void q4_0_two_tiles(const uint8_t *qs, const uint8_t *sc, const XS &xs, uint32_t qq,
                                               int lane, float (&yr)[2][NT], float (&yr8)[2][NT]) {
  XOp x[NT];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) load_x(xs, nt, qq, lane, x[nt]);
  uint4 a0[2], a1[2];
  uint2 d0[2], d1[2];
#pragma unroll
  for (int t = 0; t < 2; t++) {
    a0[t] = *reinterpret_cast<const uint4 *>(qs + t * 1024 + lane * 16);
    a1[t] = *reinterpret_cast<const uint4 *>(qs + t * 1024 + 512 + lane * 16);
    d0[t] = *reinterpret_cast<const uint2 *>(sc + t * 128 + (lane >> 2) * 8);
    d1[t] = *reinterpret_cast<const uint2 *>(sc + t * 128 + 64 + (lane >> 2) * 8);
  }
  const float lscale = (lane & 1) ? (1.0f / 256.0f) : 256.0f;
  const float cmul = (lane & 1) ? 0.0f : 8.0f;  // the -8 offset of Q4_0 codes, once per lane pair
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float sl[NT], cr[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      sl[nt] = comp(x[nt].sb, i) * lscale;
      cr[nt] = comp(x[nt].sx, i) * cmul;
    }
#pragma unroll
    for (int t = 0; t < 2; t++) {
      const uint32_t wr = comp(a0[t], i), wr8 = comp(a1[t], i);
      const uint32_t A0 = wr & M4, A1 = wr8 & M4, A2 = (wr >> 4) & M4, A3 = (wr8 >> 4) & M4;
      const float dr = half_at(d0[t], i), dr8 = half_at(d1[t], i);
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        int acc[4];
        mma_u8s8(acc, A0, A1, A2, A3, comp(x[nt].lo, i), comp(x[nt].hi, i));
        yr[t][nt] = fmaf(dr, fmaf(sl[nt], fold(acc[0], acc[1]), -cr[nt]), yr[t][nt]);
        yr8[t][nt] = fmaf(dr8, fmaf(sl[nt], fold(acc[2], acc[3]), -cr[nt]), yr8[t][nt]);
      }
    }
  }
}

// Producer: stream the weights of the CTA's range of one GEMV phase into the
// ring, one stage per U units of a sub-item. Returns false when a wait for
// a free stage ran out.
template <uint32_t T, int NT, int CONS>
__device__ bool produce(const KP &p, int k, const uint8_t *w, uint8_t *ring, uint64_t *full, uint64_t *empty,
                        uint32_t &fill) {
  using Un = Unit<T>;
  constexpr int U = kUPS<T, NT>, GT = CONS * kTPW<T, NT>;
  constexpr uint32_t GQ = GT * Un::QB, GS = GT * Un::SB;
  static_assert(U * (GQ + GS) <= kStageBytes<CONS>, "ring stage");
  const Shape &sh = p.sh[k];
  const uint8_t *qs = w, *sc = w + sh.sc_off;
  const uint32_t r0 = s_rng[k].r0, r1 = s_rng[k].r1;
  for (uint32_t pos = r0; pos < r1;) {
    const Sub s = sub_at(sh, pos, r1);
    pos += s.u1 - s.u0;
    const uint32_t nv = min((uint32_t)GT, sh.ntiles - s.g * GT);  // tiles present in the group
    const size_t tile0 = (size_t)s.g * GT;
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
  uint32_t u0;  // unit of entry 0
  bool resident;
};

template <int NT, int XPU>
__device__ __forceinline__ XArea x_area(const KP &p, const Shape &sh, uint8_t *area, uint32_t r0, uint32_t r1) {
  XArea a;
  const uint32_t L = r1 - r0;
  a.resident = L >= sh.units;
  a.nent = a.resident ? sh.units : L;
  a.u0 = a.resident ? 0u : r0 % sh.units;
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

// Unit of entry e: a range shorter than a group spans at most two groups, so
// the units run u0, u0 + 1, ... and wrap once.
__device__ __forceinline__ uint32_t entry_unit(const Shape &sh, const XArea &a, uint32_t e) {
  const uint32_t u = a.u0 + e;
  return u >= sh.units ? u - sh.units : u;
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
  for (uint32_t i0 = lane; i0 < nb; i0 += 8 * 32) {
    double v[8];
#pragma unroll
    for (int m = 0; m < 8; m++) v[m] = i0 + 32 * m < nb ? __ldcg(s + i0 + 32 * m) : 0.0;
#pragma unroll
    for (int m = 0; m < 8; m++)
      if (i0 + 32 * m < nb) acc = __dadd_rn(acc, v[m]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  const float ms = (float)__ddiv_rn(acc, (double)p.n_embd);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
}

// 16-byte asynchronous global -> shared copy (L2 only, no registers held).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n cp.async.wait_all;" ::: "memory");
}

// A GEMV operand quantised once in global memory (src), the entries' units
// of it staged by asynchronous copies. NORM: src is the unscaled x * gamma
// of an RMSNorm (xqn), and the block scales are multiplied by the norm
// scale, which warp b computes for vector b from the block sums of squares
// while the copies land.
template <int NT, int XPU, int CONS, bool NORM>
__device__ __noinline__ void stage_copy(const KP &p, const Shape &sh, const XArea &a, const b200_xq_t &src, int c,
                                        int lane, int ctid, int nthr, float *scales) {
  const uint32_t nq = a.nent * XPU, per = NT * XPU * 64;  // uint4 per entry (digits)
  uint4 *dl = reinterpret_cast<uint4 *>(const_cast<uint8_t *>(a.xs.limbs));
  const uint4 *sl = reinterpret_cast<const uint4 *>(src.limbs);
  for (uint32_t i = ctid; i < a.nent * per; i += nthr) {
    const uint32_t e = i / per, r = i % per, nt = r / (XPU * 64), o = r % (XPU * 64);
    cp_async16(dl + (((size_t)nt * nq + (size_t)e * XPU) * 1024) / 16 + o,
               sl + (((size_t)nt * src.quads + (size_t)entry_unit(sh, a, e) * XPU) * 1024) / 16 + o);
  }
  float4 *db = reinterpret_cast<float4 *>(const_cast<float *>(a.xs.sb));
  float4 *dx = reinterpret_cast<float4 *>(const_cast<float *>(a.xs.sx));
  const float4 *sb = reinterpret_cast<const float4 *>(src.sb);
  const float4 *sx = reinterpret_cast<const float4 *>(src.sx);
  const uint32_t nsc = a.nent * p.batch * XPU;
  for (uint32_t i = ctid; i < nsc; i += nthr) {
    const uint32_t e = i / (p.batch * XPU), r = i % (p.batch * XPU), vec = r / XPU, q = r % XPU;
    const size_t from = (size_t)vec * src.quads + (size_t)entry_unit(sh, a, e) * XPU + q;
    const size_t d = (size_t)vec * nq + (size_t)e * XPU + q;
    cp_async16(db + d, sb + from);
    cp_async16(dx + d, sx + from);
  }
  if (NORM)
    for (uint32_t b = c; b < p.batch; b += CONS) {  // warp b: vector b's scale
      const float sc = norm_scale(p, b, lane);
      if (lane == 0) scales[b] = sc;
    }
  cp_async_wait_all();
  cbar(nthr);  // the copies and the norm scales are in shared memory
  if (NORM)
    for (uint32_t i = ctid; i < nsc; i += nthr) {
      const uint32_t e = i / (p.batch * XPU), r = i % (p.batch * XPU), vec = r / XPU, q = r % XPU;
      const size_t d = (size_t)vec * nq + (size_t)e * XPU + q;
      const float f = scales[vec];
      float4 bv = db[d], xv = dx[d];
      bv.x = __fmul_rn(bv.x, f), bv.y = __fmul_rn(bv.y, f), bv.z = __fmul_rn(bv.z, f), bv.w = __fmul_rn(bv.w, f);
      xv.x = __fmul_rn(xv.x, f), xv.y = __fmul_rn(xv.y, f), xv.z = __fmul_rn(xv.z, f), xv.w = __fmul_rn(xv.w, f);
      db[d] = bv;
      dx[d] = xv;
    }
}

// Attention output of head hh of vector b: the attention CTAs' partials of
// its slots merged (slot order; one round of loads -- lane s holds slot s's
// statistics, lane l the dims 4l..4l+3 of every slot) and quantised into
// blocks blk0 .. blk0 + 3 of vector b of `dst` (through the warp's shared
// scratch ws, lane = element). One warp.
__device__ __forceinline__ void merge_head(const KP &p, uint32_t b, uint32_t hh, int lane, float *ws,
                                           const b200_xq_t &dst, uint32_t blk0) {
  const uint32_t ph = p.per_head;
  const float *base = p.apart + (((size_t)b * p.h + hh) * ph) * kAS;
  const float2 ml = (uint32_t)lane < ph ? __ldcg(reinterpret_cast<const float2 *>(base + (size_t)lane * kAS + kHD))
                                        : make_float2(-INFINITY, 0.0f);
  float4 ov[kMaxSlots];
#pragma unroll
  for (uint32_t m = 0; m < kMaxSlots; m++)
    ov[m] = m < ph ? __ldcg(reinterpret_cast<const float4 *>(base + (size_t)m * kAS) + lane)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
  const float M = warp_max(ml.y > 0.0f ? ml.x : -INFINITY);
  const float w = ml.y > 0.0f ? expf(ml.x - M) : 0.0f;
  const float L = warp_sum(ml.y * w);
  float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (uint32_t m = 0; m < kMaxSlots; m++) {
    const float wm = __shfl_sync(0xffffffffu, w, m);
    o[0] = fmaf(ov[m].x, wm, o[0]), o[1] = fmaf(ov[m].y, wm, o[1]);
    o[2] = fmaf(ov[m].z, wm, o[2]), o[3] = fmaf(ov[m].w, wm, o[3]);
  }
  __syncwarp();
  *reinterpret_cast<float4 *>(ws + 4 * lane) = make_float4(o[0] / L, o[1] / L, o[2] / L, o[3] / L);
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 4; q++) xq_store_block(dst, b, blk0 + q, ws[32 * q + lane]);
  __syncwarp();
}

// o's input at batches of 1-2: the heads in the entries' units merged by this
// CTA (one warp per (vector, head)).
template <int NT, int XPU, int CONS>
__device__ __noinline__ void stage_att(const KP &p, const Shape &sh, const XArea &a, int c, int lane, float *scratch) {
  const b200_xq_t v = slot_view(p, a, sh.k);
  const uint32_t heads = a.nent * XPU, nj = heads * p.batch;
  for (uint32_t j = c; j < nj; j += CONS) {
    const uint32_t b = j / heads, eh = j % heads, e = eh / XPU;
    // head (unit e XPU + eh % XPU) is x blocks 4 hh .. 4 hh + 3; in the entry
    // they are blocks 4 (e XPU + eh % XPU) .. of the slot
    merge_head(p, b, entry_unit(sh, a, e) * XPU + eh % XPU, lane, scratch + c * kHD, v, (e * XPU + eh % XPU) * 4);
  }
}

// Batches of 3+: every (vector, head) merged once into xqa, one warp each
// over the grid (o then stages xqa by copies).
template <int CONS>
__device__ __noinline__ void merge_phase(const KP &p, int c, int lane, float *scratch) {
  const uint32_t nj = p.batch * p.h;
  for (uint32_t j = blockIdx.x * CONS + c; j < nj; j += gridDim.x * CONS)
    merge_head(p, j / p.h, j % p.h, lane, scratch + c * kHD, p.xqa, 4 * (j % p.h));
}

// h = silu(gate) * up for outputs o0 .. o0 + 127 of vector b from the
// gate|up partial sums (gate|up tile t holds gate rows 8t.. then the
// matching up rows), quantised into blocks blk0 .. blk0 + 3 of vector b of
// `dst`. One warp: lane l takes outputs 4l..4l+3 -- 4 consecutive gate rows
// and the 4 up rows 8 further, one 16-byte load each per split, all splits'
// loads in flight -- and the values go through the warp's shared scratch to
// quantise with lane = element.
template <int CONS>
__device__ __forceinline__ void silu_chunk(const KP &p, uint32_t b, uint32_t o0, uint32_t k, int lane, float *ws,
                                           const b200_xq_t &dst, uint32_t blk0) {
  const Shape &gu = p.sh[M_GU];
  const size_t st4 = (size_t)p.batch * gu.npad / 4;
  constexpr int CH = 4;  // splits loaded at once (a gate|up group spans few CTAs)
  const uint32_t o = o0 + 4 * lane, oc = min(o, k - 4);
  const uint32_t grow = (oc / 8) * 16 + oc % 8;
  const uint32_t nseg = s_nseg[gu.tab + grow / (16u * gu.gt)];
  const float4 *q = reinterpret_cast<const float4 *>(p.part[0] + (size_t)b * gu.npad + grow);
  float4 gv[CH], uv[CH];
#pragma unroll
  for (int m = 0; m < CH; m++) {
    const bool in = (uint32_t)m < nseg;
    gv[m] = in ? __ldcg(q + m * st4) : make_float4(0.f, 0.f, 0.f, 0.f);
    uv[m] = in ? __ldcg(q + m * st4 + 2) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float4 gs = gv[0], us = uv[0];
#pragma unroll
  for (int m = 1; m < CH; m++)
    if ((uint32_t)m < nseg) {
      gs.x += gv[m].x, gs.y += gv[m].y, gs.z += gv[m].z, gs.w += gv[m].w;
      us.x += uv[m].x, us.y += uv[m].y, us.z += uv[m].z, us.w += uv[m].w;
    }
  for (uint32_t m = CH; m < nseg; m++) {
    const float4 g4 = __ldcg(q + m * st4), u4 = __ldcg(q + m * st4 + 2);
    gs.x += g4.x, gs.y += g4.y, gs.z += g4.z, gs.w += g4.w;
    us.x += u4.x, us.y += u4.y, us.z += u4.z, us.w += u4.w;
  }
  float4 h4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (o < k) {  // k % 32 == 0: the lane's 4 outputs are all in or all out
    // llama.c:774-781
    h4.x = __fmul_rn(__fdiv_rn(gs.x, __fadd_rn(1.0f, expf(-gs.x))), us.x);
    h4.y = __fmul_rn(__fdiv_rn(gs.y, __fadd_rn(1.0f, expf(-gs.y))), us.y);
    h4.z = __fmul_rn(__fdiv_rn(gs.z, __fadd_rn(1.0f, expf(-gs.z))), us.z);
    h4.w = __fmul_rn(__fdiv_rn(gs.w, __fadd_rn(1.0f, expf(-gs.w))), us.w);
  }
  __syncwarp();
  *reinterpret_cast<float4 *>(ws + 4 * lane) = h4;
  __syncwarp();
#pragma unroll
  for (int qq = 0; qq < 4; qq++) xq_store_block(dst, b, blk0 + qq, ws[32 * qq + lane]);
  __syncwarp();
}

// down's input at batches of 1-2: the entries' units computed by this CTA,
// one warp per (vector, 128 outputs).
template <int NT, int XPU, int CONS>
__device__ __noinline__ void stage_silu(const KP &p, const Shape &sh, const XArea &a, int c, int lane,
                                        float *scratch) {
  const b200_xq_t v = slot_view(p, a, sh.k);
  const uint32_t nch = a.nent * XPU, ni = nch * p.batch;  // 128-output chunks
  for (uint32_t it = c; it < ni; it += CONS) {
    const uint32_t b = it / nch, ch = it % nch, e = ch / XPU;
    silu_chunk<CONS>(p, b, (entry_unit(sh, a, e) * XPU + ch % XPU) * 128, sh.k, lane, scratch + c * kHD, v,
                     ch * 4);
  }
}

// Batches of 3+: h computed once into xqh, one warp per (vector, 128
// outputs) over the grid (down then stages xqh by copies).
template <int CONS>
__device__ __noinline__ void silu_phase(const KP &p, int c, int lane, float *scratch) {
  const uint32_t k = p.sh[M_DOWN].k, nch = (k + 127) / 128, ni = nch * p.batch;
  for (uint32_t it = blockIdx.x * CONS + c; it < ni; it += gridDim.x * CONS)
    silu_chunk<CONS>(p, it / nch, (it % nch) * 128, k, lane, scratch + c * kHD, p.xqh, (it % nch) * 4);
}

// ---- GEMV phases ------------------------------------------------------------------------

enum { X_NORMQ = 0, X_ATT = 1, X_SILU = 2, X_COPY_A = 3, X_COPY_H = 4 };

// Consumer side of one GEMV phase: stage the operand, run the ring, write
// the CTA's segments as partial row sums. `failed` (shared) records a ring
// wait that ran out; the loop structure is the same either way, so every
// thread reaches the same barriers.
template <uint32_t T, int NT, int CONS>
__device__ void consume(const KP &p, int k, int xsrc, float *part, uint8_t *ring, uint64_t *full,
                        uint64_t *empty, uint32_t &seq, uint8_t *area, float *scratch, float *scales, int c,
                        int lane, int ctid, int nthr, volatile int *failed) {
  using Un = Unit<T>;
  constexpr int U = kUPS<T, NT>, XPU = Un::XPU, TPW = kTPW<T, NT>, GT = CONS * TPW;
  constexpr uint32_t GQ = GT * Un::QB, GS = GT * Un::SB;
  const Shape &sh = p.sh[k];
  const uint32_t r0 = s_rng[k].r0, r1 = s_rng[k].r1, g0 = s_rng[k].g0, split0 = s_rng[k].split0;
  if (r0 >= r1) return;
  const XArea a = x_area<NT, XPU>(p, sh, area, r0, r1);
  if (xsrc == X_NORMQ)
    stage_copy<NT, XPU, CONS, true>(s_kp, s_kp.sh[k], a, s_kp.xqn, c, lane, ctid, nthr, scales);
  else if (xsrc == X_COPY_A)
    stage_copy<NT, XPU, CONS, false>(s_kp, s_kp.sh[k], a, s_kp.xqa, c, lane, ctid, nthr, scales);
  else if (xsrc == X_COPY_H)
    stage_copy<NT, XPU, CONS, false>(s_kp, s_kp.sh[k], a, s_kp.xqh, c, lane, ctid, nthr, scales);
  else if (xsrc == X_ATT)
    stage_att<NT, XPU, CONS>(s_kp, s_kp.sh[k], a, c, lane, scratch);
  else
    stage_silu<NT, XPU, CONS>(s_kp, s_kp.sh[k], a, c, lane, scratch);
  cbar(nthr);
  const uint32_t r = lane >> 2, vsel = (lane & 3) >> 1;
  const bool holder = (lane & 1) == 0;
  float yr[TPW][NT], yr8[TPW][NT];
  bool bad = false;
  for (uint32_t pos = r0; pos < r1;) {
    const Sub s = sub_at(sh, pos, r1);
    const uint32_t eoff = pos - r0;  // entry of unit s.u0 when not resident
    pos += s.u1 - s.u0;
    const uint32_t tile0 = s.g * GT + c * TPW;  // the warp's first tile of the group
    const bool active = tile0 < sh.ntiles;
#pragma unroll
    for (int t = 0; t < TPW; t++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++) yr[t][nt] = yr8[t][nt] = 0.f;
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
            const uint8_t *q = st + uu * GQ + c * TPW * Un::QB, *h = st + U * GQ + uu * GS + c * TPW * Un::SB;
            if constexpr (TPW == 2)
              q4_0_two_tiles<NT>(q, h, a.xs, e * XPU, lane, yr, yr8);
            else
              Un::template compute<NT>(q, h, a.xs, e * XPU, lane, yr[0], yr8[0]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      seq++;
    }
    if (!active || bad) continue;
    // this CTA's segment of group g: its partial row sums
    const uint32_t split = s.g == g0 ? split0 : 0u;
#pragma unroll
    for (int t = 0; t < TPW; t++) {
      const uint32_t tile = tile0 + t;
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {  // lane pairs (c, c^1) hold the two halves of one sum
        const float ya = yr[t][nt] + __shfl_xor_sync(0xffffffffu, yr[t][nt], 1);
        const float yb = yr8[t][nt] + __shfl_xor_sync(0xffffffffu, yr8[t][nt], 1);
        const uint32_t vec = 2 * nt + vsel;
        if (holder && vec < p.batch && tile < sh.ntiles) {
          float *pp = part + ((size_t)split * p.batch + vec) * sh.npad + (size_t)tile * 16 + r;
          pp[0] = ya;
          pp[8] = yb;
        }
      }
    }
  }
}

// ---- reduce phases: residual add, block sums of squares, the next norm's operand -----------

// x block (32 rows) of vector b: v = x + sum; writes x, the block's sum of
// squares (fixed shuffle order) and v * gamma quantised (unscaled); g is the
// lane's gain, loaded by the caller with its other operands. One warp.
__device__ __forceinline__ void finish_block(const KP &p, uint32_t b, uint32_t blk, float v, float g, int lane) {
  const uint32_t row = blk * 32 + lane;
  p.x[(size_t)b * p.n_embd + row] = v;
  double sq = __dmul_rn((double)v, (double)v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq = __dadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
  if (lane == 0) p.ssq[(size_t)b * (p.n_embd / 32) + blk] = sq;
  xq_store_block(p.xqn, b, blk, __fmul_rn(v, g));
}

// One GPU: x += the o or down GEMV's row sums (the residual adds of
// llama.c:747-749, 793-795); warp per 32-row block.
template <int CONS>
__device__ __noinline__ void reduce_rows(const KP &p, const Shape &sh, const float *gamma, int c, int lane) {
  const uint32_t nb = p.n_embd / 32;
  for (uint32_t wb = blockIdx.x * CONS + c; wb < p.batch * nb; wb += gridDim.x * CONS) {
    const uint32_t b = wb / nb, blk = wb % nb, row = blk * 32 + lane;
    float pv[32];
    const RowRef rr = row_load<32, CONS>(p.part[1], sh, p.batch, b, row, pv);
    const float xv = __ldcg(p.x + (size_t)b * p.n_embd + row), g = __ldg(gamma + row);  // same round
    finish_block(p, b, blk, __fadd_rn(xv, row_finish<32>(rr, pv, p.batch, sh.npad)), g, lane);
  }
}

__device__ __forceinline__ uint64_t *land_words(uint8_t *b) { return reinterpret_cast<uint64_t *>(b); }
// Row slot [parity][src] of rank r's landing buffer: batch x n_embd tagged words.
__device__ __forceinline__ uint64_t *land_rows(const KP &p, uint32_t r, uint32_t parity, uint32_t src) {
  return reinterpret_cast<uint64_t *>(p.land[r] + B200_LAND_HDR) + ((size_t)parity * p.nranks + src) * p.batch * p.n_embd;
}
__device__ __forceinline__ void st_relaxed_sys64(uint64_t *q, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(q), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys64(const uint64_t *q) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(q) : "memory");
  return v;
}

// Tensor parallelism: the same as reduce_rows with the sum over ranks, by a
// low-latency protocol. Every row value of this rank travels as one 8-byte
// word (tag << 32 | value bits; tag = low 32 bits of the exchange count + 1,
// so a word of an older exchange or the zeroed buffer never matches) stored
// into slot [parity][this rank] of every rank's landing buffer (plain peer
// stores over NVLink; an aligned 8-byte store arrives whole). The warp that
// owns a 32-row block -- the same block -> warp map on every rank -- then
// polls its own buffer for each rank's word of its rows (bounded, ends early
// when another CTA raised the abort word) and adds the ranks' values in rank
// order, so every rank holds the same bits. No fence, no flag round, no
// barrier inside the exchange. A slot is reused two exchanges later, which
// no rank reaches before every rank has read it: exchange e+1 needs every
// rank's rows of e+1, which a rank writes only after its grid barrier that
// follows its reading of e. Returns false (the same answer to every consumer
// thread of the CTA) when a wait ran out or the launch was aborted.
template <int CONS>
__device__ __noinline__ bool exchange_rows(const KP &p, const Shape &sh, const float *gamma, uint64_t e, int c,
                                           int lane, int ctid, int nthr, volatile int *sflag) {
  const uint32_t nb = p.n_embd / 32, parity = (uint32_t)(e & 1u), tag = (uint32_t)(e + 1);
  bool ok = true;
  for (uint32_t wb = blockIdx.x * CONS + c; wb < p.batch * nb && ok; wb += gridDim.x * CONS) {
    const uint32_t b = wb / nb, blk = wb % nb, row = blk * 32 + lane;
    const size_t at = (size_t)b * p.n_embd + row;
    const float v = row_sum<32, CONS>(p.part[1], sh, p.batch, b, row);
    const uint64_t word = ((uint64_t)tag << 32) | __float_as_uint(v);
    for (uint32_t q = 0; q < p.nranks; q++) st_relaxed_sys64(land_rows(p, q, parity, p.rank) + at, word);
    const float xv = __ldcg(p.x + at), g = __ldg(gamma + row);
    float sum = 0.0f;
    bool mine = true;
    for (uint32_t q = 0; q < p.nranks && mine; q++) {  // rank order
      const uint64_t *src = land_rows(p, p.rank, parity, q) + at;
      uint64_t w = ld_relaxed_sys64(src);
      uint64_t t0 = 0;
      for (uint32_t it = 0; (uint32_t)(w >> 32) != tag; it++) {
        if ((it & 63u) == 0) {
          if (*(volatile uint32_t *)(p.bar + 2)) {
            mine = false;
            break;
          }
          const uint64_t now = globaltimer_ns();
          if (it == 0) {
            t0 = now;
          } else if (now - t0 > p.wait_ns) {
            raise_abort(p);
            mine = false;
            break;
          }
        }
        w = ld_relaxed_sys64(src);
      }
      const float vq = __uint_as_float((uint32_t)w);
      sum = q == 0 ? vq : sum + vq;
    }
    ok = __all_sync(0xffffffffu, mine);
    if (ok) finish_block(p, b, blk, __fadd_rn(xv, sum), g, lane);
  }
  cbar(nthr);
  if (ctid == 0) *sflag = *(volatile uint32_t *)(p.bar + 2) ? 0 : 1;
  cbar(nthr);
  return *sflag != 0;
}

// ---- attention ---------------------------------------------------------------------------

// Attention over layer `layer`'s cache (the last row of pai_ref_attention_f32,
// cpu/reference/ref_ops.c:307-349, on the cache contents: scores scaled by
// 1/sqrtf(hd) after the dot, softmax with the maximum subtracted, sum of
// p_i v_i), after RoPE (pai_ref_rope_f32's pairs (i, i + 64)) of q and k and
// the fp16 append of k and v at the position (llama.c:700-731).
//
// Work item (sequence b, kv head, slot j): positions [j cpos, (j+1) cpos),
// slots = per_head CTAs per (sequence, kv head). The CTA first adds the
// q|k|v partial sums of its G + 2 heads' rows into shared memory (all loads
// in flight), rotates q and k there, and -- the CTA whose range holds the
// position -- appends k and v to the cache. Warp w takes the 8-position
// groups p0 + 8 w + 8 CONS t: lane 4i + r dots quarter r (32 dims) of
// position i's K row with the G q heads and two shuffles add the quarters;
// softmax statistics over the 8 positions take three shuffles; the V rows of
// the 8 positions are loaded at once with lane l on dims 4l..4l+3. The warps
// are merged in shared memory into one partial (o, max, sum) per head and
// slot. Not inlined: its arrays keep their own register allocation.
constexpr uint32_t kQP = 36;  // shared-memory q: quarter rows of 32 dims padded to 36 (banks)

template <int G, int CONS>
__device__ __noinline__ void attention(const KP &p, uint32_t layer, int warp, int lane, int ctid, int nthr,
                                       float *sm) {
  const Shape &sq = p.sh[M_QKV];
  const float *part = p.part[0];
  const uint32_t npos = s_npos, pos = npos - 1, ph = p.per_head;
  const uint32_t cpos = ((npos + ph - 1) / ph + 7u) / 8u * 8u;  // positions per slot
  const uint32_t nitems = p.batch * p.hk * ph;
  const size_t lofs = (size_t)layer * p.layer_stride;
  constexpr uint32_t R = (G + 2) * kHD;  // rows of q (G heads), k, v
  // shared memory: q [G][4][kQP] | k, v [2][kHD] | the warps' partials [CONS][G][kAS]
  float *qs = sm, *kvs = sm + G * 4 * kQP, *wpart = kvs + 2 * kHD;
  const int r4 = lane & 3, i8 = lane >> 2;  // quarter, position in the group of 8
  for (uint32_t item = blockIdx.x; item < nitems; item += gridDim.x) {
    const uint32_t b = item / (p.hk * ph), kvh = (item / ph) % p.hk, j = item % ph, h0 = kvh * G;
    const uint32_t p0 = j * cpos, p1 = min(npos, p0 + cpos);
    if (p0 >= p1) {  // no positions (CTA-uniform): the slot says so
      for (uint32_t i = ctid; i < G * kAS; i += nthr) {
        const uint32_t g = i / kAS, d = i % kAS;
        p.apart[(((size_t)b * p.h + h0 + g) * p.per_head + j) * kAS + d] = d == kHD ? -INFINITY : 0.0f;
      }
      continue;
    }
    const uint32_t nw = min((uint32_t)CONS, (p1 - p0 + 7) / 8);  // warps with positions
    // RoPE table entries of the first pair this thread rotates below (loaded with the rows)
    constexpr uint32_t NP = (G + 1) * (kHD / 2);  // pairs of the G q heads and k
    float rc = 0.f, rs = 0.f;
    if ((uint32_t)ctid < NP) {
      const uint32_t d = (uint32_t)ctid % (kHD / 2);
      rc = __ldg(p.cos_t + (size_t)pos * (kHD / 2) + d), rs = __ldg(p.sin_t + (size_t)pos * (kHD / 2) + d);
    }
    // q | k | v rows of this kv head from the q|k|v partial sums: every
    // thread's rows (RPT of them) with the first 8 parts of each loaded in
    // one round -- a q|k|v row group is split over at most 8 CTAs at the
    // shapes this kernel serves, and row_finish loads any further parts
    constexpr uint32_t RPT = (R + CONS * 32 - 1) / (CONS * 32);
    {
      float v[RPT][8];
      RowRef rr[RPT];
#pragma unroll
      for (uint32_t t = 0; t < RPT; t++) {
        const uint32_t i = min((uint32_t)ctid + t * nthr, R - 1);
        const uint32_t row = i < G * kHD ? h0 * kHD + i
                                         : (i < (G + 1) * kHD ? (p.h + kvh) * kHD + i - G * kHD
                                                              : (p.h + p.hk + kvh) * kHD + i - (G + 1) * kHD);
        rr[t] = row_load<8, CONS>(part, sq, p.batch, b, row, v[t]);
      }
#pragma unroll
      for (uint32_t t = 0; t < RPT; t++) {
        const uint32_t i = ctid + t * nthr;
        const float x = row_finish<8>(rr[t], v[t], p.batch, sq.npad);
        // q rows go to the padded quarter layout, k and v rows after them
        if (i < G * kHD) qs[(i / kHD) * 4 * kQP + ((i % kHD) / 32) * kQP + i % 32] = x;
        else if (i < R) kvs[i - G * kHD] = x;
      }
    }
    cbar(nthr);
    // RoPE of the G q heads and k at the position: pair (d, d + 64)
    for (uint32_t i = ctid; i < NP; i += nthr) {
      const uint32_t hh = i / (kHD / 2), d = i % (kHD / 2);
      float c = rc, sn = rs;
      if (i != (uint32_t)ctid)
        c = __ldg(p.cos_t + (size_t)pos * (kHD / 2) + d), sn = __ldg(p.sin_t + (size_t)pos * (kHD / 2) + d);
      float *lo, *hi;
      if (hh < (uint32_t)G) {
        lo = qs + hh * 4 * kQP + (d / 32) * kQP + d % 32;
        hi = qs + hh * 4 * kQP + ((d + 64) / 32) * kQP + d % 32;
      } else {
        lo = kvs + d;
        hi = kvs + d + 64;
      }
      float o0, o1;
      rope_pair(*lo, *hi, c, sn, o0, o1);
      *lo = o0;
      *hi = o1;
    }
    cbar(nthr);
    const size_t kvbase = lofs + (size_t)b * p.seq_stride + (size_t)kvh * p.cap * kHD;
    if (p0 <= pos && pos < p1) {  // CTA-uniform: append k and v (fp16) at the position
      for (uint32_t i = ctid; i < kHD; i += nthr) {
        const uint32_t kv = i / (kHD / 2), d = 2 * (i % (kHD / 2));
        *reinterpret_cast<__half2 *>((kv ? p.vc : p.kc) + kvbase + (size_t)pos * kHD + d) =
            __floats2half2_rn(kvs[kv * kHD + d], kvs[kv * kHD + d + 1]);
      }
      cbar(nthr);  // the appended row is read back below (from L2, by other threads)
    }
    float m[G], l[G], o[G][4];
#pragma unroll
    for (int g = 0; g < G; g++) {
      m[g] = -INFINITY, l[g] = 0.f;
#pragma unroll
      for (int e = 0; e < 4; e++) o[g][e] = 0.f;
    }
    for (uint32_t c0 = p0 + 8 * warp; c0 < p1; c0 += 8 * CONS) {
      const uint32_t cnt = min(8u, p1 - c0);
      const bool mine = (uint32_t)i8 < cnt;
      // quarter r4 of position c0 + i8's K row (32 fp16 = 4 x 16 B)
      const uint4 *kr =
          reinterpret_cast<const uint4 *>(p.kc + kvbase + (size_t)(c0 + (mine ? i8 : 0)) * kHD + 32 * r4);
      uint4 kw[4];
#pragma unroll
      for (int t = 0; t < 4; t++) kw[t] = __ldcg(kr + t);
      // the V rows of the 8 positions, lane l on dims 4l..4l+3 (loaded now, used below)
      const uint2 *vr = reinterpret_cast<const uint2 *>(p.vc + kvbase + (size_t)c0 * kHD) + lane;
      uint2 vw[8];
#pragma unroll
      for (int t = 0; t < 8; t++) vw[t] = (uint32_t)t < cnt ? __ldcg(vr + (size_t)t * (kHD / 4)) : make_uint2(0u, 0u);
      float sc[G];
#pragma unroll
      for (int g = 0; g < G; g++) sc[g] = 0.f;
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const float2 k0 = __half22float2(*reinterpret_cast<const __half2 *>(&kw[t].x));
        const float2 k1 = __half22float2(*reinterpret_cast<const __half2 *>(&kw[t].y));
        const float2 k2 = __half22float2(*reinterpret_cast<const __half2 *>(&kw[t].z));
        const float2 k3 = __half22float2(*reinterpret_cast<const __half2 *>(&kw[t].w));
#pragma unroll
        for (int g = 0; g < G; g++) {
          const float *qq = qs + g * 4 * kQP + r4 * kQP + 8 * t;
          const float4 qa = *reinterpret_cast<const float4 *>(qq), qb = *reinterpret_cast<const float4 *>(qq + 4);
          float a = sc[g];
          a = fmaf(qa.x, k0.x, a), a = fmaf(qa.y, k0.y, a), a = fmaf(qa.z, k1.x, a), a = fmaf(qa.w, k1.y, a);
          a = fmaf(qb.x, k2.x, a), a = fmaf(qb.y, k2.y, a), a = fmaf(qb.z, k3.x, a), a = fmaf(qb.w, k3.y, a);
          sc[g] = a;
        }
      }
      // quarters added (lanes 4i..4i+3), then softmax over the 8 positions
      float ew[G];
#pragma unroll
      for (int g = 0; g < G; g++) {
        float sv = sc[g] + __shfl_xor_sync(0xffffffffu, sc[g], 1);
        sv += __shfl_xor_sync(0xffffffffu, sv, 2);
        sv = mine ? sv * p.inv_scale : -INFINITY;
        float mx = fmaxf(sv, __shfl_xor_sync(0xffffffffu, sv, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m[g], mx);
        const float alpha = m[g] == -INFINITY ? 0.0f : expf(m[g] - m_new);
        ew[g] = mine ? expf(sv - m_new) : 0.0f;
        float es = ew[g] + __shfl_xor_sync(0xffffffffu, ew[g], 4);
        es += __shfl_xor_sync(0xffffffffu, es, 8);
        es += __shfl_xor_sync(0xffffffffu, es, 16);
        l[g] = fmaf(l[g], alpha, es);
        m[g] = m_new;
#pragma unroll
        for (int e = 0; e < 4; e++) o[g][e] *= alpha;
      }
      // exp-weighted V: position t's weight broadcast from lane 4t
#pragma unroll
      for (int t = 0; t < 8; t++) {
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vw[t].x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vw[t].y));
#pragma unroll
        for (int g = 0; g < G; g++) {
          const float w = __shfl_sync(0xffffffffu, ew[g], 4 * t);
          o[g][0] = fmaf(w, v01.x, o[g][0]);
          o[g][1] = fmaf(w, v01.y, o[g][1]);
          o[g][2] = fmaf(w, v23.x, o[g][2]);
          o[g][3] = fmaf(w, v23.y, o[g][3]);
        }
      }
    }
    // the warps with positions merged in shared memory
    if ((uint32_t)warp < nw) {
#pragma unroll
      for (int g = 0; g < G; g++) {
        float *w = wpart + ((size_t)warp * G + g) * kAS;
        *reinterpret_cast<float4 *>(w + 4 * lane) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
        if (lane == 0) w[kHD] = m[g], w[kHD + 1] = l[g];
      }
    }
    cbar(nthr);
    for (uint32_t i = ctid; i < G * kHD; i += nthr) {
      const uint32_t g = i / kHD, dd = i % kHD;
      float M = -INFINITY;
      for (uint32_t w = 0; w < nw; w++) M = fmaxf(M, wpart[((size_t)w * G + g) * kAS + kHD]);
      float L = 0.f, od = 0.f;
      for (uint32_t w = 0; w < nw; w++) {
        const float *ws = wpart + ((size_t)w * G + g) * kAS;
        const float wt = expf(ws[kHD] - M);
        L = fmaf(ws[kHD + 1], wt, L);
        od = fmaf(ws[dd], wt, od);
      }
      float *dst = p.apart + (((size_t)b * p.h + h0 + g) * p.per_head + j) * kAS;
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
    finish_block(p, b, blk, emb_elem(p, r, blk * 32 + lane), __ldg(gamma + blk * 32 + lane), lane);
  }
}

// The lm head's operand: xqn (x * output_norm, quantised unscaled by the last
// reduce phase) with its block scales multiplied by the norm scale.
template <int CONS>
__device__ void final_norm(const KP &p, int c, int lane, int ctid, int nthr, float *scales) {
  for (uint32_t b = c; b < p.batch; b += CONS) {
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
    s_npos = (uint32_t)__ldcg(p.pos) + 1u;
  }
  if (threadIdx.x < 4) s_rng[threadIdx.x] = make_range(p.sh[threadIdx.x]);
  static_assert(sizeof(KP) % 4 == 0, "KP copied as words");
  for (uint32_t i = threadIdx.x; i < sizeof(KP) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t *>(&s_kp)[i] = reinterpret_cast<const uint32_t *>(&p)[i];
  __syncthreads();

  if (warp == 0) {
    // ---- producer: the four matrices of every layer, in order ----
    if (lane != 0) return;
    uint32_t fill = 0;
    bool ok = true;
    for (uint32_t l = 0; l < p.n_layer && ok; l++)
      for (int k = 0; k < 4 && ok; k++) ok = produce<T, NT, CONS>(p, k, p.layers[l].w[k], ring, full, empty, fill);
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
  float *scratch = reinterpret_cast<float *>(area + p.scratch_off);
  uint32_t seq = 0, epoch = 0;
  // row exchanges this rank completed in earlier steps (written by the
  // previous launch's last CTA)
  const uint64_t xbase = p.nranks > 1 ? *(volatile uint64_t *)(land_words(p.land[p.rank]) + 1) : 0;
  bool ok = true;
  fill_split_table(p, ctid, nthr);  // the first grid barrier's named barrier publishes it
  auto gemv = [&](int k, int xsrc, int pi) {
    consume<T, NT, CONS>(p, k, xsrc, p.part[pi], ring, full, empty, seq, area, scratch, scales, c, lane, ctid,
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
      case 1: attention<1, CONS>(s_kp, l, c, lane, ctid, nthr, reinterpret_cast<float *>(area)); break;
      case 2: attention<2, CONS>(s_kp, l, c, lane, ctid, nthr, reinterpret_cast<float *>(area)); break;
      case 4: attention<4, CONS>(s_kp, l, c, lane, ctid, nthr, reinterpret_cast<float *>(area)); break;
      default: attention<8, CONS>(s_kp, l, c, lane, ctid, nthr, reinterpret_cast<float *>(area)); break;
    }
    if (!sync()) break;
    if (NT > 1) {  // batches of 3+: merge once, then stage by copies
      merge_phase<CONS>(s_kp, c, lane, scratch);
      if (!sync()) break;
      gemv(M_O, X_COPY_A, 1);
    } else {
      gemv(M_O, X_ATT, 1);
    }
    if (!sync()) break;
    if (p.nranks > 1)
      ok = exchange_rows<CONS>(s_kp, s_kp.sh[M_O], L.ffn_norm, xbase + 2ull * l, c, lane, ctid, nthr, &sflag);
    else
      reduce_rows<CONS>(s_kp, s_kp.sh[M_O], L.ffn_norm, c, lane);
    if (!sync()) break;
    gemv(M_GU, X_NORMQ, 0);
    if (!sync()) break;
    if (NT > 1) {
      silu_phase<CONS>(s_kp, c, lane, scratch);
      if (!sync()) break;
      gemv(M_DOWN, X_COPY_H, 1);
    } else {
      gemv(M_DOWN, X_SILU, 1);
    }
    if (!sync()) break;
    if (p.nranks > 1)
      ok = exchange_rows<CONS>(s_kp, s_kp.sh[M_DOWN], g_next, xbase + 2ull * l + 1, c, lane, ctid, nthr, &sflag);
    else
      reduce_rows<CONS>(s_kp, s_kp.sh[M_DOWN], g_next, c, lane);
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
