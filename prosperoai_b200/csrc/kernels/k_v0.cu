// GEMM over weights in ProsperoAI's v0 grouped-scale integer formats,
// read in place, with m <= 8 activation rows per launch.
//
// The weight is the executor's GEMM B operand [k][n] (n contiguous,
// scheduler/scheduler.c:285-343), stored as signed int8 values or as signed
// nibbles packed two per byte over the flat index (even index in the low
// nibble), with f32 scales in one of two layouts:
//   kOpScales   s[(t / g) * n + j]: one scale per (k-group, column), the
//               registered w8/w4 GEMMs (cpu/reference/ref_ops.c:447-499);
//   kFlatScales s[(t * n + j) / g]: one scale per g consecutive flat
//               elements, the blob a v0 .pai container holds for a
//               quantized tensor ([values][scales], models/quantize.c:74-181,
//               models/container.c:176-229).
// c[r][j] = sum over t of a[r][t] * q(t, j) * scale(t, j), accumulated in
// fp32. The reference rounds each product as (a*q)*s (w8/w4) or a*(s*q)
// (dequantise, then pai_ref_gemm_f32); here the scale is applied with the
// same two roundings in a different order and the sum is split over k, so
// the result agrees with the reference to fp32 accumulation noise.
//
// HBM-bound (1 or 0.5 B of values per weight plus the scales), so the
// design is about moving bytes: a CTA owns a strip of 256 columns and a
// range of k; each lane holds 8 consecutive columns (8 B of int8 or 4 B of
// nibbles per row), its warp takes every 8th row of the range, and 4-8
// rows are loaded before any is used. Values become floats without the
// integer-conversion pipe: the biased byte or nibble is placed in the low
// mantissa bits of 2^23 by one byte permute and the bias subtracted in one
// exact fp32 add. Partial sums of the warps are added in warp order in
// shared memory; k-splits write partials that the last CTA of the strip to
// finish adds in split order, so results do not depend on timing.
//
// Shapes the vector path does not take (n not a multiple of 8, unaligned
// pointers, flat groups that are not a multiple of 8) run an element-wise
// kernel with the same split and reduction order.
#include <cuda.h>  // CUtensorMap and its enums (types only; the encoder comes from the runtime)
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace {

enum { kOpScales = 0, kFlatScales = 1 };

constexpr int kCols = 8;                 // columns per lane
constexpr int kWarps = 8;                // warps per CTA; warp w takes rows t0 + w + 8i
constexpr int kThreads = kWarps * 32;    // 256
constexpr int kStrip = 32 * kCols;       // 256 columns per CTA
constexpr int kMaxRows = 8;              // activation rows per launch
constexpr uint64_t kMaxPer = 512;        // rows of k per split (activation staging)
constexpr uint64_t kMaxScaleGroups = 16; // k-groups of scales one split stages (kOpScales)
constexpr int kU8 = 8, kU4 = 16;         // rows per lane and batch: 64 B of int8, 64 B of nibbles
constexpr int kCtasPerSm = 2;            // grid target: about this many CTAs per SM
constexpr int kSplitLoads = 8;           // partials loaded at once by the split reduction

struct V0Args {
  uint64_t m, n, k;   // m <= kMaxRows
  const float *a;     // [m][k]
  const uint8_t *w;   // values
  const uint8_t *s;   // f32 scales (4-byte aligned on the vector path)
  uint64_t g;         // group size: rows (kOpScales) or flat elements (kFlatScales)
  float *c;           // [m][n]
  uint64_t per;       // rows of k per split, a multiple of kWarps
  float *part;        // [split][m][n] when gridDim.y > 1
  uint32_t *cnt;      // [strip] arrival counters, left at zero
  uint64_t wait_ns;   // the context's limit on every wait (TMA ring)
};

// Signed value of flat element f (models/quantize.c:165-172).
template <int BITS>
__device__ __forceinline__ int32_t v0_value(const uint8_t *w, uint64_t f) {
  if (BITS == 8) return (int8_t)w[f];
  const uint32_t b = w[f >> 1];
  const int32_t nib = (f & 1) ? (b >> 4) & 0xF : b & 0xF;
  return (nib ^ 8) - 8;
}

__device__ __forceinline__ float ld_scale_any(const uint8_t *s, uint64_t i) {
  const uint8_t *p = s + 4 * i;
  return __uint_as_float((uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24));
}

// Float of the biased unsigned byte `sel` of word x: 2^23 + byte, exact.
__device__ __forceinline__ float biased_byte(uint32_t x, uint32_t sel) {
  return __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540u | sel));
}

// After every thread has written its columns' results (to c when the grid
// has one split, else to its split's partials): the last CTA of the strip
// adds the splits in order.
__device__ __forceinline__ void finish_strip(const V0Args &p) {
  if (gridDim.y == 1) return;
  __shared__ uint32_t ticket;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) ticket = atomicAdd(&p.cnt[blockIdx.x], 1u);
  __syncthreads();
  if (ticket != gridDim.y - 1) return;
  __threadfence();
  const uint64_t j = (uint64_t)blockIdx.x * kStrip + threadIdx.x;
  if (j < p.n) {
    const uint64_t ys = p.m * p.n;  // stride between splits
    for (uint64_t r = 0; r < p.m; r++) {
      const float *src = p.part + r * p.n + j;
      float v = 0.0f;
      uint32_t y = 0;
      for (; y + kSplitLoads <= gridDim.y; y += kSplitLoads) {  // loads in flight together, added in order
        float b[kSplitLoads];
#pragma unroll
        for (int u = 0; u < kSplitLoads; u++) b[u] = __ldcg(src + (uint64_t)(y + u) * ys);
#pragma unroll
        for (int u = 0; u < kSplitLoads; u++) v += b[u];
      }
      for (; y < gridDim.y; y++) v += __ldcg(src + (uint64_t)y * ys);
      p.c[r * p.n + j] = v;
    }
  }
  if (threadIdx.x == 0) p.cnt[blockIdx.x] = 0;
}

__device__ __forceinline__ void put_result(const V0Args &p, uint64_t r, uint64_t j, float v) {
  if (gridDim.y == 1)
    p.c[r * p.n + j] = v;
  else
    p.part[((uint64_t)blockIdx.y * p.m + r) * p.n + j] = v;
}

// Vector path: n % 8 == 0, values 8-byte (int8) or 4-byte (nibbles)
// aligned, and g a multiple of 8 (kFlatScales: a lane's 8 columns of a row
// share one scale) or at least 8 (kOpScales: a warp's row step of 8 crosses
// at most one group boundary), scales 16-byte (kOpScales) or 4-byte
// aligned. No scale load waits on the critical path: kOpScales stages the
// split's (group, column) scales in shared memory with the activations;
// kFlatScales loads each row's scale together with the row's weights.
template <int BITS, int LAYOUT, int MB>
__global__ void __launch_bounds__(kThreads) k_gemm_v0(V0Args p) {
  extern __shared__ __align__(16) float dyn[];  // [MB][per] activations, then [ngr][kStrip] scales (kOpScales)
  __shared__ __align__(16) float red[kWarps][kStrip];  // written as float4
  constexpr int U = BITS == 8 ? kU8 : kU4;
  using Raw = typename std::conditional<BITS == 8, uint2, uint32_t>::type;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t c0 = (uint64_t)blockIdx.x * kStrip, j0 = c0 + lane * kCols;
  const uint64_t t0 = (uint64_t)blockIdx.y * p.per, t1 = min(p.k, t0 + p.per);
  const uint64_t tf = t0 + warp;
  const bool live = j0 < p.n;
  const float *sf = reinterpret_cast<const float *>(p.s);
  float *sa = dyn;
  float *ss = dyn + MB * p.per;

  // kFlatScales cursor: (f / g, f % g) of this lane's first column f of the
  // next row to load; rows advance by kWarps
  uint64_t qg = 0, rg = 0, dq = 0, dr = 0;
  if (LAYOUT == kFlatScales) {
    const uint64_t f = tf * p.n + j0, step = (uint64_t)kWarps * p.n;
    qg = f / p.g;
    rg = f - qg * p.g;
    dq = step / p.g;
    dr = step - dq * p.g;
  }
  // U rows of this lane's 8 columns from row t (rows t, t+8, ...), and for
  // kFlatScales each row's scale
  auto load_batch = [&](Raw *raw, float *rs, uint64_t t) {
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint64_t tu = t + (uint64_t)kWarps * u;
      const bool in = tu < t1;
      raw[u] = (live && in) ? __ldcs(reinterpret_cast<const Raw *>(
                                  p.w + (BITS == 8 ? tu * p.n + j0 : (tu * p.n + j0) >> 1)))
                            : Raw{};  // decodes to zeros
      if (LAYOUT == kFlatScales) {
        rs[u] = (live && in) ? __ldg(sf + qg) : 0.0f;
        if (in) {
          rg += dr;
          qg += dq;
          if (rg >= p.g) {
            rg -= p.g;
            qg++;
          }
        }
      }
    }
  };
  pdl_wait();  // a no-op unless launched as a programmatic dependent
  // the first weight batch is in flight while activations (and scales) are staged
  Raw nxt[U];
  float nsc[U];
  load_batch(nxt, nsc, tf);
  for (uint32_t i = threadIdx.x; i < MB * p.per; i += kThreads) {
    const uint32_t r = i / (uint32_t)p.per, tt = i - r * (uint32_t)p.per;
    sa[i] = (r < p.m && t0 + tt < t1) ? __ldg(p.a + r * p.k + t0 + tt) : 0.0f;
  }
  uint64_t gnext = 0;
  uint32_t gl = 0;
  if (LAYOUT == kOpScales) {
    const uint64_t gfirst = t0 / p.g, ngr = (t1 - 1) / p.g - gfirst + 1, ngroups = (p.k + p.g - 1) / p.g;
    for (uint32_t i = threadIdx.x; i < ngr * kStrip; i += kThreads) {
      const uint64_t gi = gfirst + i / kStrip, col = c0 + i % kStrip;
      ss[i] = (col < p.n && gi < ngroups) ? __ldg(sf + gi * p.n + col) : 0.0f;
    }
    const uint64_t gi = tf / p.g;
    gl = (uint32_t)(gi - gfirst);
    gnext = (gi + 1) * p.g;
  }
  __syncthreads();

  float acc[MB][kCols];
#pragma unroll
  for (int r = 0; r < MB; r++)
#pragma unroll
    for (int e = 0; e < kCols; e++) acc[r][e] = 0.0f;
  float sc[kCols];
  if (LAYOUT == kOpScales) {
    const float4 s0 = *reinterpret_cast<const float4 *>(ss + gl * kStrip + lane * kCols);
    const float4 s1 = *reinterpret_cast<const float4 *>(ss + gl * kStrip + lane * kCols + 4);
    sc[0] = s0.x, sc[1] = s0.y, sc[2] = s0.z, sc[3] = s0.w;
    sc[4] = s1.x, sc[5] = s1.y, sc[6] = s1.z, sc[7] = s1.w;
  }

  for (uint64_t t = tf; t < t1; t += (uint64_t)kWarps * U) {
    Raw raw[U];
    float rsc[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      raw[u] = nxt[u];
      rsc[u] = nsc[u];
    }
    if (t + (uint64_t)kWarps * U < t1) load_batch(nxt, nsc, t + (uint64_t)kWarps * U);  // next batch in flight
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint64_t tu = t + (uint64_t)kWarps * u;
      if (tu >= t1) break;
      float v[kCols];
      if constexpr (BITS == 8) {
        const uint32_t x0 = raw[u].x ^ 0x80808080u, x1 = raw[u].y ^ 0x80808080u;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          v[e] = biased_byte(x0, e) - 8388736.0f;  // 2^23 + 128
          v[e + 4] = biased_byte(x1, e) - 8388736.0f;
        }
      } else {
        const uint32_t x = raw[u] ^ 0x88888888u;
        const uint32_t lo = x & 0x0F0F0F0Fu, hi = (x >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          v[2 * e] = biased_byte(lo, e) - 8388616.0f;  // 2^23 + 8
          v[2 * e + 1] = biased_byte(hi, e) - 8388616.0f;
        }
      }
      const uint32_t tl = (uint32_t)(tu - t0);
      if constexpr (LAYOUT == kOpScales) {
        if (tu >= gnext) {  // uniform across the warp; g >= 8, so one group at most
          gl++;
          gnext += p.g;
          const float4 s0 = *reinterpret_cast<const float4 *>(ss + gl * kStrip + lane * kCols);
          const float4 s1 = *reinterpret_cast<const float4 *>(ss + gl * kStrip + lane * kCols + 4);
          sc[0] = s0.x, sc[1] = s0.y, sc[2] = s0.z, sc[3] = s0.w;
          sc[4] = s1.x, sc[5] = s1.y, sc[6] = s1.z, sc[7] = s1.w;
        }
#pragma unroll
        for (int e = 0; e < kCols; e++) {
          const float we = v[e] * sc[e];
#pragma unroll
          for (int r = 0; r < MB; r++) acc[r][e] = fmaf(sa[r * p.per + tl], we, acc[r][e]);
        }
      } else {
#pragma unroll
        for (int r = 0; r < MB; r++) {
          const float as = sa[r * p.per + tl] * rsc[u];
#pragma unroll
          for (int e = 0; e < kCols; e++) acc[r][e] = fmaf(as, v[e], acc[r][e]);
        }
      }
    }
  }

  // warps' partial sums, added in warp order
#pragma unroll
  for (int r = 0; r < MB; r++) {
    if (r >= (int)p.m) break;
    float4 *dst = reinterpret_cast<float4 *>(&red[warp][lane * kCols]);
    dst[0] = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    dst[1] = make_float4(acc[r][4], acc[r][5], acc[r][6], acc[r][7]);
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; w++) s += red[w][threadIdx.x];
    const uint64_t j = c0 + threadIdx.x;
    if (j < p.n) put_result(p, r, j, s);
    __syncthreads();
  }
  finish_strip(p);
}

// TMA path (the default where its alignment rules hold): the CTA's
// weights arrive by 2-D tensor copies, one box of 32 rows x one 256-byte
// (int8) or 128-byte (nibble) column strip per ring stage, issued by a
// producer warp into a 6-stage shared-memory ring (mbarrier completion,
// bounded waits), so the consumer warps never wait on their own loads.
// Consumers: warp w takes rows w, w+8, w+16, w+24 of each stage; lane =
// 8 columns, read from shared memory (8 or 4 bytes, conflict-free); the
// arithmetic is the vector path's. The tensor map's inner coordinate is
// the strip's byte offset, a multiple of 128.
constexpr int kTmaRows = 32;    // rows per box (stage)
constexpr int kTmaStages = 6;
constexpr int kTmaThreads = kThreads + 32;  // 8 consumer warps + 1 producer warp

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

template <int BITS, int LAYOUT, int MB>
__global__ void __launch_bounds__(kTmaThreads) k_gemm_v0_tma(V0Args p, uint32_t *err,
                                                             const __grid_constant__ CUtensorMap map) {
  constexpr uint32_t SB = BITS == 8 ? 256 : 128;  // bytes of a row strip
  constexpr uint32_t STAGE = SB * kTmaRows;
  using Raw = typename std::conditional<BITS == 8, uint2, uint32_t>::type;
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t *ring = dsm;                                                   // [kTmaStages][STAGE]
  float *sa = reinterpret_cast<float *>(dsm + kTmaStages * STAGE);       // [MB][per]
  float *ss = sa + MB * p.per;                                           // [ngr][kStrip] (kOpScales)
  __shared__ __align__(16) float red[kWarps][kStrip];
  __shared__ __align__(8) uint64_t full[kTmaStages], empty[kTmaStages];
  __shared__ int failed;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t c0 = (uint64_t)blockIdx.x * kStrip, j0 = c0 + lane * kCols;
  const uint64_t t0 = (uint64_t)blockIdx.y * p.per, t1 = min(p.k, t0 + p.per);
  const uint32_t nst = (uint32_t)((t1 - t0 + kTmaRows - 1) / kTmaRows);
  const float *sf = reinterpret_cast<const float *>(p.s);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTmaStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarps);
    }
    fence_mbar_init();
    failed = 0;
  }
  __syncthreads();
  pdl_wait();  // a no-op unless launched as a programmatic dependent
  uint32_t issued = 0;
  const bool producer = warp == kWarps;
  auto issue = [&](uint32_t st) -> bool {  // stage st into slot st % kTmaStages
    const uint32_t slot = st % kTmaStages;
    if (st >= (uint32_t)kTmaStages && !mbar_wait_spin(&empty[slot], ((st / kTmaStages) - 1) & 1u, p.wait_ns))
      return false;
    mbar_expect_tx(&full[slot], STAGE);
    tma_load_2d(ring + (size_t)slot * STAGE, &map, (int32_t)(blockIdx.x * SB), (int32_t)(t0 + (uint64_t)st * kTmaRows),
                &full[slot]);
    return true;
  };
  if (producer && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map)) : "memory");
    for (; issued < nst && issued < (uint32_t)kTmaStages; issued++) issue(issued);
  }
  // activations (and per-(group, column) scales) while the first boxes land
  uint64_t gnext = 0;
  uint32_t gl = 0;
  if (!producer) {
    for (uint32_t i = threadIdx.x; i < MB * p.per; i += kThreads) {
      const uint32_t r = i / (uint32_t)p.per, tt = i - r * (uint32_t)p.per;
      sa[i] = (r < p.m && t0 + tt < t1) ? __ldg(p.a + r * p.k + t0 + tt) : 0.0f;
    }
    if (LAYOUT == kOpScales) {
      const uint64_t gfirst = t0 / p.g, ngr = (t1 - 1) / p.g - gfirst + 1, ngroups = (p.k + p.g - 1) / p.g;
      for (uint32_t i = threadIdx.x; i < ngr * kStrip; i += kThreads) {
        const uint64_t gi = gfirst + i / kStrip, col = c0 + i % kStrip;
        ss[i] = (col < p.n && gi < ngroups) ? __ldg(sf + gi * p.n + col) : 0.0f;
      }
      const uint64_t gi = (t0 + warp) / p.g;
      gl = (uint32_t)(gi - gfirst);
      gnext = (gi + 1) * p.g;
    }
  }
  __syncthreads();

  if (producer) {
    if (lane == 0) {
      bool ok = true;
      for (; ok && issued < nst; issued++) ok = issue(issued);
      if (!ok) {
        // a wait ran out: raise the error and let the boxes in flight land (bounded)
        atomicExch(err, 1u);
        failed = 1;
        for (uint32_t f = issued > (uint32_t)kTmaStages ? issued - kTmaStages : 0; f < issued; f++)
          mbar_wait(&full[f % kTmaStages], (f / kTmaStages) & 1u, p.wait_ns);
      }
    }
  } else {
    const bool live = j0 < p.n;
    float acc[MB][kCols];
#pragma unroll
    for (int r = 0; r < MB; r++)
#pragma unroll
      for (int e = 0; e < kCols; e++) acc[r][e] = 0.0f;
    float sc[kCols];
    if (LAYOUT == kOpScales) {
      const float4 s0 = *reinterpret_cast<const float4 *>(ss + gl * kStrip + lane * kCols);
      const float4 s1 = *reinterpret_cast<const float4 *>(ss + gl * kStrip + lane * kCols + 4);
      sc[0] = s0.x, sc[1] = s0.y, sc[2] = s0.z, sc[3] = s0.w;
      sc[4] = s1.x, sc[5] = s1.y, sc[6] = s1.z, sc[7] = s1.w;
    }
    // kFlatScales: cursor (f / g, f % g) of this lane's first column of the
    // next row whose scale is loaded (rows advance by kWarps); the scales of
    // a stage's rows are loaded one stage ahead
    constexpr int RPW = kTmaRows / kWarps;  // rows per warp per stage
    uint64_t qg = 0, rg = 0, dq = 0, dr = 0;
    float rs_next[RPW];
    auto load_scales = [&](uint32_t st) {
#pragma unroll
      for (int u = 0; u < RPW; u++) {
        const uint64_t t = t0 + (uint64_t)st * kTmaRows + warp + kWarps * u;
        const bool in = t < t1;
        rs_next[u] = (live && in) ? __ldg(sf + qg) : 0.0f;
        if (in) {
          rg += dr;
          qg += dq;
          if (rg >= p.g) {
            rg -= p.g;
            qg++;
          }
        }
      }
    };
    if (LAYOUT == kFlatScales) {
      const uint64_t f = (t0 + warp) * p.n + j0, step = (uint64_t)kWarps * p.n;
      qg = f / p.g;
      rg = f - qg * p.g;
      dq = step / p.g;
      dr = step - dq * p.g;
      load_scales(0);
    }
    for (uint32_t st = 0; st < nst; st++) {
      const uint32_t slot = st % kTmaStages;
      if (!mbar_wait(&full[slot], (st / kTmaStages) & 1u, p.wait_ns)) {
        if (lane == 0) atomicExch(err, 1u);
        failed = 1;
        break;
      }
      float rs[RPW];
      if (LAYOUT == kFlatScales) {
#pragma unroll
        for (int u = 0; u < RPW; u++) rs[u] = rs_next[u];
        if (st + 1 < nst) load_scales(st + 1);
      }
      const uint8_t *stage = ring + (size_t)slot * STAGE;
#pragma unroll
      for (int u = 0; u < RPW; u++) {
        const uint32_t row = warp + kWarps * u;
        const uint64_t tu = t0 + (uint64_t)st * kTmaRows + row;
        if (tu >= t1) break;
        const Raw raw = *reinterpret_cast<const Raw *>(stage + (size_t)row * SB + lane * sizeof(Raw));
        float v[kCols];
        if constexpr (BITS == 8) {
          const uint32_t x0 = raw.x ^ 0x80808080u, x1 = raw.y ^ 0x80808080u;
#pragma unroll
          for (int e = 0; e < 4; e++) {
            v[e] = biased_byte(x0, e) - 8388736.0f;  // 2^23 + 128
            v[e + 4] = biased_byte(x1, e) - 8388736.0f;
          }
        } else {
          const uint32_t x = raw ^ 0x88888888u;
          const uint32_t lo = x & 0x0F0F0F0Fu, hi = (x >> 4) & 0x0F0F0F0Fu;
#pragma unroll
          for (int e = 0; e < 4; e++) {
            v[2 * e] = biased_byte(lo, e) - 8388616.0f;  // 2^23 + 8
            v[2 * e + 1] = biased_byte(hi, e) - 8388616.0f;
          }
        }
        const uint32_t tl = (uint32_t)(tu - t0);
        if constexpr (LAYOUT == kOpScales) {
          if (tu >= gnext) {  // uniform across the warp; g >= 8, so one group at most
            gl++;
            gnext += p.g;
            const float4 s0 = *reinterpret_cast<const float4 *>(ss + gl * kStrip + lane * kCols);
            const float4 s1 = *reinterpret_cast<const float4 *>(ss + gl * kStrip + lane * kCols + 4);
            sc[0] = s0.x, sc[1] = s0.y, sc[2] = s0.z, sc[3] = s0.w;
            sc[4] = s1.x, sc[5] = s1.y, sc[6] = s1.z, sc[7] = s1.w;
          }
#pragma unroll
          for (int e = 0; e < kCols; e++) {
            const float we = v[e] * sc[e];
#pragma unroll
            for (int r = 0; r < MB; r++) acc[r][e] = fmaf(sa[r * p.per + tl], we, acc[r][e]);
          }
        } else {
#pragma unroll
          for (int r = 0; r < MB; r++) {
            const float as = sa[r * p.per + tl] * rs[u];
#pragma unroll
            for (int e = 0; e < kCols; e++) acc[r][e] = fmaf(as, v[e], acc[r][e]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    // reduction of the warps' partial sums, one activation row at a time
#pragma unroll
    for (int r = 0; r < MB; r++) {
      if (r >= (int)p.m) break;
      float4 *dst = reinterpret_cast<float4 *>(&red[warp][lane * kCols]);
      dst[0] = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
      dst[1] = make_float4(acc[r][4], acc[r][5], acc[r][6], acc[r][7]);
      asm volatile("bar.sync 1, %0;" ::"r"(kThreads) : "memory");  // consumer warps only
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; w++) s += red[w][threadIdx.x];
      const uint64_t j = c0 + threadIdx.x;
      if (j < p.n) put_result(p, r, j, s);
      asm volatile("bar.sync 1, %0;" ::"r"(kThreads) : "memory");
    }
  }
  __syncthreads();
  if (failed) return;
  // k-splits: the strip's last CTA adds the partials in split order
  if (gridDim.y == 1) return;
  __shared__ uint32_t ticket;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) ticket = atomicAdd(&p.cnt[blockIdx.x], 1u);
  __syncthreads();
  if (ticket != gridDim.y - 1) return;
  __threadfence();
  if (threadIdx.x < kStrip) {
    const uint64_t j = c0 + threadIdx.x;
    if (j < p.n) {
      const uint64_t ys = p.m * p.n;
      for (uint64_t r = 0; r < p.m; r++) {
        const float *src = p.part + r * p.n + j;
        float v = 0.0f;
        uint32_t y = 0;
        for (; y + kSplitLoads <= gridDim.y; y += kSplitLoads) {
          float b[kSplitLoads];
#pragma unroll
          for (int u = 0; u < kSplitLoads; u++) b[u] = __ldcg(src + (uint64_t)(y + u) * ys);
#pragma unroll
          for (int u = 0; u < kSplitLoads; u++) v += b[u];
        }
        for (; y < gridDim.y; y++) v += __ldcg(src + (uint64_t)y * ys);
        p.c[r * p.n + j] = v;
      }
    }
  }
  if (threadIdx.x == 0) p.cnt[blockIdx.x] = 0;
}

// Element-wise path for every other shape: thread per column, all rows of
// the split in order.
template <int BITS, int LAYOUT>
__global__ void __launch_bounds__(kThreads) k_gemm_v0_any(V0Args p) {
  const uint64_t j = (uint64_t)blockIdx.x * kStrip + threadIdx.x;
  const uint64_t t0 = (uint64_t)blockIdx.y * p.per, t1 = min(p.k, t0 + p.per);
  pdl_wait();
  float acc[kMaxRows];
#pragma unroll
  for (int r = 0; r < kMaxRows; r++) acc[r] = 0.0f;
  if (j < p.n) {
    for (uint64_t t = t0; t < t1; t++) {
      const uint64_t f = t * p.n + j;
      const float sv = ld_scale_any(p.s, LAYOUT == kOpScales ? (t / p.g) * p.n + j : f / p.g);
      const float we = (float)v0_value<BITS>(p.w, f) * sv;
#pragma unroll
      for (int r = 0; r < kMaxRows; r++)
        if (r < (int)p.m) acc[r] = fmaf(__ldg(p.a + r * p.k + t), we, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < kMaxRows; r++)
      if (r < (int)p.m) put_result(p, r, j, acc[r]);
  }
  finish_strip(p);
}

// Groups of k one split of `per` rows can touch (its first row need not
// start a group).
inline uint64_t split_groups(uint64_t per, uint64_t g) { return (per + g - 1) / g + 1; }

template <int BITS, int LAYOUT>
cudaError_t launch_vec(pai_b200_ctx_t *ctx, dim3 grid, uint32_t mb, const V0Args &a) {
  size_t smem = (size_t)mb * a.per * sizeof(float);
  if (LAYOUT == kOpScales) smem += split_groups(a.per, a.g) * kStrip * sizeof(float);
  switch (mb) {
    case 1: return b200_launch(ctx, k_gemm_v0<BITS, LAYOUT, 1>, grid, dim3(kThreads), smem, a);
    case 2: return b200_launch(ctx, k_gemm_v0<BITS, LAYOUT, 2>, grid, dim3(kThreads), smem, a);
    case 4: return b200_launch(ctx, k_gemm_v0<BITS, LAYOUT, 4>, grid, dim3(kThreads), smem, a);
    default: return b200_launch(ctx, k_gemm_v0<BITS, LAYOUT, 8>, grid, dim3(kThreads), smem, a);
  }
}

template <int BITS, int LAYOUT, int MB>
cudaError_t launch_tma_mb(pai_b200_ctx_t *ctx, dim3 grid, const V0Args &a, const CUtensorMap &map) {
  constexpr uint32_t SB = BITS == 8 ? 256 : 128;
  size_t smem = (size_t)kTmaStages * SB * kTmaRows + (size_t)MB * a.per * sizeof(float);
  if (LAYOUT == kOpScales) smem += split_groups(a.per, a.g) * kStrip * sizeof(float);
  // dynamic shared memory this instantiation is opted in to, per device (the attribute is per device)
  static SmemOptIn opt;
  const cudaError_t e = opt.ensure(b200_ctx_device(ctx), smem, [](size_t b) {
    return cudaFuncSetAttribute(k_gemm_v0_tma<BITS, LAYOUT, MB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)b);
  });
  if (e != cudaSuccess) return e;
  return b200_launch(ctx, k_gemm_v0_tma<BITS, LAYOUT, MB>, grid, dim3(kTmaThreads), smem, a, b200_ctx_errflag(ctx),
                     map);
}

template <int BITS, int LAYOUT>
cudaError_t launch_tma(pai_b200_ctx_t *ctx, dim3 grid, uint32_t mb, const V0Args &a, const CUtensorMap &map) {
  switch (mb) {
    case 1: return launch_tma_mb<BITS, LAYOUT, 1>(ctx, grid, a, map);
    case 2: return launch_tma_mb<BITS, LAYOUT, 2>(ctx, grid, a, map);
    case 4: return launch_tma_mb<BITS, LAYOUT, 4>(ctx, grid, a, map);
    default: return launch_tma_mb<BITS, LAYOUT, 8>(ctx, grid, a, map);
  }
}

pai_status_t gemm_v0(pai_b200_ctx_t *ctx, uint32_t bits, int layout, uint64_t m, uint64_t n, uint64_t k,
                     const float *a, const void *w, const void *s, uint64_t g, float *c, const char *what) {
  const uintptr_t wa = (uintptr_t)w, sa = (uintptr_t)s;
  const bool vec = n % kCols == 0 && wa % (bits == 8 ? 8 : 4) == 0 &&
                   (layout == kOpScales ? (sa % 16 == 0 && g >= kCols) : (sa % 4 == 0 && g % kCols == 0));
  // TMA path: rows of whole 16-byte multiples (the tensor map's stride rule), 16-byte aligned
  // values, and the vector path's scale rules
  const uint64_t row_bytes = bits == 8 ? n : n / 2;
  PFN_cuTensorMapEncodeTiled_v12000 encode =
      vec ? reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(b200_tensor_map_encoder()) : nullptr;
  const bool tma = encode && (bits == 8 ? n % 16 == 0 : n % 32 == 0) && wa % 16 == 0 && k <= 0x7FFFFFFFull &&
                   row_bytes >= (bits == 8 ? 256u : 128u) && row_bytes < (1ull << 40);
  const uint64_t strips = (n + kStrip - 1) / kStrip;
  // about kCtasPerSm CTAs per SM, at least 64 rows per split, at most
  // kMaxPer (and, with staged scales, at most kMaxScaleGroups groups)
  const uint64_t max_per = vec && layout == kOpScales
                               ? std::min<uint64_t>(kMaxPer, (kMaxScaleGroups - 2) * g / kWarps * kWarps)
                               : kMaxPer;
  uint64_t splits = std::max<uint64_t>(1, (kCtasPerSm * 148 + strips - 1) / strips);
  splits = std::min<uint64_t>(splits, std::max<uint64_t>(1, k / 64));
  splits = std::max<uint64_t>(splits, (k + max_per - 1) / max_per);
  uint64_t per = (k + splits - 1) / splits;
  const uint64_t quantum = tma ? kTmaRows : kWarps;  // whole boxes per split on the TMA path
  per = (per + quantum - 1) / quantum * quantum;
  splits = (k + per - 1) / per;
  CUtensorMap map;
  if (tma) {
    const cuuint64_t dims[2] = {row_bytes, k};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {bits == 8 ? 256u : 128u, (cuuint32_t)kTmaRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return b200_fail(PAI_ERR_INTERNAL, "%s: cuTensorMapEncodeTiled error %d", what, (int)r);
  }
  if (strips > 0xFFFFFFFFull || splits > 65535)
    return b200_fail(PAI_ERR_INVALID_ARG, "%s: n %llu x k %llu is beyond the launch grid", what,
                     (unsigned long long)n, (unsigned long long)k);
  for (uint64_t r0 = 0; r0 < m; r0 += kMaxRows) {
    const uint64_t mm = std::min<uint64_t>(kMaxRows, m - r0);
    V0Args p{};
    p.m = mm;
    p.n = n;
    p.k = k;
    p.a = a + r0 * k;
    p.w = static_cast<const uint8_t *>(w);
    p.s = static_cast<const uint8_t *>(s);
    p.g = g;
    p.c = c + r0 * n;
    p.per = per;
    p.wait_ns = b200_ctx_wait_ns(ctx);
    if (splits > 1) {
      pai_status_t st = b200_ctx_scratch(ctx, splits * mm * n, (uint32_t)strips, &p.part, &p.cnt);
      if (st) return st;
    }
    const dim3 grid((uint32_t)strips, (uint32_t)splits);
    cudaError_t e;
    if (tma) {
      const uint32_t mb = mm == 1 ? 1 : mm == 2 ? 2 : mm <= 4 ? 4 : 8;
      if (bits == 8)
        e = layout == kOpScales ? launch_tma<8, kOpScales>(ctx, grid, mb, p, map)
                                : launch_tma<8, kFlatScales>(ctx, grid, mb, p, map);
      else
        e = layout == kOpScales ? launch_tma<4, kOpScales>(ctx, grid, mb, p, map)
                                : launch_tma<4, kFlatScales>(ctx, grid, mb, p, map);
    } else if (vec) {
      const uint32_t mb = mm == 1 ? 1 : mm == 2 ? 2 : mm <= 4 ? 4 : 8;
      if (bits == 8)
        e = layout == kOpScales ? launch_vec<8, kOpScales>(ctx, grid, mb, p) : launch_vec<8, kFlatScales>(ctx, grid, mb, p);
      else
        e = layout == kOpScales ? launch_vec<4, kOpScales>(ctx, grid, mb, p) : launch_vec<4, kFlatScales>(ctx, grid, mb, p);
    } else {
      if (bits == 8)
        e = layout == kOpScales ? b200_launch(ctx, k_gemm_v0_any<8, kOpScales>, grid, dim3(kThreads), 0, p)
                                : b200_launch(ctx, k_gemm_v0_any<8, kFlatScales>, grid, dim3(kThreads), 0, p);
      else
        e = layout == kOpScales ? b200_launch(ctx, k_gemm_v0_any<4, kOpScales>, grid, dim3(kThreads), 0, p)
                                : b200_launch(ctx, k_gemm_v0_any<4, kFlatScales>, grid, dim3(kThreads), 0, p);
    }
    if (e != cudaSuccess) return b200_cuda(e, what);
    pai_status_t st = b200_launched(ctx, 1, tma ? "k_gemm_v0_tma" : vec ? "k_gemm_v0" : "k_gemm_v0_any");
    if (st) return st;
  }
  return PAI_OK;
}

pai_status_t gemm_wq(pai_b200_ctx_t *ctx, uint32_t bits, uint64_t m, uint64_t n, uint64_t k, const float *a,
                     const int8_t *w_q, const float *b_scales, uint64_t group_size, float *c, const char *what) {
  // argument rules of ref_ops.c:450-455 / 474-479
  if (!ctx || m == 0 || n == 0 || k == 0 || !a || !w_q || !b_scales || !c)
    return b200_fail(PAI_ERR_INVALID_ARG, "%s: invalid arguments", what);
  if (group_size == 0 || group_size > k) group_size = k;
  return gemm_v0(ctx, bits, kOpScales, m, n, k, a, w_q, b_scales, group_size, c, what);
}

}  // namespace

extern "C" pai_status_t pai_b200_gemm_w8_f32(pai_b200_ctx_t *ctx, uint64_t m, uint64_t n, uint64_t k, const float *a,
                                             const int8_t *w_q, const float *b_scales, uint64_t group_size,
                                             float *c) {
  return gemm_wq(ctx, 8, m, n, k, a, w_q, b_scales, group_size, c, "gemm_w8_f32");
}

extern "C" pai_status_t pai_b200_gemm_w4_f32(pai_b200_ctx_t *ctx, uint64_t m, uint64_t n, uint64_t k, const float *a,
                                             const int8_t *w_q4, const float *b_scales, uint64_t group_size,
                                             float *c) {
  return gemm_wq(ctx, 4, m, n, k, a, w_q4, b_scales, group_size, c, "gemm_w4_f32");
}

extern "C" uint64_t pai_b200_v0_blob_bytes(uint32_t bit_width, uint32_t group_size, uint64_t numel) {
  // pai_quant_weights_bytes (models/quantize.c:53-72)
  if ((bit_width != 8 && bit_width != 4) || numel == 0) return 0;
  const uint64_t gs = group_size ? group_size : numel;
  return (bit_width == 8 ? numel : (numel + 1) / 2) + (numel + gs - 1) / gs * sizeof(float);
}

extern "C" pai_status_t pai_b200_gemm_v0_f32(pai_b200_ctx_t *ctx, uint32_t bit_width, uint32_t group_size, uint64_t m,
                                             uint64_t n, uint64_t k, const float *a, const void *blob, float *c) {
  if (!ctx || m == 0 || n == 0 || k == 0 || !a || !blob || !c)
    return b200_fail(PAI_ERR_INVALID_ARG, "gemm_v0: invalid arguments");
  // v0 executes signed q8/q4 only (models/quantize.c:14-19, models/model.c:264-267)
  if (bit_width != 8 && bit_width != 4)
    return b200_fail(PAI_ERR_UNSUPPORTED, "gemm_v0: bit width %u (v0 runs 8 and 4)", bit_width);
  const uint64_t numel = n * k, gs = group_size ? group_size : numel;
  const uint64_t vbytes = bit_width == 8 ? numel : (numel + 1) / 2;
  return gemm_v0(ctx, bit_width, kFlatScales, m, n, k, a, blob, static_cast<const uint8_t *>(blob) + vbytes, gs, c,
                 "gemm_v0");
}
