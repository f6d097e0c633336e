// Prompt prefill: the kernels that run between the GEMMs when a session
// processes many prompt positions in one pass per layer (rows = sequences x
// positions) instead of one decode step per position.
//
//   k_prefill_rope_append  RoPE of every row's q heads (in place) and k
//                          heads at the row's position, k and v appended to
//                          the fp16 cache: the same operations and rounding
//                          as the decode step (k_attn.cu), row by row.
//   k_attn_prefill         causal GQA attention of every row over its
//                          sequence's cache positions 0..pos, K/V read as
//                          fp16 (what the decode step reads); scores scaled
//                          by 1/sqrtf(hd) after the dot; single-pass softmax
//                          with a running maximum (the reference's two-pass
//                          softmax, cpu/reference/ref_ops.c:307-349, to fp32
//                          rounding).
//   k_attn_prefill_mma     the default: QK^T and PV on mma.sync tensor cores
//                          (fp16 operands with q and the softmax weights
//                          split into high and remainder parts, fp32 sums)
//                          over 32-position K/V tiles shared by 4 warps.
//   k_attn_prefill_tiled   the same with FMAs, each 32-position K/V tile staged
//                          once in shared memory for all the (row, head)
//                          warps of a GQA group and 8/G consecutive rows.
//   k_silu_glu_rows        silu(gate) * up of the fused gate/up GEMM output,
//                          whose 16-row tiles hold 8 gate rows then the 8
//                          matching up rows (ref_ops.c:219-228, 124-133 with
//                          the reference's rounding).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace {

constexpr int kHD = 128;

// Row r = b * rows_per_seq + i sits at position p0 + i of sequence b.
__global__ void __launch_bounds__(128) k_prefill_rope_append(uint32_t rows_per_seq, uint32_t p0, uint32_t h,
                                                             uint32_t hk, float *__restrict__ qkv,
                                                             const float *__restrict__ cos_t,
                                                             const float *__restrict__ sin_t, __half *__restrict__ kc,
                                                             __half *__restrict__ vc, uint64_t cap,
                                                             uint64_t seq_stride) {
  constexpr uint32_t r2 = kHD / 2;
  const uint32_t r = blockIdx.x, b = r / rows_per_seq, pos = p0 + r % rows_per_seq;
  float *row = qkv + (size_t)r * (h + 2 * hk) * kHD;
  const float *ct = cos_t + (size_t)pos * r2, *st = sin_t + (size_t)pos * r2;
  for (uint32_t i = threadIdx.x; i < h * r2; i += blockDim.x) {  // q heads, pair (j, j + r2) per thread
    float *xr = row + (size_t)(i / r2) * kHD;
    const uint32_t j = i % r2;
    float o0, o1;
    rope_pair(xr[j], xr[j + r2], ct[j], st[j], o0, o1);
    xr[j] = o0;
    xr[j + r2] = o1;
  }
  for (uint32_t i = threadIdx.x; i < hk * r2; i += blockDim.x) {  // k heads -> cache
    const uint32_t kvh = i / r2, j = i % r2;
    const float *kr = row + (size_t)(h + kvh) * kHD;
    float o0, o1;
    rope_pair(kr[j], kr[j + r2], ct[j], st[j], o0, o1);
    const size_t at = (size_t)b * seq_stride + ((size_t)kvh * cap + pos) * kHD;
    kc[at + j] = __float2half_rn(o0);
    kc[at + j + r2] = __float2half_rn(o1);
  }
  for (uint32_t i = threadIdx.x; i < hk * kHD; i += blockDim.x) {  // v heads -> cache
    const uint32_t kvh = i / kHD, d = i % kHD;
    const size_t at = (size_t)b * seq_stride + ((size_t)kvh * cap + pos) * kHD;
    vc[at + d] = __float2half_rn(row[(size_t)(h + hk + kvh) * kHD + d]);
  }
}

// One warp per (row, query head). Lanes take 32 consecutive positions at a
// time for the scores (each lane one whole key row), then each lane owns 4
// of the 128 output dimensions for the value sum.
constexpr int kAttnWarps = 4;
__global__ void __launch_bounds__(kAttnWarps * 32) k_attn_prefill(uint32_t nrows, uint32_t rows_per_seq, uint32_t p0,
                                                                  uint32_t h, uint32_t hk,
                                                                  const float *__restrict__ qkv,
                                                                  const __half *__restrict__ kc,
                                                                  const __half *__restrict__ vc, uint64_t cap,
                                                                  uint64_t seq_stride, float inv_scale,
                                                                  float *__restrict__ out) {
  __shared__ __align__(16) float qs[kAttnWarps][kHD];
  const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint64_t item = (uint64_t)blockIdx.x * kAttnWarps + w;  // row * h + head
  const bool active = item < (uint64_t)nrows * h;
  const uint32_t r = active ? (uint32_t)(item / h) : 0, head = active ? (uint32_t)(item % h) : 0;
  const uint32_t b = r / rows_per_seq, pos = p0 + r % rows_per_seq, kvh = head / (h / hk);
  const float *q = qkv + (size_t)r * (h + 2 * hk) * kHD + (size_t)head * kHD;
  for (uint32_t d = lane; d < kHD; d += 32) qs[w][d] = active ? q[d] : 0.0f;
  __syncwarp();
  if (!active) return;
  const size_t base = (size_t)b * seq_stride + (size_t)kvh * cap * kHD;
  const __half *kb = kc + base, *vb = vc + base;
  const uint32_t npos = pos + 1;
  float m = -INFINITY, l = 0.0f, acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (uint32_t j0 = 0; j0 < npos; j0 += 32) {
    const uint32_t j = j0 + lane;
    float s = -INFINITY;
    if (j < npos) {
      const uint4 *kr = reinterpret_cast<const uint4 *>(kb + (size_t)j * kHD);
      float dot = 0.0f;
#pragma unroll 4
      for (int c = 0; c < kHD / 8; c++) {
        const uint4 raw = __ldg(kr + c);
        const __half2 *hp = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 f = __half22float2(hp[e]);
          dot = fmaf(qs[w][8 * c + 2 * e], f.x, dot);
          dot = fmaf(qs[w][8 * c + 2 * e + 1], f.y, dot);
        }
      }
      s = __fmul_rn(dot, inv_scale);
    }
    const float mt = warp_max(s);
    const float mn = fmaxf(m, mt);
    const float corr = m == -INFINITY ? 0.0f : expf(m - mn);
    const float pj = j < npos ? expf(s - mn) : 0.0f;
    l = l * corr + warp_sum(pj);
#pragma unroll
    for (int e = 0; e < 4; e++) acc[e] *= corr;
    const uint32_t cnt = min(32u, npos - j0);
    for (uint32_t u = 0; u < cnt; u++) {
      const float pu = __shfl_sync(0xffffffffu, pj, u);
      const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(vb + (size_t)(j0 + u) * kHD + 4 * lane));
      const __half2 *hp = reinterpret_cast<const __half2 *>(&raw);
      const float2 v0 = __half22float2(hp[0]), v1 = __half22float2(hp[1]);
      acc[0] = fmaf(pu, v0.x, acc[0]);
      acc[1] = fmaf(pu, v0.y, acc[1]);
      acc[2] = fmaf(pu, v1.x, acc[2]);
      acc[3] = fmaf(pu, v1.y, acc[3]);
    }
    m = mn;
  }
  float4 o = make_float4(acc[0] / l, acc[1] / l, acc[2] / l, acc[3] / l);
  *reinterpret_cast<float4 *>(out + (size_t)r * h * kHD + (size_t)head * kHD + 4 * lane) = o;
}

// Two fp16 values packed in a word (low half first) as floats, exactly.
__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t w) {
  return make_float2(__half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))),
                     __half2float(__ushort_as_half((unsigned short)(w >> 16))));
}

// Tiled form: CTA per (sequence, kv head, block of 8/G consecutive rows)
// with one warp per (row, query head of the GQA group), G = h/hk dividing
// 8. The 32-position K and V tiles are loaded once per CTA into shared
// memory and read by all its warps (8x less L2 traffic than a tile per
// warp); the arithmetic per warp is k_attn_prefill's. K rows are padded to
// 136 halves so that the lanes' 16-byte reads of different rows fall in
// different banks.
constexpr int kTile = 32, kKPad = kHD + 8;
__global__ void __launch_bounds__(256) k_attn_prefill_tiled(uint32_t rows_per_seq, uint32_t p0, uint32_t h, uint32_t hk,
                                                            const float *__restrict__ qkv,
                                                            const __half *__restrict__ kc,
                                                            const __half *__restrict__ vc, uint64_t cap,
                                                            uint64_t seq_stride, float inv_scale,
                                                            float *__restrict__ out) {
  __shared__ __align__(16) __half kt[2][kTile][kKPad];  // double-buffered tiles
  __shared__ __align__(16) __half vt[2][kTile][kHD];
  __shared__ __align__(16) float qs[8][kHD];
  const uint32_t G = h / hk, RB = 8 / G;
  const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint32_t b = blockIdx.z, kvh = blockIdx.y, i0 = blockIdx.x * RB;
  const uint32_t g = w % G, i = i0 + w / G, head = kvh * G + g;
  const bool active = i < rows_per_seq;
  const uint32_t r = b * rows_per_seq + i;
  const uint32_t npos = active ? p0 + i + 1 : 0;
  const uint32_t ilast = min(i0 + RB, rows_per_seq) - 1, nmax = p0 + ilast + 1;  // positions this CTA needs
  if (active) {
    const float *q = qkv + (size_t)r * (h + 2 * hk) * kHD + (size_t)head * kHD;
    for (uint32_t d = lane; d < kHD; d += 32) qs[w][d] = q[d];
  }
  const size_t base = (size_t)b * seq_stride + (size_t)kvh * cap * kHD;
  float m = -INFINITY, l = 0.0f, acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  // tile t of positions [32t, 32t + 32) into buffer t & 1: 32 rows x 16
  // chunks of 16 B for K and for V, 2 + 2 asynchronous copies per thread;
  // rows at or beyond nmax are zero-filled (source size 0, no read)
  auto load_tile = [&](uint32_t t) {
    const uint32_t buf = t & 1u, j0 = t * kTile;
    for (uint32_t c = threadIdx.x; c < kTile * (kHD / 8); c += blockDim.x) {
      const uint32_t row = c / (kHD / 8), col = c % (kHD / 8);
      const bool in = j0 + row < nmax;
      const size_t off = base + (size_t)(in ? j0 + row : 0) * kHD + col * 8;
      const uint32_t n = in ? 16u : 0u;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(&kt[buf][row][col * 8])),
                   "l"(kc + off), "r"(n)
                   : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(&vt[buf][row][col * 8])),
                   "l"(vc + off), "r"(n)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const uint32_t ntiles = (nmax + kTile - 1) / kTile;
  load_tile(0);
  for (uint32_t t = 0; t < ntiles; t++) {
    const uint32_t j0 = t * kTile, buf = t & 1u;
    if (t + 1 < ntiles) {
      load_tile(t + 1);  // its buffer was last read in iteration t - 1, before that iteration's barrier
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // tile t is in shared memory for every thread (and qs, the first time)
    if (active && j0 < npos) {
      const uint32_t j = j0 + lane;
      float s = -INFINITY;
      if (j < npos) {
        float dot = 0.0f;
#pragma unroll 4
        for (int c = 0; c < kHD / 8; c++) {
          const uint4 raw = *reinterpret_cast<const uint4 *>(&kt[buf][lane][c * 8]);
          const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float2 f = half2_bits_to_float2(words[e]);
            dot = fmaf(qs[w][8 * c + 2 * e], f.x, dot);
            dot = fmaf(qs[w][8 * c + 2 * e + 1], f.y, dot);
          }
        }
        s = __fmul_rn(dot, inv_scale);
      }
      const float mt = warp_max(s);
      const float mn = fmaxf(m, mt);
      const float corr = m == -INFINITY ? 0.0f : expf(m - mn);
      const float pj = j < npos ? expf(s - mn) : 0.0f;
      l = l * corr + warp_sum(pj);
#pragma unroll
      for (int e = 0; e < 4; e++) acc[e] *= corr;
      const uint32_t cnt = min((uint32_t)kTile, npos - j0);
      for (uint32_t u = 0; u < cnt; u++) {
        const float pu = __shfl_sync(0xffffffffu, pj, u);
        const uint2 raw = *reinterpret_cast<const uint2 *>(&vt[buf][u][4 * lane]);
        const float2 v0 = half2_bits_to_float2(raw.x), v1 = half2_bits_to_float2(raw.y);
        acc[0] = fmaf(pu, v0.x, acc[0]);
        acc[1] = fmaf(pu, v0.y, acc[1]);
        acc[2] = fmaf(pu, v1.x, acc[2]);
        acc[3] = fmaf(pu, v1.y, acc[3]);
      }
      m = mn;
    }
    __syncthreads();  // every warp is done with buffer t & 1 before tile t + 2 is copied into it
  }
  if (!active) return;
  float4 o = make_float4(acc[0] / l, acc[1] / l, acc[2] / l, acc[3] / l);
  *reinterpret_cast<float4 *>(out + (size_t)r * h * kHD + (size_t)head * kHD + 4 * lane) = o;
}

// Tensor-core form (the default where G = h/hk divides 16): QK^T and PV
// on mma.sync m16n8k16 (fp16 operands, fp32 accumulate). A warp owns an
// M-tile of 16 (position, query head) rows: 16/G consecutive positions x
// the G heads of one KV head; a CTA is 4 such warps over 64/G consecutive
// positions and shares each 32-position K/V tile (fp16, from the cache,
// rows padded to 136 halves so fragment loads are conflict-free). K and V
// are exact in fp16. q and the softmax weights are not, so each is split
// into an fp16 high part and an fp16 remainder and multiplied twice: the
// products carry about 2^-22 relative error, fp32-like, and the sums are
// fp32. The softmax keeps a running row maximum as k_attn_prefill does.
constexpr int kMmaWarps = 4, kMPad = kHD + 8;

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (x, y) -> fp16 high parts packed (x low) and fp16 remainders packed
__device__ __forceinline__ void split2(float x, float y, uint32_t &hi, uint32_t &lo) {
  const __half hx = __float2half_rn(x), hy = __float2half_rn(y);
  const __half lx = __float2half_rn(x - __half2float(hx)), ly = __float2half_rn(y - __half2float(hy));
  hi = (uint32_t)__half_as_ushort(hx) | ((uint32_t)__half_as_ushort(hy) << 16);
  lo = (uint32_t)__half_as_ushort(lx) | ((uint32_t)__half_as_ushort(ly) << 16);
}

__global__ void __launch_bounds__(kMmaWarps * 32) k_attn_prefill_mma(uint32_t rows_per_seq, uint32_t p0, uint32_t h,
                                                                     uint32_t hk, const float *__restrict__ qkv,
                                                                     const __half *__restrict__ kc,
                                                                     const __half *__restrict__ vc, uint64_t cap,
                                                                     uint64_t seq_stride, float inv_scale,
                                                                     float *__restrict__ out) {
  __shared__ __align__(16) __half kt[kTile][kMPad];
  __shared__ __align__(16) __half vt[kTile][kMPad];
  const uint32_t G = h / hk, PW = 16 / G;  // positions per warp
  const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint32_t gq = lane >> 2, tq = lane & 3;  // fragment row group, thread in group
  const uint32_t b = blockIdx.z, kvh = blockIdx.y;
  const uint32_t ic0 = blockIdx.x * (PW * kMmaWarps);  // first position index (within the prompt) of the CTA
  const uint32_t iw0 = ic0 + w * PW;                    // first position index of this warp
  // this thread's two fragment rows: M-tile row m -> position iw0 + m / G, head kvh * G + m % G
  uint32_t npos[2];
  size_t rowq[2];
  bool live[2];
#pragma unroll
  for (int x = 0; x < 2; x++) {
    const uint32_t mrow = gq + 8 * x, i = iw0 + mrow / G;
    live[x] = i < rows_per_seq;
    npos[x] = live[x] ? p0 + i + 1 : 0;
    rowq[x] = ((size_t)b * rows_per_seq + (live[x] ? i : 0)) * (h + 2 * hk) * kHD + (size_t)(kvh * G + mrow % G) * kHD;
  }
  // q fragments, high and remainder: k-step s covers dims 16s..16s+15
  uint32_t qh[8][4], ql[8][4];
#pragma unroll
  for (int st = 0; st < 8; st++) {
#pragma unroll
    for (int x = 0; x < 2; x++) {
#pragma unroll
      for (int half = 0; half < 2; half++) {  // dims +0..7 (regs 0/1), +8..15 (regs 2/3)
        const uint32_t d = 16 * st + 8 * half + 2 * tq;
        const float2 v = live[x] ? *reinterpret_cast<const float2 *>(qkv + rowq[x] + d) : make_float2(0.f, 0.f);
        split2(v.x, v.y, qh[st][x + 2 * half], ql[st][x + 2 * half]);
      }
    }
  }
  const uint32_t ilast = min(ic0 + PW * kMmaWarps, rows_per_seq) - 1, nmax = p0 + ilast + 1;
  // The warp's last needed position + 1, the same in every lane: its rows
  // are positions [iw0, iw0 + PW), so the tile skip below is warp-uniform
  // and every mma.sync, ldmatrix and full-mask shuffle after it is reached
  // by all 32 lanes or by none (a per-lane bound here once let some lanes
  // skip a tile while the others waited in mma.sync). Rows that end earlier
  // mask their keys with npos.
  const uint32_t wmax = iw0 < rows_per_seq ? p0 + min(iw0 + PW, rows_per_seq) : 0;
  const size_t base = (size_t)b * seq_stride + (size_t)kvh * cap * kHD;
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
  for (uint32_t j0 = 0; j0 < nmax; j0 += kTile) {
    __syncthreads();
    for (uint32_t c = threadIdx.x; c < kTile * (kHD / 8); c += blockDim.x) {
      const uint32_t row = c / (kHD / 8), col = c % (kHD / 8);
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (j0 + row < nmax) {
        kv = __ldg(reinterpret_cast<const uint4 *>(kc + base + (size_t)(j0 + row) * kHD) + col);
        vv = __ldg(reinterpret_cast<const uint4 *>(vc + base + (size_t)(j0 + row) * kHD) + col);
      }
      *reinterpret_cast<uint4 *>(&kt[row][col * 8]) = kv;
      *reinterpret_cast<uint4 *>(&vt[row][col * 8]) = vv;
    }
    __syncthreads();
    if (j0 >= wmax) continue;  // uniform across the warp
    // S = q K^T for the 32 positions: 4 n-tiles of 8
    float sacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; nt++) {
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
      for (int st = 0; st < 8; st++) {
        const __half *kr = &kt[nt * 8 + gq][16 * st + 2 * tq];
        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(kr), b1 = *reinterpret_cast<const uint32_t *>(kr + 8);
        mma16816(sacc[nt], qh[st], b0, b1);
        mma16816(sacc[nt], ql[st], b0, b1);
      }
    }
    // scale, causal mask, running maximum per row (a row's 4 threads share it)
    float mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 4; nt++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int x = e >> 1;
        const uint32_t key = j0 + nt * 8 + 2 * tq + (e & 1);
        const float sv = key < npos[x] ? __fmul_rn(sacc[nt][e], inv_scale) : -INFINITY;
        sacc[nt][e] = sv;
        mt[x] = fmaxf(mt[x], sv);
      }
    float corr[2];
#pragma unroll
    for (int x = 0; x < 2; x++) {
      mt[x] = fmaxf(mt[x], __shfl_xor_sync(0xffffffffu, mt[x], 1));
      mt[x] = fmaxf(mt[x], __shfl_xor_sync(0xffffffffu, mt[x], 2));
      const float mn = fmaxf(m[x], mt[x]);
      corr[x] = (m[x] == -INFINITY) ? 0.0f : expf(m[x] - mn);
      m[x] = mn;
      l[x] *= corr[x];
    }
#pragma unroll
    for (int n = 0; n < 16; n++) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
    // softmax weights as A fragments (high and remainder) for the 2 k-steps of 16 positions
    uint32_t ph[2][4], pl[2][4];
#pragma unroll
    for (int nt = 0; nt < 4; nt++) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int x = e >> 1;
        pv[e] = m[x] == -INFINITY || sacc[nt][e] == -INFINITY ? 0.0f : expf(sacc[nt][e] - m[x]);
        l[x] += pv[e];
      }
      const int ks = nt >> 1, r = (nt & 1) * 2;  // n-tile 2ks -> regs 0/1, 2ks+1 -> regs 2/3
      split2(pv[0], pv[1], ph[ks][r], pl[ks][r]);
      split2(pv[2], pv[3], ph[ks][r + 1], pl[ks][r + 1]);
    }
    // O += P V: 16 n-tiles of 8 dims, B fragments by transposing loads of the V rows
#pragma unroll
    for (int ks = 0; ks < 2; ks++) {
#pragma unroll
      for (int n = 0; n < 16; n++) {
        uint32_t b0, b1;
        const __half *vr = &vt[16 * ks + (lane & 15)][8 * n];
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                     : "=r"(b0), "=r"(b1)
                     : "r"(smem_u32(vr)));
        mma16816(o[n], ph[ks], b0, b1);
        mma16816(o[n], pl[ks], b0, b1);
      }
    }
  }
  // row sums: each of a row's 4 threads holds a quarter
#pragma unroll
  for (int x = 0; x < 2; x++) {
    l[x] += __shfl_xor_sync(0xffffffffu, l[x], 1);
    l[x] += __shfl_xor_sync(0xffffffffu, l[x], 2);
  }
#pragma unroll
  for (int x = 0; x < 2; x++) {
    if (!live[x]) continue;
    const uint32_t mrow = gq + 8 * x, i = iw0 + mrow / G, r = b * rows_per_seq + i;
    float *dst = out + (size_t)r * h * kHD + (size_t)(kvh * G + mrow % G) * kHD;
#pragma unroll
    for (int n = 0; n < 16; n++)
      *reinterpret_cast<float2 *>(dst + 8 * n + 2 * tq) = make_float2(o[n][2 * x] / l[x], o[n][2 * x + 1] / l[x]);
  }
}

__global__ void k_silu_glu_rows(uint64_t rows, uint32_t ff, const float *__restrict__ gu, float *__restrict__ hout) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * ff) return;
  const uint64_t r = i / ff;
  const uint32_t f = (uint32_t)(i % ff), tile = f / 8, wi = f % 8;
  const float *g = gu + (size_t)r * 2 * ff;
  const float a = g[(size_t)tile * 16 + wi], u = g[(size_t)tile * 16 + 8 + wi];
  hout[i] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), u);
}

}  // namespace

extern "C" pai_status_t b200_launch_prefill_rope_append(pai_b200_ctx_t *ctx, uint32_t rows, uint32_t rows_per_seq,
                                                        uint32_t p0, uint32_t h, uint32_t hk, uint32_t hd, float *qkv,
                                                        const float *cos_t, const float *sin_t, uint16_t *kc,
                                                        uint16_t *vc, uint64_t cap, uint64_t seq_stride) {
  if (hd != kHD || rows == 0 || rows_per_seq == 0 || p0 + rows_per_seq > cap)
    return b200_fail(PAI_ERR_INVALID_ARG, "prefill_rope_append: head_dim %u, %u rows from position %u, cap %llu", hd,
                     rows, p0, (unsigned long long)cap);
  k_prefill_rope_append<<<rows, 128, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(
      rows_per_seq, p0, h, hk, qkv, cos_t, sin_t, reinterpret_cast<__half *>(kc), reinterpret_cast<__half *>(vc), cap,
      seq_stride);
  return b200_launched(ctx, 1, "k_prefill_rope_append");
}

extern "C" pai_status_t b200_launch_attn_prefill(pai_b200_ctx_t *ctx, uint32_t rows, uint32_t rows_per_seq,
                                                 uint32_t p0, uint32_t h, uint32_t hk, uint32_t hd, const float *qkv,
                                                 const uint16_t *kc, const uint16_t *vc, uint64_t cap,
                                                 uint64_t seq_stride, float *out) {
  if (hd != kHD || rows == 0 || hk == 0 || h % hk || p0 + rows_per_seq > cap)
    return b200_fail(PAI_ERR_INVALID_ARG, "attn_prefill: invalid shape");
  const uint64_t items = (uint64_t)rows * h, blocks = (items + kAttnWarps - 1) / kAttnWarps;
  if (blocks > 0x7FFFFFFFull) return b200_fail(PAI_ERR_UNSUPPORTED, "attn_prefill: too many rows");
  // 1/sqrtf(hd), the scale of the decode attention
  const float inv_scale = 1.0f / sqrtf((float)hd);
  const uint32_t G = h / hk;
  if (G <= 16 && 16 % G == 0 && rows % rows_per_seq == 0) {
    const uint32_t per_cta = (16 / G) * kMmaWarps, nseq = rows / rows_per_seq;
    if (nseq > 65535 || hk > 65535) return b200_fail(PAI_ERR_UNSUPPORTED, "attn_prefill: grid");
    k_attn_prefill_mma<<<dim3((rows_per_seq + per_cta - 1) / per_cta, hk, nseq), kMmaWarps * 32, 0,
                         (cudaStream_t)b200_ctx_stream(ctx)>>>(
        rows_per_seq, p0, h, hk, qkv, reinterpret_cast<const __half *>(kc), reinterpret_cast<const __half *>(vc),
        cap, seq_stride, inv_scale, out);
    return b200_launched(ctx, 1, "k_attn_prefill_mma");
  }
  if (G <= 8 && 8 % G == 0 && rows % rows_per_seq == 0) {
    const uint32_t RB = 8 / G, nseq = rows / rows_per_seq;
    if (nseq > 65535 || hk > 65535) return b200_fail(PAI_ERR_UNSUPPORTED, "attn_prefill: grid");
    k_attn_prefill_tiled<<<dim3((rows_per_seq + RB - 1) / RB, hk, nseq), 256, 0,
                           (cudaStream_t)b200_ctx_stream(ctx)>>>(
        rows_per_seq, p0, h, hk, qkv, reinterpret_cast<const __half *>(kc), reinterpret_cast<const __half *>(vc),
        cap, seq_stride, inv_scale, out);
    return b200_launched(ctx, 1, "k_attn_prefill_tiled");
  }
  k_attn_prefill<<<(uint32_t)blocks, kAttnWarps * 32, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(
      rows, rows_per_seq, p0, h, hk, qkv, reinterpret_cast<const __half *>(kc), reinterpret_cast<const __half *>(vc),
      cap, seq_stride, inv_scale, out);
  return b200_launched(ctx, 1, "k_attn_prefill");
}

extern "C" pai_status_t b200_launch_silu_glu_rows(pai_b200_ctx_t *ctx, uint64_t rows, uint32_t ff, const float *gu,
                                                  float *hout) {
  const uint64_t n = rows * ff, blocks = (n + 255) / 256;
  if (!n || ff % 8 || blocks > 0x7FFFFFFFull) return b200_fail(PAI_ERR_INVALID_ARG, "silu_glu_rows: shape");
  k_silu_glu_rows<<<(uint32_t)blocks, 256, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(rows, ff, gu, hout);
  return b200_launched(ctx, 1, "k_silu_glu_rows");
}
