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
//   k_attn_prefill_tiled   the same, with each 32-position K/V tile staged
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
