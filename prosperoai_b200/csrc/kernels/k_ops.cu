// Row and elementwise kernels around the GEMVs: RMSNorm, RoPE (op form
// and the decode form that also appends the new K/V rows to the fp16
// cache), SiLU-gate, residual add, embedding lookup and greedy argmax.
// Where the reference's result is a fixed sequence of IEEE operations
// (rmsnorm scale, rope, residual add, embedding) the kernels issue the
// same operations with explicit rounding (__fmul_rn, __fadd_rn, ...) so
// that nvcc cannot contract them into FMAs and the result is bit-exact.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace {

inline unsigned nblk(uint64_t work, unsigned t) { return (unsigned)((work + t - 1) / t); }

// pai_ref_rmsnorm_gamma_f32 (cpu/reference/ref_ops.c:196-216): the sum of
// squares is taken in double like the reference (products of floats are
// exact in double); scale = 1/sqrtf((float)(acc/n) + eps) and
// c = (a*gamma)*scale with single roundings.
__global__ void k_rmsnorm(uint64_t n, const float *__restrict__ a, const float *__restrict__ gamma,
                          float eps, float *__restrict__ c) {
  const float *ar = a + blockIdx.x * n;
  float *cr = c + blockIdx.x * n;
  double acc = 0.0;
  for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
    double v = (double)ar[i];
    acc = __dadd_rn(acc, __dmul_rn(v, v));
  }
  __shared__ double red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  __shared__ float scale;
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (unsigned w = 0; w < (blockDim.x + 31) / 32; w++) t += red[w];
    float ms = (float)__ddiv_rn(t, (double)n);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  }
  __syncthreads();
  float s = scale;
  for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) cr[i] = __fmul_rn(__fmul_rn(ar[i], gamma[i]), s);
}

// pai_ref_silu_f32 then pai_ref_vecmul_f32 (ref_ops.c:219-228, 124-133).
__global__ void k_silu_mul(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ o,
                           uint64_t n) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    float a = g[i];
    o[i] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), u[i]);
  }
}

__global__ void k_vecadd(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ c,
                         uint64_t n) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) c[i] = __fadd_rn(a[i], b[i]);
}

__device__ __forceinline__ void rope_pair(float x0, float x1, float c, float s, float &o0, float &o1) {
  o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  o1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

// pai_ref_rope_f32 (ref_ops.c:231-257): one thread per (row, i) with
// i < hd; i < r2 rotates the pair (i, i+r2), i >= 2*r2 copies.
__global__ void k_rope(const float *__restrict__ x, uint64_t rows, uint64_t hd, uint64_t heads,
                       const float *__restrict__ cos_t, const float *__restrict__ sin_t, uint64_t r2,
                       float *__restrict__ out) {
  uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * hd) return;
  uint64_t row = idx / hd, i = idx % hd;
  uint64_t p = row / heads;
  const float *xr = x + row * hd;
  float *orow = out + row * hd;
  if (i < r2) {
    float o0, o1;
    rope_pair(xr[i], xr[i + r2], cos_t[p * r2 + i], sin_t[p * r2 + i], o0, o1);
    orow[i] = o0;
    orow[i + r2] = o1;
  } else if (i >= 2 * r2) {
    orow[i] = xr[i];
  }
}

// Decode form: the fused q|k|v projection row of each sequence is split,
// q and k are rotated at position *pos, k and v are rounded to fp16 and
// written at *pos of the sequence's cache ([hk][cap][hd]).
__global__ void k_rope_kv(uint32_t h, uint32_t hk, uint32_t hd, const float *__restrict__ qkv,
                          const int32_t *__restrict__ pos, const float *__restrict__ cos_t,
                          const float *__restrict__ sin_t, float *__restrict__ q, __half *__restrict__ kc,
                          __half *__restrict__ vc, uint64_t cap, uint64_t seq_stride) {
  const uint32_t bi = blockIdx.x;
  const uint32_t p = (uint32_t)*pos;
  const uint32_t r2 = hd / 2;
  const uint32_t width = (h + 2 * hk) * hd;
  const float *row = qkv + (size_t)bi * width;
  float *qo = q + (size_t)bi * h * hd;
  __half *kcs = kc + (size_t)bi * seq_stride;
  __half *vcs = vc + (size_t)bi * seq_stride;
  for (uint32_t idx = threadIdx.x; idx < (h + hk) * r2; idx += blockDim.x) {
    uint32_t head = idx / r2, i = idx % r2;
    float c = cos_t[(size_t)p * r2 + i], s = sin_t[(size_t)p * r2 + i];
    const float *xr = row + (size_t)head * hd;
    float o0, o1;
    rope_pair(xr[i], xr[i + r2], c, s, o0, o1);
    if (head < h) {
      qo[(size_t)head * hd + i] = o0;
      qo[(size_t)head * hd + i + r2] = o1;
    } else {
      __half *kr = kcs + ((size_t)(head - h) * cap + p) * hd;
      kr[i] = __float2half_rn(o0);
      kr[i + r2] = __float2half_rn(o1);
    }
  }
  for (uint32_t idx = threadIdx.x; idx < hk * hd; idx += blockDim.x) {
    uint32_t head = idx / hd, d = idx % hd;
    vcs[((size_t)head * cap + p) * hd + d] = __float2half_rn(row[(size_t)(h + hk) * hd + idx]);
  }
}

// Embedding lookup: the reference multiplies a one-hot row by the
// dequantised table (adapters/llama/llama.c:490, 510-522), which yields
// the dequantised table row exactly. One thread per block of the row.
__global__ void k_embed(uint32_t type, uint32_t nb, const uint8_t *__restrict__ qs,
                        const uint8_t *__restrict__ sc, const int32_t *__restrict__ tokens,
                        float *__restrict__ x) {
  const uint32_t bi = blockIdx.x;
  const uint32_t r = (uint32_t)tokens[bi];
  const uint32_t chunks = b200_chunks(type), hdr = b200_hdr_bytes(type), el = b200_blk_elems(type);
  const uint64_t g = r / B200_RG, lr = r % B200_RG;
  float *xr = x + (size_t)bi * nb * el;
  for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
    uint64_t tile = g * nb + b;
    const uint8_t *h = sc + (tile * B200_RG + lr) * hdr;
    float d = f16_bits_to_f32((uint16_t)(h[0] | (h[1] << 8)));
    float *o = xr + (size_t)b * el;
    auto q = [&](uint32_t byte) -> uint8_t {
      return qs[((tile * chunks + byte / 16u) * B200_RG + lr) * 16u + byte % 16u];
    };
    if (type == PAI_B200_Q8_0) {
      for (int j = 0; j < 32; j++) o[j] = __fmul_rn((float)(int8_t)q(j), d);
    } else if (type == PAI_B200_Q4_0) {
      for (int j = 0; j < 16; j++) {
        uint8_t v = q(j);
        o[j] = __fmul_rn((float)((int)(v & 15) - 8), d);
        o[j + 16] = __fmul_rn((float)((int)(v >> 4) - 8), d);
      }
    } else {
      float dmin = f16_bits_to_f32((uint16_t)(h[2] | (h[3] << 8)));
      for (int c = 0; c < 4; c++) {
        uint8_t s0, m0, s1, m1;
        k4_scale_min(2 * c, h + 4, &s0, &m0);
        k4_scale_min(2 * c + 1, h + 4, &s1, &m1);
        float d1 = __fmul_rn(d, (float)s0), mm1 = __fmul_rn(dmin, (float)m0);
        float d2 = __fmul_rn(d, (float)s1), mm2 = __fmul_rn(dmin, (float)m1);
        for (int l = 0; l < 32; l++) {
          uint8_t v = q(32 * c + l);
          o[64 * c + l] = __fsub_rn(__fmul_rn(d1, (float)(v & 15)), mm1);
          o[64 * c + 32 + l] = __fsub_rn(__fmul_rn(d2, (float)(v >> 4)), mm2);
        }
      }
    }
  }
}

// Greedy pick (models/sampler.c:89-99): first index of the strict
// maximum. Each thread keeps the first maximum of its strided slice; the
// reduction prefers the larger value and, on equal values, the smaller
// index, which is the sequential scan's answer.
__global__ void k_argmax(uint64_t n, const float *__restrict__ logits, int32_t *__restrict__ out) {
  const float *row = logits + (size_t)blockIdx.x * n;
  float best = -INFINITY;
  uint32_t bidx = 0xFFFFFFFFu;
  for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
    float v = row[i];
    if (bidx == 0xFFFFFFFFu || v > best) {
      best = v;
      bidx = (uint32_t)i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    uint32_t oi = __shfl_xor_sync(0xffffffffu, bidx, o);
    if (oi != 0xFFFFFFFFu && (bidx == 0xFFFFFFFFu || ov > best || (ov == best && oi < bidx))) {
      best = ov;
      bidx = oi;
    }
  }
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bidx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (unsigned w = 1; w < blockDim.x / 32; w++) {
      if (si[w] != 0xFFFFFFFFu && (bidx == 0xFFFFFFFFu || sv[w] > best || (sv[w] == best && si[w] < bidx))) {
        best = sv[w];
        bidx = si[w];
      }
    }
    out[blockIdx.x] = (int32_t)bidx;
  }
}

// End of a device-resident decode step: advance the position and feed
// the chosen tokens back as the next step's input.
__global__ void k_step_tail(uint32_t batch, const int32_t *__restrict__ tok_out, int32_t *__restrict__ tok_in,
                            int32_t *__restrict__ pos) {
  uint32_t i = threadIdx.x;
  if (i < batch) tok_in[i] = tok_out[i];
  if (i == 0) *pos += 1;
}

}  // namespace

extern "C" pai_status_t b200_launch_rmsnorm(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, const float *a,
                                            const float *gamma, float eps, float *c) {
  if (eps == 0.0f) eps = 1e-5f;
  k_rmsnorm<<<(unsigned)rows, 256, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(n, a, gamma, eps, c);
  return b200_launched(ctx, 1, "k_rmsnorm");
}

extern "C" pai_status_t pai_b200_rmsnorm_gamma_f32(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n,
                                                   const float *a, const float *gamma, float eps, float *c) {
  if (!ctx || !a || !gamma || !c) return b200_fail(PAI_ERR_INVALID_ARG, "rmsnorm: NULL");
  if (rows == 0 || n == 0 || rows > 0x7FFFFFFFull) return b200_fail(PAI_ERR_INVALID_ARG, "rmsnorm: shape");
  return b200_launch_rmsnorm(ctx, rows, n, a, gamma, eps, c);
}

extern "C" pai_status_t pai_b200_silu_mul_f32(pai_b200_ctx_t *ctx, const float *gate, const float *up,
                                              float *out, uint64_t n) {
  if (!ctx || ((!gate || !up || !out) && n)) return b200_fail(PAI_ERR_INVALID_ARG, "silu_mul: NULL");
  if (!n) return PAI_OK;
  k_silu_mul<<<nblk(n, 256), 256, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(gate, up, out, n);
  return b200_launched(ctx, 1, "k_silu_mul");
}

extern "C" pai_status_t pai_b200_vecadd_f32(pai_b200_ctx_t *ctx, const float *a, const float *b, float *c,
                                            uint64_t n) {
  if (!ctx || ((!a || !b || !c) && n)) return b200_fail(PAI_ERR_INVALID_ARG, "vecadd: NULL");
  if (!n) return PAI_OK;
  k_vecadd<<<nblk(n, 256), 256, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(a, b, c, n);
  return b200_launched(ctx, 1, "k_vecadd");
}

extern "C" pai_status_t pai_b200_rope_f32(pai_b200_ctx_t *ctx, const float *x, uint64_t rows, uint64_t hd,
                                          uint64_t seq, uint64_t heads, const float *cos_t, const float *sin_t,
                                          uint64_t r2, float *out) {
  // Argument rules of pai_ref_rope_f32 (ref_ops.c:235-238).
  if (!ctx || rows == 0 || hd == 0 || seq == 0 || heads == 0 || r2 == 0 || 2 * r2 > hd || rows % heads != 0 ||
      !x || !out || !cos_t || !sin_t)
    return b200_fail(PAI_ERR_INVALID_ARG, "rope: invalid arguments");
  k_rope<<<nblk(rows * hd, 256), 256, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(x, rows, hd, heads, cos_t, sin_t,
                                                                               r2, out);
  return b200_launched(ctx, 1, "k_rope");
}

extern "C" pai_status_t b200_launch_rope_kv(pai_b200_ctx_t *ctx, uint32_t batch, uint32_t h, uint32_t hk,
                                            uint32_t hd, const float *qkv, const int32_t *pos,
                                            const float *cos_t, const float *sin_t, float *q, uint16_t *kc,
                                            uint16_t *vc, uint64_t cap, uint64_t seq_stride) {
  k_rope_kv<<<batch, 256, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(h, hk, hd, qkv, pos, cos_t, sin_t, q,
                                                                    (__half *)kc, (__half *)vc, cap, seq_stride);
  return b200_launched(ctx, 1, "k_rope_kv");
}

extern "C" pai_status_t b200_launch_embed(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch, uint64_t rows,
                                          uint64_t k, const void *w, const int32_t *tokens, float *x) {
  uint32_t nb = (uint32_t)(k / b200_blk_elems(type));
  const uint8_t *qs = (const uint8_t *)w;
  const uint8_t *sc = qs + b200_sc_offset(type, rows, k);
  k_embed<<<batch, 128, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(type, nb, qs, sc, tokens, x);
  return b200_launched(ctx, 1, "k_embed");
}

extern "C" pai_status_t b200_launch_argmax(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, const float *logits,
                                           int32_t *out) {
  k_argmax<<<(unsigned)rows, 1024, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(n, logits, out);
  return b200_launched(ctx, 1, "k_argmax");
}

extern "C" pai_status_t pai_b200_argmax_f32(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, const float *logits,
                                            int32_t *out) {
  if (!ctx || !logits || !out) return b200_fail(PAI_ERR_INVALID_ARG, "argmax: NULL");
  if (rows == 0 || n == 0 || n > 0xFFFFFFFEull || rows > 0x7FFFFFFFull)
    return b200_fail(PAI_ERR_INVALID_ARG, "argmax: shape");
  return b200_launch_argmax(ctx, rows, n, logits, out);
}

extern "C" pai_status_t b200_launch_step_tail(pai_b200_ctx_t *ctx, uint32_t batch, int32_t *tok_out,
                                              int32_t *tok_in, int32_t *pos) {
  k_step_tail<<<1, 32, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(batch, tok_out, tok_in, pos);
  return b200_launched(ctx, 1, "k_step_tail");
}
