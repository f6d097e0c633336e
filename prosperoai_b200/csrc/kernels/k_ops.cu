// Row and elementwise kernels around the GEMVs: RMSNorm (optionally
// writing the GEMV operand format), RoPE, SiLU-gate, residual add,
// embedding lookup and greedy argmax. The decode form of RoPE (with the
// K/V append) lives in the attention kernel (k_attn.cu).
// Where the reference's result is a fixed sequence of IEEE operations
// (rmsnorm scale, rope, residual add, embedding) the kernels issue the
// same operations with explicit rounding (__fmul_rn, __fadd_rn, ...) so
// that nvcc cannot contract them into FMAs and the result is bit-exact.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace {

inline unsigned nblk(uint64_t work, unsigned t) { return (unsigned)((work + t - 1) / t); }

// pai_ref_rmsnorm_gamma_f32 (cpu/reference/ref_ops.c:196-216): the sum of
// squares is taken in double like the reference (products of floats are
// exact in double); scale = 1/sqrtf((float)(acc/n) + eps) and
// c = (a*gamma)*scale with single roundings. CTA (slice, row): every CTA
// of a row sums the whole row (16 KB at n = 4096, in one round of loads)
// in the same order, so all get the same scale, then writes only its
// slice of 32-element blocks -- as fp32 into c and/or quantised into xq
// for the GEMV that consumes it, one block per warp.
constexpr int kNormThreads = 128;
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm(uint32_t n, uint32_t bps, const float *__restrict__ a,
                                                          const float *__restrict__ gamma, float eps,
                                                          float *__restrict__ c, b200_xq_t xq) {
  pdl_trigger();
  pdl_wait();
  const uint32_t row = blockIdx.y;
  const float *ar = a + (size_t)row * n;
  double acc = 0.0;
#pragma unroll 8
  for (uint32_t i = threadIdx.x; i < n; i += kNormThreads) {
    const double v = (double)ar[i];
    acc = __dadd_rn(acc, __dmul_rn(v, v));
  }
  __shared__ double red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < kNormThreads / 32; w++) t += red[w];
  const float ms = (float)__ddiv_rn(t, (double)n);
  const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  float *cr = c ? c + (size_t)row * n : nullptr;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t nblk = xq.limbs ? (uint32_t)(xq.quads * 4) : (n + 31) / 32;
  const uint32_t b1 = min(nblk, (blockIdx.x + 1) * bps);
  for (uint32_t b = blockIdx.x * bps + (threadIdx.x >> 5); b < b1; b += kNormThreads / 32) {
    const uint32_t i = b * 32 + lane;
    const float v = i < n ? __fmul_rn(__fmul_rn(ar[i], gamma[i]), s) : 0.0f;
    if (cr && i < n) cr[i] = v;
    if (xq.limbs) xq_store_block(xq, row, b, v);
  }
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

// Embedding lookup: the reference multiplies a one-hot row by the
// dequantised table (adapters/llama/llama.c:490, 510-522), which yields
// the dequantised table row exactly. One thread per block of the row.
__global__ void k_embed(uint32_t type, uint32_t nb, uint64_t ntiles, const uint8_t *__restrict__ qs,
                        const uint8_t *__restrict__ sc, const int32_t *__restrict__ tokens, float *__restrict__ x) {
  pdl_trigger();
  pdl_wait();
  const uint32_t bi = blockIdx.x;
  const uint64_t r = (uint32_t)tokens[bi];
  const uint32_t el = b200_blk_elems(type);
  for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x)
    dequant_block_dev(type, ntiles, qs, sc, r, b, x + ((size_t)bi * nb + b) * el);
}

// Greedy pick (models/sampler.c:89-99): first index of the strict
// maximum. CTA (slice, row) scans a contiguous slice; each thread keeps the
// first maximum of its strided part, and merges prefer the larger value
// and, on equal values, the smaller index, which is the sequential scan's
// answer. The last slice of a row to finish (ticket) merges the slices.
__device__ __forceinline__ void amax_merge(float &best, uint32_t &bidx, float ov, uint32_t oi) {
  if (oi != 0xFFFFFFFFu && (bidx == 0xFFFFFFFFu || ov > best || (ov == best && oi < bidx))) {
    best = ov;
    bidx = oi;
  }
}

__device__ __forceinline__ void amax_block(float &best, uint32_t &bidx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bidx, o);
    amax_merge(best, bidx, ov, oi);
  }
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bidx;
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (unsigned w = 1; w < blockDim.x / 32; w++) amax_merge(best, bidx, sv[w], si[w]);
  __syncthreads();
}

// Greedy argmax of each logit row: slices per CTA, the last slice to finish
// merges them (first index of the maximum, as models/sampler.c:89-99). With
// `pair` set, the row's result is written as (maximum, index + v0) for a
// merge across tensor-parallel vocabulary shards instead of to `out`.
__global__ void __launch_bounds__(256) k_argmax(uint64_t n, uint64_t per, const float *__restrict__ logits,
                                                int32_t *__restrict__ out, float *__restrict__ part,
                                                uint32_t *__restrict__ cnt, float *__restrict__ pair, uint32_t v0) {
  pdl_trigger();
  pdl_wait();
  const uint32_t row = blockIdx.y, slice = blockIdx.x, nsl = gridDim.x;
  const float *lr = logits + (size_t)row * n;
  const uint64_t lo = (uint64_t)slice * per, hi = min(n, lo + per);
  float best = -INFINITY;
  uint32_t bidx = 0xFFFFFFFFu;
  for (uint64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = lr[i];
    if (bidx == 0xFFFFFFFFu || v > best) {
      best = v;
      bidx = (uint32_t)i;
    }
  }
  amax_block(best, bidx);
  __shared__ uint32_t ticket;
  if (threadIdx.x == 0) {
    part[((size_t)row * nsl + slice) * 2] = best;
    part[((size_t)row * nsl + slice) * 2 + 1] = __uint_as_float(bidx);
    __threadfence();
    ticket = atomicAdd(&cnt[row], 1u);
  }
  __syncthreads();
  if (ticket != nsl - 1) return;
  __threadfence();
  best = -INFINITY;
  bidx = 0xFFFFFFFFu;
  for (uint32_t s = threadIdx.x; s < nsl; s += blockDim.x)
    amax_merge(best, bidx, __ldcg(&part[((size_t)row * nsl + s) * 2]),
               __float_as_uint(__ldcg(&part[((size_t)row * nsl + s) * 2 + 1])));
  amax_block(best, bidx);
  if (threadIdx.x == 0) {
    if (pair) {
      pair[(size_t)row * 2] = best;
      pair[(size_t)row * 2 + 1] = __uint_as_float(bidx == 0xFFFFFFFFu ? bidx : bidx + v0);
    } else {
      out[row] = (int32_t)bidx;
    }
    cnt[row] = 0;
  }
}

// Merge the (maximum, index) pairs of `nranks` vocabulary shards, ranks in
// order: pairs[rank][row][2]. Shard r holds the indices [r vl, (r + 1) vl),
// so the first index of the maximum over the whole vocabulary wins ties.
__global__ void k_argmax_ranks(uint32_t rows, uint32_t nranks, const float *__restrict__ pairs,
                               int32_t *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float best = -INFINITY;
  uint32_t bidx = 0xFFFFFFFFu;
  for (uint32_t r = 0; r < nranks; r++)
    amax_merge(best, bidx, pairs[((size_t)r * rows + row) * 2], __float_as_uint(pairs[((size_t)r * rows + row) * 2 + 1]));
  out[row] = (int32_t)bidx;
}

// Tensor-parallel greedy pick over NVLink peer memory, without a
// collective library call. CTA (slice, row) scans its slice of this rank's
// vocabulary shard; the last slice of a row merges the row (first index of
// the maximum) into a staged pair; the last row to finish then stores every
// row's (maximum, index + v0) into slot [parity][rank] of every rank's
// landing buffer, adds one arrival to every rank's greedy counter, waits
// (bounded) until all ranks arrived, merges the ranks' pairs in rank order
// (shard r holds the indices [r vl, (r + 1) vl), so on equal values the
// lower rank's index wins: the first index over the whole vocabulary,
// models/sampler.c:89-99), writes the tokens, feeds them back as the next
// step's input and advances the position.
struct PeerPick {
  uint8_t *land[B200_TP_MAX_RANKS];
  uint32_t rank, nranks;
  uint64_t pairs_off;  // byte offset of the pair slots in a landing buffer
  int32_t *tok_out, *tok_in, *pos;
  uint32_t *err;
  uint64_t wait_ns;
};

__global__ void __launch_bounds__(256) k_argmax_peer(uint64_t n, uint64_t per, const float *__restrict__ logits,
                                                     float *__restrict__ part, uint32_t *__restrict__ cnt, uint32_t v0,
                                                     PeerPick a) {
  pdl_trigger();
  pdl_wait();
  const uint32_t row = blockIdx.y, rows = gridDim.y, slice = blockIdx.x, nsl = gridDim.x;
  const float *lr = logits + (size_t)row * n;
  const uint64_t lo = (uint64_t)slice * per, hi = min(n, lo + per);
  float best = -INFINITY;
  uint32_t bidx = 0xFFFFFFFFu;
  for (uint64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = lr[i];
    if (bidx == 0xFFFFFFFFu || v > best) {
      best = v;
      bidx = (uint32_t)i;
    }
  }
  amax_block(best, bidx);
  __shared__ uint32_t ticket;
  float *staged = part + (size_t)rows * nsl * 2;  // [row][2]: each row's merged pair
  if (threadIdx.x == 0) {
    part[((size_t)row * nsl + slice) * 2] = best;
    part[((size_t)row * nsl + slice) * 2 + 1] = __uint_as_float(bidx);
    __threadfence();
    ticket = atomicAdd(&cnt[row], 1u);
  }
  __syncthreads();
  if (ticket != nsl - 1) return;
  __threadfence();
  best = -INFINITY;
  bidx = 0xFFFFFFFFu;
  for (uint32_t s = threadIdx.x; s < nsl; s += blockDim.x)
    amax_merge(best, bidx, __ldcg(&part[((size_t)row * nsl + s) * 2]),
               __float_as_uint(__ldcg(&part[((size_t)row * nsl + s) * 2 + 1])));
  amax_block(best, bidx);
  if (threadIdx.x != 0) return;
  staged[row * 2] = best;
  staged[row * 2 + 1] = __uint_as_float(bidx == 0xFFFFFFFFu ? bidx : bidx + v0);
  cnt[row] = 0;
  __threadfence();
  if (atomicAdd(&cnt[rows], 1u) != rows - 1) return;
  // the last row: exchange all rows' pairs with the other ranks
  __threadfence();
  cnt[rows] = 0;
  uint64_t *mine = reinterpret_cast<uint64_t *>(a.land[a.rank]);
  const uint64_t done = *(volatile uint64_t *)(mine + 3), parity = done & 1u;
  for (uint32_t q = 0; q < a.nranks; q++) {
    float *dst = reinterpret_cast<float *>(a.land[q] + a.pairs_off) + ((parity * a.nranks + a.rank) * 8) * 2;
    for (uint32_t r = 0; r < rows; r++) {
      dst[r * 2] = __ldcg(&staged[r * 2]);
      dst[r * 2 + 1] = __ldcg(&staged[r * 2 + 1]);
    }
  }
  __threadfence_system();
  for (uint32_t q = 0; q < a.nranks; q++)
    atomicAdd_system(reinterpret_cast<unsigned long long *>(a.land[q]) + 2, 1ull);
  const uint64_t target = (done + 1) * a.nranks;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; it++) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(mine + 2) : "memory");
    if (v >= target) break;
    if ((it & 255u) == 0) {
      const uint64_t now = globaltimer_ns();
      if (it == 0) {
        t0 = now;
      } else if (now - t0 > a.wait_ns) {
        atomicExch(a.err, 1u);
        return;  // the position is not advanced: the step did not complete
      }
    }
  }
  const float *pairs = reinterpret_cast<const float *>(a.land[a.rank] + a.pairs_off) + (parity * a.nranks * 8) * 2;
  for (uint32_t r = 0; r < rows; r++) {
    float b = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t q = 0; q < a.nranks; q++)
      amax_merge(b, bi, __ldcg(&pairs[(q * 8 + r) * 2]), __float_as_uint(__ldcg(&pairs[(q * 8 + r) * 2 + 1])));
    a.tok_out[r] = (int32_t)bi;
    a.tok_in[r] = (int32_t)bi;
  }
  *a.pos += 1;
  mine[3] = done + 1;
}

// End of a device-resident decode step: advance the position and feed
// the chosen tokens back as the next step's input.
__global__ void k_step_tail(uint32_t batch, const int32_t *__restrict__ tok_out, int32_t *__restrict__ tok_in,
                            int32_t *__restrict__ pos) {
  pdl_trigger();
  pdl_wait();
  uint32_t i = threadIdx.x;
  if (i < batch) tok_in[i] = tok_out[i];
  if (i == 0) *pos += 1;
}

}  // namespace

extern "C" pai_status_t b200_launch_rmsnorm_xq(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, const float *a,
                                               const float *gamma, float eps, float *c, const b200_xq_t *xq) {
  if (eps == 0.0f) eps = 1e-5f;
  if (rows > 65535) return b200_fail(PAI_ERR_UNSUPPORTED, "rmsnorm: %llu rows (at most 65535)", (unsigned long long)rows);
  b200_xq_t q{};
  if (xq) q = *xq;
  // one 32-element block per warp, up to 256 CTAs per row; with many rows
  // (a prompt) one CTA per row already fills the GPU and reads each row once
  const uint64_t nblk = xq ? xq->quads * 4 : (n + 31) / 32;
  const uint64_t nsl = rows >= 64 ? 1 : std::max<uint64_t>(1, std::min<uint64_t>(256, (nblk + 3) / 4));
  const uint32_t bps = (uint32_t)((nblk + nsl - 1) / nsl);
  b200_launch(ctx, k_rmsnorm, dim3((unsigned)nsl, (unsigned)rows), dim3(kNormThreads), 0, (uint32_t)n, bps, a, gamma,
              eps, c, q);
  return b200_launched(ctx, 1, "k_rmsnorm");
}

extern "C" pai_status_t pai_b200_rmsnorm_gamma_f32(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n,
                                                   const float *a, const float *gamma, float eps, float *c) {
  if (!ctx || !a || !gamma || !c) return b200_fail(PAI_ERR_INVALID_ARG, "rmsnorm: NULL");
  if (rows == 0 || n == 0 || rows > 0x7FFFFFFFull || n > 0x7FFFFFFFull)
    return b200_fail(PAI_ERR_INVALID_ARG, "rmsnorm: shape");
  return b200_launch_rmsnorm_xq(ctx, rows, n, a, gamma, eps, c, nullptr);
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

extern "C" pai_status_t b200_launch_embed(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch, uint64_t rows,
                                          uint64_t k, const void *w, const int32_t *tokens, float *x) {
  const uint32_t nb = (uint32_t)(k / b200_blk_elems(type));
  const uint8_t *qs = (const uint8_t *)w;
  const uint8_t *sc = qs + b200_sc_offset(type, rows, k);
  b200_launch(ctx, k_embed, dim3(batch), dim3(128), 0, type, nb, (uint64_t)b200_ntiles(rows), qs, sc, tokens, x);
  return b200_launched(ctx, 1, "k_embed");
}

extern "C" pai_status_t b200_launch_argmax(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, const float *logits,
                                           int32_t *out) {
  // slices of at least 2048 logits, at most one per SM
  const uint64_t nsl = std::min<uint64_t>(148, (n + 2047) / 2048), per = (n + nsl - 1) / nsl;
  float *part = nullptr;
  uint32_t *cnt = nullptr;
  pai_status_t st = b200_ctx_scratch(ctx, rows * nsl * 2, (uint32_t)rows, &part, &cnt);
  if (st) return st;
  b200_launch(ctx, k_argmax, dim3((unsigned)nsl, (unsigned)rows), dim3(256), 0, n, per, logits, out, part, cnt,
              (float *)nullptr, 0u);
  return b200_launched(ctx, 1, "k_argmax");
}

extern "C" pai_status_t b200_launch_argmax_pair(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, uint32_t v0,
                                                const float *logits, float *pair) {
  const uint64_t nsl = std::min<uint64_t>(148, (n + 2047) / 2048), per = (n + nsl - 1) / nsl;
  float *part = nullptr;
  uint32_t *cnt = nullptr;
  pai_status_t st = b200_ctx_scratch(ctx, rows * nsl * 2, (uint32_t)rows, &part, &cnt);
  if (st) return st;
  b200_launch(ctx, k_argmax, dim3((unsigned)nsl, (unsigned)rows), dim3(256), 0, n, per, logits, (int32_t *)nullptr,
              part, cnt, pair, v0);
  return b200_launched(ctx, 1, "k_argmax");
}

extern "C" pai_status_t b200_launch_argmax_ranks(pai_b200_ctx_t *ctx, uint32_t rows, uint32_t nranks,
                                                 const float *pairs, int32_t *out) {
  b200_launch(ctx, k_argmax_ranks, dim3((rows + 31) / 32), dim3(32), 0, rows, nranks, pairs, out);
  return b200_launched(ctx, 1, "k_argmax_ranks");
}

extern "C" pai_status_t pai_b200_argmax_f32(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, const float *logits,
                                            int32_t *out) {
  if (!ctx || !logits || !out) return b200_fail(PAI_ERR_INVALID_ARG, "argmax: NULL");
  if (rows == 0 || n == 0 || n > 0xFFFFFFFEull) return b200_fail(PAI_ERR_INVALID_ARG, "argmax: shape");
  if (rows > 65535) return b200_fail(PAI_ERR_UNSUPPORTED, "argmax: %llu rows (at most 65535)", (unsigned long long)rows);
  return b200_launch_argmax(ctx, rows, n, logits, out);
}

extern "C" pai_status_t b200_launch_argmax_peer(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, uint32_t v0,
                                                const float *logits, void *const *land, uint64_t land_rows,
                                                uint32_t rank, uint32_t nranks, int32_t *tok_out, int32_t *tok_in,
                                                int32_t *pos) {
  if (rows == 0 || rows > 8 || nranks == 0 || nranks > B200_TP_MAX_RANKS || rank >= nranks || n == 0 ||
      n > 0xFFFFFFFEull || !land || !logits)
    return b200_fail(PAI_ERR_INVALID_ARG, "argmax_peer: rows %llu, rank %u of %u", (unsigned long long)rows, rank,
                     nranks);
  const uint64_t nsl = std::min<uint64_t>(148, (n + 2047) / 2048), per = (n + nsl - 1) / nsl;
  float *part = nullptr;
  uint32_t *cnt = nullptr;
  pai_status_t st = b200_ctx_scratch(ctx, rows * nsl * 2 + rows * 2, (uint32_t)rows + 1, &part, &cnt);
  if (st) return st;
  PeerPick a{};
  for (uint32_t r = 0; r < nranks; r++) {
    if (!land[r]) return b200_fail(PAI_ERR_INVALID_ARG, "argmax_peer: landing buffer of rank %u is NULL", r);
    a.land[r] = static_cast<uint8_t *>(land[r]);
  }
  a.rank = rank;
  a.nranks = nranks;
  a.tok_out = tok_out;
  a.tok_in = tok_in;
  a.pos = pos;
  a.err = b200_ctx_errflag(ctx);
  a.wait_ns = b200_ctx_wait_ns(ctx);
  // the pair slots follow the row slots of the landing buffers
  a.pairs_off = b200_land_pairs_off(nranks, land_rows);
  b200_launch(ctx, k_argmax_peer, dim3((unsigned)nsl, (unsigned)rows), dim3(256), 0, n, per, logits, part, cnt, v0, a);
  return b200_launched(ctx, 1, "k_argmax_peer");
}

extern "C" pai_status_t b200_launch_step_tail(pai_b200_ctx_t *ctx, uint32_t batch, int32_t *tok_out,
                                              int32_t *tok_in, int32_t *pos) {
  b200_launch(ctx, k_step_tail, dim3(1), dim3(32), 0, batch, tok_out, tok_in, pos);
  return b200_launched(ctx, 1, "k_step_tail");
}
