// Fused dequantise-and-dot GEMV over the packed Q4_0 / Q8_0 / Q4_K layout.
//
// Mapping: one CTA = one group of 32 output rows x a contiguous range of
// K blocks; lane l of every warp owns row l of the group, the 8 warps
// stride over the CTA's blocks. Each lane reads its row's block with
// 128-bit loads that are coalesced across the warp (the packed layout
// puts chunk c of the 32 rows of a group side by side), unpacks nibbles
// or bytes to exact fp32 in registers, and accumulates sum_j q_j * x_j
// per block before applying the block scale once. x for the CTA's
// K-range is staged in shared memory and read as warp-wide broadcasts.
// Warps are reduced through shared memory in a fixed order; when K is
// split across several CTAs, each writes its partial row sums to scratch
// and the last CTA to arrive (an atomic ticket per row group) adds them
// in split order and applies the epilogue, so results do not depend on
// scheduling.
//
// Reference semantics: y = W.x with W = dequant_block(...) rows
// (adapters/llama/gguf.c:680-693, 750-761, 852-882) and the dot of
// pai_ref_gemv_f32 (cpu/reference/ref_ops.c:92-106); the epilogues fuse
// the executor's residual PAI_OP_ADD and the SILU -> MUL pair of the
// LLaMA MLP (adapters/llama/llama.c:747-749, 774-795).
#include <cuda_runtime.h>

#include <algorithm>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct GemvParams {
  const uint8_t *qs;
  const uint8_t *sc;
  const float *x;    // [batch][k]
  const float *res;  // [batch][n] or null
  float *y;
  float *partial;    // [kcta][batch][npad]
  uint32_t *counters;
  uint32_t n, k, nb, ngroups, kcta, bpc, npad;
  int epi;
};

// Magic constants: a 0..255 field OR'ed into the mantissa of 2^23 gives
// the exact float 2^23 + v; subtracting 2^23 + bias leaves v - bias.
constexpr float kM = 8388608.0f;

// byte i of w (i = 0..3) placed in bits 0..7 of 0x4B000000
__device__ __forceinline__ float byte_f(uint32_t w, int i, float bias) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + (uint32_t)i)) - bias;
}

template <uint32_t T>
struct Block;

// Q4_0: 16 bytes of nibbles; byte j holds element j (low) and j+16 (high).
template <>
struct Block<PAI_B200_Q4_0> {
  static constexpr uint32_t EL = 32, CH = 1, U = 4;
  struct Raw {
    uint4 q;
    uint16_t d;
  };
  __device__ static void load(const GemvParams &p, uint32_t g, uint32_t b, int lane, Raw &r) {
    size_t tile = (size_t)g * p.nb + b;
    r.q = ldg_stream(p.qs + (tile * 32 + lane) * 16);
    r.d = ldg_u16(p.sc + (tile * 32 + lane) * 2);
  }
  template <int B>
  __device__ static void dot(const Raw &r, const float *xb, uint32_t xstride, float (&acc)[B]) {
    float w[32];
    const uint32_t q[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
#pragma unroll
    for (int wi = 0; wi < 4; wi++) {
      uint32_t lo = q[wi] & 0x0F0F0F0Fu;
      uint32_t hi = (q[wi] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        w[4 * wi + i] = byte_f(lo, i, kM + 8.0f);
        w[16 + 4 * wi + i] = byte_f(hi, i, kM + 8.0f);
      }
    }
    float d = __half2float(__ushort_as_half(r.d));
#pragma unroll
    for (int bi = 0; bi < B; bi++) {
      const float4 *x4 = reinterpret_cast<const float4 *>(xb + bi * xstride);
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        float4 a = x4[j], c = x4[j + 1];
        s0 = fmaf(w[4 * j + 0], a.x, s0);
        s0 = fmaf(w[4 * j + 1], a.y, s0);
        s0 = fmaf(w[4 * j + 2], a.z, s0);
        s0 = fmaf(w[4 * j + 3], a.w, s0);
        s1 = fmaf(w[4 * j + 4], c.x, s1);
        s1 = fmaf(w[4 * j + 5], c.y, s1);
        s1 = fmaf(w[4 * j + 6], c.z, s1);
        s1 = fmaf(w[4 * j + 7], c.w, s1);
      }
      acc[bi] = fmaf(d, s0 + s1, acc[bi]);
    }
  }
};

// Q8_0: 32 signed bytes in two chunks.
template <>
struct Block<PAI_B200_Q8_0> {
  static constexpr uint32_t EL = 32, CH = 2, U = 2;
  struct Raw {
    uint4 q[2];
    uint16_t d;
  };
  __device__ static void load(const GemvParams &p, uint32_t g, uint32_t b, int lane, Raw &r) {
    size_t tile = (size_t)g * p.nb + b;
    r.q[0] = ldg_stream(p.qs + ((tile * 2 + 0) * 32 + lane) * 16);
    r.q[1] = ldg_stream(p.qs + ((tile * 2 + 1) * 32 + lane) * 16);
    r.d = ldg_u16(p.sc + (tile * 32 + lane) * 2);
  }
  template <int B>
  __device__ static void dot(const Raw &r, const float *xb, uint32_t xstride, float (&acc)[B]) {
    float w[32];
#pragma unroll
    for (int c = 0; c < 2; c++) {
      const uint32_t q[4] = {r.q[c].x ^ 0x80808080u, r.q[c].y ^ 0x80808080u, r.q[c].z ^ 0x80808080u,
                             r.q[c].w ^ 0x80808080u};
#pragma unroll
      for (int wi = 0; wi < 4; wi++)
#pragma unroll
        for (int i = 0; i < 4; i++) w[16 * c + 4 * wi + i] = byte_f(q[wi], i, kM + 128.0f);
    }
    float d = __half2float(__ushort_as_half(r.d));
#pragma unroll
    for (int bi = 0; bi < B; bi++) {
      const float4 *x4 = reinterpret_cast<const float4 *>(xb + bi * xstride);
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        float4 a = x4[j], c = x4[j + 1];
        s0 = fmaf(w[4 * j + 0], a.x, s0);
        s0 = fmaf(w[4 * j + 1], a.y, s0);
        s0 = fmaf(w[4 * j + 2], a.z, s0);
        s0 = fmaf(w[4 * j + 3], a.w, s0);
        s1 = fmaf(w[4 * j + 4], c.x, s1);
        s1 = fmaf(w[4 * j + 5], c.y, s1);
        s1 = fmaf(w[4 * j + 6], c.z, s1);
        s1 = fmaf(w[4 * j + 7], c.w, s1);
      }
      acc[bi] = fmaf(d, s0 + s1, acc[bi]);
    }
  }
};

// Q4_K: 128 bytes of nibbles in 8 chunks plus a 16-byte header
// {d, dmin, scales[12]}. Chunk t holds bytes 16t..16t+15 of qs; byte l
// of 64-group c = t/2 holds element 64c+l (sub-block 2c, low nibble) and
// 64c+32+l (sub-block 2c+1, high nibble). Per sub-block s the weight is
// (d*sc_s)*q - dmin*m_s, so W.x = sum_s d*sc_s * (q.x)_s - dmin*m_s * (sum x)_s,
// with the sub-block sums of x precomputed when x is staged.
template <>
struct Block<PAI_B200_Q4_K> {
  static constexpr uint32_t EL = 256, CH = 8, U = 1;
  struct Raw {
    uint4 q[8];
    uint4 h;
  };
  __device__ static void load(const GemvParams &p, uint32_t g, uint32_t b, int lane, Raw &r) {
    size_t tile = (size_t)g * p.nb + b;
#pragma unroll
    for (int c = 0; c < 8; c++) r.q[c] = ldg_stream(p.qs + ((tile * 8 + c) * 32 + lane) * 16);
    r.h = ldg_stream(p.sc + (tile * 32 + lane) * 16);
  }
  template <int B>
  __device__ static void dot(const Raw &r, const float *xb, uint32_t xstride, const float *xsum,
                             uint32_t sstride, float (&acc)[B]) {
    float d = __half2float(__ushort_as_half((uint16_t)(r.h.x & 0xFFFFu)));
    float dmin = __half2float(__ushort_as_half((uint16_t)(r.h.x >> 16)));
    uint8_t s12[12];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      s12[i] = (uint8_t)(r.h.y >> (8 * i));
      s12[4 + i] = (uint8_t)(r.h.z >> (8 * i));
      s12[8 + i] = (uint8_t)(r.h.w >> (8 * i));
    }
    float dsc[8], dmm[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      uint8_t s, m;
      k4_scale_min(j, s12, &s, &m);
      dsc[j] = d * (float)s;
      dmm[j] = dmin * (float)m;
    }
#pragma unroll
    for (int bi = 0; bi < B; bi++) {
      const float *xr = xb + bi * xstride;
      float tot = 0.f;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        float slo = 0.f, shi = 0.f;
#pragma unroll
        for (int half = 0; half < 2; half++) {
          const uint4 qq = r.q[2 * c + half];
          const uint32_t q[4] = {qq.x, qq.y, qq.z, qq.w};
          const float4 *xl = reinterpret_cast<const float4 *>(xr + 64 * c + 16 * half);
          const float4 *xh = reinterpret_cast<const float4 *>(xr + 64 * c + 32 + 16 * half);
#pragma unroll
          for (int wi = 0; wi < 4; wi++) {
            uint32_t lo = q[wi] & 0x0F0F0F0Fu, hi = (q[wi] >> 4) & 0x0F0F0F0Fu;
            float4 a = xl[wi], e = xh[wi];
            slo = fmaf(byte_f(lo, 0, kM), a.x, slo);
            slo = fmaf(byte_f(lo, 1, kM), a.y, slo);
            slo = fmaf(byte_f(lo, 2, kM), a.z, slo);
            slo = fmaf(byte_f(lo, 3, kM), a.w, slo);
            shi = fmaf(byte_f(hi, 0, kM), e.x, shi);
            shi = fmaf(byte_f(hi, 1, kM), e.y, shi);
            shi = fmaf(byte_f(hi, 2, kM), e.z, shi);
            shi = fmaf(byte_f(hi, 3, kM), e.w, shi);
          }
        }
        const float *xs8 = xsum + bi * sstride;
        tot = fmaf(dsc[2 * c], slo, tot);
        tot = fmaf(dsc[2 * c + 1], shi, tot);
        tot = fmaf(-dmm[2 * c], xs8[2 * c], tot);
        tot = fmaf(-dmm[2 * c + 1], xs8[2 * c + 1], tot);
      }
      acc[bi] += tot;
    }
  }
};

template <uint32_t T, int B>
__global__ void __launch_bounds__(kThreads, 2) k_gemv(GemvParams p) {
  using Blk = Block<T>;
  constexpr uint32_t EL = Blk::EL, U = Blk::U;
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[kWarps][B][32];
  __shared__ int is_last;

  const uint32_t g = blockIdx.x, ks = blockIdx.y;
  const uint32_t b0 = ks * p.bpc;
  const uint32_t b1 = min(p.nb, b0 + p.bpc);
  const uint32_t nblk = b1 - b0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t xstride = p.bpc * EL;
  float *xsum = xs + B * xstride;  // Q4_K: [B][bpc*8] sub-block sums

  // Stage this CTA's K-range of x (all batch rows).
  for (int bi = 0; bi < B; bi++) {
    const float4 *src = reinterpret_cast<const float4 *>(p.x + (size_t)bi * p.k + (size_t)b0 * EL);
    float4 *dst = reinterpret_cast<float4 *>(xs + bi * xstride);
    for (uint32_t i = threadIdx.x; i < nblk * EL / 4; i += kThreads) dst[i] = src[i];
  }
  if constexpr (T == PAI_B200_Q4_K) {
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < B * nblk * 8; i += kThreads) {
      uint32_t bi = i / (nblk * 8), j = i % (nblk * 8);
      const float *v = xs + bi * xstride + j * 32;
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 32; e++) s += v[e];
      xsum[bi * p.bpc * 8 + j] = s;
    }
  }
  __syncthreads();

  float acc[B];
#pragma unroll
  for (int bi = 0; bi < B; bi++) acc[bi] = 0.f;

  for (uint32_t base = b0 + warp; base < b1; base += kWarps * U) {
    typename Blk::Raw raw[U];
#pragma unroll
    for (uint32_t u = 0; u < U; u++) {
      uint32_t b = base + u * kWarps;
      if (b < b1) Blk::load(p, g, b, lane, raw[u]);
    }
#pragma unroll
    for (uint32_t u = 0; u < U; u++) {
      uint32_t b = base + u * kWarps;
      if (b < b1) {
        const float *xb = xs + (b - b0) * EL;
        if constexpr (T == PAI_B200_Q4_K)
          Blk::template dot<B>(raw[u], xb, xstride, xsum + (b - b0) * 8, p.bpc * 8, acc);
        else
          Blk::template dot<B>(raw[u], xb, xstride, acc);
      }
    }
  }

#pragma unroll
  for (int bi = 0; bi < B; bi++) red[warp][bi][lane] = acc[bi];
  __syncthreads();
  if (warp != 0) {
    if (p.kcta == 1) return;
  }
  float vals[B];
  if (warp == 0) {
#pragma unroll
    for (int bi = 0; bi < B; bi++) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; w++) v += red[w][bi][lane];
      vals[bi] = v;
    }
  }
  if (p.kcta > 1) {
    if (warp == 0) {
#pragma unroll
      for (int bi = 0; bi < B; bi++)
        p.partial[((size_t)ks * B + bi) * p.npad + (size_t)g * 32 + lane] = vals[bi];
      __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t prev = atomicAdd(&p.counters[g], 1u);
      is_last = (prev == p.kcta - 1);
    }
    __syncthreads();
    if (!is_last || warp != 0) return;
    __threadfence();
#pragma unroll
    for (int bi = 0; bi < B; bi++) {
      float v = 0.f;
      for (uint32_t s = 0; s < p.kcta; s++) v += __ldcg(&p.partial[((size_t)s * B + bi) * p.npad + (size_t)g * 32 + lane]);
      vals[bi] = v;
    }
    if (lane == 0) p.counters[g] = 0;
  }

  // Epilogue (warp 0 of the finishing CTA).
  const uint32_t row = g * 32 + lane;
  if (p.epi == B200_EPI_SILU_GLU) {
    const uint32_t nout = p.n / 2;
#pragma unroll
    for (int bi = 0; bi < B; bi++) {
      float up = __shfl_down_sync(0xffffffffu, vals[bi], 16);
      uint32_t orow = g * 16 + lane;
      if (lane < 16 && orow < nout) {
        float gate = vals[bi];
        float sg = __fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate)));
        p.y[(size_t)bi * nout + orow] = __fmul_rn(sg, up);
      }
    }
  } else if (row < p.n) {
#pragma unroll
    for (int bi = 0; bi < B; bi++) {
      float v = vals[bi];
      if (p.epi == B200_EPI_RESIDUAL) v = __fadd_rn(p.res[(size_t)bi * p.n + row], v);
      p.y[(size_t)bi * p.n + row] = v;
    }
  }
}

template <uint32_t T, int B>
pai_status_t launch_t(pai_b200_ctx_t *ctx, GemvParams p, int num_sms) {
  constexpr uint32_t EL = Block<T>::EL;
  auto kern = k_gemv<T, B>;
  // K split: aim for ~3 resident CTAs per SM, with at least 2 blocks per
  // warp (Q4_K: 1) and x staging within 96 KB of shared memory.
  const uint32_t min_bpc = (T == PAI_B200_Q4_K) ? kWarps : 2 * kWarps;
  const uint32_t per_blk_smem = B * EL * 4 + (T == PAI_B200_Q4_K ? B * 8 * 4 : 0);
  const uint32_t max_bpc = std::max<uint32_t>(1, (96u * 1024u) / per_blk_smem);
  uint32_t target = (uint32_t)num_sms * 3;
  uint32_t kcta = (target + p.ngroups - 1) / p.ngroups;
  kcta = std::min<uint32_t>(kcta, std::max<uint32_t>(1, p.nb / min_bpc));
  uint32_t bpc = (p.nb + kcta - 1) / kcta;
  if (bpc > max_bpc) bpc = max_bpc;
  kcta = (p.nb + bpc - 1) / bpc;
  p.bpc = bpc;
  p.kcta = kcta;
  size_t smem = (size_t)bpc * per_blk_smem;
  if (kcta > 1) {
    pai_status_t st = b200_ctx_scratch(ctx, (uint64_t)kcta * B * p.npad, p.ngroups, &p.partial, &p.counters);
    if (st) return st;
  }
  static bool attr_set = false;
  if (!attr_set) {
    pai_status_t st = b200_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024),
                                "k_gemv smem attribute");
    if (st) return st;
    attr_set = true;
  }
  dim3 grid(p.ngroups, kcta);
  kern<<<grid, kThreads, smem, (cudaStream_t)b200_ctx_stream(ctx)>>>(p);
  return b200_launched(ctx, 1, "k_gemv");
}

template <uint32_t T>
pai_status_t launch_b(pai_b200_ctx_t *ctx, GemvParams p, uint32_t batch, int sms) {
  switch (batch) {
    case 1: return launch_t<T, 1>(ctx, p, sms);
    case 2: return launch_t<T, 2>(ctx, p, sms);
    case 4: return launch_t<T, 4>(ctx, p, sms);
    case 8: return launch_t<T, 8>(ctx, p, sms);
    default: return b200_fail(PAI_ERR_UNSUPPORTED, "gemv: batch %u (1, 2, 4 or 8)", batch);
  }
}

int sm_count(pai_b200_ctx_t *ctx) {
  static int cached[64];
  int dev = b200_ctx_device(ctx);
  if (dev < 64 && cached[dev]) return cached[dev];
  int v = 148;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = v;
  return v;
}

}  // namespace

extern "C" pai_status_t b200_launch_gemv(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch, uint64_t n,
                                         uint64_t k, const void *w, const float *x, const float *residual,
                                         float *y, int epi) {
  if (!ctx || !w || !x || !y) return b200_fail(PAI_ERR_INVALID_ARG, "gemv: NULL pointer");
  if (!b200_type_ok(type)) return b200_fail(PAI_ERR_UNSUPPORTED, "gemv: block type %u", type);
  if (n == 0 || k == 0 || k % b200_blk_elems(type))
    return b200_fail(PAI_ERR_MISMATCH, "gemv: k=%llu is not a whole number of %u-element blocks",
                     (unsigned long long)k, b200_blk_elems(type));
  if (n > 0xFFFFFFFFull || k > 0x7FFFFFFFull) return b200_fail(PAI_ERR_UNSUPPORTED, "gemv: shape too large");
  if (epi == B200_EPI_RESIDUAL && !residual) return b200_fail(PAI_ERR_INVALID_ARG, "gemv: NULL residual");
  if (epi == B200_EPI_SILU_GLU && n % 32) return b200_fail(PAI_ERR_MISMATCH, "gemv: gate/up rows must be 32-aligned");
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 255)) return b200_fail(PAI_ERR_INVALID_ARG, "gemv: misaligned x or w");
  GemvParams p{};
  p.qs = (const uint8_t *)w;
  p.sc = p.qs + b200_sc_offset(type, n, k);
  p.x = x;
  p.res = residual;
  p.y = y;
  p.n = (uint32_t)n;
  p.k = (uint32_t)k;
  p.nb = (uint32_t)(k / b200_blk_elems(type));
  p.ngroups = (uint32_t)b200_ngroups(n);
  p.npad = p.ngroups * 32;
  p.epi = epi;
  int sms = sm_count(ctx);
  switch (type) {
    case PAI_B200_Q4_0: return launch_b<PAI_B200_Q4_0>(ctx, p, batch, sms);
    case PAI_B200_Q8_0: return launch_b<PAI_B200_Q8_0>(ctx, p, batch, sms);
    default: return launch_b<PAI_B200_Q4_K>(ctx, p, batch, sms);
  }
}

extern "C" pai_status_t pai_b200_gemv_f32(pai_b200_ctx_t *ctx, uint32_t type, uint64_t batch, uint64_t n,
                                          uint64_t k, const void *w, const float *x, const float *residual,
                                          float *y) {
  if (batch == 0 || batch > 0xFFFFFFFFull) return b200_fail(PAI_ERR_INVALID_ARG, "gemv: batch");
  return b200_launch_gemv(ctx, type, (uint32_t)batch, n, k, w, x, residual, y,
                          residual ? B200_EPI_RESIDUAL : B200_EPI_STORE);
}

extern "C" pai_status_t pai_b200_gemv_q8_0_f32(pai_b200_ctx_t *ctx, uint64_t n, uint64_t k, const void *w,
                                               const float *x, float *y) {
  return b200_launch_gemv(ctx, PAI_B200_Q8_0, 1, n, k, w, x, nullptr, y, B200_EPI_STORE);
}
extern "C" pai_status_t pai_b200_gemv_q4_0_f32(pai_b200_ctx_t *ctx, uint64_t n, uint64_t k, const void *w,
                                               const float *x, float *y) {
  return b200_launch_gemv(ctx, PAI_B200_Q4_0, 1, n, k, w, x, nullptr, y, B200_EPI_STORE);
}
extern "C" pai_status_t pai_b200_gemv_q4_k_f32(pai_b200_ctx_t *ctx, uint64_t n, uint64_t k, const void *w,
                                               const float *x, float *y) {
  return b200_launch_gemv(ctx, PAI_B200_Q4_K, 1, n, k, w, x, nullptr, y, B200_EPI_STORE);
}
