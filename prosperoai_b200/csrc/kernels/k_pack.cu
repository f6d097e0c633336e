// Weight-format kernels: packing ggml blocks into the GEMV layout,
// bit-exact device dequantisation, the device block quantiser and the
// seeded synthetic-weight generator. All of these run once per model
// load; the per-token path only reads the packed layout.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace {

// One thread per (padded row, padded block): moves the block's header and
// quant bytes to their places in the packed layout (b200_internal.h), or
// writes zeros for padding rows, padding blocks and ROW_ZERO rows; rows
// marked ROW_SKIP belong to another source tensor and are left alone.
__global__ void k_pack(uint32_t type, uint64_t n, uint64_t npad, uint32_t nb, uint32_t nbpad, uint64_t ntiles,
                       const uint8_t *__restrict__ src, const uint64_t *__restrict__ row_off,
                       uint8_t *__restrict__ qs, uint8_t *__restrict__ sc) {
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t r = idx / nbpad;
  const uint32_t b = (uint32_t)(idx % nbpad);
  if (r >= npad) return;
  const uint64_t off = r < n ? row_off[r] : ~0ull;
  if (off == ~0ull - 1ull) return;  // row owned by another source tensor
  const uint32_t bb = b200_blk_bytes(type);
  const uint8_t *s = (off == ~0ull || b >= nb) ? nullptr : src + off + (uint64_t)b * bb;
  const uint32_t hdr = type == PAI_B200_Q4_K ? 16u : 2u, nq = bb - hdr;
  uint8_t *h = sc + pk_hdr_off(type, ntiles, r, b);
  for (uint32_t i = 0; i < hdr; i++) h[i] = s ? s[i] : 0;
  for (uint32_t j = 0; j < nq; j++) qs[pk_qs_off(type, ntiles, r, b, j)] = s ? s[hdr + j] : 0;
}

__global__ void k_dequant(uint32_t type, uint64_t n, uint32_t nb, uint64_t ntiles, const uint8_t *__restrict__ qs,
                          const uint8_t *__restrict__ sc, float *__restrict__ out) {
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t r = idx / nb;
  const uint32_t b = (uint32_t)(idx % nb);
  if (r >= n) return;
  const uint32_t el = b200_blk_elems(type);
  dequant_block_dev(type, ntiles, qs, sc, r, b, out + r * (uint64_t)nb * el + (uint64_t)b * el);
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__device__ __forceinline__ void put_f16(uint8_t *p, float f) {
  uint16_t h = __half_as_ushort(__float2half_rn(f));
  p[0] = (uint8_t)(h & 0xFF);
  p[1] = (uint8_t)(h >> 8);
}

// Device block quantiser: the same formulas and rounding steps as the
// host quantiser (csrc/host/b200_quant.c), with IEEE division and
// round-half-even conversion (lrintf) so both produce identical bytes.
__global__ void k_quantize(uint32_t type, uint64_t nblocks, const float *__restrict__ src,
                           uint8_t *__restrict__ dst) {
  uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  if (type == PAI_B200_Q8_0) {
    const float *s = src + b * 32;
    uint8_t *o = dst + b * 34;
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(s[j]));
    float d = __fdiv_rn(amax, 127.0f);
    put_f16(o, d);
    for (int j = 0; j < 32; j++) {
      int q = d > 0.0f ? clampi(__float2int_rn(__fdiv_rn(s[j], d)), -127, 127) : 0;
      o[2 + j] = (uint8_t)(int8_t)q;
    }
  } else if (type == PAI_B200_Q4_0) {
    const float *s = src + b * 32;
    uint8_t *o = dst + b * 18;
    float amax = 0.0f, m = 0.0f;
    for (int j = 0; j < 32; j++) {
      float a = fabsf(s[j]);
      if (a > amax) {
        amax = a;
        m = s[j];
      }
    }
    float d = __fdiv_rn(m, -8.0f);
    put_f16(o, d);
    int q[32];
    for (int j = 0; j < 32; j++) q[j] = d != 0.0f ? clampi(__float2int_rn(__fdiv_rn(s[j], d)) + 8, 0, 15) : 8;
    for (int j = 0; j < 16; j++) o[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
  } else {
    const float *s = src + b * 256;
    uint8_t *o = dst + b * 144;
    float S[8], M[8], maxS = 0.0f, maxM = 0.0f;
    for (int t = 0; t < 8; t++) {
      float lo = 0.0f, hi = 0.0f;
      for (int l = 0; l < 32; l++) {
        float v = s[32 * t + l];
        lo = v < lo ? v : lo;
        hi = v > hi ? v : hi;
      }
      S[t] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
      M[t] = -lo;
      maxS = S[t] > maxS ? S[t] : maxS;
      maxM = M[t] > maxM ? M[t] : maxM;
    }
    __half d16 = __float2half_rn(__fdiv_rn(maxS, 63.0f));
    __half dm16 = __float2half_rn(__fdiv_rn(maxM, 63.0f));
    float df = __half2float(d16), dmf = __half2float(dm16);
    uint16_t db = __half_as_ushort(d16), dmb = __half_as_ushort(dm16);
    o[0] = db & 0xFF; o[1] = db >> 8; o[2] = dmb & 0xFF; o[3] = dmb >> 8;
    int sc[8], mn[8];
    for (int t = 0; t < 8; t++) {
      sc[t] = df > 0.0f ? clampi(__float2int_rn(__fdiv_rn(S[t], df)), 0, 63) : 0;
      mn[t] = dmf > 0.0f ? clampi(__float2int_rn(__fdiv_rn(M[t], dmf)), 0, 63) : 0;
    }
    for (int j = 0; j < 4; j++) {
      o[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
      o[8 + j] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
      o[12 + j] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    for (int c = 0; c < 4; c++) {
      int t0 = 2 * c, t1 = 2 * c + 1;
      float sc0 = __fmul_rn(df, (float)sc[t0]), of0 = __fmul_rn(dmf, (float)mn[t0]);
      float sc1 = __fmul_rn(df, (float)sc[t1]), of1 = __fmul_rn(dmf, (float)mn[t1]);
      for (int l = 0; l < 32; l++) {
        float v0 = s[64 * c + l], v1 = s[64 * c + 32 + l];
        int q0 = sc0 > 0.0f ? clampi(__float2int_rn(__fdiv_rn(__fadd_rn(v0, of0), sc0)), 0, 15) : 0;
        int q1 = sc1 > 0.0f ? clampi(__float2int_rn(__fdiv_rn(__fadd_rn(v1, of1), sc1)), 0, 15) : 0;
        o[16 + 32 * c + l] = (uint8_t)(q0 | (q1 << 4));
      }
    }
  }
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Seeded N(0, std) rows: row r is the splitmix64 stream started at
// mix64(seed + r); pair j draws outputs 2j and 2j+1 of that stream and
// turns them into two normals by Box-Muller in double precision.
__global__ void k_synth_normal(float *__restrict__ dst, uint64_t rows, uint64_t cols, uint64_t seed,
                               double stddev) {
  const uint64_t pairs = (cols + 1) / 2;
  uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * pairs) return;
  uint64_t r = idx / pairs, j = idx % pairs;
  const uint64_t gamma = 0x9E3779B97F4A7C15ull;
  uint64_t st = mix64(seed + r);
  uint64_t x1 = mix64(st + (2 * j + 1) * gamma);
  uint64_t x2 = mix64(st + (2 * j + 2) * gamma);
  double u1 = __dmul_rn((double)((x1 >> 11) + 1), 0x1.0p-53);
  double u2 = __dmul_rn((double)(x2 >> 11), 0x1.0p-53);
  double rad = sqrt(__dmul_rn(-2.0, log(u1)));
  double t = __dmul_rn(6.283185307179586, u2);
  double sr = __dmul_rn(stddev, rad);
  float *o = dst + r * cols + 2 * j;
  o[0] = (float)__dmul_rn(sr, cos(t));
  if (2 * j + 1 < cols) o[1] = (float)__dmul_rn(sr, sin(t));
}

__global__ void k_fill(float *dst, uint64_t n, float v) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = v;
}

inline unsigned nblk(uint64_t work, unsigned t) { return (unsigned)((work + t - 1) / t); }

}  // namespace

extern "C" uint64_t pai_b200_packed_bytes(uint32_t type, uint64_t n, uint64_t k) {
  if (!b200_type_ok(type) || n == 0 || k == 0 || k % b200_blk_elems(type)) return 0;
  return b200_sc_offset(type, n, k) + b200_align256(b200_ntiles(n) * b200_units(type, k) * b200_unit_sc_bytes(type));
}

extern "C" pai_status_t pai_b200_pack(pai_b200_ctx_t *ctx, uint32_t type, uint64_t n, uint64_t k,
                                      const void *src, const uint64_t *row_off, void *dst) {
  if (!ctx || !src || !row_off || !dst) return b200_fail(PAI_ERR_INVALID_ARG, "pack: NULL");
  if (!b200_type_ok(type)) return b200_fail(PAI_ERR_UNSUPPORTED, "pack: block type %u", type);
  if (n == 0 || k == 0 || k % b200_blk_elems(type))
    return b200_fail(PAI_ERR_MISMATCH, "pack: k=%llu not a multiple of %u", (unsigned long long)k,
                     b200_blk_elems(type));
  if ((uintptr_t)dst & 255) return b200_fail(PAI_ERR_INVALID_ARG, "pack: destination not 256-byte aligned");
  const uint32_t nb = (uint32_t)(k / b200_blk_elems(type));
  const uint32_t nbpad = (uint32_t)(b200_units(type, k) * b200_unit_blocks(type));
  const uint64_t ntiles = b200_ntiles(n), npad = ntiles * B200_TILE;
  uint8_t *qs = (uint8_t *)dst;
  uint8_t *sc = qs + b200_sc_offset(type, n, k);
  cudaStream_t s = (cudaStream_t)b200_ctx_stream(ctx);
  k_pack<<<nblk(npad * nbpad, 256), 256, 0, s>>>(type, n, npad, nb, nbpad, ntiles, (const uint8_t *)src, row_off,
                                                 qs, sc);
  return b200_launched(ctx, 1, "k_pack");
}

extern "C" pai_status_t pai_b200_dequant(pai_b200_ctx_t *ctx, uint32_t type, uint64_t n, uint64_t k,
                                         const void *packed, float *out) {
  if (!ctx || !packed || !out) return b200_fail(PAI_ERR_INVALID_ARG, "dequant: NULL");
  if (!b200_type_ok(type)) return b200_fail(PAI_ERR_UNSUPPORTED, "dequant: block type %u", type);
  if (n == 0 || k == 0 || k % b200_blk_elems(type)) return b200_fail(PAI_ERR_MISMATCH, "dequant: shape");
  const uint32_t nb = (uint32_t)(k / b200_blk_elems(type));
  const uint8_t *qs = (const uint8_t *)packed;
  const uint8_t *sc = qs + b200_sc_offset(type, n, k);
  k_dequant<<<nblk(n * nb, 128), 128, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(type, n, nb, b200_ntiles(n), qs,
                                                                                 sc, out);
  return b200_launched(ctx, 1, "k_dequant");
}

extern "C" pai_status_t b200_launch_quantize(pai_b200_ctx_t *ctx, uint32_t type, const float *src,
                                             uint64_t numel, void *dst) {
  uint64_t nb = numel / b200_blk_elems(type);
  k_quantize<<<nblk(nb, 128), 128, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(type, nb, src, (uint8_t *)dst);
  return b200_launched(ctx, 1, "k_quantize");
}

extern "C" pai_status_t b200_launch_synth_normal(pai_b200_ctx_t *ctx, float *dst, uint64_t rows,
                                                 uint64_t cols, uint64_t seed, float stddev) {
  uint64_t work = rows * ((cols + 1) / 2);
  k_synth_normal<<<nblk(work, 256), 256, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(dst, rows, cols, seed,
                                                                                     (double)stddev);
  return b200_launched(ctx, 1, "k_synth_normal");
}

extern "C" pai_status_t b200_launch_fill(pai_b200_ctx_t *ctx, float *dst, uint64_t n, float v) {
  k_fill<<<nblk(n, 256), 256, 0, (cudaStream_t)b200_ctx_stream(ctx)>>>(dst, n, v);
  return b200_launched(ctx, 1, "k_fill");
}
