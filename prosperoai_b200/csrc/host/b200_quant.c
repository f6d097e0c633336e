/*
 * Host side of the weight formats: ggml block sizes, the block quantiser
 * (Q8_0 / Q4_0 / Q4_K), RoPE tables, and the upload+pack helper.
 *
 * Compiled as ISO C11 with -ffp-contract=off, like the reference, so the
 * quantiser's divisions, additions and lrintf roundings happen exactly
 * as written; the device quantiser (csrc/kernels/k_pack.cu) issues the
 * same IEEE operations and produces the same bytes.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "../b200_internal.h"

uint64_t pai_b200_block_bytes(uint32_t type, uint64_t numel) {
  if (!b200_type_ok(type) || numel % b200_blk_elems(type)) {
    return 0;
  }
  return numel / b200_blk_elems(type) * b200_blk_bytes(type);
}

/* IEEE binary16, round to nearest even. */
static uint16_t f32_to_f16(float f) {
  uint32_t x, sign, ex, mant;
  int32_t e;
  memcpy(&x, &f, 4);
  sign = (x >> 16) & 0x8000u;
  ex = (x >> 23) & 0xFFu;
  mant = x & 0x7FFFFFu;
  if (ex == 0xFFu) {
    return (uint16_t)(sign | 0x7C00u | (mant ? (0x200u | (mant >> 13)) : 0u));
  }
  e = (int32_t)ex - 112;
  if (e >= 31) {
    return (uint16_t)(sign | 0x7C00u);
  }
  if (e <= 0) {
    uint32_t full, shift, v, rem, half;
    if (e < -10) {
      return (uint16_t)sign;
    }
    full = mant | 0x800000u;
    shift = (uint32_t)(14 - e);
    v = full >> shift;
    rem = full & ((1u << shift) - 1u);
    half = 1u << (shift - 1u);
    v += (rem > half || (rem == half && (v & 1u))) ? 1u : 0u;
    return (uint16_t)(sign | v);
  } else {
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    h += (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ? 1u : 0u;
    return (uint16_t)h;
  }
}

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
  float f;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
      uint32_t ee = 113;
      while (!(m & 0x400u)) {
        m <<= 1;
        ee--;
      }
      bits = sign | (ee << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7F800000u | (m << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  memcpy(&f, &bits, 4);
  return f;
}

static void store_f16(uint8_t *p, uint16_t h) {
  p[0] = (uint8_t)(h & 0xFFu);
  p[1] = (uint8_t)(h >> 8);
}

static int clamp_round(float v, int lo, int hi) {
  long r = lrintf(v);
  return r < lo ? lo : (r > hi ? hi : (int)r);
}

static void quant_q8_0(const float *w, uint8_t *o) {
  float amax = 0.0f, d;
  for (int j = 0; j < 32; j++) {
    float a = fabsf(w[j]);
    amax = a > amax ? a : amax;
  }
  d = amax / 127.0f;
  store_f16(o, f32_to_f16(d));
  for (int j = 0; j < 32; j++) {
    o[2 + j] = (uint8_t)(int8_t)(d > 0.0f ? clamp_round(w[j] / d, -127, 127) : 0);
  }
}

static void quant_q4_0(const float *w, uint8_t *o) {
  float amax = 0.0f, m = 0.0f, d;
  uint8_t q[32];
  for (int j = 0; j < 32; j++) {
    float a = fabsf(w[j]);
    if (a > amax) {
      amax = a;
      m = w[j];
    }
  }
  d = m / -8.0f;
  store_f16(o, f32_to_f16(d));
  for (int j = 0; j < 32; j++) {
    int v = 8;
    if (d != 0.0f) {
      v = (int)lrintf(w[j] / d) + 8;
      v = v < 0 ? 0 : (v > 15 ? 15 : v);
    }
    q[j] = (uint8_t)v;
  }
  for (int j = 0; j < 16; j++) {
    o[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
  }
}

/* Q4_K: the inverse of get_scale_min_k4 (adapters/llama/gguf.c:640-648)
 * packs sub-block scales/mins 0..3 in the low 6 bits of bytes 0..3 / 4..7
 * and sub-blocks 4..7 as low nibbles in bytes 8..11 plus their top two
 * bits in the high bits of bytes 0..7. */
static void quant_q4_k(const float *w, uint8_t *o) {
  float S[8], M[8], maxS = 0.0f, maxM = 0.0f, df, dmf;
  int sc[8], mn[8];
  uint16_t d16, dm16;
  for (int s = 0; s < 8; s++) {
    float lo = 0.0f, hi = 0.0f;
    for (int l = 0; l < 32; l++) {
      float v = w[32 * s + l];
      lo = v < lo ? v : lo;
      hi = v > hi ? v : hi;
    }
    S[s] = (hi - lo) / 15.0f;
    M[s] = -lo;
    maxS = S[s] > maxS ? S[s] : maxS;
    maxM = M[s] > maxM ? M[s] : maxM;
  }
  d16 = f32_to_f16(maxS / 63.0f);
  dm16 = f32_to_f16(maxM / 63.0f);
  df = f16_to_f32(d16);
  dmf = f16_to_f32(dm16);
  store_f16(o, d16);
  store_f16(o + 2, dm16);
  for (int s = 0; s < 8; s++) {
    sc[s] = df > 0.0f ? clamp_round(S[s] / df, 0, 63) : 0;
    mn[s] = dmf > 0.0f ? clamp_round(M[s] / dmf, 0, 63) : 0;
  }
  for (int j = 0; j < 4; j++) {
    o[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    o[8 + j] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    o[12 + j] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
  }
  for (int c = 0; c < 4; c++) {
    float s0 = df * (float)sc[2 * c], f0 = dmf * (float)mn[2 * c];
    float s1 = df * (float)sc[2 * c + 1], f1 = dmf * (float)mn[2 * c + 1];
    for (int l = 0; l < 32; l++) {
      int q0 = s0 > 0.0f ? clamp_round((w[64 * c + l] + f0) / s0, 0, 15) : 0;
      int q1 = s1 > 0.0f ? clamp_round((w[64 * c + 32 + l] + f1) / s1, 0, 15) : 0;
      o[16 + 32 * c + l] = (uint8_t)(q0 | (q1 << 4));
    }
  }
}

pai_status_t pai_b200_quantize(uint32_t type, const float *src, uint64_t numel, void *dst) {
  uint64_t el, nb;
  uint8_t *o = (uint8_t *)dst;
  if ((!src || !dst) && numel) {
    return b200_fail(PAI_ERR_INVALID_ARG, "quantize: NULL");
  }
  if (!b200_type_ok(type)) {
    return b200_fail(PAI_ERR_UNSUPPORTED, "quantize: block type %u", type);
  }
  el = b200_blk_elems(type);
  if (numel % el) {
    return b200_fail(PAI_ERR_MISMATCH, "quantize: %llu elements is not a whole number of %llu-blocks",
                     (unsigned long long)numel, (unsigned long long)el);
  }
  nb = numel / el;
  for (uint64_t b = 0; b < nb; b++) {
    const float *w = src + b * el;
    uint8_t *ob = o + b * b200_blk_bytes(type);
    if (type == PAI_B200_Q8_0) {
      quant_q8_0(w, ob);
    } else if (type == PAI_B200_Q4_0) {
      quant_q4_0(w, ob);
    } else {
      quant_q4_k(w, ob);
    }
  }
  return PAI_OK;
}

/* pai_ref_rope_cossin_f32 (cpu/reference/ref_ops.c:260-279). */
pai_status_t pai_b200_rope_cossin_f32(uint64_t ctx_len, uint64_t r2, float base, float *cos_t, float *sin_t) {
  if (ctx_len == 0 || r2 == 0 || !cos_t || !sin_t) {
    return b200_fail(PAI_ERR_INVALID_ARG, "rope_cossin: invalid arguments");
  }
  if (base == 0.0f) {
    base = 10000.0f;
  }
  for (uint64_t p = 0; p < ctx_len; p++) {
    for (uint64_t i = 0; i < r2; i++) {
      double theta = (double)p * pow((double)base, -(2.0 * (double)i) / (2.0 * (double)r2));
      cos_t[p * r2 + i] = (float)cos(theta);
      sin_t[p * r2 + i] = (float)sin(theta);
    }
  }
  return PAI_OK;
}

pai_status_t pai_b200_upload_matrix(pai_b200_ctx_t *ctx, uint32_t type, uint64_t n, uint64_t k,
                                    const void *host_blocks, void *dst_packed) {
  uint64_t row_bytes = pai_b200_block_bytes(type, k);
  uint64_t *offs = NULL;
  void *dsrc = NULL, *doff = NULL;
  pai_status_t st;
  if (!ctx || !host_blocks || !dst_packed) {
    return b200_fail(PAI_ERR_INVALID_ARG, "upload_matrix: NULL");
  }
  if (!b200_type_ok(type)) {
    return b200_fail(PAI_ERR_UNSUPPORTED, "upload_matrix: block type %u", type);
  }
  if (n == 0 || row_bytes == 0) {
    return b200_fail(PAI_ERR_MISMATCH, "upload_matrix: shape %llu x %llu", (unsigned long long)n,
                     (unsigned long long)k);
  }
  offs = (uint64_t *)malloc(n * sizeof(uint64_t));
  if (!offs) {
    return b200_fail(PAI_ERR_NOMEM, "upload_matrix: host allocation");
  }
  for (uint64_t r = 0; r < n; r++) {
    offs[r] = r * row_bytes;
  }
  st = pai_b200_alloc(ctx, n * row_bytes, &dsrc);
  if (!st) st = pai_b200_alloc(ctx, n * sizeof(uint64_t), &doff);
  if (!st) st = pai_b200_memcpy_h2d(ctx, dsrc, host_blocks, n * row_bytes);
  if (!st) st = pai_b200_memcpy_h2d(ctx, doff, offs, n * sizeof(uint64_t));
  if (!st) st = pai_b200_pack(ctx, type, n, k, dsrc, (const uint64_t *)doff, dst_packed);
  if (!st) st = pai_b200_sync(ctx);
  pai_b200_free(ctx, dsrc);
  pai_b200_free(ctx, doff);
  free(offs);
  return st;
}
