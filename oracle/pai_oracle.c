/*
 * pai_oracle — CPU restatement of ProsperoAI's quantized-weights hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never part of
 * it. See pai_oracle.h for the contract; each function cites the
 * reference file:line whose operation order it keeps.
 */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "pai_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- fp16 ---------------------------------------------------------------- */

/* adapters/llama/gguf.c:602-630: subnormals are normalised by shifting
 * the mantissa until the implicit bit appears. */
float po_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  uint32_t bits;
  float f;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
      uint32_t ee = 113; /* 127 - 15 + 1 */
      while ((m & 0x400u) == 0) {
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

uint16_t po_f32_to_f16(float f) {
  uint32_t x;
  uint32_t sign, exp, mant;
  int32_t e;
  memcpy(&x, &f, 4);
  sign = (x >> 16) & 0x8000u;
  exp = (x >> 23) & 0xFFu;
  mant = x & 0x7FFFFFu;
  if (exp == 0xFFu) {
    return (uint16_t)(sign | 0x7C00u | (mant ? (0x200u | (mant >> 13)) : 0u));
  }
  e = (int32_t)exp - 112; /* rebias 127 -> 15 */
  if (e >= 31) {
    return (uint16_t)(sign | 0x7C00u);
  }
  if (e <= 0) {
    uint32_t full, shift, q, rem, half;
    if (e < -10) {
      return (uint16_t)sign;
    }
    full = mant | 0x800000u;
    shift = (uint32_t)(14 - e);
    q = full >> shift;
    rem = full & ((1u << shift) - 1u);
    half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) {
      q++;
    }
    return (uint16_t)(sign | q);
  }
  {
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) {
      h++;
    }
    return (uint16_t)h;
  }
}

static float le_f16(const uint8_t *p) {
  return po_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
}

static void put_f16(uint8_t *p, uint16_t h) {
  p[0] = (uint8_t)(h & 0xFFu);
  p[1] = (uint8_t)(h >> 8);
}

/* ---- block formats ------------------------------------------------------- */

uint64_t po_type_bytes(uint32_t type, uint64_t numel) {
  switch (type) {
    case PO_Q4_0:
      return numel % 32 == 0 ? numel / 32 * 18 : 0;
    case PO_Q8_0:
      return numel % 32 == 0 ? numel / 32 * 34 : 0;
    case PO_Q4_K:
      return numel % 256 == 0 ? numel / 256 * 144 : 0;
    default:
      return 0;
  }
}

/* adapters/llama/gguf.c:640-648 (get_scale_min_k4): 6-bit scale and min
 * of sub-block j from the 12 packed bytes. */
static void k4_scale_min(int j, const uint8_t *q, uint8_t *sc, uint8_t *mn) {
  if (j < 4) {
    *sc = q[j] & 63;
    *mn = q[j + 4] & 63;
  } else {
    *sc = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
    *mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

int po_dequant(uint32_t type, const uint8_t *src, float *dst, uint64_t numel) {
  uint64_t nb;
  if (po_type_bytes(type, numel) == 0) {
    return -1;
  }
  switch (type) {
    case PO_Q4_0: /* gguf.c:680-693 */
      nb = numel / 32;
      for (uint64_t b = 0; b < nb; b++, src += 18, dst += 32) {
        float d = le_f16(src);
        for (int j = 0; j < 16; j++) {
          int lo = (src[2 + j] & 0x0F) - 8;
          int hi = (src[2 + j] >> 4) - 8;
          dst[j] = (float)lo * d;
          dst[j + 16] = (float)hi * d;
        }
      }
      return 0;
    case PO_Q8_0: /* gguf.c:750-761 */
      nb = numel / 32;
      for (uint64_t b = 0; b < nb; b++, src += 34, dst += 32) {
        float d = le_f16(src);
        const int8_t *qs = (const int8_t *)(src + 2);
        for (int j = 0; j < 32; j++) {
          dst[j] = (float)qs[j] * d;
        }
      }
      return 0;
    case PO_Q4_K: /* gguf.c:852-882 */
      nb = numel / 256;
      for (uint64_t b = 0; b < nb; b++, src += 144) {
        const uint8_t *sc = src + 4;
        const uint8_t *q = src + 16;
        float d = le_f16(src);
        float dmin = le_f16(src + 2);
        for (int j = 0, is = 0; j < 256; j += 64, is += 2, q += 32, dst += 64) {
          uint8_t s, m;
          float d1, m1, d2, m2;
          k4_scale_min(is, sc, &s, &m);
          d1 = d * (float)s;
          m1 = dmin * (float)m;
          k4_scale_min(is + 1, sc, &s, &m);
          d2 = d * (float)s;
          m2 = dmin * (float)m;
          for (int l = 0; l < 32; l++) {
            dst[l] = d1 * (float)(q[l] & 0x0F) - m1;
          }
          for (int l = 0; l < 32; l++) {
            dst[l + 32] = d2 * (float)(q[l] >> 4) - m2;
          }
        }
      }
      return 0;
    default:
      return -1;
  }
}

static int clampi(long v, int lo, int hi) {
  return v < lo ? lo : (v > hi ? hi : (int)v);
}

int po_quantize(uint32_t type, const float *src, uint8_t *dst, uint64_t numel) {
  uint64_t nb;
  if (po_type_bytes(type, numel) == 0) {
    return -1;
  }
  switch (type) {
    case PO_Q8_0:
      nb = numel / 32;
      for (uint64_t b = 0; b < nb; b++, src += 32, dst += 34) {
        float amax = 0.0f, d;
        for (int j = 0; j < 32; j++) {
          float a = fabsf(src[j]);
          if (a > amax) {
            amax = a;
          }
        }
        d = amax / 127.0f;
        put_f16(dst, po_f32_to_f16(d));
        for (int j = 0; j < 32; j++) {
          int q = d > 0.0f ? clampi(lrintf(src[j] / d), -127, 127) : 0;
          dst[2 + j] = (uint8_t)(int8_t)q;
        }
      }
      return 0;
    case PO_Q4_0:
      nb = numel / 32;
      for (uint64_t b = 0; b < nb; b++, src += 32, dst += 18) {
        float amax = 0.0f, m = 0.0f, d;
        int q[32];
        for (int j = 0; j < 32; j++) {
          float a = fabsf(src[j]);
          if (a > amax) {
            amax = a;
            m = src[j];
          }
        }
        d = m / -8.0f;
        put_f16(dst, po_f32_to_f16(d));
        for (int j = 0; j < 32; j++) {
          q[j] = d != 0.0f ? clampi(lrintf(src[j] / d) + 8, 0, 15) : 8;
        }
        for (int j = 0; j < 16; j++) {
          dst[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
        }
      }
      return 0;
    case PO_Q4_K:
      nb = numel / 256;
      for (uint64_t b = 0; b < nb; b++, src += 256, dst += 144) {
        float S[8], M[8], maxS = 0.0f, maxM = 0.0f, df, dmf;
        int sc[8], mn[8];
        uint16_t d16, dm16;
        uint8_t *scales = dst + 4;
        uint8_t *qs = dst + 16;
        int q[256];
        for (int s = 0; s < 8; s++) {
          float lo = 0.0f, hi = 0.0f;
          for (int l = 0; l < 32; l++) {
            float v = src[32 * s + l];
            if (v < lo) {
              lo = v;
            }
            if (v > hi) {
              hi = v;
            }
          }
          S[s] = (hi - lo) / 15.0f;
          M[s] = -lo;
          if (S[s] > maxS) {
            maxS = S[s];
          }
          if (M[s] > maxM) {
            maxM = M[s];
          }
        }
        d16 = po_f32_to_f16(maxS / 63.0f);
        dm16 = po_f32_to_f16(maxM / 63.0f);
        df = po_f16_to_f32(d16);
        dmf = po_f16_to_f32(dm16);
        put_f16(dst, d16);
        put_f16(dst + 2, dm16);
        for (int s = 0; s < 8; s++) {
          sc[s] = df > 0.0f ? clampi(lrintf(S[s] / df), 0, 63) : 0;
          mn[s] = dmf > 0.0f ? clampi(lrintf(M[s] / dmf), 0, 63) : 0;
        }
        for (int j = 0; j < 4; j++) {
          scales[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
          scales[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
          scales[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
        }
        for (int s = 0; s < 8; s++) {
          float scale = df * (float)sc[s];
          float off = dmf * (float)mn[s];
          for (int l = 0; l < 32; l++) {
            float v = src[32 * s + l];
            q[32 * s + l] =
                scale > 0.0f ? clampi(lrintf((v + off) / scale), 0, 15) : 0;
          }
        }
        for (int c = 0; c < 4; c++) {
          for (int l = 0; l < 32; l++) {
            qs[32 * c + l] =
                (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
          }
        }
      }
      return 0;
    default:
      return -1;
  }
}

/* ---- dense ops ------------------------------------------------------------ */

void po_gemv_f32(uint64_t m, uint64_t k, const float *a, const float *x,
                 float *y) {
  for (uint64_t i = 0; i < m; i++) {
    float acc = 0.0f;
    for (uint64_t j = 0; j < k; j++) {
      acc += a[i * k + j] * x[j];
    }
    y[i] = acc;
  }
}

void po_gemm_f32(uint64_t m, uint64_t n, uint64_t k, const float *a,
                 const float *b, float *c) {
  for (uint64_t i = 0; i < m; i++) {
    for (uint64_t j = 0; j < n; j++) {
      float acc = 0.0f;
      for (uint64_t l = 0; l < k; l++) {
        acc += a[i * k + l] * b[l * n + j];
      }
      c[i * n + j] = acc;
    }
  }
}

/* ---- v0 grouped-scale formats ----------------------------------------------- */

/* Signed value of element i of a v0 blob: int8, or the nibble of byte i/2
 * selected by the parity of i, sign-extended (models/quantize.c:165-172). */
static int32_t v0_value(uint32_t bits, const int8_t *q, uint64_t i) {
  if (bits == 8) {
    return q[i];
  }
  const uint8_t byte = (uint8_t)q[i / 2];
  const int32_t nib = (i & 1) ? (byte >> 4) & 0x0F : byte & 0x0F;
  return (nib & 0x08) ? nib - 16 : nib;
}

uint64_t po_quant_v0(uint32_t bits, uint64_t gs, const float *src, uint64_t n,
                     int8_t *q, float *scales) {
  if ((bits != 8 && bits != 4) || n == 0) {
    return 0;
  }
  if (gs == 0) {
    gs = n;
  }
  const int32_t qmax = bits == 8 ? 127 : 7;
  memset(q, 0, bits == 8 ? n : (n + 1) / 2);
  uint64_t g = 0;
  for (uint64_t t = 0; t < n; t += gs, g++) {
    const uint64_t t1 = t + gs < n ? t + gs : n;
    float amax = 0.0f;
    for (uint64_t i = t; i < t1; i++) {
      const float v = fabsf(src[i]);
      if (v > amax) {
        amax = v;
      }
    }
    const float scale = amax > 0.0f ? amax / (float)qmax : 0.0f;
    scales[g] = scale;
    for (uint64_t i = t; i < t1; i++) {
      int32_t v = 0;
      if (scale > 0.0f) {
        v = (int32_t)lrintf(src[i] / scale);
        v = v > qmax ? qmax : (v < -qmax ? -qmax : v);
      }
      if (bits == 8) {
        q[i] = (int8_t)v;
      } else {
        uint8_t *b = (uint8_t *)q + i / 2;
        *b = (i & 1) ? (uint8_t)((*b & 0x0F) | ((v & 0x0F) << 4)) : (uint8_t)((*b & 0xF0) | (v & 0x0F));
      }
    }
  }
  return g;
}

int po_dequant_v0(uint32_t bits, uint64_t gs, const int8_t *q,
                  const float *scales, uint64_t n, float *out) {
  if (bits != 8 && bits != 4) {
    return -1;
  }
  if (gs == 0) {
    gs = n;
  }
  for (uint64_t i = 0; i < n; i++) {
    out[i] = scales[i / gs] * (float)v0_value(bits, q, i);
  }
  return 0;
}

int po_gemm_wq_f32(uint32_t bits, uint64_t m, uint64_t n, uint64_t k,
                   const float *a, const int8_t *w_q, const float *s,
                   uint64_t g, float *c) {
  if ((bits != 8 && bits != 4) || m == 0 || n == 0 || k == 0) {
    return -1;
  }
  if (g == 0 || g > k) {
    g = k;
  }
  for (uint64_t i = 0; i < m; i++) {
    for (uint64_t j = 0; j < n; j++) {
      float acc = 0.0f;
      for (uint64_t t = 0; t < k; t++) {
        const float prod = a[i * k + t] * (float)v0_value(bits, w_q, t * n + j);
        acc += prod * s[(t / g) * n + j];
      }
      c[i * n + j] = acc;
    }
  }
  return 0;
}

typedef struct {
  uint32_t type;
  uint64_t r0, r1, k, row_bytes;
  const uint8_t *w;
  const float *x;
  float *y;
  int rc;
} gemv_job_t;

static void *gemv_q_worker(void *arg) {
  gemv_job_t *j = (gemv_job_t *)arg;
  float *row = (float *)malloc((size_t)j->k * sizeof(float));
  if (row == NULL) {
    j->rc = -1;
    return NULL;
  }
  for (uint64_t r = j->r0; r < j->r1; r++) {
    if (po_dequant(j->type, j->w + r * j->row_bytes, row, j->k) != 0) {
      j->rc = -1;
      break;
    }
    po_gemv_f32(1, j->k, row, j->x, j->y + r);
  }
  free(row);
  return NULL;
}

int po_gemv_q(uint32_t type, uint64_t n, uint64_t k, const uint8_t *w,
              const float *x, float *y, int threads) {
  uint64_t row_bytes = po_type_bytes(type, k);
  gemv_job_t jobs[64];
  pthread_t tid[64];
  int nt = threads < 1 ? 1 : (threads > 64 ? 64 : threads);
  int rc = 0;
  if (row_bytes == 0 || n == 0) {
    return -1;
  }
  if ((uint64_t)nt > n) {
    nt = (int)n;
  }
  for (int t = 0; t < nt; t++) {
    jobs[t].type = type;
    jobs[t].r0 = n * (uint64_t)t / (uint64_t)nt;
    jobs[t].r1 = n * (uint64_t)(t + 1) / (uint64_t)nt;
    jobs[t].k = k;
    jobs[t].row_bytes = row_bytes;
    jobs[t].w = w;
    jobs[t].x = x;
    jobs[t].y = y;
    jobs[t].rc = 0;
  }
  if (nt == 1) {
    gemv_q_worker(&jobs[0]);
    return jobs[0].rc;
  }
  for (int t = 0; t < nt; t++) {
    if (pthread_create(&tid[t], NULL, gemv_q_worker, &jobs[t]) != 0) {
      gemv_q_worker(&jobs[t]);
      tid[t] = 0;
    }
  }
  for (int t = 0; t < nt; t++) {
    if (tid[t] != 0) {
      pthread_join(tid[t], NULL);
    }
    rc |= jobs[t].rc;
  }
  return rc;
}

void po_rmsnorm_gamma_f32(const float *a, float *c, uint64_t n,
                          const float *gamma, float eps) {
  double acc = 0.0;
  float rms;
  if (eps == 0.0f) {
    eps = 1e-5f;
  }
  for (uint64_t i = 0; i < n; i++) {
    acc += (double)a[i] * (double)a[i];
  }
  rms = 1.0f / sqrtf((float)(acc / (double)n) + eps);
  for (uint64_t i = 0; i < n; i++) {
    c[i] = a[i] * gamma[i] * rms;
  }
}

void po_silu_f32(const float *a, float *c, uint64_t n) {
  for (uint64_t i = 0; i < n; i++) {
    c[i] = a[i] / (1.0f + expf(-a[i]));
  }
}

void po_vecmul_f32(const float *a, const float *b, float *c, uint64_t n) {
  for (uint64_t i = 0; i < n; i++) {
    c[i] = a[i] * b[i];
  }
}

void po_vecadd_f32(const float *a, const float *b, float *c, uint64_t n) {
  for (uint64_t i = 0; i < n; i++) {
    c[i] = a[i] + b[i];
  }
}

static void rope_row(const float *xr, float *o, uint64_t hd, uint64_t p,
                     const float *cos_t, const float *sin_t, uint64_t r2) {
  for (uint64_t i = 0; i < r2; i++) {
    float c = cos_t[p * r2 + i];
    float s = sin_t[p * r2 + i];
    float x0 = xr[i];
    float x1 = xr[i + r2];
    o[i] = x0 * c - x1 * s;
    o[i + r2] = x0 * s + x1 * c;
  }
  for (uint64_t i = 2 * r2; i < hd; i++) {
    o[i] = xr[i];
  }
}

void po_rope_f32(const float *x, uint64_t rows, uint64_t hd, uint64_t heads,
                 const float *cos_t, const float *sin_t, uint64_t r2,
                 float *out) {
  for (uint64_t row = 0; row < rows; row++) {
    rope_row(x + row * hd, out + row * hd, hd, row / heads, cos_t, sin_t, r2);
  }
}

void po_rope_at_f32(const float *x, uint64_t heads, uint64_t hd, uint64_t p,
                    const float *cos_t, const float *sin_t, uint64_t r2,
                    float *out) {
  for (uint64_t h = 0; h < heads; h++) {
    rope_row(x + h * hd, out + h * hd, hd, p, cos_t, sin_t, r2);
  }
}

void po_rope_cossin_f32(uint64_t ctx, uint64_t r2, float base, float *cos_t,
                        float *sin_t) {
  if (base == 0.0f) {
    base = 10000.0f;
  }
  for (uint64_t p = 0; p < ctx; p++) {
    for (uint64_t i = 0; i < r2; i++) {
      double theta = (double)p *
                     pow((double)base, -(2.0 * (double)i) / (2.0 * (double)r2));
      cos_t[p * r2 + i] = (float)cos(theta);
      sin_t[p * r2 + i] = (float)sin(theta);
    }
  }
}

/* One attention row: the body of ref_ops.c:307-349 for query qp over
 * positions 0..np-1 of one KV head, K/V rows fetched by callbacks. */
typedef float (*kv_get_fn)(const void *base, uint64_t pos, uint64_t d);

static void attn_row(const float *qp, uint64_t np, uint64_t hd,
                     const void *kb, const void *vb, kv_get_fn get,
                     float *scores, float *op) {
  float inv_scale = 1.0f / sqrtf((float)hd);
  float maxv, sum = 0.0f;
  for (uint64_t i = 0; i < np; i++) {
    float dot = 0.0f;
    for (uint64_t d = 0; d < hd; d++) {
      dot += qp[d] * get(kb, i, d);
    }
    scores[i] = dot * inv_scale;
  }
  maxv = scores[0];
  for (uint64_t i = 1; i < np; i++) {
    if (scores[i] > maxv) {
      maxv = scores[i];
    }
  }
  for (uint64_t i = 0; i < np; i++) {
    float e = expf(scores[i] - maxv);
    scores[i] = e;
    sum += e;
  }
  for (uint64_t i = 0; i < np; i++) {
    scores[i] /= sum;
  }
  for (uint64_t d = 0; d < hd; d++) {
    float acc = 0.0f;
    for (uint64_t i = 0; i < np; i++) {
      acc += scores[i] * get(vb, i, d);
    }
    op[d] = acc;
  }
}

typedef struct {
  const float *base;
  uint64_t stride;
} f32_view_t;

static float get_f32(const void *b, uint64_t pos, uint64_t d) {
  const f32_view_t *v = (const f32_view_t *)b;
  return v->base[pos * v->stride + d];
}

typedef struct {
  const uint16_t *base;
  uint64_t stride;
} f16_view_t;

static float get_f16(const void *b, uint64_t pos, uint64_t d) {
  const f16_view_t *v = (const f16_view_t *)b;
  return po_f16_to_f32(v->base[pos * v->stride + d]);
}

int po_attention_f32(uint64_t h, uint64_t hk, uint64_t seq, uint64_t hd,
                     const float *q, const float *k, const float *v,
                     float *out) {
  float *scores;
  if (h == 0 || hk == 0 || seq == 0 || hd == 0 || h % hk != 0) {
    return -1;
  }
  scores = (float *)malloc((size_t)seq * sizeof(float));
  if (scores == NULL) {
    return -1;
  }
  for (uint64_t p = 0; p < seq; p++) {
    for (uint64_t hh = 0; hh < h; hh++) {
      uint64_t kvh = (hh * hk) / h;
      f32_view_t kv = {k + kvh * hd, hk * hd};
      f32_view_t vv = {v + kvh * hd, hk * hd};
      attn_row(q + (p * h + hh) * hd, p + 1, hd, &kv, &vv, get_f32, scores,
               out + (p * h + hh) * hd);
    }
  }
  free(scores);
  return 0;
}

int po_attention_decode_f16(uint64_t h, uint64_t hk, uint64_t hd,
                            uint64_t npos, uint64_t cap, const float *q,
                            const uint16_t *kc, const uint16_t *vc,
                            float *out) {
  float *scores;
  if (h == 0 || hk == 0 || hd == 0 || npos == 0 || npos > cap || h % hk != 0) {
    return -1;
  }
  scores = (float *)malloc((size_t)npos * sizeof(float));
  if (scores == NULL) {
    return -1;
  }
  for (uint64_t hh = 0; hh < h; hh++) {
    uint64_t kvh = (hh * hk) / h;
    f16_view_t kv = {kc + kvh * cap * hd, hd};
    f16_view_t vv = {vc + kvh * cap * hd, hd};
    attn_row(q + hh * hd, npos, hd, &kv, &vv, get_f16, scores, out + hh * hd);
  }
  free(scores);
  return 0;
}

uint32_t po_argmax_f32(const float *logits, uint64_t n) {
  float best = logits[0];
  uint32_t chosen = 0;
  for (uint64_t i = 1; i < n; i++) {
    if (logits[i] > best) {
      best = logits[i];
      chosen = (uint32_t)i;
    }
  }
  return chosen;
}

/* ---- synthetic data ------------------------------------------------------- */

uint64_t po_splitmix64(uint64_t *state) {
  uint64_t z = (*state += 0x9E3779B97F4A7C15ULL);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

void po_fill_normal(float *dst, uint64_t n, uint64_t seed, double mean,
                    double std) {
  uint64_t st = seed;
  for (uint64_t i = 0; i < n; i += 2) {
    double u1 = (double)((po_splitmix64(&st) >> 11) + 1) * 0x1.0p-53;
    double u2 = (double)(po_splitmix64(&st) >> 11) * 0x1.0p-53;
    double r = sqrt(-2.0 * log(u1));
    double t = 6.283185307179586 * u2;
    dst[i] = (float)(mean + std * r * cos(t));
    if (i + 1 < n) {
      dst[i + 1] = (float)(mean + std * r * sin(t));
    }
  }
}

/* ---- composed decode -------------------------------------------------------- */

struct po_session {
  po_model_cfg_t cfg;
  po_model_w_t w;
  uint32_t max_ctx, pos;
  int threads;
  uint16_t *kc, *vc; /* [layer][hk][max_ctx][hd] fp16 */
  float *cos_t, *sin_t;
  float *x, *xn, *q, *k, *v, *qr, *kr, *att, *o, *hn, *g, *u, *h, *dn,
      *logits;
};

po_session_t *po_session_create(const po_model_cfg_t *cfg,
                                const po_model_w_t *w, uint32_t max_ctx,
                                int threads) {
  po_session_t *s = (po_session_t *)calloc(1, sizeof(*s));
  uint64_t kv;
  uint64_t qd, kd;
  if (s == NULL) {
    return NULL;
  }
  s->cfg = *cfg;
  s->w = *w;
  s->max_ctx = max_ctx;
  s->threads = threads;
  qd = (uint64_t)cfg->n_head * cfg->head_dim;
  kd = (uint64_t)cfg->n_head_kv * cfg->head_dim;
  kv = (uint64_t)cfg->n_layer * kd * max_ctx;
  s->kc = (uint16_t *)calloc(kv, 2);
  s->vc = (uint16_t *)calloc(kv, 2);
  s->cos_t = (float *)malloc((size_t)max_ctx * cfg->head_dim / 2 * 4);
  s->sin_t = (float *)malloc((size_t)max_ctx * cfg->head_dim / 2 * 4);
  s->x = (float *)calloc(cfg->n_embd, 4);
  s->xn = (float *)calloc(cfg->n_embd, 4);
  s->q = (float *)calloc(qd, 4);
  s->qr = (float *)calloc(qd, 4);
  s->att = (float *)calloc(qd, 4);
  s->k = (float *)calloc(kd, 4);
  s->kr = (float *)calloc(kd, 4);
  s->v = (float *)calloc(kd, 4);
  s->o = (float *)calloc(cfg->n_embd, 4);
  s->hn = (float *)calloc(cfg->n_embd, 4);
  s->dn = (float *)calloc(cfg->n_embd, 4);
  s->g = (float *)calloc(cfg->n_ff, 4);
  s->u = (float *)calloc(cfg->n_ff, 4);
  s->h = (float *)calloc(cfg->n_ff, 4);
  s->logits = (float *)calloc(cfg->vocab, 4);
  if (!s->kc || !s->vc || !s->cos_t || !s->sin_t || !s->x || !s->xn ||
      !s->q || !s->qr || !s->att || !s->k || !s->kr || !s->v || !s->o ||
      !s->hn || !s->dn || !s->g || !s->u || !s->h || !s->logits) {
    po_session_destroy(s);
    return NULL;
  }
  po_rope_cossin_f32(max_ctx, cfg->head_dim / 2, cfg->rope_theta, s->cos_t,
                     s->sin_t);
  return s;
}

void po_session_destroy(po_session_t *s) {
  if (s == NULL) {
    return;
  }
  free(s->kc);
  free(s->vc);
  free(s->cos_t);
  free(s->sin_t);
  free(s->x);
  free(s->xn);
  free(s->q);
  free(s->qr);
  free(s->att);
  free(s->k);
  free(s->kr);
  free(s->v);
  free(s->o);
  free(s->hn);
  free(s->dn);
  free(s->g);
  free(s->u);
  free(s->h);
  free(s->logits);
  free(s);
}

const float *po_session_hidden(const po_session_t *s) { return s->x; }

/* Cache rows of layer l ([hk][max_ctx][hd] fp16), for tests that start
 * from a given cache, and the position of the next step (the positions
 * below it must hold the cache contents to attend over). */
uint16_t *po_session_kv(po_session_t *s, uint32_t layer, int v) {
  const uint64_t kd = (uint64_t)s->cfg.n_head_kv * s->cfg.head_dim;
  if (layer >= s->cfg.n_layer) {
    return NULL;
  }
  return (v ? s->vc : s->kc) + (uint64_t)layer * kd * s->max_ctx;
}

int po_session_seek(po_session_t *s, uint32_t pos) {
  if (pos > s->max_ctx) {
    return -1;
  }
  s->pos = pos;
  return 0;
}

int64_t po_session_step(po_session_t *s, uint32_t token, float *logits) {
  const po_model_cfg_t *c = &s->cfg;
  uint64_t E = c->n_embd, hd = c->head_dim, r2 = hd / 2;
  uint64_t qd = (uint64_t)c->n_head * hd, kd = (uint64_t)c->n_head_kv * hd;
  uint64_t erow = po_type_bytes(c->etype, E);
  uint64_t p = s->pos;
  int T = s->threads;
  if (p >= s->max_ctx || token >= c->vocab) {
    return -1;
  }
  /* Embedding: one-hot GEMM row (llama.c:510-522) == dequantised row. */
  if (po_dequant(c->etype, s->w.tok_embd + (uint64_t)token * erow, s->x, E)) {
    return -1;
  }
  for (uint32_t l = 0; l < c->n_layer; l++) {
    uint64_t kvoff = (uint64_t)l * c->n_head_kv * s->max_ctx * hd;
    po_rmsnorm_gamma_f32(s->x, s->xn, E, s->w.attn_norm[l], c->eps);
    if (po_gemv_q(c->wtype, qd, E, s->w.wq[l], s->xn, s->q, T) ||
        po_gemv_q(c->wtype, kd, E, s->w.wk[l], s->xn, s->k, T) ||
        po_gemv_q(c->wtype, kd, E, s->w.wv[l], s->xn, s->v, T)) {
      return -1;
    }
    po_rope_at_f32(s->q, c->n_head, hd, p, s->cos_t, s->sin_t, r2, s->qr);
    po_rope_at_f32(s->k, c->n_head_kv, hd, p, s->cos_t, s->sin_t, r2, s->kr);
    for (uint64_t kh = 0; kh < c->n_head_kv; kh++) {
      for (uint64_t d = 0; d < hd; d++) {
        uint64_t at = kvoff + (kh * s->max_ctx + p) * hd + d;
        s->kc[at] = po_f32_to_f16(s->kr[kh * hd + d]);
        s->vc[at] = po_f32_to_f16(s->v[kh * hd + d]);
      }
    }
    if (po_attention_decode_f16(c->n_head, c->n_head_kv, hd, p + 1,
                                s->max_ctx, s->qr, s->kc + kvoff,
                                s->vc + kvoff, s->att)) {
      return -1;
    }
    if (po_gemv_q(c->wtype, E, qd, s->w.wo[l], s->att, s->o, T)) {
      return -1;
    }
    po_vecadd_f32(s->x, s->o, s->x, E);
    po_rmsnorm_gamma_f32(s->x, s->hn, E, s->w.ffn_norm[l], c->eps);
    if (po_gemv_q(c->wtype, c->n_ff, E, s->w.wgate[l], s->hn, s->g, T) ||
        po_gemv_q(c->wtype, c->n_ff, E, s->w.wup[l], s->hn, s->u, T)) {
      return -1;
    }
    po_silu_f32(s->g, s->g, c->n_ff);
    po_vecmul_f32(s->g, s->u, s->h, c->n_ff);
    if (po_gemv_q(c->wtype, E, c->n_ff, s->w.wdown[l], s->h, s->dn, T)) {
      return -1;
    }
    po_vecadd_f32(s->x, s->dn, s->x, E);
  }
  po_rmsnorm_gamma_f32(s->x, s->xn, E, s->w.output_norm, c->eps);
  if (po_gemv_q(c->etype, c->vocab, E, s->w.output, s->xn, s->logits, T)) {
    return -1;
  }
  if (logits != NULL) {
    memcpy(logits, s->logits, (size_t)c->vocab * 4);
  }
  s->pos++;
  return po_argmax_f32(s->logits, c->vocab);
}
