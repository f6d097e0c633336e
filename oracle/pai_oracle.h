/*
 * pai_oracle — CPU restatement of ProsperoAI's quantized-weights hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links, loads
 * or calls this code: it is the checker that the CUDA path is compared
 * against (tests/, the smoke check and bench.py's CPU-baseline leg).
 *
 * Every function restates one reference function with the same
 * operation order, so that the dequantisers, RMSNorm, RoPE, residual
 * and SiLU-gate results are bit-identical to the reference's
 * cpu/reference + adapters/llama code on the same inputs. The reference
 * file:line each one follows is cited beside it. The restatement is
 * pinned against the reference itself (oracle/_ref, built from the
 * reference sources by oracle/Makefile) and against the reference's
 * known-answer vectors (tests/golden/).
 *
 * Compile with -std=c11 -ffp-contract=off: the reference is built as ISO
 * C11, where GCC does not fuse a*b+c into an FMA, and bit-exactness of
 * the restated ops depends on the same rounding steps.
 */
#ifndef PAI_ORACLE_H
#define PAI_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml block type ids, as in adapters/llama/gguf.h:36-51. */
#define PO_Q4_0 2u
#define PO_Q8_0 8u
#define PO_Q4_K 12u

/* fp16 <-> fp32 ---------------------------------------------------------- */

/* adapters/llama/gguf.c:602-630 (f16_to_f32). */
float po_f16_to_f32(uint16_t h);
/* IEEE binary16 round-to-nearest-even (the quantiser's scale store). */
uint16_t po_f32_to_f16(float f);

/* ggml block formats ------------------------------------------------------ */

/* Bytes of `numel` elements of `type` (adapters/llama/gguf.c:563-599);
 * 0 when numel is not a whole number of blocks or type is unknown. */
uint64_t po_type_bytes(uint32_t type, uint64_t numel);

/* dequant_block for Q4_0 / Q8_0 / Q4_K (adapters/llama/gguf.c:680-693,
 * 750-761, 852-882). Returns 0, or -1 for an unsupported type or a
 * ragged element count. */
int po_dequant(uint32_t type, const uint8_t *src, float *dst, uint64_t numel);

/* Block quantisers restating the benchmark specification's formulas (the reference ships
 * dequantisers only, so this part is parity-unpinned by the reference):
 *   Q8_0: d = max|w|/127, q = lrintf(w/d) clamped to [-127,127]
 *   Q4_0: d = m/-8 with m the first element of largest |w|,
 *         q = clamp(lrintf(w/d) + 8, 0, 15)
 *   Q4_K: per 32-element sub-block lo=min(0,min w), hi=max(0,max w),
 *         S=(hi-lo)/15, M=-lo; d=max S/63, dmin=max M/63 stored fp16;
 *         sc=lrintf(S/d), m=lrintf(M/dmin) clamped to [0,63];
 *         q = clamp(lrintf((w + dmin*m)/(d*sc)), 0, 15).
 * The product library's quantiser must produce the same bytes. */
int po_quantize(uint32_t type, const float *src, uint8_t *dst, uint64_t numel);

/* dense ops (cpu/reference/ref_ops.c) ------------------------------------ */

/* ref_ops.c:92-106 */
void po_gemv_f32(uint64_t m, uint64_t k, const float *a, const float *x,
                 float *y);
/* Dequantise row r of W[n,k] (ggml row-major blocks) and run the
 * ref_ops.c:92-106 row loop: bit-identical to pai_gguf_dequant followed
 * by pai_ref_gemv_f32. Rows are split over `threads` pthreads; the
 * per-row operation order does not change. */
int po_gemv_q(uint32_t type, uint64_t n, uint64_t k, const uint8_t *w,
              const float *x, float *y, int threads);
/* ref_ops.c:428-444: c[m,n] = sum over l ascending of a[m,l] * b[l,n]. */
void po_gemm_f32(uint64_t m, uint64_t n, uint64_t k, const float *a,
                 const float *b, float *c);

/* v0 grouped-scale formats (models/quantize.c, cpu/reference/ref_ops.c) -- */

/* models/quantize.c:74-143 (pai_quantize_f32): signed symmetric, one f32
 * scale max|w|/qmax per `gs` consecutive elements (gs 0: all n), q =
 * lrintf(w/scale) clamped to [-qmax, qmax], qmax 127 (bits 8) or 7 (bits
 * 4, two per byte: even index low nibble). Returns the number of groups,
 * or 0 for an unsupported width. q must hold value_bytes(n) bytes. */
uint64_t po_quant_v0(uint32_t bits, uint64_t gs, const float *src, uint64_t n,
                     int8_t *q, float *scales);
/* models/quantize.c:146-181 (pai_dequantize_f32): out[i] =
 * scales[i / gs] * (float)q(i), nibbles sign-extended. */
int po_dequant_v0(uint32_t bits, uint64_t gs, const int8_t *q,
                  const float *scales, uint64_t n, float *out);
/* ref_ops.c:447-499 (pai_ref_gemm_w8_f32 / pai_ref_gemm_w4_f32):
 * c[i,j] = sum over t ascending of (a[i,t] * (float)q(t,j)) * s[(t/g)*n + j],
 * q(t,j) the int8 w_q[t*n+j] (bits 8) or the signed nibble at flat index
 * t*n+j (bits 4); g 0 or > k selects k. */
int po_gemm_wq_f32(uint32_t bits, uint64_t m, uint64_t n, uint64_t k,
                   const float *a, const int8_t *w_q, const float *s,
                   uint64_t g, float *c);

/* ref_ops.c:196-216 (eps == 0 selects 1e-5) */
void po_rmsnorm_gamma_f32(const float *a, float *c, uint64_t n,
                          const float *gamma, float eps);
/* ref_ops.c:219-228 */
void po_silu_f32(const float *a, float *c, uint64_t n);
/* ref_ops.c:124-133 */
void po_vecmul_f32(const float *a, const float *b, float *c, uint64_t n);
/* ref_ops.c:8-17 */
void po_vecadd_f32(const float *a, const float *b, float *c, uint64_t n);
/* ref_ops.c:231-257: half-split pairs (i, i+r2), row = p*heads + h. */
void po_rope_f32(const float *x, uint64_t rows, uint64_t hd, uint64_t heads,
                 const float *cos_t, const float *sin_t, uint64_t r2,
                 float *out);
/* Rotate one position-p row block of `heads` rows (decode form of the
 * above: identical arithmetic, the table row is p). */
void po_rope_at_f32(const float *x, uint64_t heads, uint64_t hd, uint64_t p,
                    const float *cos_t, const float *sin_t, uint64_t r2,
                    float *out);
/* ref_ops.c:260-279 (double pow/cos/sin, base 0 selects 10000) */
void po_rope_cossin_f32(uint64_t ctx, uint64_t r2, float base, float *cos_t,
                        float *sin_t);
/* ref_ops.c:287-354, causal GQA over position-major q/k/v. */
int po_attention_f32(uint64_t h, uint64_t hk, uint64_t seq, uint64_t hd,
                     const float *q, const float *k, const float *v,
                     float *out);
/* The last-row (p = npos-1) iteration of ref_ops.c:307-349 over an fp16
 * KV cache laid out [hk][cap][hd] (position stride hd, head stride
 * cap*hd). K/V widen exactly to fp32, so this is the reference loop on
 * the cache contents. q is [h][hd]; out is [h][hd]. */
int po_attention_decode_f16(uint64_t h, uint64_t hk, uint64_t hd,
                            uint64_t npos, uint64_t cap, const float *q,
                            const uint16_t *kc, const uint16_t *vc,
                            float *out);
/* models/sampler.c:89-99 greedy: first index of the strict maximum. */
uint32_t po_argmax_f32(const float *logits, uint64_t n);

/* seeded synthetic data ---------------------------------------------------- */

/* splitmix64 step (Steele, Lea, Flood 2014). */
uint64_t po_splitmix64(uint64_t *state);
/* n samples of mean + std*Z, Z ~ N(0,1) by Box-Muller in double over a
 * splitmix64 stream seeded with `seed`; pairs (cos, sin) in order. */
void po_fill_normal(float *dst, uint64_t n, uint64_t seed, double mean,
                    double std);

/* composed LLaMA decode (adapters/llama/llama.c:669-797 op order) ------ */

typedef struct po_model_cfg {
  uint32_t n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff, vocab;
  float eps, rope_theta;
  uint32_t wtype;              /* block type of the layer matrices   */
  uint32_t etype;              /* block type of embedding and lm head */
} po_model_cfg_t;

/* Weights of one model in ggml row-major blocks ([out][in]). */
typedef struct po_model_w {
  const uint8_t *tok_embd;     /* [vocab][n_embd] etype               */
  const uint8_t *output;       /* [vocab][n_embd] etype               */
  const float *output_norm;    /* [n_embd]                            */
  const uint8_t **wq, **wk, **wv, **wo, **wgate, **wup, **wdown;
  const float **attn_norm, **ffn_norm;
} po_model_w_t;

typedef struct po_session po_session_t;

po_session_t *po_session_create(const po_model_cfg_t *cfg,
                                const po_model_w_t *w, uint32_t max_ctx,
                                int threads);
void po_session_destroy(po_session_t *s);
/* Feed one token at the next position; writes logits[vocab] when
 * non-NULL and returns the greedy token. */
int64_t po_session_step(po_session_t *s, uint32_t token, float *logits);
/* Hidden state after the last step (n_embd floats). */
const float *po_session_hidden(const po_session_t *s);
/* K (v = 0) or V (v = 1) cache of one layer: [hk][max_ctx][hd] fp16. */
uint16_t *po_session_kv(po_session_t *s, uint32_t layer, int v);
/* Continue at position pos (0 <= pos <= max_ctx). */
int po_session_seek(po_session_t *s, uint32_t pos);

#ifdef __cplusplus
}
#endif

#endif /* PAI_ORACLE_H */
