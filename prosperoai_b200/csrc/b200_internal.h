/*
 * Internal interface between the C host code (csrc/host) and the CUDA
 * shim (csrc/kernels). C-compatible: the host side never sees a CUDA
 * type; streams, graphs and events are opaque pointers.
 */
#ifndef B200_INTERNAL_H
#define B200_INTERNAL_H

#include "pai_b200.h"

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- packed weight layout -------------------------------------------------------
 * Rows are grouped by B200_RG = 32. For row group g and block b, the
 * block's quant bytes are split into 16-byte chunks and chunk c of all
 * 32 rows is stored contiguously (512 B), so a warp with one lane per row
 * reads a chunk with a single fully coalesced 128-bit load per lane:
 *     qs plane: [ngroups][nb][chunks][32 rows][16 B]
 * The per-row block header (the fp16 d of Q4_0/Q8_0; d, dmin and the 12
 * packed scale bytes of Q4_K) goes to a second plane:
 *     sc plane: [ngroups][nb][32 rows][hdr bytes]
 * starting at the 256-byte aligned end of the qs plane. The bytes are
 * those of the ggml block (adapters/llama/gguf.c:680-693, 750-761,
 * 852-882) moved, never re-encoded, so the total equals the ggml size up
 * to alignment and zero rows that pad n to a multiple of 32. */
#define B200_RG 32u

#ifdef __CUDACC__
#define B200_HD __host__ __device__
#else
#define B200_HD
#endif

static inline B200_HD uint32_t b200_blk_elems(uint32_t t) { return t == PAI_B200_Q4_K ? 256u : 32u; }
static inline B200_HD uint32_t b200_blk_bytes(uint32_t t) {
  return t == PAI_B200_Q4_0 ? 18u : (t == PAI_B200_Q8_0 ? 34u : 144u);
}
static inline B200_HD uint32_t b200_chunks(uint32_t t) {
  return t == PAI_B200_Q4_0 ? 1u : (t == PAI_B200_Q8_0 ? 2u : 8u);
}
static inline B200_HD uint32_t b200_hdr_bytes(uint32_t t) { return t == PAI_B200_Q4_K ? 16u : 2u; }
static inline B200_HD int b200_type_ok(uint32_t t) {
  return t == PAI_B200_Q4_0 || t == PAI_B200_Q8_0 || t == PAI_B200_Q4_K;
}
static inline B200_HD uint64_t b200_align256(uint64_t v) { return (v + 255u) & ~(uint64_t)255u; }
static inline B200_HD uint64_t b200_ngroups(uint64_t n) { return (n + B200_RG - 1) / B200_RG; }
static inline B200_HD uint64_t b200_qs_bytes(uint32_t t, uint64_t n, uint64_t k) {
  return b200_ngroups(n) * (k / b200_blk_elems(t)) * b200_chunks(t) * B200_RG * 16u;
}
static inline B200_HD uint64_t b200_sc_offset(uint32_t t, uint64_t n, uint64_t k) {
  return b200_align256(b200_qs_bytes(t, n, k));
}

/* ---- errors ------------------------------------------------------------------------- */

pai_status_t b200_fail(pai_status_t st, const char *fmt, ...);
/* Map a CUDA runtime error code to a status (PAI_OK for 0). */
pai_status_t b200_cuda(int err, const char *what);

/* ---- context ------------------------------------------------------------------------ */

void *b200_ctx_stream(pai_b200_ctx_t *ctx);
int b200_ctx_device(pai_b200_ctx_t *ctx);
void b200_ctx_count_launch(pai_b200_ctx_t *ctx, uint32_t kernels);
/* Count `kernels` launches and report a launch error under `name`. With
 * PAI_B200_SYNC_CHECK=1 in the environment (and outside graph capture)
 * it also waits for the kernels and reports their execution errors,
 * which localises a failing kernel. */
pai_status_t b200_launched(pai_b200_ctx_t *ctx, uint32_t kernels, const char *name);
/* Per-context split-K scratch: float partial sums and zeroed counters
 * (each kernel that uses the counters leaves them at zero). */
pai_status_t b200_ctx_scratch(pai_b200_ctx_t *ctx, uint64_t partial_floats,
                              uint32_t counters, float **partial,
                              uint32_t **counter);

/* CUDA graph capture of everything launched on the context stream. */
pai_status_t b200_graph_begin(pai_b200_ctx_t *ctx);
pai_status_t b200_graph_end(pai_b200_ctx_t *ctx, void **exec, uint32_t *kernels);
pai_status_t b200_graph_launch(pai_b200_ctx_t *ctx, void *exec, uint32_t kernels);
void b200_graph_destroy(void *exec);

/* ---- kernel launchers (csrc/kernels) ----------------------------------------------- */

enum { B200_EPI_STORE = 0, B200_EPI_RESIDUAL = 1, B200_EPI_SILU_GLU = 2 };

/* GEMV over a packed matrix. For B200_EPI_SILU_GLU the packed rows come
 * in groups of 16 gate rows followed by the 16 matching up rows, n counts
 * both, and y receives n/2 values silu(gate)*up per batch row. */
pai_status_t b200_launch_gemv(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch,
                              uint64_t n, uint64_t k, const void *w, const float *x,
                              const float *residual, float *y, int epi);
/* x[b] = dequantised row tokens[b] of a packed rows x k table. */
pai_status_t b200_launch_embed(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch,
                               uint64_t rows, uint64_t k, const void *w,
                               const int32_t *tokens, float *x);
/* q/k/v from the fused projection ([batch][(H+2HK)*hd]), rotate q and k
 * at position *pos, write q (fp32) and the new k/v rows into the fp16
 * caches [hk][cap][hd] of each sequence (cache stride per sequence
 * seq_stride elements). */
pai_status_t b200_launch_rope_kv(pai_b200_ctx_t *ctx, uint32_t batch, uint32_t h,
                                 uint32_t hk, uint32_t hd, const float *qkv,
                                 const int32_t *pos, const float *cos_t,
                                 const float *sin_t, float *q, uint16_t *kc,
                                 uint16_t *vc, uint64_t cap, uint64_t seq_stride);
/* Decode attention at position *pos (npos = *pos + 1) when pos is a
 * device pointer; max_npos bounds the launch. */
pai_status_t b200_launch_attn_decode(pai_b200_ctx_t *ctx, uint32_t batch, uint32_t h,
                                     uint32_t hk, uint32_t hd, const int32_t *pos,
                                     uint64_t npos_host, uint64_t max_npos,
                                     uint64_t cap, uint64_t seq_stride,
                                     const float *q, const uint16_t *kc,
                                     const uint16_t *vc, float *out);
pai_status_t b200_launch_rmsnorm(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n,
                                 const float *a, const float *gamma, float eps,
                                 float *c);
pai_status_t b200_launch_argmax(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n,
                                const float *logits, int32_t *out);
pai_status_t b200_launch_step_tail(pai_b200_ctx_t *ctx, uint32_t batch,
                                   int32_t *tok_out, int32_t *tok_in, int32_t *pos);
pai_status_t b200_launch_synth_normal(pai_b200_ctx_t *ctx, float *dst, uint64_t rows,
                                      uint64_t cols, uint64_t seed, float stddev);
pai_status_t b200_launch_quantize(pai_b200_ctx_t *ctx, uint32_t type, const float *src,
                                  uint64_t numel, void *dst);
pai_status_t b200_launch_fill(pai_b200_ctx_t *ctx, float *dst, uint64_t n, float v);

#ifdef __cplusplus
}
#endif

#endif /* B200_INTERNAL_H */
