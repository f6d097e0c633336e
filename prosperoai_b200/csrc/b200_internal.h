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

/* ---- packed weight layout ------------------------------------------------------
 * Built once at load from ggml blocks; bytes are moved, never re-encoded.
 * Rows are taken 16 at a time (a "tile": the M of one m16n8k32 int8 MMA)
 * and K in "units": 4 blocks (128 weights) for Q4_0/Q8_0, one 256-weight
 * super-block for Q4_K. Each (tile, unit) holds
 *   qs plane: CH chunks x 32 lanes x 16 B, in the order the MMA A-fragment
 *             wants them: lane l (row r = l/4, column group c = l%4) finds in
 *             one 16-byte load the 4-byte words it needs of 4 blocks (or of
 *             the 4 64-weight groups of a Q4_K super-block):
 *     Q4_0 (CH 2):  chunk h      = word c of qs[16] of row r+8h, blocks 0..3
 *     Q8_0 (CH 4):  chunk 2h+p   = bytes 16p+4c..+3 of row r+8h, blocks 0..3
 *     Q4_K (CH 4):  chunk 2h+p   = bytes 32g+16p+4c..+3 of row r+8h, g 0..3
 *   sc plane: the block headers, [16 rows][4 blocks] fp16 d (Q4_0/Q8_0) or
 *             [16 rows][16 B] {d, dmin, scales[12]} (Q4_K), at the 256-byte
 *             aligned end of the qs plane.
 * The (tile, unit) pieces are stored unit-major (all tiles of unit 0, then
 * unit 1, ...), so the pieces of consecutive tiles for one unit are one
 * contiguous run: a GEMV CTA that owns a group of tiles fetches a unit of
 * all of them with one bulk copy per plane.
 * Rows beyond n and blocks beyond k (to a whole unit) are zero. */
#define B200_TILE 16u

#ifdef __CUDACC__
#define B200_HD __host__ __device__
#else
#define B200_HD
#endif

static inline B200_HD uint32_t b200_blk_elems(uint32_t t) { return t == PAI_B200_Q4_K ? 256u : 32u; }
static inline B200_HD uint32_t b200_blk_bytes(uint32_t t) {
  return t == PAI_B200_Q4_0 ? 18u : (t == PAI_B200_Q8_0 ? 34u : 144u);
}
static inline B200_HD int b200_type_ok(uint32_t t) {
  return t == PAI_B200_Q4_0 || t == PAI_B200_Q8_0 || t == PAI_B200_Q4_K;
}
static inline B200_HD uint64_t b200_align256(uint64_t v) { return (v + 255u) & ~(uint64_t)255u; }
static inline B200_HD uint64_t b200_ntiles(uint64_t n) { return (n + B200_TILE - 1) / B200_TILE; }
/* Blocks per unit, units per row of k elements. */
static inline B200_HD uint32_t b200_unit_blocks(uint32_t t) { return t == PAI_B200_Q4_K ? 1u : 4u; }
static inline B200_HD uint64_t b200_units(uint32_t t, uint64_t k) {
  uint64_t nb = k / b200_blk_elems(t);
  return (nb + b200_unit_blocks(t) - 1) / b200_unit_blocks(t);
}
static inline B200_HD uint32_t b200_unit_qs_bytes(uint32_t t) { return t == PAI_B200_Q4_0 ? 1024u : 2048u; }
static inline B200_HD uint32_t b200_unit_sc_bytes(uint32_t t) { return t == PAI_B200_Q4_K ? 256u : 128u; }
static inline B200_HD uint64_t b200_sc_offset(uint32_t t, uint64_t n, uint64_t k) {
  return b200_align256(b200_ntiles(n) * b200_units(t, k) * b200_unit_qs_bytes(t));
}

/* ---- quantised activations ("xq") ----------------------------------------------
 * A GEMV reads x as 24-bit fixed point per 32-element block: x_j ~ s_b * X_j
 * with X_j = L2*65536 + L1*256 + L0 in balanced base-256 digits (each an
 * int8), s_b = max|x_b| / 8355711. The digits are stored in the order of
 * the MMA B-fragment: vectors go in pairs (a pair fills the 8 columns of
 * one MMA: columns 0..3 = L2, L1, L0, 0 of the even vector, 4..7 of the
 * odd one), and for pair t, x-quad q (4 blocks), part p (elements 16p..):
 *   limbs: [pair][quad][2][32 lanes][16 B]; lane l = column*4 + c holds
 *          bytes 4c..4c+3 of elements 16p.. of blocks 0..3 of its column
 *   sb:    [vec][quad*4] f32 block scales s_b
 *   sx:    [vec][quad*4] f32 s_b * sum_j X_j (for the Q4_0 -8 offset and
 *          the Q4_K mins)
 * Writers fill every byte of a block, zero column included; the bytes of
 * an absent odd vector are never weighted (its scales read as 0). */
#define B200_XQ_MAX 8355711
static inline B200_HD uint64_t b200_xq_quads(uint64_t k) { return (k / 32u + 3u) / 4u; }
static inline B200_HD uint64_t b200_xq_limb_bytes(uint32_t batch, uint64_t k) {
  return (uint64_t)((batch + 1u) / 2u) * b200_xq_quads(k) * 1024u;
}
static inline B200_HD uint64_t b200_xq_bytes(uint32_t batch, uint64_t k) {
  return b200_align256(b200_xq_limb_bytes(batch, k)) + 2u * b200_align256((uint64_t)batch * b200_xq_quads(k) * 16u);
}

typedef struct b200_xq {
  uint8_t *limbs;
  float *sb, *sx;
  uint32_t batch;
  uint64_t k, quads;
} b200_xq_t;

/* Carve an xq view out of `base` (b200_xq_bytes(batch, k) bytes). */
static inline B200_HD b200_xq_t b200_xq_view(void *base, uint32_t batch, uint64_t k) {
  b200_xq_t v;
  uint8_t *p = (uint8_t *)base;
  v.batch = batch;
  v.k = k;
  v.quads = b200_xq_quads(k);
  v.limbs = p;
  p += b200_align256(b200_xq_limb_bytes(batch, k));
  v.sb = (float *)p;
  p += b200_align256((uint64_t)batch * v.quads * 16u);
  v.sx = (float *)p;
  return v;
}

/* ---- model files (csrc/host/b200_gguf.c, b200_pai.c) ------------------------------- */

/* One tensor of a model file, viewed in place: ggml type (0 = f32), ggml
 * shape rows x cols ([out][in]), bytes. */
typedef struct b200_named_tensor {
  char name[128];
  uint32_t type;
  uint64_t rows, cols, bytes;
  const uint8_t *data;
} b200_named_tensor_t;
typedef struct b200_gguf_view b200_gguf_view_t;
/* The tensors a LLaMA GGUF file's model uses (views into the mapped file,
 * valid until b200_gguf_release); info as pai_b200_gguf_inspect. */
pai_status_t b200_gguf_llama_tensors(const char *path, pai_b200_gguf_info_t *info, b200_named_tensor_t **out,
                                     uint32_t *count, b200_gguf_view_t **view);
void b200_gguf_release(b200_gguf_view_t *view);

/* ---- errors ------------------------------------------------------------------------- */

pai_status_t b200_fail(pai_status_t st, const char *fmt, ...);
/* Map a CUDA runtime error code to a status (PAI_OK for 0). */
pai_status_t b200_cuda(int err, const char *what);
/* The driver's cuTensorMapEncodeTiled, looked up once through the runtime
 * (no link-time dependency on libcuda); NULL where unavailable. */
void *b200_tensor_map_encoder(void);

/* ---- context ------------------------------------------------------------------------ */

void *b200_ctx_stream(pai_b200_ctx_t *ctx);
int b200_ctx_device(pai_b200_ctx_t *ctx);
/* Make ctx's device current on the calling thread. */
pai_status_t b200_ctx_use_device(pai_b200_ctx_t *ctx);
void b200_ctx_count_launch(pai_b200_ctx_t *ctx, uint32_t kernels);
/* Count `kernels` launches and report a launch error under `name`. With
 * PAI_B200_SYNC_CHECK=1 in the environment (and outside graph capture)
 * it also waits for the kernels and reports their execution errors,
 * which localises a failing kernel. */
pai_status_t b200_launched(pai_b200_ctx_t *ctx, uint32_t kernels, const char *name);
/* Per-context scratch: float partial sums and zeroed counters (each
 * kernel that uses the counters leaves them at zero). Kernels on the
 * context stream use it one after another. */
pai_status_t b200_ctx_scratch(pai_b200_ctx_t *ctx, uint64_t partial_floats,
                              uint32_t counters, float **partial,
                              uint32_t **counter);
/* Activation scratch of the public GEMV entry points (grown on demand). */
pai_status_t b200_ctx_xq(pai_b200_ctx_t *ctx, uint64_t bytes, void **buf);
/* Device address of the context's error word: kernels whose bounded waits
 * run out set it, and pai_b200_sync then reports PAI_ERR_TIMEOUT. */
uint32_t *b200_ctx_errflag(pai_b200_ctx_t *ctx);
/* Programmatic dependent launch for the kernels of the model's decode
 * step: while on, those kernels are launched so that each may become
 * resident before its predecessor in the stream finishes; each waits
 * (griddepcontrol.wait) before it touches memory the predecessor writes,
 * and only the GEMV does work before that wait: it prefetches weights,
 * which nothing in the step writes. Off for the public single-op entry
 * points, whose inputs a preceding kernel may just have written.
 * PAI_B200_PDL=0 in the environment keeps it off. */
int b200_ctx_pdl(pai_b200_ctx_t *ctx);
/* Limit in nanoseconds on every bounded device wait of the context's
 * kernels (pai_b200_set_wait_limit; 2 s by default). */
uint64_t b200_ctx_wait_ns(pai_b200_ctx_t *ctx);
void b200_ctx_set_pdl(pai_b200_ctx_t *ctx, int on);

/* CUDA graph capture of everything launched on the context stream. */
pai_status_t b200_graph_begin(pai_b200_ctx_t *ctx);
pai_status_t b200_graph_end(pai_b200_ctx_t *ctx, void **exec, uint32_t *kernels);
pai_status_t b200_graph_launch(pai_b200_ctx_t *ctx, void *exec, uint32_t kernels);
void b200_graph_destroy(void *exec);

/* ---- kernel launchers (csrc/kernels) ----------------------------------------------- */

enum { B200_EPI_STORE = 0, B200_EPI_RESIDUAL = 1, B200_EPI_SILU_GLU = 2 };

/* GEMV over a packed matrix with x given as xq (batch vectors of k).
 * B200_EPI_SILU_GLU: each 16-row tile holds 8 gate rows then the 8 matching
 * up rows, n counts both, y receives n/2 values silu(gate)*up per vector,
 * and when xq_out is non-NULL they are also quantised into it (the next
 * GEMV's input). */
pai_status_t b200_launch_gemv(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch,
                              uint64_t n, uint64_t k, const void *w, const b200_xq_t *xq,
                              const float *residual, float *y, int epi,
                              const b200_xq_t *xq_out);
/* The same GEMV with x = rmsnorm_gamma(x_f32, gamma, eps) computed by
 * every CTA in its prologue (pai_ref_rmsnorm_gamma_f32's arithmetic) and
 * quantised into shared memory: no norm kernel, no xq round trip.
 * PAI_ERR_UNSUPPORTED, before any launch, when the quantised x does not
 * fit in a CTA's shared memory: use rmsnorm_xq + gemv then. */
pai_status_t b200_launch_gemv_norm(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch,
                                   uint64_t n, uint64_t k, const void *w, const float *x,
                                   const float *gamma, float eps, const float *residual,
                                   float *y, int epi, const b200_xq_t *xq_out);
/* Quantise x[batch][k] (fp32) into xq. */
pai_status_t b200_launch_xprep(pai_b200_ctx_t *ctx, uint32_t batch, uint64_t k,
                               const float *x, const b200_xq_t *xq);
/* rmsnorm_gamma of each of `rows` rows of n; writes c (fp32) when non-NULL
 * and the quantised result into xq when non-NULL. */
pai_status_t b200_launch_rmsnorm_xq(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n,
                                    const float *a, const float *gamma, float eps,
                                    float *c, const b200_xq_t *xq);
/* x[b] = dequantised row tokens[b] of a packed rows x k table. */
pai_status_t b200_launch_embed(pai_b200_ctx_t *ctx, uint32_t type, uint32_t batch,
                               uint64_t rows, uint64_t k, const void *w,
                               const int32_t *tokens, float *x);
/* Decode attention at position *pos (npos = *pos + 1) when pos is a
 * device pointer; max_npos bounds the launch. q is already rotated. */
pai_status_t b200_launch_attn_decode(pai_b200_ctx_t *ctx, uint32_t batch, uint32_t h,
                                     uint32_t hk, uint32_t hd, const int32_t *pos,
                                     uint64_t npos_host, uint64_t max_npos,
                                     uint64_t cap, uint64_t seq_stride,
                                     const float *q, const uint16_t *kc,
                                     const uint16_t *vc, float *out,
                                     const b200_xq_t *xq_out);
/* Decode-step attention straight from the fused projection rows qkv
 * [batch][(h + 2 hk) hd]: rotates q and k at *pos (tables cos_t/sin_t),
 * appends k and v (fp16) at *pos of each sequence's cache ([hk][cap][hd],
 * seq_stride elements apart), attends over positions 0..*pos and merges
 * the position chunks in the same kernel; out (and xq_out when non-NULL)
 * receive the attention output. */
pai_status_t b200_launch_attn_step(pai_b200_ctx_t *ctx, uint32_t batch, uint32_t h, uint32_t hk,
                                   uint32_t hd, const int32_t *pos, uint64_t max_npos, uint64_t cap,
                                   uint64_t seq_stride, const float *qkv, const float *cos_t,
                                   const float *sin_t, uint16_t *kc, uint16_t *vc, float *out,
                                   const b200_xq_t *xq_out);
pai_status_t b200_launch_argmax(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n,
                                const float *logits, int32_t *out);
/* Tensor-parallel argmax: this shard's (maximum, index + v0) per row into
 * pair[row][2]; then the merge of all ranks' pairs, pairs[rank][row][2]. */
pai_status_t b200_launch_argmax_pair(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, uint32_t v0,
                                     const float *logits, float *pair);
pai_status_t b200_launch_argmax_ranks(pai_b200_ctx_t *ctx, uint32_t rows, uint32_t nranks, const float *pairs,
                                      int32_t *out);
/* Tensor-parallel greedy pick over peer memory: this shard's (maximum,
 * index + v0) per row is stored into every rank's landing buffer, the last
 * CTA waits (bounded) for all ranks' pairs, merges them in rank order,
 * writes tok_out and the next step's tok_in and advances *pos. */
pai_status_t b200_launch_argmax_peer(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n, uint32_t v0,
                                     const float *logits, void *const *land, uint64_t land_rows, uint32_t rank,
                                     uint32_t nranks, int32_t *tok_out, int32_t *tok_in, int32_t *pos);

/* Tensor-parallel exchange over NVLink peer memory (kernels/k_tp.cu). */
#define B200_TP_MAX_RANKS 8
#define B200_TP_HANDLE_BYTES 64
/* This rank's exchange buffer (header + 2 slots of `cap` floats), zeroed,
 * and its IPC handle for the other ranks. */
pai_status_t b200_tp_xbuf_alloc(pai_b200_ctx_t *ctx, uint64_t cap, void **buf, uint8_t handle[B200_TP_HANDLE_BYTES]);
pai_status_t b200_tp_xbuf_open(pai_b200_ctx_t *ctx, const uint8_t handle[B200_TP_HANDLE_BYTES], void **buf);
/* `bytes` of zeroed device memory and its IPC handle (close with
 * b200_tp_xbuf_free; peers map it with b200_tp_xbuf_open). */
pai_status_t b200_ipc_alloc(pai_b200_ctx_t *ctx, uint64_t bytes, void **buf, uint8_t handle[B200_TP_HANDLE_BYTES]);
void b200_tp_xbuf_close(void *buf);
void b200_tp_xbuf_free(void *buf);
float *b200_tp_xbuf_slot(void *buf, uint32_t slot, uint64_t cap);
/* x[0..n) += sum over ranks (in rank order) of slot `slot` of every rank's
 * buffer; bufs[r] = rank r's buffer as mapped in this process. */
pai_status_t b200_launch_tp_allreduce_add(pai_b200_ctx_t *ctx, void *const *bufs, uint32_t rank, uint32_t nranks,
                                          uint32_t slot, uint64_t cap, float *x, uint64_t n);
/* Prompt prefill (kernels/k_prefill.cu). Row r = b * rows_per_seq + i is
 * position p0 + i of sequence b; qkv rows are [(h + 2 hk) hd]. */
pai_status_t b200_launch_prefill_rope_append(pai_b200_ctx_t *ctx, uint32_t rows, uint32_t rows_per_seq,
                                             uint32_t p0, uint32_t h, uint32_t hk, uint32_t hd, float *qkv,
                                             const float *cos_t, const float *sin_t, uint16_t *kc, uint16_t *vc,
                                             uint64_t cap, uint64_t seq_stride);
pai_status_t b200_launch_attn_prefill(pai_b200_ctx_t *ctx, uint32_t rows, uint32_t rows_per_seq, uint32_t p0,
                                      uint32_t h, uint32_t hk, uint32_t hd, const float *qkv, const uint16_t *kc,
                                      const uint16_t *vc, uint64_t cap, uint64_t seq_stride, float *out);
pai_status_t b200_launch_silu_glu_rows(pai_b200_ctx_t *ctx, uint64_t rows, uint32_t ff, const float *gu,
                                       float *hout);
/* ---- persistent decode step (kernels/k_decode*.cu) --------------------------------
 * One cooperative launch runs the layers of a decode step over one CTA per
 * SM: a weight producer streams every matrix of the step, in order, into a
 * shared-memory ring (it never waits for activations, so the next matrix is
 * in flight while the current phase finishes); consumer warps run the
 * phases of each layer in order and meet at a grid barrier between them. */

/* Landing buffer of the tensor-parallel persistent decode: one per rank in
 * its HBM, mapped into every other rank with CUDA IPC.
 *   header (B200_LAND_HDR bytes): u64 words [1] row exchanges this rank
 *   completed, [2] arrivals of greedy pairs (every rank adds 1 per step),
 *   [3] greedy exchanges this rank completed;
 *   row slots [2 parities][ranks][rows] u64 (rows = batch x n_embd): the
 *   rows a rank reduced from its o/down partial sums, each an fp32 value in
 *   the low word and the exchange's tag in the high word, stored by that
 *   rank into slot [parity][rank] of every rank's buffer;
 *   pair slots [2 parities][ranks][8][2] fp32: each rank's (maximum, index)
 *   of its vocabulary shard per sequence. */
#define B200_LAND_HDR 16384u
static inline B200_HD uint64_t b200_land_bytes(uint32_t nranks, uint64_t rows) {
  return B200_LAND_HDR + 2ull * nranks * rows * 8u + 2ull * nranks * 16u * 4u;
}
static inline B200_HD uint64_t b200_land_pairs_off(uint32_t nranks, uint64_t rows) {
  return B200_LAND_HDR + 2ull * nranks * rows * 8u;
}

/* The matrices and norm gains of one layer (packed, this rank's shard). */
typedef struct b200_decode_layer {
  const void *wqkv, *wo, *wgu, *wdown;
  const float *attn_norm, *ffn_norm;
} b200_decode_layer_t;

typedef struct b200_decode_args {
  uint32_t type;                  /* block type of the layer matrices */
  uint32_t batch, n_layer;
  float eps;                      /* RMSNorm epsilon */
  /* embedding: x[b] = row tok_in[b] of the packed vocab x n_embd table */
  uint32_t etype;
  const void *emb;
  uint64_t vocab, n_embd;
  const int32_t *tok_in;
  /* this rank's shapes: q|k|v rows, o input columns, ffn rows per gate/up half */
  uint64_t n_qkv, k_o, ffl;
  /* attention: fp16 cache [layer][seq][kv head][cap][hd], rotary tables [cap][hd/2] */
  uint32_t h, hk, hd;
  int32_t *pos;                   /* device position of the step's token */
  uint64_t cap, seq_stride, layer_stride;
  uint16_t *kc, *vc;
  const float *cos_t, *sin_t;
  /* outputs: the hidden state after the last layer and RMSNorm(x) * out_norm
   * quantised for the lm head */
  const float *out_norm;
  float *x;
  b200_xq_t xq_out;
  /* tensor parallelism: rank of nranks, every rank's landing buffer as
   * mapped here (nranks = 1: none) */
  uint32_t rank, nranks;
  void *land[B200_TP_MAX_RANKS];
} b200_decode_args_t;

typedef struct b200_decode_plan b200_decode_plan_t;
/* Check the shapes against the kernel's limits, size and allocate its
 * scratch (split-K partials, attention partials, the normed operand, block
 * sums of squares, barrier words) and upload the layer table.
 * PAI_ERR_UNSUPPORTED when a shape does not fit. */
pai_status_t b200_decode_plan_create(pai_b200_ctx_t *ctx, const b200_decode_args_t *args,
                                     const b200_decode_layer_t *layers, b200_decode_plan_t **out);
pai_status_t b200_decode_launch(pai_b200_ctx_t *ctx, b200_decode_plan_t *plan);
void b200_decode_plan_destroy(b200_decode_plan_t *plan);

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
