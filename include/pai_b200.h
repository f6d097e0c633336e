/*
 * pai_b200.h — the `cuda-b200` backend of the ProsperoAI runtime: a C ABI
 * over hand-written sm_100a kernels for the quantized-weights hot path.
 *
 * Everything here is plain C: integers, floats and pointers. Device
 * pointers are returned by pai_b200_alloc and passed back unchanged;
 * nothing in the signatures is a CUDA or PyTorch type. All calls return
 * a ProsperoAI status code (pai/error.h:13-23): PAI_ERR_INVALID_ARG for a
 * NULL or ill-shaped argument, PAI_ERR_MISMATCH for inconsistent shapes,
 * PAI_ERR_UNSUPPORTED for a block type or size the backend does not run,
 * PAI_ERR_NOMEM when device memory is exhausted, PAI_ERR_TIMEOUT when a
 * bounded device wait ran out, and PAI_ERR_INTERNAL for a CUDA or NCCL
 * failure (the message is kept for pai_b200_last_error).
 *
 * Operations are asynchronous on the context's stream, like kernel
 * launches; pai_b200_sync() waits. The reference executor is synchronous
 * (scheduler/scheduler.c:346-632 returns when every step is done), so
 * the integration shim syncs at the same boundaries.
 */
#ifndef PAI_B200_H
#define PAI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- types shared with the reference ABI --------------------------------
 * When the reference headers are included first, theirs are used; the
 * definitions below are layout-identical restatements of them.          */

#ifndef PAI_ERROR_H
typedef int32_t pai_status_t; /* pai/error.h:11 */
#define PAI_OK 0
#define PAI_ERR_INVALID_ARG -1
#define PAI_ERR_NOMEM -2
#define PAI_ERR_UNSUPPORTED -3
#define PAI_ERR_CAPABILITY -4
#define PAI_ERR_TIMEOUT -5
#define PAI_ERR_MISMATCH -6
#define PAI_ERR_IO -7
#define PAI_ERR_INIT -8
#define PAI_ERR_INTERNAL -9
#define PAI_ERR_PROTOCOL -10
#endif

#ifndef PAI_OP_H
typedef int32_t pai_kernel_id_t;               /* pai/op.h:28 */
typedef pai_status_t (*pai_op_ref_fn)(void);   /* pai/op.h:69 */
typedef struct pai_op_descriptor {             /* pai/op.h:71-84 */
  const char *name;
  uint32_t version;
  uint32_t num_inputs;
  uint32_t num_outputs;
  int32_t in_dtype;  /* pai_dtype_t (pai/dtype.h:13-24), an int-sized enum */
  int32_t out_dtype;
  uint32_t caps;
  pai_op_ref_fn ref_fn;
  pai_kernel_id_t kernel_id;
  uint32_t reserved[2];
} pai_op_descriptor_t;
#define PAI_OP_REGISTRY_MAX_OPS 64u            /* pai/op.h:88 */
typedef struct pai_op_registry {               /* pai/op.h:90-94 */
  uint32_t version;
  uint32_t count;
  const pai_op_descriptor_t *ops[PAI_OP_REGISTRY_MAX_OPS];
} pai_op_registry_t;
#endif

/* Capability bit of this backend: the next free bit after
 * PAI_OP_CAP_HOST_REF (pai/op.h:59-61). */
#define PAI_OP_CAP_CUDA_B200 (1u << 3)

/* Kernel ids of this backend, after the reference's 1..13 (pai/op.h:37-51). */
enum {
  PAI_KERNEL_B200_GEMV_Q8_0 = 14,
  PAI_KERNEL_B200_GEMV_Q4_0 = 15,
  PAI_KERNEL_B200_GEMV_Q4_K = 16,
  PAI_KERNEL_B200_GEMM_Q4_0 = 17,
  PAI_KERNEL_B200_RMSNORM = 18,
  PAI_KERNEL_B200_ROPE = 19,
  PAI_KERNEL_B200_ATTN_DECODE = 20,
  PAI_KERNEL_B200_ATTENTION = 21,
  PAI_KERNEL_B200_SILU_MUL = 22,
  PAI_KERNEL_B200_VECADD = 23,
  PAI_KERNEL_B200_DEQUANT = 24,
  PAI_KERNEL_B200_ARGMAX = 25,
  PAI_KERNEL_B200_GEMM_W8 = 26,
  PAI_KERNEL_B200_GEMM_W4 = 27,
  PAI_KERNEL_B200_GEMM_V0 = 28,
  PAI_KERNEL_B200_GEMM_Q8_0 = 29,
  PAI_KERNEL_B200_GEMM_Q4_K = 30
};

/* Quantized weight operand of a descriptor: pai_op_descriptor_t.reserved[0]
 * holds its format -- a ggml block type below, or one of these -- and
 * reserved[1] holds 1 + its input index (0: the op has none). */
#define PAI_B200_WEIGHT_ANY_GGML 0x100u /* any of the ggml block types below            */
#define PAI_B200_WEIGHT_W8_COLS 0x101u  /* int8 [k][n], f32 scales per (k group, column) */
#define PAI_B200_WEIGHT_W4_COLS 0x102u  /* nibbles of the same layout                    */
#define PAI_B200_WEIGHT_V0_BLOB 0x103u  /* a v0 .pai tensor blob (values, flat-group scales) */

/* ggml block types, numbered as adapters/llama/gguf.h:36-51. */
#define PAI_B200_Q4_0 2u  /* 32 weights: fp16 d, 16 B of nibbles       (18 B) */
#define PAI_B200_Q8_0 8u  /* 32 weights: fp16 d, 32 int8                (34 B) */
#define PAI_B200_Q4_K 12u /* 256 weights: fp16 d, fp16 dmin, 12 B packed
                             6-bit scales/mins, 128 B of nibbles      (144 B) */

typedef struct pai_b200_ctx pai_b200_ctx_t;

/* ---- runtime ---------------------------------------------------------------- */

/* Open device `device` and create a context with its own stream and
 * scratch memory. Replaces the PS5 HAL's device bring-up
 * (runtime/runtime.c:18-80, gpu/hal/hal.h:45-61). */
pai_status_t pai_b200_init(int device, pai_b200_ctx_t **out);
pai_status_t pai_b200_shutdown(pai_b200_ctx_t *ctx);
pai_status_t pai_b200_device_count(int *out);
/* Text of the last failure on this thread ("" when none). */
const char *pai_b200_last_error(void);
/* Library build string (kernels, arch). */
const char *pai_b200_version(void);

/* Device memory (the planner region of models/model.c:236 moves here). */
pai_status_t pai_b200_alloc(pai_b200_ctx_t *ctx, uint64_t bytes, void **out);
pai_status_t pai_b200_free(pai_b200_ctx_t *ctx, void *p);
/* Page-locked host memory for copies that overlap compute. */
pai_status_t pai_b200_host_alloc(pai_b200_ctx_t *ctx, uint64_t bytes, void **out);
pai_status_t pai_b200_host_free(pai_b200_ctx_t *ctx, void *p);
pai_status_t pai_b200_memcpy_h2d(pai_b200_ctx_t *ctx, void *dst, const void *src,
                                 uint64_t bytes);
pai_status_t pai_b200_memcpy_d2h(pai_b200_ctx_t *ctx, void *dst, const void *src,
                                 uint64_t bytes);
pai_status_t pai_b200_memcpy_d2d(pai_b200_ctx_t *ctx, void *dst, const void *src,
                                 uint64_t bytes);
pai_status_t pai_b200_memset(pai_b200_ctx_t *ctx, void *dst, int value,
                             uint64_t bytes);
/* Wait for all work queued on the context; reports any device error. */
pai_status_t pai_b200_sync(pai_b200_ctx_t *ctx);
/* Launch this context's kernels with programmatic dependent launch (1) or
 * plainly (0, the default outside a decode step): each kernel then starts
 * its prologue (weight prefetch) while its predecessor on the stream
 * finishes, and waits for the predecessor before it reads dependent data.
 * No reference counterpart. The environment variable PAI_B200_PDL=0
 * disables it for the process. */
pai_status_t pai_b200_set_pdl(pai_b200_ctx_t *ctx, int on);
/* Limit on every bounded wait inside this context's kernels (a bulk copy
 * landing, a peer rank's stamp, a grid barrier), in nanoseconds; 0 restores
 * the default of 2 s, the range is 1 ms to 60 s. A wait that runs out ends
 * its kernel early and the next pai_b200_sync answers PAI_ERR_TIMEOUT: the
 * counterpart of the reference's pai_gpu_wait_label(..., timeout_ns)
 * (gpu/hal/hal.h:106-108). */
pai_status_t pai_b200_set_wait_limit(pai_b200_ctx_t *ctx, uint64_t ns);

/* Stream-ordered timing: event_record places a marker, event_elapsed
 * waits for both markers and returns milliseconds between them. */
pai_status_t pai_b200_event_create(pai_b200_ctx_t *ctx, void **ev);
pai_status_t pai_b200_event_destroy(pai_b200_ctx_t *ctx, void *ev);
pai_status_t pai_b200_event_record(pai_b200_ctx_t *ctx, void *ev);
pai_status_t pai_b200_event_elapsed(void *start, void *stop, float *ms);

/* Number of this library's kernels launched on the context so far
 * (graph replays count every kernel node they run). */
uint64_t pai_b200_launch_count(pai_b200_ctx_t *ctx);

/* CUDA graph capture of the ops enqueued on the context's stream between
 * begin and end (for sequences of small ops whose host launch cost
 * exceeds their device time). Ops that would grow the context's scratch
 * fail during a capture: run each op once before capturing it.
 * pai_b200_graph_launch replays the graph on the context's stream. */
typedef struct pai_b200_graph pai_b200_graph_t;
pai_status_t pai_b200_graph_begin(pai_b200_ctx_t *ctx);
pai_status_t pai_b200_graph_end(pai_b200_ctx_t *ctx, pai_b200_graph_t **graph);
pai_status_t pai_b200_graph_launch(pai_b200_ctx_t *ctx, pai_b200_graph_t *graph);
pai_status_t pai_b200_graph_destroy(pai_b200_graph_t *graph);

/* ---- weight blocks ------------------------------------------------------------- */

/* ggml byte size of numel elements (adapters/llama/gguf.c:563-599);
 * 0 when numel is not a whole number of blocks. */
uint64_t pai_b200_block_bytes(uint32_t type, uint64_t numel);
/* Host block quantiser: numel fp32 values -> ggml blocks.
 *   Q8_0: d = max|w|/127, q = lrintf(w/d) in [-127,127]
 *   Q4_0: d = m/-8 (m the first element of largest |w|),
 *         q = clamp(lrintf(w/d)+8, 0, 15)
 *   Q4_K: per 32-sub-block scale (max-min)/15 and offset -min, 6-bit
 *         codes against fp16 d/dmin = their maxima/63.
 * Dequantising the result with gguf.c:651-967 gives w back to within the
 * block's step. The reference has no ggml quantiser (it dequantises at
 * import, adapters/llama/llama.c:408-457), so these formulas are the
 * benchmark specification's. */
pai_status_t pai_b200_quantize(uint32_t type, const float *src, uint64_t numel,
                               void *dst_blocks);

/* Weights live on the device in a packed layout built once at load from
 * ggml blocks: rows in tiles of 16 and K in units of 128 weights (one
 * super-block for Q4_K), each (tile, unit) piece holding the quant bytes
 * in the operand order of the int8 tensor-core MMA and the block headers
 * in a separate plane; pieces are stored unit-major. Bytes are moved,
 * never re-encoded. Byte count of an n x k matrix in that layout: */
uint64_t pai_b200_packed_bytes(uint32_t type, uint64_t n, uint64_t k);
/* Pack rows of ggml blocks already on the device. Packed row r is taken
 * from src + row_offsets[r] (a device array of n byte offsets; ~0 gives
 * a zero row, ~0-1 leaves the row untouched), reading k/block_elems
 * blocks starting there. Concatenation,
 * interleaving and tensor-parallel slicing are all row-offset tables. */
pai_status_t pai_b200_pack(pai_b200_ctx_t *ctx, uint32_t type, uint64_t n,
                           uint64_t k, const void *src,
                           const uint64_t *row_offsets, void *dst_packed);
/* Upload an n x k ggml matrix from host memory and pack it (convenience
 * over pai_b200_pack with contiguous rows). */
pai_status_t pai_b200_upload_matrix(pai_b200_ctx_t *ctx, uint32_t type, uint64_t n,
                                    uint64_t k, const void *host_blocks,
                                    void *dst_packed);
/* Device dequantisation of a packed n x k matrix to fp32 [n][k],
 * bit-identical to dequant_block (adapters/llama/gguf.c:680-693,
 * 750-761, 852-882). */
pai_status_t pai_b200_dequant(pai_b200_ctx_t *ctx, uint32_t type, uint64_t n,
                              uint64_t k, const void *packed, float *out);

/* ---- hot-path ops (device pointers; asynchronous) ----------------------------- */

/* y[n] = W[n,k] . x[k] with the dequantisation fused into the dot product,
 * fp32 accumulation. Replaces the GEMM/GEMV step of the executor
 * (scheduler/scheduler.c:413-428 -> run_gemm :285-343 -> pai_ref_gemm_f32,
 * ref_ops.c:428-444) for a quantized B operand; the reference result is
 * pai_gguf_dequant + pai_ref_gemv_f32 (ref_ops.c:92-106). */
pai_status_t pai_b200_gemv_q8_0_f32(pai_b200_ctx_t *ctx, uint64_t n, uint64_t k,
                                    const void *w, const float *x, float *y);
pai_status_t pai_b200_gemv_q4_0_f32(pai_b200_ctx_t *ctx, uint64_t n, uint64_t k,
                                    const void *w, const float *x, float *y);
pai_status_t pai_b200_gemv_q4_k_f32(pai_b200_ctx_t *ctx, uint64_t n, uint64_t k,
                                    const void *w, const float *x, float *y);
/* Batched form with optional fused residual: for each of `batch` rows,
 * y[b][n] = (residual ? residual[b][n] : 0) + W . x[b]. The residual add
 * is the executor's following PAI_OP_ADD (scheduler.c:396-403,
 * adapters/llama/llama.c:747-749,793-795), fused. residual may equal y. */
pai_status_t pai_b200_gemv_f32(pai_b200_ctx_t *ctx, uint32_t type, uint64_t batch,
                               uint64_t n, uint64_t k, const void *w,
                               const float *x, const float *residual, float *y);
/* The same GEMV with the activations prepared once for several matrices
 * (the q, k and v projections of one x, for instance). pai_b200_prepare_x_f32
 * writes x[batch][k] into a device buffer of pai_b200_xq_bytes(batch, k)
 * bytes (256-byte aligned) in the GEMV kernels' operand format (24-bit
 * fixed point per 32-element block); pai_b200_gemv_prepared_f32 then
 * multiplies without re-reading x in fp32. Results equal pai_b200_gemv_f32's
 * bit for bit. No counterpart in the reference, whose GEMVs take f32 x
 * each time. */
uint64_t pai_b200_xq_bytes(uint64_t batch, uint64_t k);
pai_status_t pai_b200_prepare_x_f32(pai_b200_ctx_t *ctx, uint64_t batch, uint64_t k,
                                    const float *x, void *xq);
pai_status_t pai_b200_gemv_prepared_f32(pai_b200_ctx_t *ctx, uint32_t type, uint64_t batch,
                                        uint64_t n, uint64_t k, const void *w,
                                        const void *xq, const float *residual, float *y);
/* y[b] = (residual ? residual[b] : 0) + W . rmsnorm_gamma(x[b], gamma, eps):
 * pai_ref_rmsnorm_gamma_f32 (ref_ops.c:196-216) followed by the GEMV, the
 * executor's PAI_OP_RMSNORM -> PAI_OP_GEMM pair (llama.c:674-697), with the
 * norm computed inside the GEMV kernel. PAI_ERR_UNSUPPORTED when x is too
 * long to stay in one CTA's shared memory (k above about 4096 at batch 8,
 * 16384 at batch 1). */
pai_status_t pai_b200_gemv_rmsnorm_f32(pai_b200_ctx_t *ctx, uint32_t type, uint64_t batch,
                                       uint64_t n, uint64_t k, const void *w, const float *x,
                                       const float *gamma, float eps, const float *residual,
                                       float *y);
/* Prefill GEMM with Q4_0 weights: Y[m][n] = X[m][k] . W^T (W packed n x k,
 * X and Y fp32, row-major). pai_ref_gemm_f32 (cpu/reference/ref_ops.c:428-444)
 * on the dequantised weights -- the executor's GEMM for a prompt of m tokens
 * (scheduler/scheduler.c:285-343). Runs on the tcgen05 tensor cores with the
 * weights dequantised to bf16 tiles in shared memory and X rounded to bf16,
 * fp32 accumulation: results match the fp32 reference to about 2^-8
 * relative (the benchmark's bar is max-abs-rel 2e-2). */
pai_status_t pai_b200_gemm_q4_0_f32(pai_b200_ctx_t *ctx, uint64_t m, uint64_t n, uint64_t k,
                                    const float *x, const void *w, float *y);
/* The same GEMM for any packed layer block type: PAI_B200_Q4_0, PAI_B200_Q8_0
 * or PAI_B200_Q4_K (k a whole number of blocks: 32, 32, 256). Each weight is
 * the reference's fp32 dequantised value (gguf.c's arithmetic) rounded once
 * to bf16; same bar as the Q4_0 form. PAI_ERR_UNSUPPORTED for other types. */
pai_status_t pai_b200_gemm_f32(pai_b200_ctx_t *ctx, uint32_t type, uint64_t m, uint64_t n, uint64_t k,
                               const float *x, const void *w, float *y);

/* v0 grouped-scale integer weights (models/quantize.h), read in place.
 * The weight is a [k][n] GEMM B operand (n contiguous), c[m][n] = a[m][k] x W.
 *
 * pai_b200_gemm_w8_f32 / pai_b200_gemm_w4_f32: the registered quantized
 * GEMMs pai_ref_gemm_w8_f32 / pai_ref_gemm_w4_f32 (cpu/reference/ref_ops.c:
 * 447-499, ref_ops.h:164-180) with device pointers and the same arguments:
 * W(t, j) = q(t, j) * b_scales[(t / g) * n + j], q the int8 w_q[t*n + j] or
 * the signed nibble at flat index t*n + j of w_q4 (even index: low nibble),
 * g = group_size (0 or > k: k). Same status codes (PAI_ERR_INVALID_ARG for
 * a zero dimension or a NULL pointer). */
pai_status_t pai_b200_gemm_w8_f32(pai_b200_ctx_t *ctx, uint64_t m, uint64_t n, uint64_t k,
                                  const float *a, const int8_t *w_q, const float *b_scales,
                                  uint64_t group_size, float *c);
pai_status_t pai_b200_gemm_w4_f32(pai_b200_ctx_t *ctx, uint64_t m, uint64_t n, uint64_t k,
                                  const float *a, const int8_t *w_q4, const float *b_scales,
                                  uint64_t group_size, float *c);
/* A quantized tensor of a v0 .pai container as stored: blob = [values]
 * [f32 scales] (pai_quant_weights_bytes bytes, models/quantize.c:53-72;
 * manifest size_bytes, models/container.c:176-182), one scale per
 * group_size consecutive flat elements (0: the whole tensor). c is what the
 * reference computes with pai_dequantize_f32 (models/model.c:259-290) then
 * pai_ref_gemm_f32 (ref_ops.c:428-444), to fp32 accumulation noise, without
 * dequantising. bit_width other than 8 or 4: PAI_ERR_UNSUPPORTED
 * (models/model.c:264-267). */
pai_status_t pai_b200_gemm_v0_f32(pai_b200_ctx_t *ctx, uint32_t bit_width, uint32_t group_size,
                                  uint64_t m, uint64_t n, uint64_t k, const float *a,
                                  const void *blob, float *c);
/* Bytes of such a blob for numel elements; 0 for an unsupported width. */
uint64_t pai_b200_v0_blob_bytes(uint32_t bit_width, uint32_t group_size, uint64_t numel);

/* c = a * gamma * (1/sqrtf(mean(a^2) + eps)) per row of n
 * (pai_ref_rmsnorm_gamma_f32, ref_ops.c:196-216; eps 0 selects 1e-5). */
pai_status_t pai_b200_rmsnorm_gamma_f32(pai_b200_ctx_t *ctx, uint64_t rows,
                                        uint64_t n, const float *a,
                                        const float *gamma, float eps, float *c);
/* out = silu(gate) * up (pai_ref_silu_f32 + pai_ref_vecmul_f32,
 * ref_ops.c:219-228, 124-133). */
pai_status_t pai_b200_silu_mul_f32(pai_b200_ctx_t *ctx, const float *gate,
                                   const float *up, float *out, uint64_t n);
/* c = a + b (pai_ref_vecadd_f32, ref_ops.c:8-17). */
pai_status_t pai_b200_vecadd_f32(pai_b200_ctx_t *ctx, const float *a,
                                 const float *b, float *c, uint64_t n);
/* Rotary embedding, same arguments as pai_ref_rope_f32 (ref_ops.c:231-257;
 * ref_ops.h:96-99): half-split pairs (i, i+r2), row = p*heads + h. */
pai_status_t pai_b200_rope_f32(pai_b200_ctx_t *ctx, const float *x, uint64_t rows,
                               uint64_t hd, uint64_t seq, uint64_t heads,
                               const float *cos_t, const float *sin_t, uint64_t r2,
                               float *out);
/* Host: RoPE tables as pai_ref_rope_cossin_f32 (ref_ops.c:260-279). */
pai_status_t pai_b200_rope_cossin_f32(uint64_t ctx_len, uint64_t r2, float base,
                                      float *cos_t, float *sin_t);
/* Causal GQA attention over position-major fp32 q/k/v
 * (pai_ref_attention_f32, ref_ops.c:287-354). */
pai_status_t pai_b200_attention_f32(pai_b200_ctx_t *ctx, uint64_t h, uint64_t hk,
                                    uint64_t seq, uint64_t hd, const float *q,
                                    const float *k, const float *v, float *out);
/* Decode attention of one query position over an fp16 KV cache laid out
 * [hk][cap][hd]: out[h][hd] for positions 0..npos-1. This is the last row
 * of pai_ref_attention_f32 on the cache contents. */
pai_status_t pai_b200_attn_decode_f16kv(pai_b200_ctx_t *ctx, uint64_t h,
                                        uint64_t hk, uint64_t hd, uint64_t npos,
                                        uint64_t cap, const float *q,
                                        const uint16_t *kcache,
                                        const uint16_t *vcache, float *out);
/* Allocation-free form of pai_b200_attn_decode_f16kv, for callers that
 * cannot allocate device memory when they run attention (a runtime that
 * reserved the whole GPU for its own arena, code running inside CUDA-graph
 * capture, a latency-critical loop). No counterpart in the reference: its
 * attention is CPU-only. Same arguments and result; the chunk partials go
 * to a fixed 4 MiB device array that the library holds on every GPU it is
 * loaded on, so h x ceil(npos/chunk) x 130 floats must fit in 2^20 (about
 * 8000 head-chunks), else PAI_ERR_UNSUPPORTED. The first call on a device
 * looks the array up on that device; make it before any stream capture.
 * Calls share the array: two calls that overlap on the GPU (different
 * streams or contexts of one device) race. Allocates nothing. */
pai_status_t pai_b200_attn_decode_f16kv_noalloc(pai_b200_ctx_t *ctx, uint64_t h,
                                                uint64_t hk, uint64_t hd,
                                                uint64_t npos, uint64_t cap,
                                                const float *q,
                                                const uint16_t *kcache,
                                                const uint16_t *vcache,
                                                float *out);
/* First index of the strict maximum of each row of logits[rows][n]
 * (models/sampler.c:89-99 greedy). out is device int32[rows]. */
pai_status_t pai_b200_argmax_f32(pai_b200_ctx_t *ctx, uint64_t rows, uint64_t n,
                                 const float *logits, int32_t *out);

/* ---- registry ------------------------------------------------------------------- */

/* Register this backend's op descriptors (caps PAI_OP_CAP_CUDA_B200,
 * ref_fn NULL: the CPU twin stays the builtin op of the same meaning) into
 * a registry filled by pai_op_registry_builtin (runtime/op_registry.c:
 * 367-397). Descriptors are static and outlive any registry (pai/op.h:
 * 98-100). Returns PAI_ERR_NOMEM when the 64-op table is full. */
pai_status_t pai_b200_register_ops(pai_op_registry_t *reg);
/* Number of descriptors pai_b200_register_ops adds, and access to them. */
uint32_t pai_b200_op_count(void);
const pai_op_descriptor_t *pai_b200_op(uint32_t i);

/* ---- decoder model and session ---------------------------------------------- */

/* A LLaMA-shaped decoder in the op order of adapters/llama/llama.c:669-797
 * (rmsnorm, q/k/v, rope(q,k), attention, o, add, rmsnorm, gate/up,
 * silu*up, down, add; then final rmsnorm, lm head, greedy). */
typedef struct pai_b200_model_cfg {
  uint32_t n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff, vocab;
  float eps, rope_theta;
  uint32_t wtype; /* block type of the layer matrices (Q4_0/Q8_0/Q4_K) */
  uint32_t etype; /* block type of token embedding and lm head        */
} pai_b200_model_cfg_t;

typedef struct pai_b200_model pai_b200_model_t;
typedef struct pai_b200_session pai_b200_session_t;

/* Tensor kinds for pai_b200_model_set_tensor. */
enum {
  PAI_B200_T_TOK_EMBD = 0, /* [vocab][n_embd] etype blocks  */
  PAI_B200_T_OUTPUT = 1,   /* [vocab][n_embd] etype blocks  */
  PAI_B200_T_OUTPUT_NORM = 2, /* [n_embd] f32               */
  PAI_B200_T_WQ = 3, PAI_B200_T_WK = 4, PAI_B200_T_WV = 5, PAI_B200_T_WO = 6,
  PAI_B200_T_WGATE = 7, PAI_B200_T_WUP = 8, PAI_B200_T_WDOWN = 9,
  PAI_B200_T_ATTN_NORM = 10, PAI_B200_T_FFN_NORM = 11
};

/* Create the model for tensor-parallel rank tp_rank of tp_size (1 for a
 * single GPU). Column-parallel q/k/v/gate/up and vocab-sharded lm head are
 * split by output rows, row-parallel o/down by input columns. */
pai_status_t pai_b200_model_create(pai_b200_ctx_t *ctx,
                                   const pai_b200_model_cfg_t *cfg,
                                   uint32_t tp_rank, uint32_t tp_size,
                                   pai_b200_model_t **out);
pai_status_t pai_b200_model_destroy(pai_b200_model_t *m);

/* ---- GGUF import ------------------------------------------------------------------ */

/* What a LLaMA-family GGUF file describes (adapters/llama/llama.c:304-375
 * reads the same keys): the model configuration (eps is the executor's
 * default 1e-5; wtype/etype the ggml types of the layer matrices and of
 * the embedding/lm head), the container version, context length, rotary
 * dims, whether output.weight is absent (the lm head is then the
 * embedding, llama.c:445-470) and the bytes of the tensors the model uses. */
typedef struct pai_b200_gguf_info {
  pai_b200_model_cfg_t cfg;
  uint32_t version, context_length, n_rot, tied_output;
  uint64_t tensor_count, weight_bytes;
  char architecture[64];
} pai_b200_gguf_info_t;

/* Parse and validate a GGUF file without a GPU (the file is mapped, not
 * read into memory; no size cap). PAI_ERR_IO: the file cannot be opened;
 * PAI_ERR_PROTOCOL: malformed container or tensor bytes outside the file;
 * PAI_ERR_UNSUPPORTED: version, architecture, tensor count over 1024, or
 * a shape/type the backend does not run (head_dim 128 fully rotated, one
 * of Q4_0/Q8_0/Q4_K for all matrices, f32 norms); PAI_ERR_MISMATCH: an
 * absent key or tensor, or inconsistent shapes. */
pai_status_t pai_b200_gguf_inspect(const char *path, pai_b200_gguf_info_t *info);
/* Create the model (pai_b200_model_create for tp_rank of tp_size) and load
 * every tensor's ggml blocks from the file as stored: no f32 dequantisation
 * at import (the reference dequantises and transposes, llama.c:402-470).
 * info, when non-NULL, receives what pai_b200_gguf_inspect reports. */
pai_status_t pai_b200_model_load_gguf(pai_b200_ctx_t *ctx, const char *path, uint32_t tp_rank,
                                      uint32_t tp_size, pai_b200_model_t **out,
                                      pai_b200_gguf_info_t *info);
/* ---- .pai containers holding ggml blocks ---------------------------------------------
 * The reference's .pai container (pai/pai.h:1-20) keeps u32 section offsets
 * and sizes (a 4 GiB file limit) and its IR quantization descriptor
 * (ir/ir.h:95-103) has no ggml block kind, so its LLaMA import dequantises
 * every weight to f32 (llama.c:408-457). Version 2 of the container, read
 * and written here, keeps the magic ("PAIC"), the header and the META
 * payload of version 1 and changes three things:
 *   - section table entries are 24 bytes: u32 type, u32 flags, u64 offset,
 *     u64 size (no 4 GiB limit);
 *   - a MANIFEST entry appends the tensor's pai_ir_quant_t (8 bytes) to the
 *     version-1 entry; ggml-blocked tensors use block structure
 *     PAI_IR_QUANT_BLOCK_GGML with dtype U8 (bytes of blocks, stored as
 *     in GGUF, [out][in]);
 *   - an HPARAMS section (type PAI_B200_PAI_SEC_HPARAMS) holds the LLaMA
 *     configuration: u32 n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff,
 *     vocab, f32 eps, f32 rope_theta, u32 wtype, u32 etype, u32 n_rot,
 *     u32 tied_output (52 bytes).
 * The header CRC-32 (IEEE) covers the header's first 12 bytes, the section
 * table and every payload except WEIGHTS (weights carry no checksum, as in
 * GGUF). A version-1 reader rejects version 2 (pai_pai_open checks the
 * version), so the two never mix. */
#ifndef PAI_IR_H
typedef struct pai_ir_quant { /* ir/ir.h:95-103 */
  uint8_t present, bit_width, scale_repr, zero_point_repr, is_signed, block_structure;
  uint16_t group_size;
} pai_ir_quant_t;
#endif
/* Block structure after PAI_IR_QUANT_BLOCK_GROUP (ir/ir.h:88-93): ggml
 * blocks; group_size = weights per block, bit_width = code bits, scale_repr
 * = F16. Q4_0: 4 bits, 32, signed (codes - 8); Q8_0: 8 bits, 32, signed;
 * Q4_K: 4 bits, 256, unsigned (with per-sub-block mins). */
#define PAI_IR_QUANT_BLOCK_GGML 3u
#define PAI_B200_PAI_VERSION 2u
#define PAI_B200_PAI_SEC_HPARAMS 0x100u
pai_status_t pai_b200_ir_quant_ggml(uint32_t ggml_type, pai_ir_quant_t *out);
/* The ggml type a descriptor names; PAI_ERR_UNSUPPORTED for any other. */
pai_status_t pai_b200_ir_quant_ggml_type(const pai_ir_quant_t *q, uint32_t *ggml_type);
/* Convert a LLaMA-family GGUF file into a version-2 .pai container, blocks
 * copied as stored (no dequantisation, no size limit). */
pai_status_t pai_b200_pai_from_gguf(const char *gguf_path, const char *pai_path);
/* Parse and validate a version-2 .pai container without a GPU; info as for
 * pai_b200_gguf_inspect (version = 2). Status codes as the GGUF reader's. */
pai_status_t pai_b200_pai_inspect(const char *path, pai_b200_gguf_info_t *info);
/* Create the model and load its blocks from a version-2 .pai file, as
 * stored (the file is mapped, not read). */
pai_status_t pai_b200_model_load_pai(pai_b200_ctx_t *ctx, const char *path, uint32_t tp_rank,
                                     uint32_t tp_size, pai_b200_model_t **out,
                                     pai_b200_gguf_info_t *info);
/* Load one whole (unsharded) tensor from host memory: ggml blocks
 * [out][in] for matrices, fp32 for norms. The model keeps its shard. */
pai_status_t pai_b200_model_set_tensor(pai_b200_model_t *m, uint32_t kind,
                                       uint32_t layer, const void *host);
/* Fill every tensor with the seeded synthetic model: weights N(0, 0.02)
 * quantised to the configured block types, norm gains 1.0. */
pai_status_t pai_b200_model_synthesize(pai_b200_model_t *m, uint64_t seed);
/* Seed of one synthetic tensor (kind, layer) of the model seeded `seed`. */
uint64_t pai_b200_tensor_seed(uint64_t seed, uint32_t kind, uint32_t layer);
/* Device generator behind pai_b200_model_synthesize: rows x cols values
 * N(0, stddev) into tmp_f32 (row r is the splitmix64 stream from
 * mix64(seed + r), Box-Muller in double), then ggml blocks of `type`
 * into dst_blocks. Exposed so tests can hand the same blocks to a CPU
 * checker. */
pai_status_t pai_b200_synth_blocks(pai_b200_ctx_t *ctx, uint32_t type, uint64_t rows,
                                   uint64_t cols, uint64_t seed, float stddev,
                                   float *tmp_f32, void *dst_blocks);
/* Device bytes held by the model's weights on this rank. */
uint64_t pai_b200_model_weight_bytes(const pai_b200_model_t *m);
/* Bytes of weights one decode step reads on this rank (all layers plus
 * the lm-head shard plus one embedding row). */
uint64_t pai_b200_model_step_weight_bytes(const pai_b200_model_t *m);

/* ---- tensor parallelism (NCCL over NVLink, one process per GPU) ----------- */

/* No reference counterpart: the reference runs on one device. Ranks of
 * one node share a communicator; the exchange steps of a tensor-parallel
 * decode (all-reduce of the o/down partial sums, argmax across lm-head
 * vocabulary shards) run on it, captured into the session's CUDA graph. */
typedef struct pai_b200_tp pai_b200_tp_t;
#define PAI_B200_TP_ID_BYTES 128
/* Make a communicator id on one rank; hand it to every rank out of band. */
pai_status_t pai_b200_tp_unique_id(uint8_t id[PAI_B200_TP_ID_BYTES]);
/* Join the communicator as `rank` of `size` on ctx's device. Collective:
 * every rank calls it with the same id. */
pai_status_t pai_b200_tp_create(pai_b200_ctx_t *ctx, const uint8_t id[PAI_B200_TP_ID_BYTES],
                                uint32_t rank, uint32_t size, pai_b200_tp_t **out);
pai_status_t pai_b200_tp_destroy(pai_b200_tp_t *tp);
uint32_t pai_b200_tp_rank(const pai_b200_tp_t *tp);
uint32_t pai_b200_tp_size(const pai_b200_tp_t *tp);
/* In-place sum over all ranks of n fp32 values, on the context's stream. */
pai_status_t pai_b200_tp_allreduce_f32(pai_b200_tp_t *tp, float *buf, uint64_t n);
/* The one-shot exchange the tensor-parallel decode uses, for callers that
 * run their own ranks: every rank owns an exchange buffer (a header of
 * arrival stamps and two slots of `cap` floats) in its HBM, maps the other
 * ranks' buffers with their IPC handles, writes its partial sums into a
 * slot of its own buffer, then calls pai_b200_tp_allreduce_add_f32, which
 * stamps its arrival into every rank's header, waits (bounded by the
 * context's wait limit) for all ranks' stamps, and adds the sum of all
 * ranks' slots, in rank order, to x. Plain peer loads and stores over
 * NVLink; no multicast. A rank whose peers never stamp gets
 * PAI_ERR_TIMEOUT from the next pai_b200_sync; the buffers are then out of
 * step and must be made again. No reference counterpart (the reference
 * runs on one device). */
#define PAI_B200_TP_HANDLE_BYTES 64
pai_status_t pai_b200_tp_xbuf_create(pai_b200_ctx_t *ctx, uint64_t cap, void **buf,
                                     uint8_t handle[PAI_B200_TP_HANDLE_BYTES]);
pai_status_t pai_b200_tp_xbuf_open(pai_b200_ctx_t *ctx, const uint8_t handle[PAI_B200_TP_HANDLE_BYTES],
                                   void **buf);
/* Release a buffer: owned = 1 for one made by xbuf_create, 0 for a mapping. */
pai_status_t pai_b200_tp_xbuf_release(pai_b200_ctx_t *ctx, void *buf, int owned);
/* Device address of slot 0 or 1 of a buffer made with capacity `cap`. */
float *pai_b200_tp_xbuf_slot(void *buf, uint32_t slot, uint64_t cap);
/* x[0..n) += sum over ranks r (in rank order) of slot `slot` of bufs[r]
 * (bufs[r] = rank r's buffer as mapped on this rank). */
pai_status_t pai_b200_tp_allreduce_add_f32(pai_b200_ctx_t *ctx, void *const *bufs, uint32_t rank,
                                           uint32_t nranks, uint32_t slot, uint64_t cap, float *x,
                                           uint64_t n);
/* Attach the communicator to a model created for the same rank and size
 * (before pai_b200_session_create; the model does not own it). */
pai_status_t pai_b200_model_set_tp(pai_b200_model_t *m, pai_b200_tp_t *tp);

/* A decode session of `batch` independent sequences with an fp16 KV cache
 * of max_ctx positions per sequence, rounded up to whole 128-position
 * blocks ([layer][sequence][kv_head][pos][head_dim], split by KV head
 * across tensor-parallel ranks). */
pai_status_t pai_b200_session_create(pai_b200_model_t *m, uint32_t batch,
                                     uint32_t max_ctx, pai_b200_session_t **out);
pai_status_t pai_b200_session_destroy(pai_b200_session_t *s);
/* Position of the next token (equal for all sequences). */
uint32_t pai_b200_session_pos(const pai_b200_session_t *s);
/* Reset to position 0 (pai_kv_cache_reset: the count of positions and
 * reservations goes to zero; the cache contents are left, positions >= pos
 * are never read). */
pai_status_t pai_b200_session_reset(pai_b200_session_t *s);
/* One decode step from host memory: feed tokens[batch], run every layer
 * and the lm head, and write the greedy next tokens to next[batch]
 * (host). logits (host, [batch][vocab]) may be NULL. Synchronous: the
 * call returns when `next` is written, like pai_sched_execute. */
pai_status_t pai_b200_session_step(pai_b200_session_t *s, const int32_t *tokens,
                                   int32_t *next, float *logits);
/* Device-resident decode: run `steps` greedy steps, each feeding back the
 * previous step's token, without host round trips (CUDA-graph replays).
 * The first step reads the device token buffer set by the last
 * session_step or session_set_tokens. Asynchronous. */
pai_status_t pai_b200_session_run(pai_b200_session_t *s, uint32_t steps);
/* Prompt prefill: n positions of every sequence (tokens[batch][n], host)
 * appended in one pass per layer instead of n decode steps -- RMSNorm over
 * all rows, the layer matrices as GEMMs over all rows (the tcgen05 GEMM
 * for Q4_0 layers, bf16 tiles with fp32 accumulation; the batched GEMV for
 * Q8_0/Q4_K), RoPE and the fp16 K/V append for every position, causal
 * attention over the cache, SiLU*up, residual adds. next[batch] receives
 * the greedy token after the last position, which is also the input of the
 * next pai_b200_session_run step. Equivalent to stepping the prompt; with
 * Q4_0 layers the bf16 GEMM tiles put the hidden state within about 1e-2
 * (max-abs-rel) of the stepped result. Under tensor parallelism every rank
 * calls it with the same tokens (a collective): the row-parallel o/down
 * outputs of all prompt rows are summed over ranks by an NCCL all-reduce
 * before the residual add. */
pai_status_t pai_b200_session_prefill(pai_b200_session_t *s, const int32_t *tokens, uint32_t n,
                                      int32_t *next);
pai_status_t pai_b200_session_set_tokens(pai_b200_session_t *s,
                                         const int32_t *tokens);
pai_status_t pai_b200_session_get_tokens(pai_b200_session_t *s, int32_t *tokens);
/* Hidden state after the last step (device pointer, [batch][n_embd]). */
const float *pai_b200_session_hidden(const pai_b200_session_t *s);
/* Kernels one decode step launches: 4 when the layers run as the persistent
 * decode kernel (layers, lm head GEMV, greedy pick, token feedback), else one
 * launch per op. */
uint32_t pai_b200_session_step_kernels(const pai_b200_session_t *s);
/* Launch only the persistent layer kernel of a step, `reps` times, on the
 * context's stream (asynchronous): for timing that kernel by itself. The
 * position does not advance, so every launch appends at the same cache
 * position and reads the same positions. PAI_ERR_UNSUPPORTED when the
 * session runs one launch per op. */
pai_status_t pai_b200_session_run_layers(pai_b200_session_t *s, uint32_t reps);

/* ---- KV-cache position accounting ---------------------------------------------
 * The session's cache keeps the bookkeeping of the reference's
 * pai_kv_cache_t (cache/kv_cache.h:29-56): capacity in token positions,
 * whole blocks of PAI_B200_KV_BLOCK_TOKENS positions (PAI_KV_BLOCK_TOKENS,
 * kv_cache.h:27; the session's max_ctx is rounded up to whole blocks), a
 * count of written positions, and reserve/reset with the status codes of
 * pai_kv_cache_reserve (kv_cache.c:125-152). The blocks own device K/V:
 * block b of (layer, sequence, kv head) is positions [128 b, 128 b + 128)
 * of that head's contiguous fp16 rows. Decode steps and prompt prefill
 * reserve their positions through the same accounting, so a full cache
 * answers PAI_ERR_NOMEM as the reference's does. */
#define PAI_B200_KV_BLOCK_TOKENS 128u
typedef struct pai_b200_kv_info {
  uint32_t capacity_tokens; /* positions per sequence (whole blocks)            */
  uint32_t positions;       /* positions written (the next token's position)    */
  uint32_t block_tokens;    /* PAI_B200_KV_BLOCK_TOKENS                          */
  uint32_t n_layer, batch, kv_heads, head_dim; /* kv_heads: this rank's share   */
  uint64_t layer_stride;    /* fp16 elements between layers                     */
  uint64_t seq_stride;      /* ... between sequences of one layer               */
  uint64_t head_stride;     /* ... between kv heads of one sequence (capacity x head_dim) */
  uint64_t stats_blocks;    /* successful reservations (pai_kv_cache_t.stats_blocks) */
  void *k, *v;              /* device: [layer][sequence][kv head][position][head_dim] fp16 */
} pai_b200_kv_info_t;
pai_status_t pai_b200_session_kv_info(const pai_b200_session_t *s, pai_b200_kv_info_t *out);
/* pai_kv_cache_reserve for all sequences of the session: *out_pos = the
 * first of `tokens` new positions, which the caller fills through the
 * pointers of pai_b200_session_kv_info (device memory, e.g. a cache handed
 * over from elsewhere); the next decode step attends over them and writes
 * position *out_pos + tokens. PAI_ERR_INVALID_ARG for tokens == 0 or a NULL
 * pointer; PAI_ERR_NOMEM when the positions do not fit. */
pai_status_t pai_b200_session_kv_reserve(pai_b200_session_t *s, uint32_t tokens, uint32_t *out_pos);

#ifdef __cplusplus
}
#endif

#endif /* PAI_B200_H */
