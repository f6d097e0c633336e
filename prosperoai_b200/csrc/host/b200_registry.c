/*
 * Op descriptors of the cuda-b200 backend, registered into a ProsperoAI
 * op registry (runtime/op_registry.c:367-377). The descriptor fields are
 * those of pai/op.h:71-84; names follow the builtin table's convention
 * (runtime/op_registry.c:65-343: "<op>_<dtype>"). Every op advertises
 * PAI_OP_CAP_CUDA_B200 only: its CPU twin is the builtin op of the same
 * meaning (gemm_f32 / rmsnorm_f32 / rope_f32 / attention_f32 ...), which
 * keeps PAI_OP_CAP_CPU_REF and the pai_ref_* function.
 */
#include "../b200_internal.h"

/* in/out dtype 0 is PAI_DTYPE_F32 (pai/dtype.h:14): the activation operands
 * and the outputs are f32. The reference's dtype carries only storage, and
 * quantization is metadata (pai/dtype.h:1-5), so a descriptor names its
 * quantized weight operand in reserved[]: reserved[0] = block format
 * (PAI_B200_WEIGHT_*: a ggml type id, or a v0 .pai grouped format),
 * reserved[1] = 1 + the index of that operand among the inputs (0: none).
 * ref_fn is NULL: these ops have no CPU path (pai_op_eval_f32 answers
 * PAI_ERR_UNSUPPORTED for them, op_registry.c:479-480); their CPU twins are
 * the builtin ops of the same meaning (gemm_f32, rmsnorm_f32, ...). */
#define B200_DESC(nm, nin, kid, wfmt, warg)                                              \
  {                                                                                      \
    .name = nm, .version = 1, .num_inputs = nin, .num_outputs = 1, .in_dtype = 0,        \
    .out_dtype = 0, .caps = PAI_OP_CAP_CUDA_B200, .ref_fn = 0, .kernel_id = kid,          \
    .reserved = {wfmt, warg}                                                             \
  }

static const pai_op_descriptor_t s_ops[] = {
    B200_DESC("gemv_q8_0_f32", 2, PAI_KERNEL_B200_GEMV_Q8_0, PAI_B200_Q8_0, 1), /* W blocks, x */
    B200_DESC("gemv_q4_0_f32", 2, PAI_KERNEL_B200_GEMV_Q4_0, PAI_B200_Q4_0, 1),
    B200_DESC("gemv_q4_k_f32", 2, PAI_KERNEL_B200_GEMV_Q4_K, PAI_B200_Q4_K, 1),
    B200_DESC("gemm_q4_0_f32", 2, PAI_KERNEL_B200_GEMM_Q4_0, PAI_B200_Q4_0, 2), /* X, W blocks */
    B200_DESC("gemm_q8_0_f32", 2, PAI_KERNEL_B200_GEMM_Q8_0, PAI_B200_Q8_0, 2),
    B200_DESC("gemm_q4_k_f32", 2, PAI_KERNEL_B200_GEMM_Q4_K, PAI_B200_Q4_K, 2),
    B200_DESC("rmsnorm_gamma_f32_b200", 2, PAI_KERNEL_B200_RMSNORM, 0, 0),     /* a, gamma */
    B200_DESC("rope_f32_b200", 3, PAI_KERNEL_B200_ROPE, 0, 0),                 /* x, cos, sin */
    B200_DESC("attention_decode_f16kv", 3, PAI_KERNEL_B200_ATTN_DECODE, 0, 0), /* q, K, V (fp16 cache) */
    B200_DESC("attention_f32_b200", 3, PAI_KERNEL_B200_ATTENTION, 0, 0),       /* q, k, v */
    B200_DESC("silu_mul_f32", 2, PAI_KERNEL_B200_SILU_MUL, 0, 0),              /* gate, up */
    B200_DESC("vecadd_f32_b200", 2, PAI_KERNEL_B200_VECADD, 0, 0),
    B200_DESC("dequant_block_f32", 1, PAI_KERNEL_B200_DEQUANT, PAI_B200_WEIGHT_ANY_GGML, 1),
    B200_DESC("argmax_f32", 1, PAI_KERNEL_B200_ARGMAX, 0, 0),
    B200_DESC("gemm_w8_f32_b200", 3, PAI_KERNEL_B200_GEMM_W8, PAI_B200_WEIGHT_W8_COLS, 2), /* a, w_q, scales */
    B200_DESC("gemm_w4_f32_b200", 3, PAI_KERNEL_B200_GEMM_W4, PAI_B200_WEIGHT_W4_COLS, 2), /* a, w_q4, scales */
    B200_DESC("gemm_v0_f32", 2, PAI_KERNEL_B200_GEMM_V0, PAI_B200_WEIGHT_V0_BLOB, 2),      /* a, .pai blob */
};

#define B200_NOPS (sizeof(s_ops) / sizeof(s_ops[0]))

uint32_t pai_b200_op_count(void) { return (uint32_t)B200_NOPS; }

const pai_op_descriptor_t *pai_b200_op(uint32_t i) { return i < B200_NOPS ? &s_ops[i] : 0; }

pai_status_t pai_b200_register_ops(pai_op_registry_t *reg) {
  if (!reg) {
    return b200_fail(PAI_ERR_INVALID_ARG, "register_ops: NULL registry");
  }
  if (reg->count + B200_NOPS > PAI_OP_REGISTRY_MAX_OPS) {
    return b200_fail(PAI_ERR_NOMEM, "register_ops: %u ops registered, %u more do not fit in %u", reg->count,
                     (unsigned)B200_NOPS, PAI_OP_REGISTRY_MAX_OPS);
  }
  /* Same append as pai_op_registry_register (op_registry.c:367-377). */
  for (uint32_t i = 0; i < B200_NOPS; i++) {
    reg->ops[reg->count++] = &s_ops[i];
  }
  return PAI_OK;
}
