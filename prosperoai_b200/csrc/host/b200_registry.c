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

#define B200_DESC(nm, nin, kid)                                                         \
  {                                                                                      \
    .name = nm, .version = 1, .num_inputs = nin, .num_outputs = 1, .in_dtype = 0,        \
    .out_dtype = 0, .caps = PAI_OP_CAP_CUDA_B200, .ref_fn = 0, .kernel_id = kid,          \
    .reserved = {0, 0}                                                                   \
  }

/* in/out dtype 0 is PAI_DTYPE_F32 (pai/dtype.h:14): activations are f32;
 * the quantized weight operand is described by the op name. */
static const pai_op_descriptor_t s_ops[] = {
    B200_DESC("gemv_q8_0_f32", 2, PAI_KERNEL_B200_GEMV_Q8_0),     /* W blocks, x     */
    B200_DESC("gemv_q4_0_f32", 2, PAI_KERNEL_B200_GEMV_Q4_0),
    B200_DESC("gemv_q4_k_f32", 2, PAI_KERNEL_B200_GEMV_Q4_K),
    B200_DESC("gemm_q4_0_f32", 2, PAI_KERNEL_B200_GEMM_Q4_0),     /* X, W blocks     */
    B200_DESC("rmsnorm_gamma_f32_b200", 2, PAI_KERNEL_B200_RMSNORM), /* a, gamma     */
    B200_DESC("rope_f32_b200", 3, PAI_KERNEL_B200_ROPE),          /* x, cos, sin     */
    B200_DESC("attention_decode_f16kv", 3, PAI_KERNEL_B200_ATTN_DECODE), /* q, K, V  */
    B200_DESC("attention_f32_b200", 3, PAI_KERNEL_B200_ATTENTION), /* q, k, v        */
    B200_DESC("silu_mul_f32", 2, PAI_KERNEL_B200_SILU_MUL),       /* gate, up        */
    B200_DESC("vecadd_f32_b200", 2, PAI_KERNEL_B200_VECADD),
    B200_DESC("dequant_block_f32", 1, PAI_KERNEL_B200_DEQUANT),
    B200_DESC("argmax_f32", 1, PAI_KERNEL_B200_ARGMAX),
    B200_DESC("gemm_w8_f32_b200", 3, PAI_KERNEL_B200_GEMM_W8),    /* a, w_q, b_scales */
    B200_DESC("gemm_w4_f32_b200", 3, PAI_KERNEL_B200_GEMM_W4),    /* a, w_q4, b_scales */
    B200_DESC("gemm_v0_f32", 2, PAI_KERNEL_B200_GEMM_V0),         /* a, .pai blob    */
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
