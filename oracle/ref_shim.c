/*
 * ref_shim — exposes the reference's own dequantiser to the test suite.
 *
 * TEST INFRASTRUCTURE ONLY. This translation unit is compiled by
 * oracle/Makefile together with the unmodified reference sources found
 * under $(REF) (the ProsperoAI checkout); nothing from the reference is
 * copied into this repository. adapters/llama/gguf.c keeps its block
 * dequantiser `dequant_block` (gguf.c:651-967) file-static, so the shim
 * includes that source file and re-exports the function under a public
 * name. The result, oracle/_ref/libpai_ref.so, also exports the
 * reference's pai_ref_* (cpu/reference/ref_ops.c), pai_opt_*
 * (cpu/optimized/opt_ops.c), pai_quantize_f32 (models/quantize.c) and
 * pai_sampler_* (models/sampler.c) symbols as built from their sources.
 */
#include "gguf.c"

pai_status_t pai_refshim_dequant(uint32_t type, const uint8_t *src, float *dst,
                                 uint64_t numel) {
  if (pai_gguf_type_bytes(type, numel) == 0) {
    return PAI_ERR_UNSUPPORTED;
  }
  return dequant_block(type, src, dst, numel);
}

/* Byte size of numel elements of a ggml type (gguf.c:563-599). */
uint64_t pai_refshim_type_bytes(uint32_t type, uint64_t numel) {
  return pai_gguf_type_bytes(type, numel);
}
