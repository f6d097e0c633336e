/*
 * Tensor-parallel exchange steps of the decode (all-reduce of the
 * row-parallel o/down partial sums, sharded lm-head argmax). The
 * single-GPU build path never calls these; a model created with
 * tp_size > 1 needs a communicator before a session can be created.
 */
#include "../b200_internal.h"

pai_status_t b200_tp_allreduce(void *tp, pai_b200_ctx_t *ctx, float *buf, uint64_t n) {
  (void)ctx;
  (void)buf;
  (void)n;
  if (!tp) return b200_fail(PAI_ERR_INIT, "tp_allreduce: no communicator");
  return b200_fail(PAI_ERR_UNSUPPORTED, "tp_allreduce: not built");
}

pai_status_t b200_tp_argmax(void *tp, pai_b200_ctx_t *ctx, uint32_t batch, uint32_t vl, uint32_t v0,
                            const float *logits, int32_t *tok_out) {
  (void)ctx;
  (void)batch;
  (void)vl;
  (void)v0;
  (void)logits;
  (void)tok_out;
  if (!tp) return b200_fail(PAI_ERR_INIT, "tp_argmax: no communicator");
  return b200_fail(PAI_ERR_UNSUPPORTED, "tp_argmax: not built");
}
