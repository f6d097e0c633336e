/*
 * ref_dispatch -- the reference's graph executor with a cuda-b200 branch.
 *
 * TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file into
 * _ref/libpai_ref.so beside the unmodified reference sources; nothing of
 * the reference is copied here. It drives the reference's own graph
 * builder (graph/graph.c), memory planner (memory/planner.c), scheduler
 * (scheduler/scheduler.c: pai_sched_build, pai_kernel_select,
 * pai_kernel_plan_check, pai_sched_execute) and op registry
 * (runtime/op_registry.c) over a small decoder slice
 *
 *     h = rmsnorm(x, gamma);  y = h . W^T;  out = y + res
 *
 * (adapters/llama/llama.c:674-697 and 747-749: the attention-input norm,
 * one projection and the residual add), and adds what a maintainer adds
 * to pai_sched_execute_hooked (scheduler.c:346-632) for GPU-placed steps:
 *
 *  - b200_op_name: graph op -> this backend's registry name, the
 *    counterpart of op_registry_name (scheduler.c:647-682). The weight's
 *    block format comes from a side table: a graph value carries only its
 *    storage dtype (graph/graph.h:46-55), and the reference's executor
 *    refuses every non-f32 value (scheduler.c:366-377).
 *  - b200_plan_check: the capability gate over that name map, the
 *    counterpart of pai_kernel_plan_check (scheduler.c:721-748) asked for
 *    PAI_OP_CAP_CUDA_B200.
 *  - b200_step: dispatch on the selected descriptor's kernel_id into the
 *    backend's C ABI, bound with dlopen/dlsym as an optional plugin.
 *
 * The reference executor runs the same plan on the host with the weights
 * dequantised by the reference's own dequant_block (ref_shim.c), which is
 * the result the GPU branch is compared with.
 */
#include <dlfcn.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <graph/graph.h>
#include <pai/error.h>
#include <pai/op.h>
#include <scheduler/scheduler.h>

#include "../include/pai_b200.h"

pai_status_t pai_refshim_dequant(uint32_t type, const uint8_t *src, float *dst,
                                 uint64_t numel);

/* Outcome of one refdisp_run, read by the tests through ctypes. */
typedef struct refdisp_report {
  int32_t gate_cpu_ref;      /* pai_kernel_plan_check(..., PAI_OP_CAP_CPU_REF, reg)  */
  int32_t gate_b200_ref_map; /* pai_kernel_plan_check(..., PAI_OP_CAP_CUDA_B200, reg) */
  int32_t gate_b200;         /* b200_plan_check: the gate over the extended name map */
  int32_t cpu_status;        /* pai_sched_execute on the host                         */
  int32_t gpu_status;        /* the GPU branch (1: not run)                           */
  uint32_t num_steps;
  uint32_t gpu_steps;        /* steps the plan placed on the GPU                      */
  int32_t kernel_ids[4];     /* descriptor kernel_id each step was dispatched through */
  uint8_t devices[4];        /* pai_sched_device_t of each step                       */
  char error[256];
} refdisp_report_t;

/* The backend's entry points, resolved from the plugin. */
typedef struct b200_api {
  void *lib;
  __typeof__(pai_b200_init) *init;
  __typeof__(pai_b200_shutdown) *shutdown;
  __typeof__(pai_b200_alloc) *alloc;
  __typeof__(pai_b200_free) *free_;
  __typeof__(pai_b200_memcpy_h2d) *h2d;
  __typeof__(pai_b200_memcpy_d2h) *d2h;
  __typeof__(pai_b200_sync) *sync;
  __typeof__(pai_b200_last_error) *last_error;
  __typeof__(pai_b200_packed_bytes) *packed_bytes;
  __typeof__(pai_b200_upload_matrix) *upload_matrix;
  __typeof__(pai_b200_gemv_f32) *gemv_f32;
  __typeof__(pai_b200_gemm_f32) *gemm_f32;
  __typeof__(pai_b200_rmsnorm_gamma_f32) *rmsnorm_gamma_f32;
  __typeof__(pai_b200_vecadd_f32) *vecadd_f32;
  __typeof__(pai_b200_register_ops) *register_ops;
} b200_api_t;

static int bind_api(const char *path, b200_api_t *api, char *err, size_t errn) {
  memset(api, 0, sizeof(*api));
  api->lib = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!api->lib) {
    snprintf(err, errn, "dlopen %s: %s", path, dlerror());
    return -1;
  }
#define BIND(field, sym)                                          \
  do {                                                            \
    *(void **)&api->field = dlsym(api->lib, #sym);                \
    if (!api->field) {                                            \
      snprintf(err, errn, "%s: missing symbol %s", path, #sym);   \
      return -1;                                                  \
    }                                                             \
  } while (0)
  BIND(init, pai_b200_init);
  BIND(shutdown, pai_b200_shutdown);
  BIND(alloc, pai_b200_alloc);
  BIND(free_, pai_b200_free);
  BIND(h2d, pai_b200_memcpy_h2d);
  BIND(d2h, pai_b200_memcpy_d2h);
  BIND(sync, pai_b200_sync);
  BIND(last_error, pai_b200_last_error);
  BIND(packed_bytes, pai_b200_packed_bytes);
  BIND(upload_matrix, pai_b200_upload_matrix);
  BIND(gemv_f32, pai_b200_gemv_f32);
  BIND(gemm_f32, pai_b200_gemm_f32);
  BIND(rmsnorm_gamma_f32, pai_b200_rmsnorm_gamma_f32);
  BIND(vecadd_f32, pai_b200_vecadd_f32);
  BIND(register_ops, pai_b200_register_ops);
#undef BIND
  return 0;
}

/* A quantized weight value of the graph: its ggml block type and, once
 * uploaded, the backend's packed copy on the device. */
typedef struct quant_side {
  pai_graph_value_id value;
  uint32_t type;
  void *packed;
} quant_side_t;

static const char *block_suffix(uint32_t type) {
  switch (type) {
    case PAI_B200_Q4_0: return "q4_0";
    case PAI_B200_Q8_0: return "q8_0";
    case PAI_B200_Q4_K: return "q4_k";
    default: return NULL;
  }
}

/* Index of the op's input that the side table marks quantized, or -1. */
static int quant_input(const pai_graph_op_t *op, const quant_side_t *q) {
  for (uint32_t i = 0; i < op->num_inputs; i++) {
    if (op->inputs[i] == q->value) {
      return (int)i;
    }
  }
  return -1;
}

/* Registry name of this backend's implementation of a graph op (NULL: none).
 * GEMV's A operand and GEMM/MATMUL's B operand are the weight
 * (scheduler.c:285-343), the positions the descriptors' reserved[1] name. */
static const char *b200_op_name(const pai_graph_op_t *op, const quant_side_t *q,
                                char *buf, size_t bufn) {
  int qi = quant_input(op, q);
  const char *sfx = block_suffix(q->type);
  switch (op->kind) {
    case PAI_OP_GEMV:
      if (qi != 0 || !sfx) return NULL;
      snprintf(buf, bufn, "gemv_%s_f32", sfx);
      return buf;
    case PAI_OP_GEMM:
    case PAI_OP_MATMUL:
      if (qi != 1 || !sfx) return NULL;
      snprintf(buf, bufn, "gemm_%s_f32", sfx);
      return buf;
    case PAI_OP_RMSNORM:
      return op->num_inputs == 2 ? "rmsnorm_gamma_f32_b200" : NULL;
    case PAI_OP_ADD:
      return "vecadd_f32_b200";
    default:
      return NULL;
  }
}

/* The selected descriptor for a GPU-placed step, checked against the
 * capability bit and the quantized operand it declares in reserved[]. */
static const pai_op_descriptor_t *b200_select(const pai_graph_op_t *op, const quant_side_t *q,
                                              const pai_op_registry_t *reg) {
  char buf[64];
  const char *name = b200_op_name(op, q, buf, sizeof(buf));
  const pai_op_descriptor_t *d = name ? pai_op_registry_lookup(reg, name) : NULL;
  if (!d || !pai_op_supports(d, PAI_OP_CAP_CUDA_B200)) {
    return NULL;
  }
  if (d->reserved[1] != 0) {
    int qi = quant_input(op, q);
    if (qi < 0 || d->reserved[0] != q->type || d->reserved[1] != (uint32_t)qi + 1) {
      return NULL;
    }
  }
  return d;
}

static pai_status_t b200_plan_check(const pai_graph_t *g, const pai_sched_plan_t *plan,
                                    const pai_op_registry_t *reg, const quant_side_t *q) {
  for (uint32_t i = 0; i < plan->num_steps; i++) {
    const pai_sched_step_t *s = &plan->steps[i];
    if (s->device == PAI_SCHED_DEV_GPU && !b200_select(&g->ops[s->op_id], q, reg)) {
      return PAI_ERR_UNSUPPORTED;
    }
  }
  return PAI_OK;
}

static uint64_t nelem(const pai_graph_value_t *v) {
  uint64_t e = 1;
  for (uint32_t d = 0; d < v->rank; d++) {
    e *= v->shape[d];
  }
  return e;
}

/* One GPU-placed step: dispatch on the descriptor's kernel_id. dev is the
 * device copy of the planned region (the reference memory plan's offsets). */
static pai_status_t b200_step(const b200_api_t *api, pai_b200_ctx_t *ctx, const pai_graph_t *g,
                              const pai_graph_mem_plan_t *mp, uint8_t *dev,
                              const pai_graph_op_t *op, const pai_op_descriptor_t *d,
                              const quant_side_t *q) {
#define DPTR(v) ((float *)(dev + pai_graph_mem_plan_offset(mp, (v))))
  const pai_graph_value_t *a = &g->values[op->inputs[0]];
  const pai_graph_value_t *b = op->num_inputs > 1 ? &g->values[op->inputs[1]] : NULL;
  switch (d->kernel_id) {
    case PAI_KERNEL_B200_GEMV_Q8_0:
    case PAI_KERNEL_B200_GEMV_Q4_0:
    case PAI_KERNEL_B200_GEMV_Q4_K: /* y[n] = W[n,k] . x[k] */
      return api->gemv_f32(ctx, d->reserved[0], 1, a->shape[0], a->shape[1], q->packed,
                           DPTR(op->inputs[1]), NULL, DPTR(op->outputs[0]));
    case PAI_KERNEL_B200_GEMM_Q4_0:
    case PAI_KERNEL_B200_GEMM_Q8_0:
    case PAI_KERNEL_B200_GEMM_Q4_K: /* Y[m,n] = X[m,k] . B[k,n], B = W^T */
      return api->gemm_f32(ctx, d->reserved[0], a->shape[0], b->shape[1], a->shape[1],
                           DPTR(op->inputs[0]), q->packed, DPTR(op->outputs[0]));
    case PAI_KERNEL_B200_RMSNORM: {
      uint64_t cols = a->shape[a->rank - 1];
      return api->rmsnorm_gamma_f32(ctx, nelem(a) / cols, cols, DPTR(op->inputs[0]),
                                    DPTR(op->inputs[1]), 0.0f, DPTR(op->outputs[0]));
    }
    case PAI_KERNEL_B200_VECADD:
      return api->vecadd_f32(ctx, DPTR(op->inputs[0]), DPTR(op->inputs[1]),
                             DPTR(op->outputs[0]), nelem(a));
    default:
      return PAI_ERR_UNSUPPORTED;
  }
#undef DPTR
}

typedef struct slice {
  pai_graph_t *g;
  pai_graph_mem_plan_t mp;
  pai_sched_plan_t *plan;
  pai_graph_value_id x, gamma, w, h, y, res, out;
} slice_t;

/* The decoder slice as the reference's graph: m == 1 is a decode step
 * (GEMV, A = W[n,k]), m > 1 a prompt (MATMUL, B = W^T[k,n]). */
static pai_status_t build_slice(slice_t *s, uint64_t m, uint64_t n, uint64_t k) {
  uint64_t row[2] = {m, k}, vk[1] = {k}, wnk[2] = {n, k}, wkn[2] = {k, n};
  uint64_t orow[2] = {m, n};
  int rank = m == 1 ? 1 : 2;
  const uint64_t *xs = m == 1 ? vk : row;
  const uint64_t *os = m == 1 ? &orow[1] : orow;
  uint8_t *hints;
  pai_status_t st;

  pai_graph_init(s->g);
  s->x = pai_graph_add_value(s->g, PAI_DTYPE_F32, rank, xs, 0);
  s->gamma = pai_graph_add_value(s->g, PAI_DTYPE_F32, 1, vk, 0);
  s->w = pai_graph_add_value(s->g, PAI_DTYPE_F32, 2, m == 1 ? wnk : wkn, 0);
  s->h = pai_graph_add_value(s->g, PAI_DTYPE_F32, rank, xs, 0);
  s->y = pai_graph_add_value(s->g, PAI_DTYPE_F32, rank, os, 0);
  s->res = pai_graph_add_value(s->g, PAI_DTYPE_F32, rank, os, 0);
  s->out = pai_graph_add_value(s->g, PAI_DTYPE_F32, rank, os, 0);
  if (!s->x || !s->gamma || !s->w || !s->h || !s->y || !s->res || !s->out) {
    return PAI_ERR_INVALID_ARG;
  }
  pai_graph_set_input(s->g, s->x);
  pai_graph_set_input(s->g, s->gamma);
  pai_graph_set_input(s->g, s->w);
  pai_graph_set_input(s->g, s->res);
  pai_graph_set_output(s->g, s->out);

  pai_graph_value_id norm_in[2] = {s->x, s->gamma};
  pai_graph_value_id gemv_in[2] = {s->w, s->h};
  pai_graph_value_id gemm_in[2] = {s->h, s->w};
  pai_graph_value_id add_in[2] = {s->y, s->res};
  pai_graph_op_id o1 = pai_graph_add_op(s->g, PAI_OP_RMSNORM, 2, 1, norm_in, &s->h);
  pai_graph_op_id o2 = m == 1 ? pai_graph_add_op(s->g, PAI_OP_GEMV, 2, 1, gemv_in, &s->y)
                              : pai_graph_add_op(s->g, PAI_OP_MATMUL, 2, 1, gemm_in, &s->y);
  pai_graph_op_id o3 = pai_graph_add_op(s->g, PAI_OP_ADD, 2, 1, add_in, &s->out);
  if (!o1 || !o2 || !o3) {
    return PAI_ERR_INVALID_ARG;
  }
  st = pai_graph_memory_plan_persistent(s->g, &s->mp);
  if (st != PAI_OK) {
    return st;
  }
  /* every op hinted to the GPU (RMSNORM and ADD default to the CPU) */
  hints = calloc(PAI_GRAPH_MAX_OPS + 1, 1);
  if (!hints) {
    return PAI_ERR_NOMEM;
  }
  hints[o1] = hints[o2] = hints[o3] = PAI_SCHED_DEV_GPU;
  st = pai_sched_build(s->g, &s->mp, PAI_SCHED_INTERACTIVE, hints, s->plan);
  free(hints);
  return st;
}

/* Runs the slice through the reference executor on the host (out_cpu) and,
 * when run_gpu, through the GPU branch (out_gpu). w_blocks: n rows of k
 * weights as ggml blocks of wtype; x and h are [m][k], res and out [m][n].
 * Returns 0 when the harness itself ran; the statuses are in *rep. */
int32_t refdisp_run(const char *backend_so, int32_t run_gpu, uint32_t wtype, uint64_t m,
                    uint64_t n, uint64_t k, const void *w_blocks, const float *x,
                    const float *gamma, const float *res, float *out_cpu, float *out_gpu,
                    refdisp_report_t *rep) {
  slice_t s;
  b200_api_t api;
  pai_op_registry_t reg;
  quant_side_t q = {0, wtype, NULL};
  uint8_t *host = NULL;
  float *wf = NULL;
  int32_t rc = -1;

  memset(rep, 0, sizeof(*rep));
  memset(&s, 0, sizeof(s));
  rep->gpu_status = 1;
  if (m == 0 || n == 0 || k == 0) {
    snprintf(rep->error, sizeof(rep->error), "empty slice");
    return -1;
  }
  s.g = calloc(1, sizeof(pai_graph_t));
  s.plan = calloc(1, sizeof(pai_sched_plan_t));
  if (!s.g || !s.plan || bind_api(backend_so, &api, rep->error, sizeof(rep->error)) != 0) {
    goto done;
  }
  if (build_slice(&s, m, n, k) != PAI_OK || s.plan->num_steps != 3) {
    snprintf(rep->error, sizeof(rep->error), "graph/plan build failed");
    goto done;
  }
  q.value = s.w;
  rep->num_steps = s.plan->num_steps;
  rep->gpu_steps = s.plan->gpu_steps;
  for (uint32_t i = 0; i < s.plan->num_steps; i++) {
    rep->devices[i] = s.plan->steps[i].device;
  }

  /* the registry: the reference's builtins, then this backend's descriptors */
  if (pai_op_registry_builtin(&reg) != PAI_OK || api.register_ops(&reg) != PAI_OK) {
    snprintf(rep->error, sizeof(rep->error), "registry setup failed");
    goto done;
  }
  rep->gate_cpu_ref = pai_kernel_plan_check(s.g, s.plan, PAI_OP_CAP_CPU_REF, &reg);
  rep->gate_b200_ref_map = pai_kernel_plan_check(s.g, s.plan, PAI_OP_CAP_CUDA_B200, &reg);
  rep->gate_b200 = b200_plan_check(s.g, s.plan, &reg, &q);

  /* host run of the reference executor on the dequantised weights */
  uint64_t region = s.plan->region_bytes;
  for (pai_graph_value_id v = 1; v <= s.g->num_values; v++) {
    if (pai_graph_mem_plan_offset(&s.mp, v) + s.g->values[v].size_bytes > region) {
      snprintf(rep->error, sizeof(rep->error), "value %u lies outside the planned region", v);
      goto done;
    }
  }
  host = aligned_alloc(64, (region + 63) / 64 * 64);
  wf = malloc(n * k * sizeof(float));
  if (!host || !wf) {
    snprintf(rep->error, sizeof(rep->error), "host allocation failed");
    goto done;
  }
#define HPTR(v) ((float *)(host + pai_graph_mem_plan_offset(&s.mp, (v))))
  memcpy(HPTR(s.x), x, m * k * sizeof(float));
  memcpy(HPTR(s.gamma), gamma, k * sizeof(float));
  memcpy(HPTR(s.res), res, m * n * sizeof(float));
  if (pai_refshim_dequant(wtype, w_blocks, wf, n * k) != PAI_OK) {
    snprintf(rep->error, sizeof(rep->error), "dequant of type %u failed", wtype);
    goto done;
  }
  if (m == 1) {
    memcpy(HPTR(s.w), wf, n * k * sizeof(float));
  } else {
    float *wt = HPTR(s.w);
    for (uint64_t r = 0; r < n; r++) {
      for (uint64_t c = 0; c < k; c++) {
        wt[c * n + r] = wf[r * k + c];
      }
    }
  }
  rep->cpu_status = pai_sched_execute(s.g, &s.mp, s.plan, host, NULL);
  memcpy(out_cpu, HPTR(s.out), m * n * sizeof(float));
#undef HPTR

  if (run_gpu) {
    pai_b200_ctx_t *ctx = NULL;
    uint8_t *dev = NULL;
    pai_status_t st = api.init(0, &ctx);
    if (st == PAI_OK) st = api.alloc(ctx, region, (void **)&dev);
    if (st == PAI_OK) st = api.alloc(ctx, api.packed_bytes(wtype, n, k), &q.packed);
    if (st == PAI_OK) st = api.upload_matrix(ctx, wtype, n, k, w_blocks, q.packed);
#define DOFF(v) (dev + pai_graph_mem_plan_offset(&s.mp, (v)))
    if (st == PAI_OK) st = api.h2d(ctx, DOFF(s.x), x, m * k * sizeof(float));
    if (st == PAI_OK) st = api.h2d(ctx, DOFF(s.gamma), gamma, k * sizeof(float));
    if (st == PAI_OK) st = api.h2d(ctx, DOFF(s.res), res, m * n * sizeof(float));
    /* the executor loop's GPU branch (scheduler.c:362-622) */
    for (uint32_t i = 0; st == PAI_OK && i < s.plan->num_steps; i++) {
      const pai_sched_step_t *step = &s.plan->steps[i];
      const pai_graph_op_t *op = &s.g->ops[step->op_id];
      const pai_op_descriptor_t *d;
      if (step->device != PAI_SCHED_DEV_GPU || !(d = b200_select(op, &q, &reg))) {
        st = PAI_ERR_UNSUPPORTED;
        break;
      }
      rep->kernel_ids[i] = d->kernel_id;
      st = b200_step(&api, ctx, s.g, &s.mp, dev, op, d, &q);
    }
    if (st == PAI_OK) st = api.sync(ctx);
    if (st == PAI_OK) st = api.d2h(ctx, out_gpu, DOFF(s.out), m * n * sizeof(float));
    if (st == PAI_OK) st = api.sync(ctx);
#undef DOFF
    if (st != PAI_OK) {
      snprintf(rep->error, sizeof(rep->error), "GPU branch: %s", api.last_error());
    }
    rep->gpu_status = st;
    if (q.packed) api.free_(ctx, q.packed);
    if (dev) api.free_(ctx, dev);
    if (ctx) api.shutdown(ctx);
  }
  rc = 0;

done:
  free(wf);
  free(host);
  if (s.g) {
    pai_graph_mem_plan_free(&s.mp);
  }
  free(s.plan);
  free(s.g);
  /* the plugin stays loaded: the process may hold it through ctypes too */
  return rc;
}
