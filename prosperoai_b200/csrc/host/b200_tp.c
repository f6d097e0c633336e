/*
 * Tensor-parallel exchange steps of the decode over NCCL (NVLink /
 * NVSwitch inside one node): the all-reduce of the row-parallel o/down
 * partial sums and the argmax across vocabulary shards of the lm head.
 * The reference runs on one device; its layer order (adapters/llama/
 * llama.c:669-797) is kept, with the sums split across ranks.
 *
 * NCCL is loaded at run time (dlopen of libnccl.so.2, or the file named by
 * PAI_B200_NCCL), so a process that already loaded NCCL (PyTorch's
 * torch.distributed) shares that copy. Only the handful of entry points
 * and constants used here are declared, with the types of NCCL's public
 * API: ncclUniqueId is 128 opaque bytes passed by value, ncclComm_t an
 * opaque pointer, ncclResult_t 0 on success; data type 1 = uint8,
 * 7 = float32; reduction 0 = sum.
 *
 * The all-reduce of the o/down partial outputs does not use NCCL: it runs
 * over NVLink peer memory, fused with the residual add (kernels/k_tp.cu),
 * on exchange buffers mapped between the ranks with CUDA IPC (handles
 * exchanged with an NCCL all-gather). NCCL carries the lm-head argmax
 * pairs and the public pai_b200_tp_allreduce_f32.
 */
#include <dlfcn.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../b200_internal.h"

typedef struct {
  char internal[PAI_B200_TP_ID_BYTES];
} nccl_uid_t;
typedef void *nccl_comm_t;
enum { NCCL_SUCCESS = 0, NCCL_UINT8 = 1, NCCL_FLOAT32 = 7, NCCL_SUM = 0 };

static struct {
  void *lib;
  char why[256];
  int (*get_unique_id)(nccl_uid_t *);
  int (*comm_init_rank)(nccl_comm_t *, int, nccl_uid_t, int);
  int (*comm_destroy)(nccl_comm_t);
  int (*all_reduce)(const void *, void *, size_t, int, int, nccl_comm_t, void *);
  int (*all_gather)(const void *, void *, size_t, int, nccl_comm_t, void *);
  const char *(*error_string)(int);
} g_nccl;
static pthread_once_t g_nccl_once = PTHREAD_ONCE_INIT;

static void nccl_load(void) {
  const char *path = getenv("PAI_B200_NCCL");
  void *h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    const char *e = dlerror();
    snprintf(g_nccl.why, sizeof g_nccl.why, "cannot load NCCL: %s", e ? e : "dlopen failed");
    return;
  }
#define NCCL_SYM(field, name)                                                   \
  do {                                                                          \
    *(void **)&g_nccl.field = dlsym(h, name);                                   \
    if (!g_nccl.field) {                                                        \
      snprintf(g_nccl.why, sizeof g_nccl.why, "NCCL lacks %s", name);           \
      return;                                                                   \
    }                                                                           \
  } while (0)
  NCCL_SYM(get_unique_id, "ncclGetUniqueId");
  NCCL_SYM(comm_init_rank, "ncclCommInitRank");
  NCCL_SYM(comm_destroy, "ncclCommDestroy");
  NCCL_SYM(all_reduce, "ncclAllReduce");
  NCCL_SYM(all_gather, "ncclAllGather");
  NCCL_SYM(error_string, "ncclGetErrorString");
#undef NCCL_SYM
  g_nccl.lib = h;
}

static pai_status_t nccl_ready(void) {
  pthread_once(&g_nccl_once, nccl_load);
  if (!g_nccl.lib) return b200_fail(PAI_ERR_UNSUPPORTED, "tensor parallelism: %s", g_nccl.why);
  return PAI_OK;
}

static pai_status_t nccl_check(int r, const char *what) {
  if (r == NCCL_SUCCESS) return PAI_OK;
  return b200_fail(PAI_ERR_INTERNAL, "%s: NCCL error %d (%s)", what, r, g_nccl.error_string(r));
}

struct pai_b200_tp {
  pai_b200_ctx_t *ctx;
  nccl_comm_t comm;
  uint32_t rank, size;
  float *pairs;                     /* argmax exchange: [rank][row][2] for up to 8 rows */
  void *xbuf[B200_TP_MAX_RANKS];    /* exchange buffers: own (allocated), peers (IPC-mapped) */
  uint64_t cap;                     /* floats per exchange slot */
  void *land[B200_TP_MAX_RANKS];    /* landing buffers of the persistent decode: own, peers */
  uint64_t land_rows;               /* rows per landing slot */
  int failed;                       /* an exchange timed out: the buffers are out of step */
};

void b200_tp_mark_failed(pai_b200_tp_t *tp) {
  if (tp) tp->failed = 1;
}

int b200_tp_failed(const pai_b200_tp_t *tp) { return tp ? tp->failed : 0; }

static void lands_release(pai_b200_tp_t *tp) {
  for (uint32_t r = 0; r < tp->size; r++) {
    if (!tp->land[r]) continue;
    if (r == tp->rank)
      b200_tp_xbuf_free(tp->land[r]);
    else
      b200_tp_xbuf_close(tp->land[r]);
    tp->land[r] = NULL;
  }
  tp->land_rows = 0;
}

/* Allocate `bytes` of zeroed device memory on every rank and map every
 * rank's allocation here (out[r]). Collective: the IPC handles travel by an
 * NCCL all-gather. */
static pai_status_t ipc_exchange(pai_b200_tp_t *tp, uint64_t bytes, void **out) {
  uint8_t *dev_h = NULL, *host_h = NULL, mine[B200_TP_HANDLE_BYTES];
  pai_status_t st = b200_ipc_alloc(tp->ctx, bytes, &out[tp->rank], mine);
  if (!st) st = pai_b200_alloc(tp->ctx, (uint64_t)tp->size * B200_TP_HANDLE_BYTES, (void **)&dev_h);
  if (!st) {
    host_h = (uint8_t *)malloc((size_t)tp->size * B200_TP_HANDLE_BYTES);
    if (!host_h) st = b200_fail(PAI_ERR_NOMEM, "tp: host allocation");
  }
  if (!st) st = pai_b200_memcpy_h2d(tp->ctx, dev_h + (uint64_t)tp->rank * B200_TP_HANDLE_BYTES, mine, sizeof mine);
  if (!st)
    st = nccl_check(g_nccl.all_gather(dev_h + (uint64_t)tp->rank * B200_TP_HANDLE_BYTES, dev_h, B200_TP_HANDLE_BYTES,
                                      NCCL_UINT8, tp->comm, b200_ctx_stream(tp->ctx)),
                    "ncclAllGather (exchange handles)");
  if (!st) st = pai_b200_memcpy_d2h(tp->ctx, host_h, dev_h, (uint64_t)tp->size * B200_TP_HANDLE_BYTES);
  if (!st) st = pai_b200_sync(tp->ctx);
  for (uint32_t r = 0; !st && r < tp->size; r++)
    if (r != tp->rank) st = b200_tp_xbuf_open(tp->ctx, host_h + (uint64_t)r * B200_TP_HANDLE_BYTES, &out[r]);
  free(host_h);
  pai_b200_free(tp->ctx, dev_h);
  return st;
}

/* Landing buffers of `rows` floats per slot on every rank (the persistent
 * decode's row exchanges and greedy pairs), mapped here; collective, every
 * rank with the same rows. They start zeroed, so every rank's counters
 * begin in step. */
pai_status_t b200_tp_land(pai_b200_tp_t *tp, uint64_t rows, void **out) {
  pai_status_t st;
  if (!tp || !out) return b200_fail(PAI_ERR_INVALID_ARG, "tp_land: NULL");
  if (tp->failed) return b200_fail(PAI_ERR_INIT, "tp_land: the communicator's exchange timed out earlier");
  if (rows > tp->land_rows) {
    st = pai_b200_sync(tp->ctx);
    if (st) return st;
    lands_release(tp);
    st = ipc_exchange(tp, b200_land_bytes(tp->size, rows), tp->land);
    if (st) {
      lands_release(tp);
      return st;
    }
    tp->land_rows = rows;
  }
  for (uint32_t r = 0; r < tp->size; r++) out[r] = tp->land[r];
  return PAI_OK;
}

static void xbufs_release(pai_b200_tp_t *tp) {
  for (uint32_t r = 0; r < tp->size; r++) {
    if (!tp->xbuf[r]) continue;
    if (r == tp->rank)
      b200_tp_xbuf_free(tp->xbuf[r]);
    else
      b200_tp_xbuf_close(tp->xbuf[r]);
    tp->xbuf[r] = NULL;
  }
  tp->cap = 0;
}

/* Make every rank's exchange buffer hold `cap` floats per slot and map all
 * of them here. Collective: every rank calls it with the same cap. */
pai_status_t b200_tp_reserve(pai_b200_tp_t *tp, uint64_t cap) {
  uint8_t *dev_h = NULL, *host_h = NULL, mine[B200_TP_HANDLE_BYTES];
  pai_status_t st;
  if (cap <= tp->cap) return PAI_OK;
  st = pai_b200_sync(tp->ctx);
  if (st) return st;
  xbufs_release(tp);
  st = b200_tp_xbuf_alloc(tp->ctx, cap, &tp->xbuf[tp->rank], mine);
  if (!st) st = pai_b200_alloc(tp->ctx, (uint64_t)tp->size * B200_TP_HANDLE_BYTES, (void **)&dev_h);
  if (!st) {
    host_h = (uint8_t *)malloc((size_t)tp->size * B200_TP_HANDLE_BYTES);
    if (!host_h) st = b200_fail(PAI_ERR_NOMEM, "tp_reserve: host allocation");
  }
  if (!st) st = pai_b200_memcpy_h2d(tp->ctx, dev_h + (uint64_t)tp->rank * B200_TP_HANDLE_BYTES, mine, sizeof mine);
  if (!st)
    st = nccl_check(g_nccl.all_gather(dev_h + (uint64_t)tp->rank * B200_TP_HANDLE_BYTES, dev_h, B200_TP_HANDLE_BYTES,
                                      NCCL_UINT8, tp->comm, b200_ctx_stream(tp->ctx)),
                    "ncclAllGather (exchange handles)");
  if (!st) st = pai_b200_memcpy_d2h(tp->ctx, host_h, dev_h, (uint64_t)tp->size * B200_TP_HANDLE_BYTES);
  if (!st) st = pai_b200_sync(tp->ctx);
  for (uint32_t r = 0; !st && r < tp->size; r++)
    if (r != tp->rank) st = b200_tp_xbuf_open(tp->ctx, host_h + (uint64_t)r * B200_TP_HANDLE_BYTES, &tp->xbuf[r]);
  free(host_h);
  pai_b200_free(tp->ctx, dev_h);
  if (st) {
    xbufs_release(tp);
    return st;
  }
  tp->cap = cap;
  return PAI_OK;
}

float *b200_tp_slot(pai_b200_tp_t *tp, uint32_t slot) { return b200_tp_xbuf_slot(tp->xbuf[tp->rank], slot, tp->cap); }

pai_status_t b200_tp_allreduce_add(pai_b200_tp_t *tp, pai_b200_ctx_t *ctx, uint32_t slot, float *x, uint64_t n) {
  if (!tp) return b200_fail(PAI_ERR_INIT, "tp_allreduce_add: no communicator");
  return b200_launch_tp_allreduce_add(ctx, tp->xbuf, tp->rank, tp->size, slot, tp->cap, x, n);
}

pai_status_t pai_b200_tp_unique_id(uint8_t id[PAI_B200_TP_ID_BYTES]) {
  nccl_uid_t u;
  pai_status_t st;
  if (!id) return b200_fail(PAI_ERR_INVALID_ARG, "tp_unique_id: NULL");
  st = nccl_ready();
  if (st) return st;
  st = nccl_check(g_nccl.get_unique_id(&u), "ncclGetUniqueId");
  if (!st) memcpy(id, u.internal, PAI_B200_TP_ID_BYTES);
  return st;
}

pai_status_t pai_b200_tp_create(pai_b200_ctx_t *ctx, const uint8_t id[PAI_B200_TP_ID_BYTES], uint32_t rank,
                                uint32_t size, pai_b200_tp_t **out) {
  nccl_uid_t u;
  pai_b200_tp_t *tp;
  pai_status_t st;
  if (!ctx || !id || !out) return b200_fail(PAI_ERR_INVALID_ARG, "tp_create: NULL");
  *out = NULL;
  if (size == 0 || size > B200_TP_MAX_RANKS || rank >= size)
    return b200_fail(PAI_ERR_INVALID_ARG, "tp_create: rank %u of %u (at most %u ranks)", rank, size, B200_TP_MAX_RANKS);
  st = nccl_ready();
  if (st) return st;
  st = b200_ctx_use_device(ctx);
  if (st) return st;
  tp = (pai_b200_tp_t *)calloc(1, sizeof(*tp));
  if (!tp) return b200_fail(PAI_ERR_NOMEM, "tp_create: host allocation");
  tp->ctx = ctx;
  tp->rank = rank;
  tp->size = size;
  memcpy(u.internal, id, PAI_B200_TP_ID_BYTES);
  st = nccl_check(g_nccl.comm_init_rank(&tp->comm, (int)size, u, (int)rank), "ncclCommInitRank");
  if (!st) st = pai_b200_alloc(ctx, (uint64_t)size * 8 * 2 * sizeof(float), (void **)&tp->pairs);
  if (st) {
    if (tp->comm) g_nccl.comm_destroy(tp->comm);
    free(tp);
    return st;
  }
  *out = tp;
  return PAI_OK;
}

pai_status_t pai_b200_tp_destroy(pai_b200_tp_t *tp) {
  pai_status_t st = PAI_OK;
  if (!tp) return PAI_OK;
  pai_b200_sync(tp->ctx);
  xbufs_release(tp);
  lands_release(tp);
  pai_b200_free(tp->ctx, tp->pairs);
  if (tp->comm) st = nccl_check(g_nccl.comm_destroy(tp->comm), "ncclCommDestroy");
  free(tp);
  return st;
}

uint32_t pai_b200_tp_rank(const pai_b200_tp_t *tp) { return tp ? tp->rank : 0; }
uint32_t pai_b200_tp_size(const pai_b200_tp_t *tp) { return tp ? tp->size : 0; }

pai_status_t b200_tp_allreduce(void *tpv, pai_b200_ctx_t *ctx, float *buf, uint64_t n) {
  pai_b200_tp_t *tp = (pai_b200_tp_t *)tpv;
  if (!tp) return b200_fail(PAI_ERR_INIT, "tp_allreduce: no communicator");
  return nccl_check(g_nccl.all_reduce(buf, buf, (size_t)n, NCCL_FLOAT32, NCCL_SUM, tp->comm, b200_ctx_stream(ctx)),
                    "ncclAllReduce");
}

pai_status_t pai_b200_tp_allreduce_f32(pai_b200_tp_t *tp, float *buf, uint64_t n) {
  if (!tp || !buf) return b200_fail(PAI_ERR_INVALID_ARG, "tp_allreduce: NULL");
  return b200_tp_allreduce(tp, tp->ctx, buf, n);
}

pai_status_t b200_tp_argmax(void *tpv, pai_b200_ctx_t *ctx, uint32_t batch, uint32_t vl, uint32_t v0,
                            const float *logits, int32_t *tok_out) {
  pai_b200_tp_t *tp = (pai_b200_tp_t *)tpv;
  pai_status_t st;
  float *mine;
  if (!tp) return b200_fail(PAI_ERR_INIT, "tp_argmax: no communicator");
  if (batch > 8) return b200_fail(PAI_ERR_UNSUPPORTED, "tp_argmax: batch %u", batch);
  /* this shard's (maximum, global index) per row, gathered in place into
   * pairs[rank][row][2] on every rank, then merged in rank order */
  mine = tp->pairs + (uint64_t)tp->rank * batch * 2;
  st = b200_launch_argmax_pair(ctx, batch, vl, v0, logits, mine);
  if (!st)
    st = nccl_check(g_nccl.all_gather(mine, tp->pairs, (size_t)batch * 2, NCCL_FLOAT32, tp->comm, b200_ctx_stream(ctx)),
                    "ncclAllGather");
  if (!st) st = b200_launch_argmax_ranks(ctx, batch, tp->size, tp->pairs, tok_out);
  return st;
}
