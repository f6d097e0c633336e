// Runtime shim: device context, memory, copies, events, CUDA graphs and
// error reporting behind the C ABI of include/pai_b200.h. The PS5 backend
// this replaces kept the same duties in gpu/hal (hal.h:45-61: device
// open, allocation, submit/wait); here a context owns one CUDA stream and
// the split-K scratch the kernels share.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

#include "../b200_internal.h"

// Bounded device waits (bulk copies landing, peers stamping, grid
// barriers): the default limit and the range a caller may set.
constexpr uint64_t kDefaultWaitNs = 2000000000ull;
constexpr uint64_t kMinWaitNs = 1000000ull;
constexpr uint64_t kMaxWaitNs = 60000000000ull;

struct pai_b200_ctx {
  int device;
  cudaStream_t stream;
  float *partial;         // split-K partial sums
  uint64_t partial_floats;
  uint32_t *counters;     // split-K arrival counters, left at zero
  uint32_t ncounters;
  uint32_t *err_host;     // host-mapped error word (bounded device waits)
  uint32_t *err_dev;
  void *xq;               // activation scratch of the public GEMV entry points
  uint64_t xq_bytes;
  uint64_t launches;
  uint32_t captured;  // this library's launches recorded into the graph being captured
  int capturing;
  int pdl;          // launch the decode-step kernels with programmatic dependent launch
  int pdl_allowed;  // PAI_B200_PDL=0 in the environment turns it off
  uint64_t wait_ns; // limit on every bounded device wait of this context's kernels
  // Scratch buffers replaced by larger ones. A CUDA graph captured earlier
  // (a session's decode step) keeps the old addresses, so they are released
  // only at shutdown; growth at least doubles, which bounds their number.
  void *retired[64];
  uint32_t nretired;
};

// Retire a scratch buffer (see pai_b200_ctx::retired). With growth that at
// least doubles, 64 retirements cannot happen; should the list ever be full,
// the growth is refused rather than a buffer a captured graph may still use
// being freed or lost.
static pai_status_t retire(pai_b200_ctx_t *c, void *p) {
  if (!p) return PAI_OK;
  if (c->nretired >= sizeof(c->retired) / sizeof(c->retired[0]))
    return b200_fail(PAI_ERR_NOMEM, "scratch growth: %u buffers already retired", c->nretired);
  c->retired[c->nretired++] = p;
  return PAI_OK;
}

static thread_local char g_err[512];

extern "C" pai_status_t b200_fail(pai_status_t st, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return st;
}

extern "C" pai_status_t b200_cuda(int err, const char *what) {
  if (err == cudaSuccess) return PAI_OK;
  cudaError_t e = (cudaError_t)err;
  if (e == cudaErrorMemoryAllocation)
    return b200_fail(PAI_ERR_NOMEM, "%s: %s", what, cudaGetErrorString(e));
  return b200_fail(PAI_ERR_INTERNAL, "%s: %s", what, cudaGetErrorString(e));
}

extern "C" void *b200_tensor_map_encoder(void) {
  static void *fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = f;
  });
  return fn;
}

extern "C" const char *pai_b200_last_error(void) { return g_err; }

extern "C" const char *pai_b200_version(void) {
  return "pai_b200 0.1 (sm_100a; packed Q4_0/Q8_0/Q4_K GEMV, fp16-KV decode)";
}

extern "C" pai_status_t pai_b200_device_count(int *out) {
  if (!out) return b200_fail(PAI_ERR_INVALID_ARG, "device_count: NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *out = 0;
    return PAI_OK;
  }
  *out = n;
  return PAI_OK;
}

extern "C" pai_status_t pai_b200_init(int device, pai_b200_ctx_t **out) {
  if (!out) return b200_fail(PAI_ERR_INVALID_ARG, "init: NULL out");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return b200_fail(PAI_ERR_INIT, "init: no CUDA device (%s)", cudaGetErrorString(e));
  }
  if (device < 0 || device >= n) return b200_fail(PAI_ERR_INVALID_ARG, "init: device %d of %d", device, n);
  pai_status_t st = b200_cuda(cudaSetDevice(device), "cudaSetDevice");
  if (st) return st;
  cudaDeviceProp prop;
  st = b200_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (st) return st;
  if (prop.major != 10) {
    return b200_fail(PAI_ERR_UNSUPPORTED, "init: device %d is sm_%d%d; this library is built for sm_100a only",
                     device, prop.major, prop.minor);
  }
  pai_b200_ctx *c = new (std::nothrow) pai_b200_ctx();
  if (!c) return b200_fail(PAI_ERR_NOMEM, "init: host allocation");
  c->device = device;
  c->wait_ns = kDefaultWaitNs;
  {
    const char *e = getenv("PAI_B200_PDL");
    c->pdl_allowed = !(e && e[0] == '0');
  }
  st = b200_cuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  if (st) {
    delete c;
    return st;
  }
  st = b200_cuda(cudaHostAlloc((void **)&c->err_host, sizeof(uint32_t), cudaHostAllocMapped), "error word");
  if (!st) st = b200_cuda(cudaHostGetDevicePointer((void **)&c->err_dev, c->err_host, 0), "error word mapping");
  if (st) {
    if (c->err_host) cudaFreeHost(c->err_host);
    cudaStreamDestroy(c->stream);
    delete c;
    return st;
  }
  *c->err_host = 0;
  *out = c;
  return PAI_OK;
}

extern "C" pai_status_t pai_b200_shutdown(pai_b200_ctx_t *c) {
  if (!c) return PAI_OK;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  if (c->partial) cudaFree(c->partial);
  if (c->counters) cudaFree(c->counters);
  if (c->xq) cudaFree(c->xq);
  for (uint32_t i = 0; i < c->nretired; i++) cudaFree(c->retired[i]);
  if (c->err_host) cudaFreeHost(c->err_host);
  cudaStreamDestroy(c->stream);
  delete c;
  return PAI_OK;
}

extern "C" void *b200_ctx_stream(pai_b200_ctx_t *c) { return c->stream; }
extern "C" int b200_ctx_device(pai_b200_ctx_t *c) { return c->device; }
extern "C" pai_status_t b200_ctx_use_device(pai_b200_ctx_t *c) {
  return b200_cuda(cudaSetDevice(c->device), "cudaSetDevice");
}
extern "C" int b200_ctx_pdl(pai_b200_ctx_t *c) { return c->pdl; }
extern "C" void b200_ctx_set_pdl(pai_b200_ctx_t *c, int on) { c->pdl = on && c->pdl_allowed; }
extern "C" pai_status_t pai_b200_set_pdl(pai_b200_ctx_t *c, int on) {
  if (!c) return b200_fail(PAI_ERR_INVALID_ARG, "set_pdl: NULL context");
  b200_ctx_set_pdl(c, on);
  return PAI_OK;
}
extern "C" uint32_t *b200_ctx_errflag(pai_b200_ctx_t *c) { return c->err_dev; }
extern "C" uint64_t b200_ctx_wait_ns(pai_b200_ctx_t *c) { return c->wait_ns; }
extern "C" pai_status_t pai_b200_set_wait_limit(pai_b200_ctx_t *c, uint64_t ns) {
  if (!c) return b200_fail(PAI_ERR_INVALID_ARG, "set_wait_limit: NULL context");
  if (ns == 0) ns = kDefaultWaitNs;
  if (ns < kMinWaitNs || ns > kMaxWaitNs)
    return b200_fail(PAI_ERR_INVALID_ARG, "set_wait_limit: %llu ns outside [%llu, %llu]", (unsigned long long)ns,
                     (unsigned long long)kMinWaitNs, (unsigned long long)kMaxWaitNs);
  c->wait_ns = ns;
  return PAI_OK;
}

extern "C" pai_status_t b200_ctx_xq(pai_b200_ctx_t *c, uint64_t bytes, void **buf) {
  if (bytes > c->xq_bytes) {
    if (c->capturing) return b200_fail(PAI_ERR_INTERNAL, "activation scratch growth during graph capture");
    const uint64_t want = std::max<uint64_t>(std::max<uint64_t>(bytes, 1u << 20), 2 * c->xq_bytes);
    pai_status_t rs = retire(c, c->xq);
    if (rs) return rs;
    c->xq = nullptr;
    c->xq_bytes = 0;
    pai_status_t st = b200_cuda(cudaMalloc(&c->xq, want), "activation scratch alloc");
    if (st) return st;
    c->xq_bytes = want;
  }
  *buf = c->xq;
  return PAI_OK;
}
extern "C" void b200_ctx_count_launch(pai_b200_ctx_t *c, uint32_t k) {
  if (c->capturing)
    c->captured += k;
  else
    c->launches += k;
}
extern "C" uint64_t pai_b200_launch_count(pai_b200_ctx_t *c) { return c ? c->launches : 0; }

static int sync_check_enabled() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("PAI_B200_SYNC_CHECK");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v;
}

extern "C" pai_status_t b200_launched(pai_b200_ctx_t *c, uint32_t k, const char *name) {
  b200_ctx_count_launch(c, k);
  pai_status_t st = b200_cuda(cudaGetLastError(), name);
  if (st || c->capturing || !sync_check_enabled()) return st;
  st = b200_cuda(cudaStreamSynchronize(c->stream), name);
  if (st) return st;
  return b200_cuda(cudaGetLastError(), name);
}

extern "C" pai_status_t b200_ctx_scratch(pai_b200_ctx_t *c, uint64_t partial_floats,
                                         uint32_t counters, float **partial,
                                         uint32_t **counter) {
  if (partial_floats > c->partial_floats) {
    if (c->capturing) return b200_fail(PAI_ERR_INTERNAL, "scratch growth during graph capture");
    const uint64_t want =
        std::max<uint64_t>(std::max<uint64_t>(partial_floats, 1u << 20), 2 * c->partial_floats);
    pai_status_t rs = retire(c, c->partial);
    if (rs) return rs;
    c->partial = nullptr;
    pai_status_t st = b200_cuda(cudaMalloc(&c->partial, want * sizeof(float)), "scratch alloc");
    if (st) {
      c->partial_floats = 0;
      return st;
    }
    c->partial_floats = want;
  }
  if (counters > c->ncounters) {
    if (c->capturing) return b200_fail(PAI_ERR_INTERNAL, "scratch growth during graph capture");
    const uint32_t want = std::max<uint32_t>(std::max<uint32_t>(counters, 16384u), 2 * c->ncounters);
    pai_status_t rs = retire(c, c->counters);
    if (rs) return rs;
    c->counters = nullptr;
    pai_status_t st = b200_cuda(cudaMalloc(&c->counters, want * sizeof(uint32_t)), "counter alloc");
    if (st) {
      c->ncounters = 0;
      return st;
    }
    st = b200_cuda(cudaMemsetAsync(c->counters, 0, want * sizeof(uint32_t), c->stream), "counter clear");
    if (st) return st;
    c->ncounters = want;
  }
  *partial = c->partial;
  *counter = c->counters;
  return PAI_OK;
}

// ---- memory -------------------------------------------------------------------------------

extern "C" pai_status_t pai_b200_alloc(pai_b200_ctx_t *c, uint64_t bytes, void **out) {
  if (!c || !out) return b200_fail(PAI_ERR_INVALID_ARG, "alloc: NULL");
  *out = nullptr;
  if (bytes == 0) bytes = 256;
  cudaSetDevice(c->device);
  return b200_cuda(cudaMalloc(out, bytes), "cudaMalloc");
}

extern "C" pai_status_t pai_b200_free(pai_b200_ctx_t *c, void *p) {
  if (!c) return b200_fail(PAI_ERR_INVALID_ARG, "free: NULL ctx");
  if (!p) return PAI_OK;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  return b200_cuda(cudaFree(p), "cudaFree");
}

extern "C" pai_status_t pai_b200_host_alloc(pai_b200_ctx_t *c, uint64_t bytes, void **out) {
  if (!c || !out) return b200_fail(PAI_ERR_INVALID_ARG, "host_alloc: NULL");
  return b200_cuda(cudaMallocHost(out, bytes ? bytes : 64), "cudaMallocHost");
}

extern "C" pai_status_t pai_b200_host_free(pai_b200_ctx_t *c, void *p) {
  if (!c) return b200_fail(PAI_ERR_INVALID_ARG, "host_free: NULL ctx");
  return p ? b200_cuda(cudaFreeHost(p), "cudaFreeHost") : PAI_OK;
}

static pai_status_t copy(pai_b200_ctx_t *c, void *dst, const void *src, uint64_t bytes,
                         cudaMemcpyKind kind, const char *what) {
  if (!c || ((!dst || !src) && bytes)) return b200_fail(PAI_ERR_INVALID_ARG, "%s: NULL", what);
  if (!bytes) return PAI_OK;
  return b200_cuda(cudaMemcpyAsync(dst, src, bytes, kind, c->stream), what);
}

extern "C" pai_status_t pai_b200_memcpy_h2d(pai_b200_ctx_t *c, void *d, const void *s, uint64_t n) {
  return copy(c, d, s, n, cudaMemcpyHostToDevice, "memcpy_h2d");
}
extern "C" pai_status_t pai_b200_memcpy_d2h(pai_b200_ctx_t *c, void *d, const void *s, uint64_t n) {
  return copy(c, d, s, n, cudaMemcpyDeviceToHost, "memcpy_d2h");
}
extern "C" pai_status_t pai_b200_memcpy_d2d(pai_b200_ctx_t *c, void *d, const void *s, uint64_t n) {
  return copy(c, d, s, n, cudaMemcpyDeviceToDevice, "memcpy_d2d");
}

extern "C" pai_status_t pai_b200_memset(pai_b200_ctx_t *c, void *dst, int v, uint64_t n) {
  if (!c || (!dst && n)) return b200_fail(PAI_ERR_INVALID_ARG, "memset: NULL");
  return n ? b200_cuda(cudaMemsetAsync(dst, v, n, c->stream), "memset") : PAI_OK;
}

extern "C" pai_status_t pai_b200_sync(pai_b200_ctx_t *c) {
  if (!c) return b200_fail(PAI_ERR_INVALID_ARG, "sync: NULL ctx");
  pai_status_t st = b200_cuda(cudaPeekAtLastError(), "earlier unchecked CUDA call");
  if (st) {
    cudaGetLastError();
    return st;
  }
  st = b200_cuda(cudaStreamSynchronize(c->stream), "stream sync");
  if (st) return st;
  st = b200_cuda(cudaGetLastError(), "kernel execution");
  if (st) return st;
  if (*(volatile uint32_t *)c->err_host) {
    *(volatile uint32_t *)c->err_host = 0;
    return b200_fail(PAI_ERR_TIMEOUT, "a bounded device wait ran out (a bulk copy or peer never completed)");
  }
  return PAI_OK;
}

// ---- events -------------------------------------------------------------------------------

extern "C" pai_status_t pai_b200_event_create(pai_b200_ctx_t *c, void **ev) {
  if (!c || !ev) return b200_fail(PAI_ERR_INVALID_ARG, "event_create: NULL");
  return b200_cuda(cudaEventCreate((cudaEvent_t *)ev), "cudaEventCreate");
}
extern "C" pai_status_t pai_b200_event_destroy(pai_b200_ctx_t *c, void *ev) {
  (void)c;
  return ev ? b200_cuda(cudaEventDestroy((cudaEvent_t)ev), "cudaEventDestroy") : PAI_OK;
}
extern "C" pai_status_t pai_b200_event_record(pai_b200_ctx_t *c, void *ev) {
  if (!c || !ev) return b200_fail(PAI_ERR_INVALID_ARG, "event_record: NULL");
  return b200_cuda(cudaEventRecord((cudaEvent_t)ev, c->stream), "cudaEventRecord");
}
extern "C" pai_status_t pai_b200_event_elapsed(void *a, void *b, float *ms) {
  if (!a || !b || !ms) return b200_fail(PAI_ERR_INVALID_ARG, "event_elapsed: NULL");
  pai_status_t st = b200_cuda(cudaEventSynchronize((cudaEvent_t)b), "cudaEventSynchronize");
  if (st) return st;
  return b200_cuda(cudaEventElapsedTime(ms, (cudaEvent_t)a, (cudaEvent_t)b), "cudaEventElapsedTime");
}

// ---- graphs -------------------------------------------------------------------------------

extern "C" pai_status_t b200_graph_begin(pai_b200_ctx_t *c) {
  pai_status_t st = b200_cuda(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal),
                              "cudaStreamBeginCapture");
  if (st) return st;
  c->capturing = 1;
  c->captured = 0;
  return PAI_OK;
}

extern "C" pai_status_t b200_graph_end(pai_b200_ctx_t *c, void **exec, uint32_t *kernels) {
  cudaGraph_t g = nullptr;
  c->capturing = 0;
  pai_status_t st = b200_cuda(cudaStreamEndCapture(c->stream, &g), "cudaStreamEndCapture");
  if (st) return st;
  cudaGraphExec_t ge = nullptr;
  st = b200_cuda(cudaGraphInstantiate(&ge, g, 0), "cudaGraphInstantiate");
  cudaGraphDestroy(g);
  if (st) return st;
  *exec = ge;
  // This library's kernels in the graph (collective kernels of NCCL, when
  // the step holds tensor-parallel exchanges, are not counted).
  *kernels = c->captured;
  return PAI_OK;
}

extern "C" pai_status_t b200_graph_launch(pai_b200_ctx_t *c, void *exec, uint32_t kernels) {
  pai_status_t st = b200_cuda(cudaGraphLaunch((cudaGraphExec_t)exec, c->stream), "cudaGraphLaunch");
  if (!st) c->launches += kernels;
  return st;
}

extern "C" void b200_graph_destroy(void *exec) {
  if (exec) cudaGraphExecDestroy((cudaGraphExec_t)exec);
}

// ---- public graph capture -------------------------------------------------------------------

struct pai_b200_graph {
  void *exec;
  uint32_t kernels;  // this library's kernels per replay
};

extern "C" pai_status_t pai_b200_graph_begin(pai_b200_ctx_t *c) {
  if (!c) return b200_fail(PAI_ERR_INVALID_ARG, "graph_begin: NULL");
  if (c->capturing) return b200_fail(PAI_ERR_INVALID_ARG, "graph_begin: a capture is already open");
  pai_status_t st = b200_ctx_use_device(c);
  return st ? st : b200_graph_begin(c);
}

extern "C" pai_status_t pai_b200_graph_end(pai_b200_ctx_t *c, pai_b200_graph_t **out) {
  if (!c || !out) return b200_fail(PAI_ERR_INVALID_ARG, "graph_end: NULL");
  if (!c->capturing) return b200_fail(PAI_ERR_INVALID_ARG, "graph_end: no capture open");
  pai_b200_graph_t *g = (pai_b200_graph_t *)calloc(1, sizeof(*g));
  void *exec = nullptr;
  uint32_t kernels = 0;
  pai_status_t st = b200_graph_end(c, &exec, &kernels);
  if (st || !g) {
    b200_graph_destroy(exec);
    free(g);
    return st ? st : b200_fail(PAI_ERR_NOMEM, "graph_end: host allocation");
  }
  g->exec = exec;
  g->kernels = kernels;
  *out = g;
  return PAI_OK;
}

extern "C" pai_status_t pai_b200_graph_launch(pai_b200_ctx_t *c, pai_b200_graph_t *g) {
  if (!c || !g) return b200_fail(PAI_ERR_INVALID_ARG, "graph_launch: NULL");
  return b200_graph_launch(c, g->exec, g->kernels);
}

extern "C" pai_status_t pai_b200_graph_destroy(pai_b200_graph_t *g) {
  if (g) {
    b200_graph_destroy(g->exec);
    free(g);
  }
  return PAI_OK;
}
