// Tensor-parallel exchange over NVLink peer memory: the all-reduce of the
// row-parallel o/down partial outputs fused with the residual add that
// follows it in the layer (adapters/llama/llama.c:747-749, 793-795).
//
// Every rank owns one exchange buffer in its HBM, mapped into the other
// ranks' address spaces with CUDA IPC:
//   [header: per-CTA call counters, per-(rank, CTA) arrival flags]
//   [slot 0][slot 1]: the rank's partial outputs, written by its o/down GEMV
//   (double-buffered by call parity).
// One launch per exchange, CTA j of every rank handles the same element
// slice: it stamps flag[my rank][j] = epoch into every rank's header (plain
// peer stores after a system-scope fence; the GEMV that wrote the partial
// finished before this kernel passed its dependency wait), waits until
// flag[r][j] >= epoch for all r (bounded), then reads all ranks' partials of
// its slice in rank order, sums them and adds the residual: every rank
// computes the same bits. Epochs are the CTA's own call counter + 1, so no
// rank synchronisation other than the flags is needed.
//
// Why two slots are enough: rank A rewrites slot s = c % 2 only in call
// c + 2, whose GEMV starts after A's exchange c + 1 completed on every CTA,
// which required every rank's CTA j to have stamped call c + 1, which each
// does only after finishing call c (its reads of slot s).
//
// No multicast, no NVLink SHARP: plain peer loads and stores. Every wait is
// bounded (2 s); on timeout the kernel raises the context's error flag and
// returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace {

constexpr uint32_t kMaxCtas = 64;
constexpr size_t kHeader = 8192;  // counters [kMaxCtas] u64, flags [B200_TP_MAX_RANKS][kMaxCtas] u64
static_assert(kMaxCtas * 8 + B200_TP_MAX_RANKS * kMaxCtas * 8 <= kHeader, "header");

struct TpArgs {
  uint8_t *buf[B200_TP_MAX_RANKS];  // every rank's exchange buffer, as mapped here
  uint32_t rank, nranks, slot;
  uint64_t cap;  // floats per slot
  float *x;      // residual in, sum out
  uint64_t n;
  uint32_t *err;
  uint64_t wait_ns;  // the context's limit on the wait for the other ranks
};

__device__ __forceinline__ uint64_t *counters(uint8_t *b) { return reinterpret_cast<uint64_t *>(b); }
__device__ __forceinline__ uint64_t *flags(uint8_t *b) { return reinterpret_cast<uint64_t *>(b) + kMaxCtas; }
__device__ __forceinline__ float *slot_of(uint8_t *b, uint32_t s, uint64_t cap) {
  return reinterpret_cast<float *>(b + kHeader) + (size_t)s * cap;
}

__device__ __forceinline__ void store_release_sys(uint64_t *p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t load_acquire_sys(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) k_tp_allreduce_add(TpArgs a) {
  pdl_trigger();
  pdl_wait();  // the partial outputs of this call are complete
  __shared__ uint64_t epoch_s;
  __shared__ int ok_s;
  const uint32_t j = blockIdx.x;
  uint8_t *mine = a.buf[a.rank];
  if (threadIdx.x == 0) {
    const uint64_t epoch = counters(mine)[j] + 1;
    epoch_s = epoch;
    // the partial was written by a kernel that has completed, in this GPU's
    // memory, which peers read through this GPU's L2: the release store
    // orders the stamp after it
    for (uint32_t r = 0; r < a.nranks; r++) store_release_sys(flags(a.buf[r]) + (size_t)a.rank * kMaxCtas + j, epoch);
    // wait for every rank's CTA j to arrive at this call
    bool ok = true;
    for (uint32_t r = 0; r < a.nranks && ok; r++) {
      const uint64_t *f = flags(mine) + (size_t)r * kMaxCtas + j;
      uint64_t t0 = 0;
      for (uint32_t it = 0;; it++) {
        if (load_acquire_sys(f) >= epoch) break;
        if ((it & 255u) == 0) {
          const uint64_t now = globaltimer_ns();
          if (it == 0) {
            t0 = now;
          } else if (now - t0 > a.wait_ns) {
            ok = false;
            break;
          }
        }
      }
    }
    ok_s = ok;
    if (!ok) atomicExch(a.err, 1u);
  }
  __syncthreads();
  if (!ok_s) return;
  // groups of 4 elements; every rank's value of a group is loaded before the
  // sum, so the peer reads are one round trip per group
  const uint64_t n4 = (a.n + 3) / 4, per = (n4 + gridDim.x - 1) / gridDim.x;
  const uint64_t lo = (uint64_t)j * per, hi = min(n4, lo + per);
  for (uint64_t g = lo + threadIdx.x; g < hi; g += blockDim.x) {
    float4 v[B200_TP_MAX_RANKS];
    const bool full = 4 * g + 3 < a.n;
#pragma unroll
    for (uint32_t r = 0; r < B200_TP_MAX_RANKS; r++) {
      if (r < a.nranks) {
        const float *src = slot_of(a.buf[r], a.slot, a.cap) + 4 * g;
        if (full) {
          v[r] = __ldcv(reinterpret_cast<const float4 *>(src));
        } else {
          v[r].x = __ldcv(src);
          v[r].y = 4 * g + 1 < a.n ? __ldcv(src + 1) : 0.f;
          v[r].z = 4 * g + 2 < a.n ? __ldcv(src + 2) : 0.f;
          v[r].w = 0.f;
        }
      }
    }
    float4 s = v[0];
#pragma unroll
    for (uint32_t r = 1; r < B200_TP_MAX_RANKS; r++) {  // rank order: the same sum on every rank
      if (r < a.nranks) {
        s.x += v[r].x;
        s.y += v[r].y;
        s.z += v[r].z;
        s.w += v[r].w;
      }
    }
    float *x = a.x + 4 * g;
    if (full) {
      float4 xv = *reinterpret_cast<float4 *>(x);
      xv.x += s.x;
      xv.y += s.y;
      xv.z += s.z;
      xv.w += s.w;
      *reinterpret_cast<float4 *>(x) = xv;
    } else {
      x[0] += s.x;
      if (4 * g + 1 < a.n) x[1] += s.y;
      if (4 * g + 2 < a.n) x[2] += s.z;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) counters(mine)[j] = epoch_s;  // read only by this CTA index, next call
}

}  // namespace

extern "C" pai_status_t b200_tp_xbuf_alloc(pai_b200_ctx_t *ctx, uint64_t cap, void **buf,
                                           uint8_t handle[B200_TP_HANDLE_BYTES]) {
  return b200_ipc_alloc(ctx, kHeader + 2 * (size_t)cap * sizeof(float), buf, handle);
}

extern "C" pai_status_t b200_ipc_alloc(pai_b200_ctx_t *ctx, uint64_t bytes, void **buf,
                                       uint8_t handle[B200_TP_HANDLE_BYTES]) {
  pai_status_t st = b200_ctx_use_device(ctx);
  if (st) return st;
  void *p = nullptr;
  st = b200_cuda(cudaMalloc(&p, bytes), "exchange buffer alloc");
  if (st) return st;
  st = b200_cuda(cudaMemset(p, 0, bytes), "exchange buffer clear");
  cudaIpcMemHandle_t h;
  if (!st) st = b200_cuda(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  if (!st) st = b200_cuda(cudaDeviceSynchronize(), "exchange buffer clear");
  if (st) {
    cudaFree(p);
    return st;
  }
  static_assert(sizeof(h) == B200_TP_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *buf = p;
  return PAI_OK;
}

extern "C" pai_status_t b200_tp_xbuf_open(pai_b200_ctx_t *ctx, const uint8_t handle[B200_TP_HANDLE_BYTES],
                                          void **buf) {
  pai_status_t st = b200_ctx_use_device(ctx);
  if (st) return st;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return b200_cuda(cudaIpcOpenMemHandle(buf, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" void b200_tp_xbuf_close(void *buf) {
  if (buf) cudaIpcCloseMemHandle(buf);
}

extern "C" void b200_tp_xbuf_free(void *buf) {
  if (buf) cudaFree(buf);
}

extern "C" float *b200_tp_xbuf_slot(void *buf, uint32_t slot, uint64_t cap) {
  return reinterpret_cast<float *>(static_cast<uint8_t *>(buf) + kHeader) + (size_t)slot * cap;
}

extern "C" pai_status_t b200_launch_tp_allreduce_add(pai_b200_ctx_t *ctx, void *const *bufs, uint32_t rank,
                                                     uint32_t nranks, uint32_t slot, uint64_t cap, float *x,
                                                     uint64_t n) {
  if (nranks == 0 || nranks > B200_TP_MAX_RANKS || rank >= nranks || slot > 1 || n > cap)
    return b200_fail(PAI_ERR_INVALID_ARG, "tp_allreduce_add: rank %u of %u, slot %u, n %llu of %llu", rank, nranks,
                     slot, (unsigned long long)n, (unsigned long long)cap);
  TpArgs a{};
  for (uint32_t r = 0; r < nranks; r++) a.buf[r] = static_cast<uint8_t *>(bufs[r]);
  a.rank = rank;
  a.nranks = nranks;
  a.slot = slot;
  a.cap = cap;
  a.x = x;
  a.n = n;
  a.err = b200_ctx_errflag(ctx);
  a.wait_ns = b200_ctx_wait_ns(ctx);
  // one group of 4 elements per thread when it fits in kMaxCtas CTAs of 256
  const uint32_t ctas = (uint32_t)std::min<uint64_t>(kMaxCtas, std::max<uint64_t>(1, (n + 1023) / 1024));
  if ((uintptr_t)x % 16 || (cap * sizeof(float)) % 16)
    return b200_fail(PAI_ERR_INVALID_ARG, "tp_allreduce_add: x and slots must be 16-byte aligned");
  b200_launch(ctx, k_tp_allreduce_add, dim3(ctas), dim3(256), 0, a);
  return b200_launched(ctx, 1, "k_tp_allreduce_add");
}

// ---- public form of the exchange ------------------------------------------------------------

extern "C" pai_status_t pai_b200_tp_xbuf_create(pai_b200_ctx_t *ctx, uint64_t cap, void **buf,
                                                uint8_t handle[PAI_B200_TP_HANDLE_BYTES]) {
  if (!ctx || !buf || !handle) return b200_fail(PAI_ERR_INVALID_ARG, "tp_xbuf_create: NULL");
  if (cap == 0 || cap % 4 || cap > (1ull << 32)) return b200_fail(PAI_ERR_INVALID_ARG, "tp_xbuf_create: capacity");
  static_assert(PAI_B200_TP_HANDLE_BYTES == B200_TP_HANDLE_BYTES, "handle size");
  return b200_tp_xbuf_alloc(ctx, cap, buf, handle);
}

extern "C" pai_status_t pai_b200_tp_xbuf_open(pai_b200_ctx_t *ctx, const uint8_t handle[PAI_B200_TP_HANDLE_BYTES],
                                              void **buf) {
  if (!ctx || !buf || !handle) return b200_fail(PAI_ERR_INVALID_ARG, "tp_xbuf_open: NULL");
  return b200_tp_xbuf_open(ctx, handle, buf);
}

extern "C" pai_status_t pai_b200_tp_xbuf_release(pai_b200_ctx_t *ctx, void *buf, int owned) {
  if (!ctx) return b200_fail(PAI_ERR_INVALID_ARG, "tp_xbuf_release: NULL");
  pai_status_t st = b200_ctx_use_device(ctx);
  if (st) return st;
  st = b200_cuda(cudaStreamSynchronize((cudaStream_t)b200_ctx_stream(ctx)), "tp_xbuf_release");
  if (owned)
    b200_tp_xbuf_free(buf);
  else
    b200_tp_xbuf_close(buf);
  return st;
}

extern "C" float *pai_b200_tp_xbuf_slot(void *buf, uint32_t slot, uint64_t cap) {
  return (buf && slot < 2) ? b200_tp_xbuf_slot(buf, slot, cap) : nullptr;
}

extern "C" pai_status_t pai_b200_tp_allreduce_add_f32(pai_b200_ctx_t *ctx, void *const *bufs, uint32_t rank,
                                                      uint32_t nranks, uint32_t slot, uint64_t cap, float *x,
                                                      uint64_t n) {
  if (!ctx || !bufs || !x) return b200_fail(PAI_ERR_INVALID_ARG, "tp_allreduce_add: NULL");
  for (uint32_t r = 0; r < nranks && r < B200_TP_MAX_RANKS; r++)
    if (!bufs[r]) return b200_fail(PAI_ERR_INVALID_ARG, "tp_allreduce_add: buffer of rank %u is NULL", r);
  return b200_launch_tp_allreduce_add(ctx, bufs, rank, nranks, slot, cap, x, n);
}
