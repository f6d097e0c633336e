// Device helpers shared by the kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../b200_internal.h"

// Per-device opt-in of a kernel's dynamic shared memory (the attribute is
// per device and per kernel): raised, never lowered, to at least the bytes a
// launch needs, once per device; safe when several host threads launch.
struct SmemOptIn {
  std::atomic<size_t> bytes[64];
  std::mutex mu;
  template <typename F>
  cudaError_t ensure(int dev, size_t want, F &&set) {
    if (dev < 0 || dev >= 64) return set(want);
    if (bytes[dev].load(std::memory_order_acquire) >= want) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu);
    if (bytes[dev].load(std::memory_order_relaxed) >= want) return cudaSuccess;
    const cudaError_t e = set(want);
    if (e == cudaSuccess) bytes[dev].store(want, std::memory_order_release);
    return e;
  }
};

// ---- programmatic dependent launch ---------------------------------------------------------
// pdl_wait blocks the calling thread until the previous kernel in the
// stream has completed and its writes are visible (a no-op when the kernel
// was launched normally); pdl_trigger lets the next kernel be scheduled
// once every CTA of this grid has called it or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch `kern` on the context's stream, with programmatic dependent
// launch when the context has it on.
template <typename... KArgs, typename... Args>
static inline cudaError_t b200_launch(pai_b200_ctx_t *ctx, void (*kern)(KArgs...), dim3 grid, dim3 block,
                                      size_t smem, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)b200_ctx_stream(ctx);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = b200_ctx_pdl(ctx) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// fp16 bits -> fp32 by integer manipulation, value- and payload-identical
// to the reference's f16_to_f32 (adapters/llama/gguf.c:602-630),
// including subnormals and NaN payloads.
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
      // normalise: the leading 1 of m sits at bit (31 - clz); shift it to bit 10
      int lead = 31 - __clz(m);
      int sh = 10 - lead;
      bits = sign | ((uint32_t)(113 - sh) << 23) | (((m << sh) & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7F800000u | (m << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  return __uint_as_float(bits);
}

// 6-bit scale and min of Q4_K sub-block j (adapters/llama/gguf.c:640-648).
__device__ __forceinline__ void k4_scale_min(int j, const uint8_t *q, uint8_t *sc, uint8_t *mn) {
  if (j < 4) {
    *sc = q[j] & 63;
    *mn = q[j + 4] & 63;
  } else {
    *sc = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
    *mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- packed weight layout (b200_internal.h) --------------------------------------------------
// Byte offset, in the qs plane, of byte j of the ggml quant bytes of block
// b of row r (j < 16 for Q4_0, < 32 for Q8_0, < 128 for Q4_K).
__device__ __forceinline__ uint64_t pk_qs_off(uint32_t t, uint64_t ntiles, uint64_t r, uint64_t b, uint32_t j) {
  const uint64_t rr = r % B200_TILE, rlo = rr % 8, h = rr / 8;
  const uint64_t ub = b200_unit_blocks(t), piece = (b / ub) * ntiles + r / B200_TILE, i = b % ub;
  if (t == PAI_B200_Q4_0)
    return piece * 1024u + h * 512u + (rlo * 4u + j / 4u) * 16u + i * 4u + j % 4u;
  if (t == PAI_B200_Q8_0)
    return piece * 2048u + (2u * h + j / 16u) * 512u + (rlo * 4u + (j % 16u) / 4u) * 16u + i * 4u + j % 4u;
  const uint32_t g = j / 32u, w = j % 32u;
  return piece * 2048u + (2u * h + w / 16u) * 512u + (rlo * 4u + (w % 16u) / 4u) * 16u + g * 4u + j % 4u;
}
// Byte offset, in the sc plane, of the header of block b of row r (the
// fp16 d; for Q4_K the 16 bytes d, dmin, scales[12]).
__device__ __forceinline__ uint64_t pk_hdr_off(uint32_t t, uint64_t ntiles, uint64_t r, uint64_t b) {
  const uint64_t rr = r % B200_TILE, ub = b200_unit_blocks(t);
  const uint64_t piece = (b / ub) * ntiles + r / B200_TILE;
  if (t == PAI_B200_Q4_K) return piece * 256u + rr * 16u;
  return piece * 128u + rr * 8u + (b % ub) * 2u;
}

// Bit-exact dequantisation of block b of row r from the packed layout
// (adapters/llama/gguf.c:680-693, 750-761, 852-882). Products of an fp16
// scale and a small integer are exact in fp32; the Q4_K form keeps
// gguf.c's rounding steps (d*sc, dmin*m, then (d*sc)*q - dmin*m) with
// explicitly rounded operations.
__device__ __forceinline__ void dequant_block_dev(uint32_t t, uint64_t ntiles, const uint8_t *__restrict__ qs,
                                                  const uint8_t *__restrict__ sc, uint64_t r, uint64_t b,
                                                  float *__restrict__ o) {
  const uint8_t *h = sc + pk_hdr_off(t, ntiles, r, b);
  const float d = f16_bits_to_f32((uint16_t)(h[0] | (h[1] << 8)));
  if (t == PAI_B200_Q4_0) {
    for (uint32_t j = 0; j < 16; j++) {
      const uint8_t v = qs[pk_qs_off(t, ntiles, r, b, j)];
      o[j] = __fmul_rn((float)((int)(v & 15) - 8), d);
      o[j + 16] = __fmul_rn((float)((int)(v >> 4) - 8), d);
    }
  } else if (t == PAI_B200_Q8_0) {
    for (uint32_t j = 0; j < 32; j++) o[j] = __fmul_rn((float)(int8_t)qs[pk_qs_off(t, ntiles, r, b, j)], d);
  } else {
    const float dmin = f16_bits_to_f32((uint16_t)(h[2] | (h[3] << 8)));
    for (uint32_t c = 0; c < 4; c++) {
      uint8_t s0, m0, s1, m1;
      k4_scale_min(2 * c, h + 4, &s0, &m0);
      k4_scale_min(2 * c + 1, h + 4, &s1, &m1);
      const float d1 = __fmul_rn(d, (float)s0), mm1 = __fmul_rn(dmin, (float)m0);
      const float d2 = __fmul_rn(d, (float)s1), mm2 = __fmul_rn(dmin, (float)m1);
      for (uint32_t l = 0; l < 32; l++) {
        const uint8_t v = qs[pk_qs_off(t, ntiles, r, b, 32 * c + l)];
        o[64 * c + l] = __fsub_rn(__fmul_rn(d1, (float)(v & 15)), mm1);
        o[64 * c + 32 + l] = __fsub_rn(__fmul_rn(d2, (float)(v >> 4)), mm2);
      }
    }
  }
}

// One RoPE rotation of the pair (x0, x1) = (x[i], x[i + r2]) with
// explicitly rounded operations (pai_ref_rope_f32, ref_ops.c:240-262).
__device__ __forceinline__ void rope_pair(float x0, float x1, float c, float s, float &o0, float &o1) {
  o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  o1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

// ---- activation quantisation (the xq format of b200_internal.h) ----------------------------
// One full warp quantises block b of vector vec: lane j holds element j.
// Writes every byte of the block (digit columns and the zero column) and
// its two scales, so a buffer reused with another layout needs no clearing.
__device__ __forceinline__ void xq_store_block(const b200_xq_t &xq, uint32_t vec, uint32_t b, float v) {
  const uint32_t lane = threadIdx.x & 31;
  // |v| bit patterns order as unsigned integers: one warp reduction gives the maximum
  const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
  const float s = __fdiv_rn(amax, (float)B200_XQ_MAX);
  int X = 0;
  if (s > 0.0f) {
    X = __float2int_rn(__fdiv_rn(v, s));
    X = X > B200_XQ_MAX ? B200_XQ_MAX : (X < -B200_XQ_MAX ? -B200_XQ_MAX : X);
  }
  const int L0 = ((X + 128) & 255) - 128;
  const int t1 = (X - L0) >> 8;
  const int L1 = ((t1 + 128) & 255) - 128;
  const int L2 = (t1 - L1) >> 8;
  const int sum = __reduce_add_sync(0xffffffffu, X);
  const uint32_t part = lane >> 4, c = (lane & 15) >> 2, q = b >> 2, i = b & 3;
  const uint32_t pair = vec >> 1, vs = vec & 1;
  uint8_t *base = xq.limbs + (((uint64_t)pair * xq.quads + q) * 2 + part) * 512 + i * 4 + (lane & 3);
  base[((vs * 4 + 0) * 4 + c) * 16] = (uint8_t)(int8_t)L2;
  base[((vs * 4 + 1) * 4 + c) * 16] = (uint8_t)(int8_t)L1;
  base[((vs * 4 + 2) * 4 + c) * 16] = (uint8_t)(int8_t)L0;
  base[((vs * 4 + 3) * 4 + c) * 16] = 0;
  if (lane == 0) {
    xq.sb[(uint64_t)vec * xq.quads * 4 + b] = s;
    xq.sx[(uint64_t)vec * xq.quads * 4 + b] = __fmul_rn((float)sum, s);
  }
}

// ---- int8 tensor-core MMA (m16n8k32, s32 accumulate from zero) -----------------------------
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// ---- mbarriers and bulk asynchronous copies --------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Arrive on `bar` (count 1) and add `bytes` to the transactions it waits for.
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// global -> shared bulk copy completing on `bar`; size and both addresses multiples of 16 B
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for phase `parity` of `bar` to complete, giving up after about
// `limit_ns` nanoseconds of wall time (%globaltimer). Returns false on
// timeout, so a copy that never lands ends the wait instead of hanging.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; it++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    const uint64_t now = globaltimer_ns();
    if (it == 0)
      t0 = now;
    else if (now - t0 > limit_ns)
      return false;
  }
}
// As mbar_wait, but each probe lets the thread sleep until the phase
// completes or `hint_ns` passes (mbarrier.try_wait's suspend-time hint), so
// warps waiting in a warp-specialised pipeline take no issue slots from the
// warps doing the work.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, uint64_t limit_ns,
                                                uint32_t hint_ns = 100000u) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; it++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(hint_ns)
        : "memory");
    if (done) return true;
    const uint64_t now = globaltimer_ns();
    if (it == 0)
      t0 = now;
    else if (now - t0 > limit_ns)
      return false;
  }
}
// As mbar_wait, but polls with the non-blocking mbarrier.test_wait, so the
// thread sees the phase complete without a suspend/wake-up round trip: for
// the single threads (copy producers, MMA issuer) on a pipeline's critical
// path. Reads the clock only every 256 polls.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; it++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 255u) == 0) {
      const uint64_t now = globaltimer_ns();
      if (it == 0)
        t0 = now;
      else if (now - t0 > limit_ns)
        return false;
    }
  }
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
