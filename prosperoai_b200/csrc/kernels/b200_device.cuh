// Device helpers shared by the kernels.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

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

// Streaming 128-bit load of weights that are read once per step: read-only
// path, no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint16_t ldg_u16(const void *p) {
  uint16_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// Exact conversion of a 4-bit field (already isolated in bits 0..3) to
// float: 2^23 + v is representable, subtracting 2^23 + bias is exact.
__device__ __forceinline__ float nib_to_f(uint32_t v_in_low_bits, float bias_plus_2p23) {
  return __uint_as_float(0x4B000000u | v_in_low_bits) - bias_plus_2p23;
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
