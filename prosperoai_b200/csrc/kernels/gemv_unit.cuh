// The per-unit arithmetic of the fused dequantise-and-dot GEMV, shared by
// the single-matrix GEMV kernel (k_gemv.cu) and the persistent decode-step
// kernel (k_decode.cu): how one consumer warp turns one K unit of its
// 16-row tile (packed weight codes and block headers in shared memory) and
// the staged activation digits into row sums on the int8 tensor cores.
// See k_gemv.cu for the operand formats and the error argument.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace gemv {

constexpr uint32_t M4 = 0x0F0F0F0Fu;

__device__ __forceinline__ uint32_t comp(const uint4 &v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
__device__ __forceinline__ float comp(const float4 &v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
__device__ __forceinline__ float half_at(const uint2 &v, int i) {
  uint32_t w = (i < 2) ? v.x : v.y;
  return __half2float(__ushort_as_half((uint16_t)((i & 1) ? (w >> 16) : (w & 0xFFFFu))));
}

// Activation operand: the CTA's staged copy of the xq digits and block
// scales for the K range of the current sub-item: digits [pair][quad][1024 B],
// then sb and sx, each [vec][quad*4] floats.
struct XS {
  const uint8_t *limbs;
  const float *sb, *sx;
  uint32_t quads, batch;
};

struct XOp {
  uint4 lo, hi;
  float4 sb, sx;
};

__device__ __forceinline__ void load_x(const XS &xs, uint32_t nt, uint32_t qq, int lane, XOp &o) {
  const uint8_t *l = xs.limbs + ((size_t)nt * xs.quads + qq) * 1024 + lane * 16;
  o.lo = *reinterpret_cast<const uint4 *>(l);
  o.hi = *reinterpret_cast<const uint4 *>(l + 512);
  const uint32_t vec = 2 * nt + ((lane & 3) >> 1);
  if (vec < xs.batch) {
    o.sb = *reinterpret_cast<const float4 *>(xs.sb + ((size_t)vec * xs.quads + qq) * 4);
    o.sx = *reinterpret_cast<const float4 *>(xs.sx + ((size_t)vec * xs.quads + qq) * 4);
  } else {
    o.sb = make_float4(0.f, 0.f, 0.f, 0.f);
    o.sx = o.sb;
  }
}

// Fold a lane's two accumulator columns: even lanes hold (L2, L1) sums,
// odd lanes (L0, 0); 256*c_even + c_odd/256 over the lane pair is
// sum_j q_j X_j. |c| < 2^16, so the folded integer (< 2^24) converts exactly.
__device__ __forceinline__ float fold(int c_a, int c_b) { return (float)(c_a * 256 + c_b); }

template <uint32_t T>
struct Unit;

// Q4_0: unit = 4 blocks; qs: chunk h = word c of row r+8h for blocks 0..3;
// sc: [16 rows][4 blocks] fp16.
template <>
struct Unit<PAI_B200_Q4_0> {
  static constexpr int U = 2;  // units per pipeline stage
  static constexpr uint32_t QB = 1024, SB = 128;
  static constexpr int XPU = 1;  // x-quads per unit
  template <int NT>
  __device__ static void compute(const uint8_t *qs, const uint8_t *sc, const XS &xs, uint32_t qq, int lane,
                                 float (&yr)[NT], float (&yr8)[NT]) {
    XOp x[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) load_x(xs, nt, qq, lane, x[nt]);
    const uint4 a0 = *reinterpret_cast<const uint4 *>(qs + lane * 16);
    const uint4 a1 = *reinterpret_cast<const uint4 *>(qs + 512 + lane * 16);
    const uint2 d0 = *reinterpret_cast<const uint2 *>(sc + (lane >> 2) * 8);
    const uint2 d1 = *reinterpret_cast<const uint2 *>(sc + 64 + (lane >> 2) * 8);
    const float lscale = (lane & 1) ? (1.0f / 256.0f) : 256.0f;
    const float cmul = (lane & 1) ? 0.0f : 8.0f;  // the -8 offset of Q4_0 codes, once per lane pair
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint32_t wr = comp(a0, i), wr8 = comp(a1, i);
      const uint32_t A0 = wr & M4, A1 = wr8 & M4, A2 = (wr >> 4) & M4, A3 = (wr8 >> 4) & M4;
      const float dr = half_at(d0, i), dr8 = half_at(d1, i);
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        int acc[4];
        mma_u8s8(acc, A0, A1, A2, A3, comp(x[nt].lo, i), comp(x[nt].hi, i));
        const float sl = comp(x[nt].sb, i) * lscale;
        const float cr = comp(x[nt].sx, i) * cmul;
        yr[nt] = fmaf(dr, fmaf(sl, fold(acc[0], acc[1]), -cr), yr[nt]);
        yr8[nt] = fmaf(dr8, fmaf(sl, fold(acc[2], acc[3]), -cr), yr8[nt]);
      }
    }
  }
};

// Q8_0: unit = 4 blocks; qs: chunk 2h+p = bytes 16p+4c.. of row r+8h.
template <>
struct Unit<PAI_B200_Q8_0> {
  static constexpr int U = 1;
  static constexpr uint32_t QB = 2048, SB = 128;
  static constexpr int XPU = 1;
  template <int NT>
  __device__ static void compute(const uint8_t *qs, const uint8_t *sc, const XS &xs, uint32_t qq, int lane,
                                 float (&yr)[NT], float (&yr8)[NT]) {
    XOp x[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) load_x(xs, nt, qq, lane, x[nt]);
    uint4 a[4];
#pragma unroll
    for (int j = 0; j < 4; j++) a[j] = *reinterpret_cast<const uint4 *>(qs + j * 512 + lane * 16);
    const uint2 d0 = *reinterpret_cast<const uint2 *>(sc + (lane >> 2) * 8);
    const uint2 d1 = *reinterpret_cast<const uint2 *>(sc + 64 + (lane >> 2) * 8);
    const float lscale = (lane & 1) ? (1.0f / 256.0f) : 256.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint32_t A0 = comp(a[0], i), A2 = comp(a[1], i), A1 = comp(a[2], i), A3 = comp(a[3], i);
      const float dr = half_at(d0, i), dr8 = half_at(d1, i);
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        int acc[4];
        mma_s8s8(acc, A0, A1, A2, A3, comp(x[nt].lo, i), comp(x[nt].hi, i));
        const float sl = comp(x[nt].sb, i) * lscale;
        yr[nt] = fmaf(dr * sl, fold(acc[0], acc[1]), yr[nt]);
        yr8[nt] = fmaf(dr8 * sl, fold(acc[2], acc[3]), yr8[nt]);
      }
    }
  }
};

// Q4_K: unit = one super-block (8 sub-blocks of 32 = 2 x-quads). qs: chunk
// 2h+p holds, for each 64-group g, bytes 32g+16p+4c.. of row r+8h (low
// nibbles = sub-block 2g, high = 2g+1); sc: [16 rows][16 B] headers.
template <>
struct Unit<PAI_B200_Q4_K> {
  static constexpr int U = 1;
  static constexpr uint32_t QB = 2048, SB = 256;
  static constexpr int XPU = 2;
  // scale and min of sub-block s from the 12 packed bytes (gguf.c:640-648)
  __device__ static void scale_min(const uint4 &h, int s, float &dsc, float &dmm) {
    const float d = __half2float(__ushort_as_half((uint16_t)(h.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
    auto byte = [&](int i) -> uint32_t { return (comp(h, 1 + i / 4) >> (8 * (i % 4))) & 0xFFu; };
    uint32_t sc, m;
    if (s < 4) {
      sc = byte(s) & 63;
      m = byte(s + 4) & 63;
    } else {
      sc = (byte(s + 4) & 0x0F) | ((byte(s - 4) >> 6) << 4);
      m = (byte(s + 4) >> 4) | ((byte(s) >> 6) << 4);
    }
    dsc = d * (float)sc;
    dmm = dmin * (float)m;
  }
  template <int NT>
  __device__ static void compute(const uint8_t *qs, const uint8_t *sc, const XS &xs, uint32_t qq, int lane,
                                 float (&yr)[NT], float (&yr8)[NT]) {
    uint4 a[4];
#pragma unroll
    for (int j = 0; j < 4; j++) a[j] = *reinterpret_cast<const uint4 *>(qs + j * 512 + lane * 16);
    const uint4 h0 = *reinterpret_cast<const uint4 *>(sc + (lane >> 2) * 16);
    const uint4 h1 = *reinterpret_cast<const uint4 *>(sc + 128 + (lane >> 2) * 16);
    const float lscale = (lane & 1) ? (1.0f / 256.0f) : 256.0f;
    const float cmul = (lane & 1) ? 0.0f : 1.0f;
#pragma unroll
    for (int half = 0; half < 2; half++) {  // x-quads 2u, 2u+1 = sub-blocks 0..3, 4..7
      XOp x[NT];
#pragma unroll
      for (int nt = 0; nt < NT; nt++) load_x(xs, nt, qq + half, lane, x[nt]);
#pragma unroll
      for (int gg = 0; gg < 2; gg++) {
        const int g = 2 * half + gg;
        const uint32_t w0 = comp(a[0], g), w1 = comp(a[1], g), w2 = comp(a[2], g), w3 = comp(a[3], g);
#pragma unroll
        for (int nib = 0; nib < 2; nib++) {
          const int s = 2 * g + nib;  // sub-block
          const int i = s & 3;        // block within the x-quad
          const uint32_t A0 = (w0 >> (4 * nib)) & M4, A2 = (w1 >> (4 * nib)) & M4;
          const uint32_t A1 = (w2 >> (4 * nib)) & M4, A3 = (w3 >> (4 * nib)) & M4;
          float dsc, dmm, dsc8, dmm8;
          scale_min(h0, s, dsc, dmm);
          scale_min(h1, s, dsc8, dmm8);
#pragma unroll
          for (int nt = 0; nt < NT; nt++) {
            int acc[4];
            mma_u8s8(acc, A0, A1, A2, A3, comp(x[nt].lo, i), comp(x[nt].hi, i));
            const float sl = comp(x[nt].sb, i) * lscale;
            const float sx = comp(x[nt].sx, i) * cmul;
            yr[nt] = fmaf(dsc, sl * fold(acc[0], acc[1]), fmaf(-dmm, sx, yr[nt]));
            yr8[nt] = fmaf(dsc8, sl * fold(acc[2], acc[3]), fmaf(-dmm8, sx, yr8[nt]));
          }
        }
      }
    }
  }
};


}  // namespace gemv
