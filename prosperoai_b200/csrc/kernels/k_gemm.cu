// Prefill GEMM Y[M][N] = X[M][K] . W[N][K]^T with Q4_0 weights on the
// 5th-generation tensor cores (tcgen05 + TMEM), bf16 operands, fp32
// accumulation. Reference: pai_ref_gemm_f32 (cpu/reference/ref_ops.c:428-444)
// on the dequantised weights (adapters/llama/gguf.c:680-693); the benchmark
// bar for bf16 tiles is max-abs-rel 2e-2.
//
// Tiling ("swap AB"): a CTA owns 256 output features x BN tokens. The
// weights are the MMA's A operand (two M=128 MMAs, one TMEM accumulator
// each) and the activations its B operand (N = BN = 16, 64, 128 or 256), so
// a 16-token prefill wastes no MMA rows. K advances 64 at a time through a
// 2- to 4-stage shared-memory ring:
//   - W: one thread streams the packed Q4_0 pieces of the CTA's 16 tiles,
//     one 128-wide K unit at a time, into a 3-deep raw ring (bulk copies);
//     16 warps, one per tile, dequantise them to bf16 (each weight rounded
//     once from the reference's fp32 value, see dq_pair) and store them in
//     the canonical K-major 128-byte-swizzle layout;
//   - X: converted to bf16 once per call by k_gemm_xprep into the same
//     swizzled layout, tile by tile, so one bulk copy (cp.async.bulk, no
//     multicast) moves a stage's activations;
//   - one thread issues the tcgen05.mma instructions of a stage once both
//     halves are in place and commits them to the stage's mbarrier, which
//     frees the stage for refilling.
// The epilogue reads each accumulator from TMEM (tcgen05.ld, 32 lanes per
// warp) and writes fp32 Y; with a K split, each split writes its part and
// the last to finish adds all parts in split order (bit-reproducible). Every mbarrier wait is bounded (2 s); on timeout
// the CTA raises the context's error flag, still frees its TMEM and exits.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "../b200_internal.h"
#include "b200_device.cuh"
#include "gemv_unit.cuh"

namespace {

constexpr int kFT = 256;          // output features per CTA (two M=128 MMAs)
constexpr int kBK = 64;           // K per stage: one 128-byte row of bf16
constexpr int kAStage = kFT * kBK * 2;  // 32 KB of bf16 weights per stage

// Stages are [rows][64] bf16 in the 128-byte swizzle layout: 16-byte chunk c
// of row r sits at chunk position c ^ (r % 8).

// Shared-memory matrix descriptor (tcgen05): K-major, 128-byte swizzle,
// 8-row groups 1024 bytes apart (stride byte offset), leading byte offset
// unused for this layout (1), descriptor version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;                 // leading byte offset (ignored)
  d |= (uint64_t)(1024u >> 4) << 32;       // stride byte offset
  d |= (uint64_t)1u << 46;                 // version
  d |= (uint64_t)2u << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both
// K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct GemmP {
  const uint8_t *qs, *sc;  // packed Q4_0 weights
  const uint8_t *xp;       // activations, bf16, swizzled, [token tile][K chunk][BN][128 B]
  float *y;                // [M][N]
  float *partial;          // split output tiles: [2 slots per CTA][BN][256] fp32
  uint32_t *cnt;           // tickets, one per (output tile, epilogue warp), left at zero
  uint32_t *err;
  uint64_t wait_ns;  // the context's limit on every wait
  uint32_t m, n, ntiles, nunits;  // tokens, features, weight tiles, K units of 128
  uint32_t mtiles;                // token tiles; output tile t = (feature tile t / mtiles, token tile t % mtiles)
  uint64_t work;                  // output tiles x K units: the stream every CTA takes an equal run of
};

// Stream-K partition: CTA c of G processes work units [c W / G, (c + 1) W / G)
// of the (output tile, K unit) stream, tile-major.
__host__ __device__ __forceinline__ uint64_t sk_begin(uint64_t c, uint64_t work, uint64_t g) { return c * work / g; }
// the CTA whose run holds unit w: the largest c with floor(c W / G) <= w
__host__ __device__ __forceinline__ uint64_t sk_owner(uint64_t w, uint64_t work, uint64_t g) {
  return ((w + 1) * g - 1) / work;
}

// K order inside each 64-wide stage. Both operands use it, so the
// contraction is unchanged: 16-byte chunk 2c + b (b = which of the stage's
// two Q4_0 blocks, c = the packed 32-bit word of the block row) holds
// elements e(c, 0..7) of block b,
//   e(c, j) = 4c + {0, 2, 1, 3}[j]            j < 4  (low nibbles)
//           = 16 + 4c + {0, 2, 1, 3}[j - 4]   j >= 4 (high nibbles),
// which is the order in which masking a packed word at bits 0/16, 8/24,
// 4/20 and 12/28 yields the nibbles (Q4_0 byte i: low nibble element i, high
// nibble element i + 16). Chunks 2c + b keep the 8 rows x 4 words a quarter
// warp stores in distinct banks after the 128-byte swizzle.
__host__ __device__ constexpr uint32_t kperm(uint32_t c, uint32_t j) {
  return (j < 4 ? 0u : 16u) + 4u * c + ((j & 1u) << 1) + ((j >> 1) & 1u);
}

// fp16 block scale d -> bf16x2 pairs (dh, dh) and (dl, dl) with dh + dl == d
// exactly: dh is d truncated to 8 significant bits, dl the remaining 3 bits.
__device__ __forceinline__ void split_scale(uint32_t hbits, uint32_t &dh2, uint32_t &dl2) {
  const float d = __half2float(__ushort_as_half((uint16_t)hbits));
  const uint32_t hb = __float_as_uint(d) & 0xFFFF0000u;
  const uint32_t lb = __float_as_uint(d - __uint_as_float(hb));  // exact, low 16 bits zero
  dh2 = hb | (hb >> 16);
  dl2 = (lb & 0xFFFF0000u) | (lb >> 16);
}

__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// Two nibbles q (at bits 0-3 and 16-19 of v) -> bf16x2 of (q - 8) * d rounded
// once to bf16, the reference's fp32 dequantised weight (q - 8) * d (exact in
// fp32) rounded to nearest. Three bf16x2 fused multiply-adds: 0x4300 | q is
// the bf16 128 + q, times 1 minus 136 gives q - 8 exactly; (q - 8) * dl is
// exact (at most 7 significant bits; the -0 addend keeps it a product); the
// last one rounds (q - 8) * dh + (q - 8) * dl once.
__device__ __forceinline__ uint32_t dq_pair(uint32_t v, uint32_t dh2, uint32_t dl2) {
  const uint32_t t = bf2_fma((v & 0x000F000Fu) | 0x43004300u, 0x3F803F80u, 0xC308C308u);  // x 1 + (-136)
  return bf2_fma(t, dh2, bf2_fma(t, dl2, 0x80008000u));
}

// Dequantise half a unit (2 blocks, 64 weights) of one 16-row tile into the
// swizzled bf16 stage: lane (rl, c) converts word c of both blocks of rows
// rl and rl + 8 (q[h] = the lane's 16 packed bytes of row rl + 8h: word c of
// blocks 0..3), one 16-byte store each at stage + soff[h][b]. `sclp` points
// at the lane's row in the tile's split scales ([16 rows][2 block pairs] x
// {dh2, dl2, dh2', dl2'}).
template <int HALF>
__device__ __forceinline__ void dequant_half(uint8_t *stage, const uint32_t (&soff)[2][2], const uint4 (&q)[2],
                                             const uint4 *sclp) {
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const uint4 sp = sclp[h * 16 + HALF];  // {dh2, dl2} of blocks 2 HALF and 2 HALF + 1
#pragma unroll
    for (int b = 0; b < 2; b++) {
      const uint32_t w = HALF ? (b ? q[h].w : q[h].z) : (b ? q[h].y : q[h].x);
      const uint32_t dh2 = b ? sp.z : sp.x, dl2 = b ? sp.w : sp.y;
      uint4 o;
      o.x = dq_pair(w, dh2, dl2);
      o.y = dq_pair(w >> 8, dh2, dl2);
      o.z = dq_pair(w >> 4, dh2, dl2);
      o.w = dq_pair(w >> 12, dh2, dl2);
      *reinterpret_cast<uint4 *>(stage + soff[h][b]) = o;
    }
  }
}

// tcgen05.ld of 8 or 32 consecutive accumulator columns for the warp's 32 lanes
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}

// N consecutive accumulator columns of the warp's 32 lanes
template <uint32_t N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&v)[N]) {
  static_assert(N == 8 || N == 16, "8 or 16 columns");
  if constexpr (N == 8) {
    tmem_ld8(taddr, v);
  } else {
    tmem_ld16(taddr, v);
  }
}

// Q8_0 and Q4_K: K order inside each 64-wide stage. 16-byte chunk 2c + b
// (b = which of the stage's two 32-weight (sub-)blocks) holds elements
// 4c..4c+3 and 16+4c..16+4c+3 of (sub-)block b, in that order: the bytes a
// lane finds in chunks (row, 0) and (row, 1) of the packed piece (k_gemv.cu's
// Q8_0 / Q4_K layouts), so no nibble or byte is moved between lanes.
__host__ __device__ constexpr uint32_t kperm_nat(uint32_t c, uint32_t j) { return (j < 4 ? 0u : 16u) + 4u * c + (j & 3u); }

// Per block type: bytes of one tile's codes (QB) and headers (SB) per K unit,
// 64-wide stages per unit, raw-unit stages in flight.
template <uint32_t T>
struct GT;
template <>
struct GT<PAI_B200_Q4_0> {
  static constexpr uint32_t QB = 1024, SB = 128;
  static constexpr int SPU = 2, RAW = 3;
};
template <>
struct GT<PAI_B200_Q8_0> {
  static constexpr uint32_t QB = 2048, SB = 128;
  static constexpr int SPU = 2, RAW = 2;
};
template <>
struct GT<PAI_B200_Q4_K> {
  static constexpr uint32_t QB = 2048, SB = 256;
  static constexpr int SPU = 4, RAW = 2;  // one 256-weight super-block per unit
};

constexpr int kWorkers = 16;                      // dequantising warps, one weight tile each
constexpr int kGThreadsWS = (kWorkers + 3) * 32;  // + raw-W producer, X producer, MMA issuer
template <uint32_t T>
constexpr uint32_t kRawStage = 16 * (GT<T>::QB + GT<T>::SB);  // one unit of the CTA's 16 tiles: codes, then headers
template <uint32_t T>
constexpr uint32_t kSclBytes = T == PAI_B200_Q4_0 ? kWorkers * 16 * 4 * 8 : 0;  // Q4_0's split scales, per warp
// bf16 weight / activation stages (shared memory bound; the 2-byte-code types
// have raw units twice as large)
// With few tokens (BN 16, 64) an MMA drains its stage at once, so the bf16
// ring stays short and the rest of shared memory holds raw weight units in
// flight: the copies' latency, not the tensor core, bounds those tiles.
template <uint32_t T, int BN>
constexpr int kAStages = BN == 16 ? 2 : (T == PAI_B200_Q4_0 ? (BN == 256 ? 2 : 3) : (BN >= 128 ? 2 : 3));
template <uint32_t T, int BN>
constexpr int kBStages = BN == 16 ? 16 : (T == PAI_B200_Q4_0 ? (BN == 256 ? 3 : 4) : (BN == 256 ? 2 : 4));
template <uint32_t T, int BN>
constexpr size_t gemm_fixed_bytes() {
  return 1024 + (size_t)kAStages<T, BN> * kAStage + (size_t)kBStages<T, BN> * BN * 128 + kSclBytes<T>;
}
// raw units in flight: as many as fit beside the rest (at most 8; 1 KB of the
// 227 KB left for the static mbarriers), at least the type's minimum
template <uint32_t T, int BN>
constexpr int kRawStages = std::max<int>(GT<T>::RAW, std::min<int>(8, (int)((226 * 1024 - gemm_fixed_bytes<T, BN>()) /
                                                                              kRawStage<T>)));
template <uint32_t T, int BN>
constexpr size_t gemm_smem_bytes() {
  return gemm_fixed_bytes<T, BN>() + (size_t)kRawStages<T, BN> * kRawStage<T>;
}

// Eight fp32 values -> one 16-byte chunk of bf16, each rounded once (RN).
__device__ __forceinline__ uint4 bf16x8(const float (&v)[8]) {
  uint4 o;
  __nv_bfloat162 b0 = __floats2bfloat162_rn(v[0], v[1]), b1 = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 b2 = __floats2bfloat162_rn(v[4], v[5]), b3 = __floats2bfloat162_rn(v[6], v[7]);
  o.x = *reinterpret_cast<uint32_t *>(&b0);
  o.y = *reinterpret_cast<uint32_t *>(&b1);
  o.z = *reinterpret_cast<uint32_t *>(&b2);
  o.w = *reinterpret_cast<uint32_t *>(&b3);
  return o;
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// A dequantising lane's part of one K unit of its tile, Q8_0 or Q4_K: the
// packed chunks (row rl + 8h, bytes 16p..) j = 2h + p, and the headers of
// rows rl and rl + 8.
struct RawLane {
  uint4 c[4];
  uint4 hd[2];  // Q4_K: the 16-byte header; Q8_0: .x, .y = the 4 fp16 block scales
};

// Stage s of the unit into the swizzled bf16 stage: for each row (h) and
// (sub-)block b of the stage, the lane's 8 weights, each the reference's
// fp32 dequantised value (gguf.c's arithmetic, explicitly rounded) rounded
// once to bf16.
//   Q8_0 (gguf.c:680-693 form y = q * d; exact in fp32): stage s holds
//   blocks 2s, 2s + 1.
//   Q4_K (y = d*sc * q - dmin*m, gguf.c:750-761): stage s is 64-group s,
//   sub-block 2s + b in the low (b = 0) or high (b = 1) nibbles.
template <uint32_t T>
__device__ __forceinline__ void dequant_stage_nat(uint8_t *stage, const uint32_t (&soff)[2][2], const RawLane &r,
                                                  int s) {
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int b = 0; b < 2; b++) {
      float v[8];
      if constexpr (T == PAI_B200_Q8_0) {
        const int i = 2 * s + b;
        const uint32_t w0 = word_of(r.c[2 * h], i), w1 = word_of(r.c[2 * h + 1], i);
        const uint32_t dw = i < 2 ? r.hd[h].x : r.hd[h].y;
        const float d = __half2float(__ushort_as_half((uint16_t)((i & 1) ? (dw >> 16) : (dw & 0xFFFFu))));
#pragma unroll
        for (int t = 0; t < 4; t++) {
          v[t] = __fmul_rn((float)(int8_t)(w0 >> (8 * t)), d);
          v[4 + t] = __fmul_rn((float)(int8_t)(w1 >> (8 * t)), d);
        }
      } else {
        float dsc, dmm;
        gemv::Unit<PAI_B200_Q4_K>::scale_min(r.hd[h], 2 * s + b, dsc, dmm);
        const uint32_t w0 = word_of(r.c[2 * h], s), w1 = word_of(r.c[2 * h + 1], s);
#pragma unroll
        for (int t = 0; t < 4; t++) {
          v[t] = __fsub_rn(__fmul_rn(dsc, (float)((w0 >> (8 * t + 4 * b)) & 15u)), dmm);
          v[4 + t] = __fsub_rn(__fmul_rn(dsc, (float)((w1 >> (8 * t + 4 * b)) & 15u)), dmm);
        }
      }
      *reinterpret_cast<uint4 *>(stage + soff[h][b]) = bf16x8(v);
    }
}

template <uint32_t T, int BN>
__global__ void __launch_bounds__(kGThreadsWS, 1) k_gemm(GemmP p) {
  constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;  // power of two for BN in {16, 64, 128, 256}
  constexpr uint32_t kBStage = BN * 128;
  constexpr uint32_t kIdesc = idesc_bf16(BN);
  constexpr int SA = kAStages<T, BN>, SB = kBStages<T, BN>;
  constexpr int RS = kRawStages<T, BN>, SPU = GT<T>::SPU;
  constexpr uint32_t QB = GT<T>::QB, HB = GT<T>::SB, kRaw = kRawStage<T>;
  static_assert(gemm_smem_bytes<T, BN>() <= 226 * 1024, "shared memory of one CTA");
  constexpr uint32_t kECols = BN / 2;                      // epilogue columns (tokens) per warp
  constexpr uint32_t kEChunk = kECols < 16 ? kECols : 16;  // columns per TMEM load round
  constexpr uint32_t kFChunk = kECols < 16 ? kECols : 16;  // columns per round of the split-tile sum
  extern __shared__ __align__(1024) uint8_t gsm_raw[];
  // 1024-byte alignment of the swizzled stages
  uint8_t *gsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *a_st = gsm;                                // [SA][2 acc][128 rows][128 B]
  uint8_t *b_st = a_st + (size_t)SA * kAStage;        // [SB][BN rows][128 B]
  uint8_t *r_st = b_st + (size_t)SB * kBStage;        // [RS][16 tiles' codes | 16 tiles' headers]
  uint4 *scl_all = reinterpret_cast<uint4 *>(r_st + (size_t)RS * kRaw);
  __shared__ __align__(8) uint64_t rfull[RS], rempty[RS];
  __shared__ __align__(8) uint64_t afull[SA], aempty[SA], bfull[SB], bempty[SB];
  __shared__ __align__(8) uint64_t accfull, accempty;
  __shared__ uint32_t tmem_base_s;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint64_t G = gridDim.x, cta = blockIdx.x, U = p.nunits;
  const uint64_t w_begin = sk_begin(cta, p.work, G), w_end = sk_begin(cta + 1, p.work, G);
  const uint32_t first_tile = (uint32_t)(w_begin / U);
  if (tid == 0) {
    for (int s = 0; s < RS; s++) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], kWorkers);
    }
    for (int s = 0; s < SA; s++) {
      mbar_init(&afull[s], kWorkers);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < SB; s++) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], 1);
    }
    mbar_init(&accfull, 1);
    mbar_init(&accempty, kWorkers);
    fence_mbar_init();
  }
  if (warp == kWorkers + 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  bool ok = true;

  if (warp == kWorkers) {
    // ---- packed weights: one K unit of the output tile's 16 weight tiles per raw stage ----
    if (lane == 0) {
      uint32_t i = 0, u = (uint32_t)(w_begin % U), tile0 = (first_tile / p.mtiles) * 16, mt = first_tile % p.mtiles;
      for (uint64_t w = w_begin; w < w_end && ok; w++, i++) {
        const uint32_t nv = min(16u, p.ntiles - tile0);
        const uint32_t rs = i % RS;
        if (i >= (uint32_t)RS && !mbar_wait(&rempty[rs], ((i / RS) - 1) & 1u, p.wait_ns)) {
          ok = false;
          break;
        }
        uint8_t *dst = r_st + (size_t)rs * kRaw;
        const size_t piece = (size_t)u * p.ntiles + tile0;
        mbar_expect_tx(&rfull[rs], nv * (QB + HB));
        bulk_g2s(dst, p.qs + piece * QB, nv * QB, &rfull[rs]);
        bulk_g2s(dst + 16 * QB, p.sc + piece * HB, nv * HB, &rfull[rs]);
        if (++u == U) {  // next output tile: token tile fastest
          u = 0;
          if (++mt == p.mtiles) {
            mt = 0;
            tile0 += 16;
          }
        }
      }
    }
  } else if (warp == kWorkers + 1) {
    // ---- activations: one 64-wide K chunk per stage ----
    if (lane == 0) {
      uint32_t j = 0, u = (uint32_t)(w_begin % U), mt = first_tile % p.mtiles;
      for (uint64_t w = w_begin; w < w_end && ok; w++) {
        for (uint32_t hs = 0; hs < (uint32_t)SPU; hs++, j++) {
          const uint32_t s = j % SB;
          if (j >= (uint32_t)SB && !mbar_wait(&bempty[s], ((j / SB) - 1) & 1u, p.wait_ns)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bfull[s], kBStage);
          bulk_g2s(b_st + (size_t)s * kBStage, p.xp + ((size_t)mt * (SPU * U) + SPU * u + hs) * kBStage, kBStage,
                   &bfull[s]);
        }
        if (++u == U) {
          u = 0;
          if (++mt == p.mtiles) mt = 0;
        }
      }
    }
  } else if (warp == kWorkers + 2) {
    // ---- MMA issue: each segment (the run's part of one output tile) into the TMEM accumulators ----
    if (lane == 0) {
      const uint64_t a_desc0 = sdesc(smem_u32(a_st)), b_desc0 = sdesc(smem_u32(b_st));
      uint32_t j = 0, e = 0, u = (uint32_t)(w_begin % U);
      for (uint64_t w = w_begin; w < w_end && ok; w++, u = (u + 1 == U) ? 0 : u + 1) {
        const bool seg_first = w == w_begin || u == 0, seg_last = w + 1 == w_end || u == U - 1;
        if (seg_first && e > 0) {  // the previous segment's epilogue has read the accumulators
          if (!mbar_wait(&accempty, (e - 1) & 1u, p.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        for (uint32_t hs = 0; hs < (uint32_t)SPU; hs++, j++) {
          const uint32_t s = j % SA, sb = j % SB;
          if (!mbar_wait(&afull[s], (j / SA) & 1u, p.wait_ns) || !mbar_wait(&bfull[sb], (j / SB) & 1u, p.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // descriptors are linear in the start address (bits 0-13 = address / 16):
          // build the stage's two once, then step 32 bytes per K slice and 16 KB
          // to the second accumulator's rows
          const uint64_t ad = a_desc0 + (uint64_t)(s * (kAStage >> 4)), bd = b_desc0 + (uint64_t)(sb * (kBStage >> 4));
          const bool fresh = seg_first && hs == 0;
          // alternate the two accumulators so consecutive MMAs are independent
#pragma unroll
          for (int k = 0; k < kBK / 16; k++)
#pragma unroll
            for (int acc = 0; acc < 2; acc++)
              mma_bf16(tmem + acc * BN, ad + (uint64_t)(acc * (128 * 128 >> 4) + k * 2), bd + (uint64_t)(k * 2), kIdesc,
                       (!fresh || k > 0) ? 1u : 0u);
          mma_commit(&aempty[s]);
          mma_commit(&bempty[sb]);
        }
        if (!ok) break;
        if (seg_last) {
          mma_commit(&accfull);
          e++;
        }
      }
    }
  } else {
    // ---- dequantising warps: warp w owns weight tile w of the output tile; then its epilogue slice ----
    const uint4 *scl = scl_all + warp * (16 * 2);
    uint32_t soff[2][2];  // the lane's store offsets within a stage: rows rl, rl + 8; blocks 0, 1
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int b = 0; b < 2; b++) {
        const uint32_t fr = 16u * warp + (lane >> 2) + 8u * h, c = lane & 3;
        soff[h][b] = (fr >> 7) * (128 * 128) + (fr & 127) * 128 + ((((2u * c + b) ^ fr) & 7u) << 4);
      }
    const uint4 *sclp = scl + (lane >> 2) * 2;
    uint4 q[2];
    bool mine = false;
    // one stage (half a unit): wait for its slot, dequantise, publish
    auto stage_half = [&](uint32_t j, auto half_tag) -> bool {
      constexpr int HALF = decltype(half_tag)::value;
      const uint32_t s = j % SA;
      if (j >= (uint32_t)SA && !mbar_wait_sleep(&aempty[s], ((j / SA) - 1) & 1u, p.wait_ns)) return false;
      if (mine) dequant_half<HALF>(a_st + (size_t)s * kAStage, soff, q, sclp);
      fence_proxy_async();  // each lane's generic-proxy stores -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[s]);  // one arrival per warp
      return true;
    };
    // Q8_0 / Q4_K: stage hs of the unit, the same publication protocol
    auto stage_nat = [&](uint32_t j, int hs, const RawLane &rl) -> bool {
      const uint32_t s = j % SA;
      if (j >= (uint32_t)SA && !mbar_wait_sleep(&aempty[s], ((j / SA) - 1) & 1u, p.wait_ns)) return false;
      if (mine) dequant_stage_nat<T>(a_st + (size_t)s * kAStage, soff, rl, hs);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[s]);
      return true;
    };
    // epilogue slice of this warp: TMEM lanes 32 (w % 4).. of accumulator (w / 4) % 2 (features),
    // columns [w / 8 * BN / 2, + BN / 2) (tokens)
    const uint32_t g = warp & 3, acc = (warp >> 2) & 1, cbase = (warp >> 3) * kECols;
    const uint32_t fin = acc * 128 + g * 32 + lane;  // feature within the output tile
    const uint32_t taddr = tmem + ((g * 32u) << 16) + acc * BN + cbase;
    uint32_t i = 0, e = 0, tile = first_tile, u = (uint32_t)(w_begin % U);
    uint32_t ft = first_tile / p.mtiles, mt = first_tile % p.mtiles;
    bool seg_full_start = u == 0;  // the current segment starts at the tile's first K unit
    for (uint64_t w = w_begin; w < w_end && ok; w++, i++) {
      mine = (uint32_t)warp < min(16u, p.ntiles - ft * 16);
      const uint32_t rs = i % RS;
      if (!mbar_wait_sleep(&rfull[rs], (i / RS) & 1u, p.wait_ns)) {
        ok = false;
        break;
      }
      const uint8_t *raw = r_st + (size_t)rs * kRaw;
      if constexpr (T != PAI_B200_Q4_0) {
        RawLane rl{};
        if (mine) {
#pragma unroll
          for (int j = 0; j < 4; j++) rl.c[j] = *reinterpret_cast<const uint4 *>(raw + warp * QB + j * 512 + lane * 16);
          const uint8_t *hp = raw + 16 * QB + warp * HB;
          if constexpr (T == PAI_B200_Q8_0) {
            const uint2 a = *reinterpret_cast<const uint2 *>(hp + (lane >> 2) * 8);
            const uint2 b = *reinterpret_cast<const uint2 *>(hp + 64 + (lane >> 2) * 8);
            rl.hd[0] = make_uint4(a.x, a.y, 0u, 0u);
            rl.hd[1] = make_uint4(b.x, b.y, 0u, 0u);
          } else {
            rl.hd[0] = *reinterpret_cast<const uint4 *>(hp + (lane >> 2) * 16);
            rl.hd[1] = *reinterpret_cast<const uint4 *>(hp + 128 + (lane >> 2) * 16);
          }
        }
#pragma unroll
        for (int hs = 0; hs < SPU; hs++)
          if (ok) ok = stage_nat(SPU * i + hs, hs, rl);
      } else if (mine) {
        // split the tile's 64 block scales once: lane l takes row l / 2, blocks 2 (l % 2) + {0, 1}
        const uint32_t dd = *reinterpret_cast<const uint32_t *>(raw + 16 * 1024 + warp * 128 + lane * 4);
        uint4 sp;
        split_scale(dd & 0xFFFFu, sp.x, sp.y);
        split_scale(dd >> 16, sp.z, sp.w);
        __syncwarp();  // the previous unit's scales are no longer read
        scl_all[warp * (16 * 2) + lane] = sp;
        __syncwarp();
        const uint8_t *pq = raw + warp * 1024 + lane * 16;
        q[0] = *reinterpret_cast<const uint4 *>(pq);
        q[1] = *reinterpret_cast<const uint4 *>(pq + 512);
      }
      if constexpr (T == PAI_B200_Q4_0)
        ok = stage_half(2 * i, std::integral_constant<int, 0>{}) &&
             stage_half(2 * i + 1, std::integral_constant<int, 1>{});
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[rs]);
      if (!ok) break;
      if (!(w + 1 == w_end || u == U - 1)) {
        u++;
        continue;
      }

      // ---- segment end: epilogue of this warp's slice ----
      if (!mbar_wait_sleep(&accfull, e & 1u, p.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t f0 = ft * kFT, m0 = mt * BN;
      const uint32_t feat = f0 + fin;
      const bool whole = seg_full_start && u == U - 1;
      if (whole) {
#pragma unroll 1
        for (uint32_t c0 = 0; c0 < kECols; c0 += kEChunk) {
          uint32_t v[kEChunk];
          tmem_ld_cols(taddr + c0, v);
          tmem_ld_wait();
          if (feat < p.n) {
#pragma unroll
            for (uint32_t jj = 0; jj < kEChunk; jj++) {
              const uint32_t m = m0 + cbase + c0 + jj;
              if (m < p.m) p.y[(size_t)m * p.n + feat] = __uint_as_float(v[jj]);
            }
          }
        }
      } else {
        // part of a tile shared with neighbouring runs: park it in this CTA's
        // slot, and the last of the tile's contributors to finish adds all
        // parts in K order, its own straight from TMEM. Slot layout per warp:
        // [column / 4][lane][4 columns], so a warp's float4 access is 512
        // contiguous bytes.
        const uint32_t slot = 2u * (uint32_t)cta + (tile == first_tile ? 0u : 1u);
        float4 *part = reinterpret_cast<float4 *>(p.partial + (size_t)slot * (BN * kFT)) +
                       (size_t)warp * (kECols / 4) * 32 + lane;
#pragma unroll 1
        for (uint32_t c0 = 0; c0 < kECols; c0 += kEChunk) {
          uint32_t v[kEChunk];
          tmem_ld_cols(taddr + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (uint32_t jj = 0; jj < kEChunk; jj += 4)
            part[(size_t)((c0 + jj) / 4) * 32] = make_float4(__uint_as_float(v[jj]), __uint_as_float(v[jj + 1]),
                                                             __uint_as_float(v[jj + 2]), __uint_as_float(v[jj + 3]));
        }
        __threadfence();
        __syncwarp();
        uint32_t ticket = 0;
        if (lane == 0) ticket = atomicAdd(&p.cnt[(size_t)tile * kWorkers + warp], 1u);
        ticket = __shfl_sync(0xFFFFFFFFu, ticket, 0);
        const uint64_t tw0 = (uint64_t)tile * U;
        const uint32_t c_lo = (uint32_t)sk_owner(tw0, p.work, G), c_hi = (uint32_t)sk_owner(tw0 + U - 1, p.work, G);
        if (ticket == c_hi - c_lo) {
          __threadfence();
#pragma unroll 1
          for (uint32_t c0 = 0; c0 < kECols; c0 += kFChunk) {
            float a[kFChunk];
#pragma unroll 1
            for (uint32_t cc = c_lo; cc <= c_hi; cc++) {
              uint32_t v[kFChunk];
              if (cc == (uint32_t)cta) {
                tmem_ld_cols(taddr + c0, v);
                tmem_ld_wait();
              } else {
                const uint32_t ccf = (uint32_t)(sk_begin(cc, p.work, G) / U);
                const float4 *pp = reinterpret_cast<const float4 *>(
                                       p.partial + (size_t)(2u * cc + (tile == ccf ? 0u : 1u)) * (BN * kFT)) +
                                   ((size_t)warp * (kECols / 4) + c0 / 4) * 32 + lane;
#pragma unroll
                for (uint32_t jj = 0; jj < kFChunk; jj += 4) {
                  const float4 f = __ldcg(pp + (size_t)(jj / 4) * 32);
                  v[jj] = __float_as_uint(f.x);
                  v[jj + 1] = __float_as_uint(f.y);
                  v[jj + 2] = __float_as_uint(f.z);
                  v[jj + 3] = __float_as_uint(f.w);
                }
              }
#pragma unroll
              for (uint32_t jj = 0; jj < kFChunk; jj++)
                a[jj] = cc == c_lo ? __uint_as_float(v[jj]) : a[jj] + __uint_as_float(v[jj]);
            }
            if (feat < p.n) {
#pragma unroll
              for (uint32_t jj = 0; jj < kFChunk; jj++) {
                const uint32_t m = m0 + cbase + c0 + jj;
                if (m < p.m) p.y[(size_t)m * p.n + feat] = a[jj];
              }
            }
          }
          if (lane == 0) p.cnt[(size_t)tile * kWorkers + warp] = 0;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty);  // this warp is done with the accumulators
      e++;
      // next output tile: token tile fastest
      u = 0;
      seg_full_start = true;
      tile++;
      if (++mt == p.mtiles) {
        mt = 0;
        ft++;
      }
    }
  }
  if (!ok) atomicExch(p.err, 1u);
  tc_fence_before();
  __syncthreads();
  if (warp == kWorkers + 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// X fp32 [M][K] -> bf16 in the GEMM's operand layout: [token tile][K chunk of
// 64][BN rows][128 B swizzled]; rows beyond M and columns beyond K are zero.
// NAT: the K order of the Q8_0 / Q4_K stages (kperm_nat), else Q4_0's.
template <int BN, bool NAT>
__global__ void __launch_bounds__(256) k_gemm_xprep(const float *__restrict__ x, uint32_t m, uint32_t k,
                                                    uint32_t nkc, uint8_t *__restrict__ xp) {
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 8-element chunk
  const uint32_t chunks_per_row = nkc * 8;
  const uint64_t row = idx / chunks_per_row;
  const uint32_t ch = (uint32_t)(idx % chunks_per_row);
  const uint32_t mtiles = (m + BN - 1) / BN;
  if (row >= (uint64_t)mtiles * BN) return;
  const uint32_t kt = ch / 8, c = ch % 8;
  // chunk c of the stage: (sub-)block c & 1, packed word c >> 1, in the weights' K order
  const uint32_t kb = kt * 64 + (c & 1u) * 32;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const uint32_t kk = kb + (NAT ? kperm_nat(c >> 1, j) : kperm(c >> 1, j));
    v[j] = (row < m && kk < k) ? x[row * k + kk] : 0.0f;
  }
  const uint4 o = bf16x8(v);
  const uint32_t tt = (uint32_t)(row / BN), r = (uint32_t)(row % BN);
  uint8_t *dst = xp + ((size_t)tt * nkc + kt) * (BN * 128) + r * 128 + (((c ^ r) & 7u) << 4);
  *reinterpret_cast<uint4 *>(dst) = o;
}

template <uint32_t T, int BN>
pai_status_t gemm_launch(pai_b200_ctx_t *ctx, uint32_t m, uint32_t n, uint32_t k, const float *x, const void *w,
                         float *y) {
  const uint32_t nunits = (uint32_t)b200_units(T, k), nkc = GT<T>::SPU * nunits;  // K chunks of 64
  const uint32_t mtiles = (m + BN - 1) / BN, ftiles = (n + kFT - 1) / kFT;
  const uint64_t tiles = (uint64_t)ftiles * mtiles, work = tiles * nunits;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, b200_ctx_device(ctx));
  // Grid: with at least as many output tiles as SMs, one persistent CTA per
  // SM over the whole stream (tiles split only where runs meet). With fewer,
  // each tile is split evenly over floor(SMs / tiles) CTAs, so no tile has
  // more contributors than it needs (measured: stream-K over 112 tiles on
  // 148 CTAs is 23 % slower at M = 512, the split tiles' sums costing more
  // than the extra SMs give). Runs are at least 4 K units long.
  const uint64_t g_want = tiles >= (uint64_t)sms ? (uint64_t)sms : tiles * ((uint64_t)sms / tiles);
  const uint32_t grid = (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(g_want, work / 4));
  const uint64_t xp_bytes = (uint64_t)mtiles * nkc * BN * 128;
  void *xp = nullptr;
  pai_status_t st = b200_ctx_xq(ctx, xp_bytes, &xp);
  if (st) return st;
  float *partial = nullptr;
  uint32_t *cnt = nullptr;
  st = b200_ctx_scratch(ctx, (uint64_t)2 * grid * BN * kFT, (uint32_t)(tiles * kWorkers), &partial, &cnt);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)b200_ctx_stream(ctx);
  const uint64_t nchunks = (uint64_t)mtiles * BN * nkc * 8;
  k_gemm_xprep<BN, T != PAI_B200_Q4_0><<<(unsigned)((nchunks + 255) / 256), 256, 0, s>>>(x, m, k, nkc, (uint8_t *)xp);
  st = b200_launched(ctx, 1, "k_gemm_xprep");
  if (st) return st;
  GemmP p{};
  p.qs = (const uint8_t *)w;
  p.sc = p.qs + b200_sc_offset(T, n, k);
  p.xp = (const uint8_t *)xp;
  p.y = y;
  p.partial = partial;
  p.cnt = cnt;
  p.err = b200_ctx_errflag(ctx);
  p.wait_ns = b200_ctx_wait_ns(ctx);
  p.m = m;
  p.n = n;
  p.ntiles = (uint32_t)b200_ntiles(n);
  p.nunits = nunits;
  p.mtiles = mtiles;
  p.work = work;
  const size_t smem = gemm_smem_bytes<T, BN>();
  static SmemOptIn opt;
  st = b200_cuda(opt.ensure(b200_ctx_device(ctx), smem,
                            [](size_t b) {
                              return cudaFuncSetAttribute(k_gemm<T, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                          (int)b);
                            }),
                 "k_gemm smem attribute");
  if (st) return st;
  k_gemm<T, BN><<<grid, kGThreadsWS, smem, s>>>(p);
  return b200_launched(ctx, 1, "k_gemm");
}

template <uint32_t T>
pai_status_t gemm_typed(pai_b200_ctx_t *ctx, uint32_t m, uint32_t n, uint32_t k, const float *x, const void *w,
                        float *y) {
  if (m <= 16) return gemm_launch<T, 16>(ctx, m, n, k, x, w, y);
  if (m <= 64) return gemm_launch<T, 64>(ctx, m, n, k, x, w, y);
  if (m <= 128) return gemm_launch<T, 128>(ctx, m, n, k, x, w, y);
  return gemm_launch<T, 256>(ctx, m, n, k, x, w, y);
}

}  // namespace

extern "C" pai_status_t pai_b200_gemm_f32(pai_b200_ctx_t *ctx, uint32_t type, uint64_t m, uint64_t n, uint64_t k,
                                          const float *x, const void *w, float *y) {
  if (!ctx || !x || !w || !y) return b200_fail(PAI_ERR_INVALID_ARG, "gemm: NULL pointer");
  if (type != PAI_B200_Q4_0 && type != PAI_B200_Q8_0 && type != PAI_B200_Q4_K)
    return b200_fail(PAI_ERR_UNSUPPORTED, "gemm: block type %u", type);
  if (m == 0 || n == 0 || k == 0 || k % b200_blk_elems(type))
    return b200_fail(PAI_ERR_MISMATCH, "gemm: k=%llu is not a whole number of blocks", (unsigned long long)k);
  if (m > 0x7FFFFFFFull || n > 0x7FFFFFF0ull || k > 0x7FFFFFFFull || (n + kFT - 1) / kFT > 0x7FFFFFFFull ||
      (m + 15) / 16 > 65535 || m * n > (1ull << 40))
    return b200_fail(PAI_ERR_UNSUPPORTED, "gemm: shape too large");
  if ((uintptr_t)w & 255) return b200_fail(PAI_ERR_INVALID_ARG, "gemm: weights not 256-byte aligned");
  switch (type) {
    case PAI_B200_Q4_0: return gemm_typed<PAI_B200_Q4_0>(ctx, (uint32_t)m, (uint32_t)n, (uint32_t)k, x, w, y);
    case PAI_B200_Q8_0: return gemm_typed<PAI_B200_Q8_0>(ctx, (uint32_t)m, (uint32_t)n, (uint32_t)k, x, w, y);
    default: return gemm_typed<PAI_B200_Q4_K>(ctx, (uint32_t)m, (uint32_t)n, (uint32_t)k, x, w, y);
  }
}

extern "C" pai_status_t pai_b200_gemm_q4_0_f32(pai_b200_ctx_t *ctx, uint64_t m, uint64_t n, uint64_t k,
                                               const float *x, const void *w, float *y) {
  return pai_b200_gemm_f32(ctx, PAI_B200_Q4_0, m, n, k, x, w, y);
}
