// Prefill GEMM Y[M][N] = X[M][K] . W[N][K]^T with Q4_0 weights on the
// 5th-generation tensor cores (tcgen05 + TMEM), bf16 operands, fp32
// accumulation. Reference: pai_ref_gemm_f32 (cpu/reference/ref_ops.c:428-444)
// on the dequantised weights (adapters/llama/gguf.c:680-693); the benchmark
// bar for bf16 tiles is max-abs-rel 2e-2.
//
// Tiling ("swap AB"): a CTA owns 256 output features x BN tokens. The
// weights are the MMA's A operand (two M=128 MMAs, one TMEM accumulator
// each) and the activations its B operand (N = BN = 16, 64 or 128), so a
// 16-token prefill wastes no MMA rows. K advances 64 at a time through a
// 4-stage shared-memory ring:
//   - W: the 8 warps dequantise the packed Q4_0 pieces of the stage (2
//     tiles of 16 rows each, loaded into registers one unit ahead) to bf16
//     and store them in the canonical K-major 128-byte-swizzle layout;
//   - X: converted to bf16 once per call by k_gemm_xprep into the same
//     swizzled layout, tile by tile, so one bulk copy (cp.async.bulk, no
//     multicast) moves a stage's activations;
//   - one thread issues the tcgen05.mma instructions of a stage once both
//     halves are in place and commits them to the stage's mbarrier, which
//     frees the stage for refilling.
// The epilogue reads each accumulator from TMEM (tcgen05.ld, 32 lanes per
// warp) and writes fp32 Y. Every mbarrier wait is bounded (2 s); on timeout
// the CTA raises the context's error flag, still frees its TMEM and exits.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace {

constexpr int kFT = 256;          // output features per CTA (two M=128 MMAs)
constexpr int kBK = 64;           // K per stage: one 128-byte row of bf16
constexpr int kAStage = kFT * kBK * 2;  // 32 KB of bf16 weights per stage
constexpr uint64_t kGWaitLimit = 2000000000ull;

// Byte offset of element (row, k) of a [rows][64] bf16 block in the 128-byte
// swizzle layout: 16-byte chunk c of row r sits at chunk c ^ (r % 8).
__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t k) {
  return row * 128u + ((((k >> 3) ^ row) & 7u) << 4) + (k & 7u) * 2u;
}

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
  float *partial;          // split-K: [split][M][N]
  uint32_t *cnt;           // split-K tickets, one per output tile, left at zero
  uint32_t *err;
  uint32_t m, n, ntiles, nunits, ksplit;  // tokens, features, weight tiles, K units of 128, K splits
};

// Dequantise half a unit (2 blocks, 64 weights) of one 16-row tile from its
// packed piece in shared memory into the swizzled bf16 stage.
__device__ __forceinline__ void dequant_half(uint8_t *a_stage, uint32_t tile_row0, const uint8_t *piece_qs,
                                             const uint8_t *piece_sc, int half, int lane) {
  const uint32_t rl = lane >> 2, c = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const uint4 q = *reinterpret_cast<const uint4 *>(piece_qs + h * 512 + lane * 16);
    const uint2 dd = *reinterpret_cast<const uint2 *>(piece_sc + h * 64 + rl * 8);
    const uint32_t fr = tile_row0 + rl + 8 * h;  // feature row within the CTA's 256
    uint8_t *blk = a_stage + (fr >> 7) * (128 * 128);
    const uint32_t r = fr & 127;
#pragma unroll
    for (int ii = 0; ii < 2; ii++) {
      const int i = 2 * half + ii;  // block within the unit
      const uint32_t w = i == 0 ? q.x : (i == 1 ? q.y : (i == 2 ? q.z : q.w));
      const uint32_t dw = i < 2 ? dd.x : dd.y;
      const float d = __half2float(__ushort_as_half((uint16_t)((i & 1) ? (dw >> 16) : (dw & 0xFFFFu))));
      __nv_bfloat162 lo0 = __floats2bfloat162_rn((float)((int)(w & 15) - 8) * d, (float)((int)((w >> 8) & 15) - 8) * d);
      __nv_bfloat162 lo1 =
          __floats2bfloat162_rn((float)((int)((w >> 16) & 15) - 8) * d, (float)((int)((w >> 24) & 15) - 8) * d);
      __nv_bfloat162 hi0 =
          __floats2bfloat162_rn((float)((int)((w >> 4) & 15) - 8) * d, (float)((int)((w >> 12) & 15) - 8) * d);
      __nv_bfloat162 hi1 =
          __floats2bfloat162_rn((float)((int)((w >> 20) & 15) - 8) * d, (float)((int)((w >> 28) & 15) - 8) * d);
      // low nibbles: elements 4c..4c+3 of the block; high: 16+4c..
      const uint32_t k_lo = ii * 32 + 4 * c, k_hi = ii * 32 + 16 + 4 * c;
      uint2 vlo, vhi;
      vlo.x = *reinterpret_cast<uint32_t *>(&lo0);
      vlo.y = *reinterpret_cast<uint32_t *>(&lo1);
      vhi.x = *reinterpret_cast<uint32_t *>(&hi0);
      vhi.y = *reinterpret_cast<uint32_t *>(&hi1);
      *reinterpret_cast<uint2 *>(blk + sw128(r, k_lo)) = vlo;
      *reinterpret_cast<uint2 *>(blk + sw128(r, k_hi)) = vhi;
    }
  }
}

constexpr int kWorkers = 8;                       // dequantising warps
constexpr int kGThreadsWS = (kWorkers + 3) * 32;  // + raw-W producer, X producer, MMA issuer
constexpr int kRawStages = 3;                     // packed-weight units in flight
constexpr uint32_t kRawStage = 16 * 1024 + 16 * 128;  // one unit of the CTA's 16 tiles: codes, then headers
template <int BN>
constexpr int kAStages = BN == 256 ? 2 : 3;       // bf16 stages (shared memory bound)

template <int BN>
__global__ void __launch_bounds__(kGThreadsWS, 1) k_gemm_q4_0(GemmP p) {
  constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;  // power of two for BN in {16, 64, 128, 256}
  constexpr uint32_t kBStage = BN * 128;
  constexpr uint32_t kIdesc = idesc_bf16(BN);
  constexpr int SA = kAStages<BN>;
  extern __shared__ __align__(1024) uint8_t gsm_raw[];
  // 1024-byte alignment of the swizzled stages
  uint8_t *gsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *a_st = gsm;                                // [SA][2 acc][128 rows][128 B]
  uint8_t *b_st = a_st + (size_t)SA * kAStage;        // [SA][BN rows][128 B]
  uint8_t *r_st = b_st + (size_t)SA * kBStage;        // [kRawStages][16 KB codes | 2 KB headers]
  __shared__ __align__(8) uint64_t rfull[kRawStages], rempty[kRawStages];
  __shared__ __align__(8) uint64_t afull[SA], bfull[SA], aempty[SA];
  __shared__ uint32_t tmem_base_s, ticket_s;
  __shared__ int abort_s;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t f0 = blockIdx.x * kFT, tile0 = f0 / 16;        // first feature and weight tile
  const uint32_t tt = blockIdx.y, m0 = tt * BN;                  // token tile
  const uint32_t z = blockIdx.z;                                 // K split
  const uint32_t u0 = z * p.nunits / p.ksplit, u1 = (z + 1) * p.nunits / p.ksplit;
  const uint32_t nu = u1 - u0, nkt = 2 * nu;                    // units and 64-wide K chunks of this CTA
  const uint32_t nv = min(16u, p.ntiles - min(p.ntiles, tile0));  // weight tiles present
  if (tid == 0) {
    for (int s = 0; s < kRawStages; s++) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], kWorkers * 32);
    }
    for (int s = 0; s < SA; s++) {
      mbar_init(&afull[s], kWorkers * 32);
      mbar_init(&bfull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    abort_s = 0;
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
    // ---- packed weights: one unit of the CTA's tiles per raw stage ----
    if (lane == 0) {
      for (uint32_t i = 0; i < nu && ok; i++) {
        const uint32_t rs = i % kRawStages;
        if (i >= (uint32_t)kRawStages && !mbar_wait(&rempty[rs], ((i / kRawStages) - 1) & 1u, kGWaitLimit)) {
          ok = false;
          break;
        }
        uint8_t *dst = r_st + (size_t)rs * kRawStage;
        const size_t piece = (size_t)(u0 + i) * p.ntiles + tile0;
        if (nv) {
          mbar_expect_tx(&rfull[rs], nv * (1024 + 128));
          bulk_g2s(dst, p.qs + piece * 1024, nv * 1024, &rfull[rs]);
          bulk_g2s(dst + 16 * 1024, p.sc + piece * 128, nv * 128, &rfull[rs]);
        } else {
          mbar_arrive(&rfull[rs]);
        }
      }
    }
  } else if (warp == kWorkers + 1) {
    // ---- activations: one 64-wide K chunk per stage ----
    if (lane == 0) {
      for (uint32_t j = 0; j < nkt && ok; j++) {
        const uint32_t s = j % SA;
        if (j >= (uint32_t)SA && !mbar_wait(&aempty[s], ((j / SA) - 1) & 1u, kGWaitLimit)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&bfull[s], kBStage);
        bulk_g2s(b_st + (size_t)s * kBStage, p.xp + ((size_t)tt * (2 * p.nunits) + 2 * u0 + j) * kBStage, kBStage,
                 &bfull[s]);
      }
    }
  } else if (warp == kWorkers + 2) {
    // ---- MMA issue ----
    if (lane == 0) {
      for (uint32_t j = 0; j < nkt && ok; j++) {
        const uint32_t s = j % SA, ph = (j / SA) & 1u;
        if (!mbar_wait(&afull[s], ph, kGWaitLimit) || !mbar_wait(&bfull[s], ph, kGWaitLimit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t abase = smem_u32(a_st + (size_t)s * kAStage), bbase = smem_u32(b_st + (size_t)s * kBStage);
#pragma unroll
        for (int acc = 0; acc < 2; acc++)
#pragma unroll
          for (int k = 0; k < kBK / 16; k++)
            mma_bf16(tmem + acc * BN, sdesc(abase + acc * (128 * 128) + k * 32), sdesc(bbase + k * 32), kIdesc,
                     (j > 0 || k > 0) ? 1u : 0u);
        mma_commit(&aempty[s]);
      }
    }
  } else {
    // ---- dequantising warps: warp w owns tiles 2w, 2w+1 of the CTA ----
    for (uint32_t i = 0; i < nu && ok; i++) {
      const uint32_t rs = i % kRawStages;
      if (!mbar_wait(&rfull[rs], (i / kRawStages) & 1u, kGWaitLimit)) {
        ok = false;
        break;
      }
      const uint8_t *raw = r_st + (size_t)rs * kRawStage;
      for (int half = 0; half < 2 && ok; half++) {
        const uint32_t j = 2 * i + half, s = j % SA;
        if (j >= (uint32_t)SA && !mbar_wait(&aempty[s], ((j / SA) - 1) & 1u, kGWaitLimit)) {
          ok = false;
          break;
        }
        uint8_t *as = a_st + (size_t)s * kAStage;
        for (int tl = 0; tl < 2; tl++) {
          const uint32_t lt = 2 * warp + tl;  // tile within the CTA
          if (lt < nv) dequant_half(as, 16 * lt, raw + lt * 1024, raw + 16 * 1024 + lt * 128, half, lane);
        }
        fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
        mbar_arrive(&afull[s]);
      }
      mbar_arrive(&rempty[rs]);
    }
  }
  if (!ok) {
    atomicExch(p.err, 1u);
    abort_s = 1;
  }
  // all MMAs done: the commit of the last stage
  if (nkt && !mbar_wait(&aempty[(nkt - 1) % SA], ((nkt - 1) / SA) & 1u, kGWaitLimit)) {
    atomicExch(p.err, 1u);
    abort_s = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const bool split = p.ksplit > 1;
  if (!abort_s && warp < kWorkers) {
    // epilogue: warp w reads TMEM lanes 32(w%4).. of accumulator w/4
    const uint32_t g = warp & 3, acc = warp >> 2;
    const uint32_t feat = f0 + acc * 128 + g * 32 + lane;
    float *dst = split ? p.partial + (size_t)z * p.m * p.n : p.y;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t v[16];
      tmem_ld16(tmem + ((g * 32u) << 16) + acc * BN + c0, v);
      tmem_ld_wait();
      if (feat < p.n) {
#pragma unroll
        for (int jj = 0; jj < 16; jj++) {
          const uint32_t m = m0 + c0 + jj;
          if (m < p.m) dst[(size_t)m * p.n + feat] = __uint_as_float(v[jj]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWorkers + 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  if (!split || abort_s) return;
  // split K: the last split of this output tile to finish adds the parts in order
  __threadfence();
  __syncthreads();
  const uint32_t tile_id = blockIdx.y * gridDim.x + blockIdx.x;
  if (tid == 0) ticket_s = atomicAdd(&p.cnt[tile_id], 1u);
  __syncthreads();
  if (ticket_s != p.ksplit - 1) return;
  __threadfence();
  for (uint32_t e = tid; e < kFT * BN; e += blockDim.x) {
    const uint32_t f = f0 + e % kFT, m = m0 + e / kFT;
    if (f >= p.n || m >= p.m) continue;
    float part[8];  // ksplit <= 8: all loads in flight, then the sum in split order
#pragma unroll
    for (uint32_t q = 0; q < 8; q++)
      if (q < p.ksplit) part[q] = __ldcg(&p.partial[((size_t)q * p.m + m) * p.n + f]);
    float a = 0.f;
#pragma unroll
    for (uint32_t q = 0; q < 8; q++)
      if (q < p.ksplit) a += part[q];
    p.y[(size_t)m * p.n + f] = a;
  }
  if (tid == 0) p.cnt[tile_id] = 0;
}

// X fp32 [M][K] -> bf16 in the GEMM's operand layout: [token tile][K chunk of
// 64][BN rows][128 B swizzled]; rows beyond M and columns beyond K are zero.
template <int BN>
__global__ void __launch_bounds__(256) k_gemm_xprep(const float *__restrict__ x, uint32_t m, uint32_t k,
                                                    uint32_t nkc, uint8_t *__restrict__ xp) {
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 8-element chunk
  const uint32_t chunks_per_row = nkc * 8;
  const uint64_t row = idx / chunks_per_row;
  const uint32_t ch = (uint32_t)(idx % chunks_per_row);
  const uint32_t mtiles = (m + BN - 1) / BN;
  if (row >= (uint64_t)mtiles * BN) return;
  const uint32_t kt = ch / 8, c = ch % 8, k0 = ch * 8;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = (row < m && k0 + j < k) ? x[row * k + k0 + j] : 0.0f;
  uint4 o;
  __nv_bfloat162 b0 = __floats2bfloat162_rn(v[0], v[1]), b1 = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 b2 = __floats2bfloat162_rn(v[4], v[5]), b3 = __floats2bfloat162_rn(v[6], v[7]);
  o.x = *reinterpret_cast<uint32_t *>(&b0);
  o.y = *reinterpret_cast<uint32_t *>(&b1);
  o.z = *reinterpret_cast<uint32_t *>(&b2);
  o.w = *reinterpret_cast<uint32_t *>(&b3);
  const uint32_t tt = (uint32_t)(row / BN), r = (uint32_t)(row % BN);
  uint8_t *dst = xp + ((size_t)tt * nkc + kt) * (BN * 128) + r * 128 + (((c ^ r) & 7u) << 4);
  *reinterpret_cast<uint4 *>(dst) = o;
}

template <int BN>
pai_status_t gemm_launch(pai_b200_ctx_t *ctx, uint32_t m, uint32_t n, uint32_t k, const float *x, const void *w,
                         float *y) {
  const uint32_t nunits = (uint32_t)b200_units(PAI_B200_Q4_0, k), nkc = 2 * nunits;  // K chunks of 64
  const uint32_t mtiles = (m + BN - 1) / BN, ftiles = (n + kFT - 1) / kFT;
  // K split when the output tiles alone leave SMs idle (small prompts)
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, b200_ctx_device(ctx));
  uint32_t ksplit = 1;
  while (ksplit < 8 && (uint64_t)ftiles * mtiles * ksplit * 2 <= (uint64_t)sms && nunits / (ksplit * 2) >= 4)
    ksplit *= 2;
  const uint64_t xp_bytes = (uint64_t)mtiles * nkc * BN * 128;
  void *xp = nullptr;
  pai_status_t st = b200_ctx_xq(ctx, xp_bytes, &xp);
  if (st) return st;
  float *partial = nullptr;
  uint32_t *cnt = nullptr;
  st = b200_ctx_scratch(ctx, ksplit > 1 ? (uint64_t)ksplit * m * n : 0, ftiles * mtiles, &partial, &cnt);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)b200_ctx_stream(ctx);
  const uint64_t nchunks = (uint64_t)mtiles * BN * nkc * 8;
  k_gemm_xprep<BN><<<(unsigned)((nchunks + 255) / 256), 256, 0, s>>>(x, m, k, nkc, (uint8_t *)xp);
  st = b200_launched(ctx, 1, "k_gemm_xprep");
  if (st) return st;
  GemmP p{};
  p.qs = (const uint8_t *)w;
  p.sc = p.qs + b200_sc_offset(PAI_B200_Q4_0, n, k);
  p.xp = (const uint8_t *)xp;
  p.y = y;
  p.partial = partial;
  p.cnt = cnt;
  p.err = b200_ctx_errflag(ctx);
  p.m = m;
  p.n = n;
  p.ntiles = (uint32_t)b200_ntiles(n);
  p.nunits = nunits;
  p.ksplit = ksplit;
  const size_t smem = 1024 + (size_t)kAStages<BN> * (kAStage + BN * 128) + (size_t)kRawStages * kRawStage;
  static bool attr_set[64];
  const int dev = b200_ctx_device(ctx);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    st = b200_cuda(cudaFuncSetAttribute(k_gemm_q4_0<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                   "k_gemm smem attribute");
    if (st) return st;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const dim3 grid(ftiles, mtiles, ksplit);
  k_gemm_q4_0<BN><<<grid, kGThreadsWS, smem, s>>>(p);
  return b200_launched(ctx, 1, "k_gemm_q4_0");
}

}  // namespace

extern "C" pai_status_t pai_b200_gemm_q4_0_f32(pai_b200_ctx_t *ctx, uint64_t m, uint64_t n, uint64_t k,
                                               const float *x, const void *w, float *y) {
  if (!ctx || !x || !w || !y) return b200_fail(PAI_ERR_INVALID_ARG, "gemm: NULL pointer");
  if (m == 0 || n == 0 || k == 0 || k % 32)
    return b200_fail(PAI_ERR_MISMATCH, "gemm: k=%llu is not a whole number of Q4_0 blocks", (unsigned long long)k);
  if (m > 0x7FFFFFFFull || n > 0x7FFFFFF0ull || k > 0x7FFFFFFFull || (n + kFT - 1) / kFT > 0x7FFFFFFFull ||
      (m + 15) / 16 > 65535 || m * n > (1ull << 40))
    return b200_fail(PAI_ERR_UNSUPPORTED, "gemm: shape too large");
  if ((uintptr_t)w & 255) return b200_fail(PAI_ERR_INVALID_ARG, "gemm: weights not 256-byte aligned");
  if (m <= 16) return gemm_launch<16>(ctx, (uint32_t)m, (uint32_t)n, (uint32_t)k, x, w, y);
  if (m <= 64) return gemm_launch<64>(ctx, (uint32_t)m, (uint32_t)n, (uint32_t)k, x, w, y);
  if (m <= 128) return gemm_launch<128>(ctx, (uint32_t)m, (uint32_t)n, (uint32_t)k, x, w, y);
  return gemm_launch<256>(ctx, (uint32_t)m, (uint32_t)n, (uint32_t)k, x, w, y);
}
