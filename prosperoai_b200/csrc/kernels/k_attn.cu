// GQA attention.
//
// Decode (one new query position over the fp16 KV cache) is split over
// positions, flash-decoding style: CTA (kv head, chunk, sequence) scores
// the chunk for all G = H/HK query heads that share the KV head (K rows
// are read once for the G heads), takes the chunk's max and exp-sum,
// and accumulates exp-weighted V rows; a second kernel merges the chunks
// with the usual max-rescaling. In the decode step the same kernel also
// rotates q and k at the position, appends k and v to the cache, and the
// last chunk of each kv head to finish merges the chunks (no separate
// RoPE or merge kernel). Reference: the last-row iteration of
// pai_ref_attention_f32 (cpu/reference/ref_ops.c:307-349) on the cache
// contents: scores scaled by 1/sqrtf(hd) after the dot, softmax with the
// max subtracted, then sum_i p_i v_i.
//
// Prefill (pai_b200_attention_f32) keeps the reference's loop structure
// per (position, head) -- sequential dots, sequential max and sum, then
// p_i = e_i/sum and a sequential weighted sum per dimension -- with
// explicitly rounded operations, so only expf's last bit can differ.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../b200_internal.h"
#include "b200_device.cuh"

namespace {

constexpr int HD = 128;
constexpr uint32_t kMaxStage = 256;  // most K/V positions staged in shared memory per round
constexpr int kMaxStepSplit = 64;  // most position chunks per kv head in the decode step

struct AttnParams {
  const float *q;  // [B][H][HD]
  const __half *kc, *vc;
  float *opart;  // [B][H][nsplit][HD]
  float *ml;     // [B][H][nsplit][2]
  float *out;    // [B][H][HD]
  const int32_t *pos;
  uint32_t npos_host;
  uint32_t h, hk, chunk, nsplit;
  uint64_t cap, seq_stride;
  float inv_scale;
  b200_xq_t xo;  // when xo.limbs is set, the merged output is also quantised for the o projection
  // decode-step form: q, k, v come unrotated from the fused projection row
  // qkv [B][(H + 2 HK) HD]; the kernel rotates q and k at the position, the
  // CTA holding the position appends k and v to the cache, and the last
  // CTA of each (sequence, kv head) merges the chunks (ticket in cnt)
  const float *qkv, *cos_t, *sin_t;
  __half *kw, *vw;
  uint32_t *cnt;
  uint32_t *err;   // the context's error word (a bounded wait ran out)
  uint64_t wait_ns;  // the context's limit on every wait
  uint32_t stage;  // positions of K (and of V) staged in shared memory per round
};

__device__ __forceinline__ uint32_t npos_of(const AttnParams &p) {
  return p.pos ? (uint32_t)(*p.pos) + 1u : p.npos_host;
}
// Positions per chunk: fixed by the host when it knows the length; when the
// position lives on the device, the nsplit chunks cover it evenly (a
// multiple of 32, at most the host's p.chunk, which sized shared memory).
__device__ __forceinline__ uint32_t chunk_of(const AttnParams &p, uint32_t npos) {
  if (!p.pos) return p.chunk;
  const uint32_t c = ((npos + p.nsplit - 1) / p.nsplit + 31) / 32 * 32;
  return c < 32 ? 32 : c;
}

// Merge the chunk partials of query head hh; every thread of the CTA
// calls it (block-wide max), thread d gets output dimension d. The sums
// run over chunks in order, eight loads in flight at a time.
__device__ __forceinline__ float merge_chunks(const AttnParams &p, uint32_t bi, uint32_t hh, uint32_t ns, uint32_t d,
                                              float *sred) {
  const size_t base = ((size_t)bi * p.h + hh) * p.nsplit;
  float M = -INFINITY;
  for (uint32_t s = threadIdx.x; s < ns; s += blockDim.x) M = fmaxf(M, __ldcg(&p.ml[(base + s) * 2]));
  M = warp_max(M);
  if ((threadIdx.x & 31) == 0) sred[threadIdx.x >> 5] = M;
  __syncthreads();
  M = sred[0];
  for (uint32_t w = 1; w < blockDim.x / 32; w++) M = fmaxf(M, sred[w]);
  __syncthreads();
  float L = 0.f, o = 0.f;
  for (uint32_t s0 = 0; s0 < ns; s0 += 8) {
    float mv[8], lv[8], ov[8];
#pragma unroll
    for (int m = 0; m < 8; m++) {
      if (s0 + m < ns) {
        mv[m] = __ldcg(&p.ml[(base + s0 + m) * 2]);
        lv[m] = __ldcg(&p.ml[(base + s0 + m) * 2 + 1]);
        ov[m] = __ldcg(&p.opart[(base + s0 + m) * HD + d]);
      }
    }
#pragma unroll
    for (int m = 0; m < 8; m++) {
      if (s0 + m < ns) {
        const float w = expf(mv[m] - M);
        L = fmaf(lv[m], w, L);
        o = fmaf(ov[m], w, o);
      }
    }
  }
  return o / L;
}

template <int G, bool STEP>
__global__ void __launch_bounds__(128) k_attn_split(AttnParams p) {
  pdl_trigger();
  pdl_wait();
  const uint32_t kvh = blockIdx.x, split = blockIdx.y, bi = blockIdx.z;
  const uint32_t npos = npos_of(p);
  const uint32_t chunk = chunk_of(p, npos);
  const uint32_t start = split * chunk;
  if (start >= npos) return;
  const uint32_t len = min(chunk, npos - start);
  extern __shared__ __align__(16) float sm[];
  float *qs = sm;               // [G][HD]
  float *sc = sm + G * HD;      // [G][chunk]
  // staged K and V rows, p.stage positions each (16-byte aligned: the
  // float parts above are multiples of 4 floats)
  __half (*kst)[HD] = reinterpret_cast<__half (*)[HD]>(sc + (size_t)G * p.chunk);
  __half (*vst)[HD] = kst + p.stage;
  __shared__ float red[2][G][HD];
  __shared__ float mls[G][2];
  __shared__ uint32_t ticket;
  __shared__ __align__(8) uint64_t kvbar;  // completion of the K/V bulk copies
  __shared__ int kvfail;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint32_t h0 = kvh * G;
  const bool one = len <= p.stage;
  if (t == 0) {
    mbar_init(&kvbar, 1);
    fence_mbar_init();
    kvfail = 0;
  }
  if (STEP) {
    // rotate this CTA's G query heads at the position (pai_ref_rope_f32 on
    // the q part of the projection row, adapters/llama/llama.c:713-724)
    const uint32_t pos = npos - 1, r2 = HD / 2;
    const float *row = p.qkv + (size_t)bi * (p.h + 2 * p.hk) * HD;
    for (int i = t; i < G * (int)r2; i += 128) {
      const uint32_t g = i / r2, j = i % r2;
      const float *xr = row + (size_t)(h0 + g) * HD;
      float o0, o1;
      rope_pair(xr[j], xr[j + r2], p.cos_t[(size_t)pos * r2 + j], p.sin_t[(size_t)pos * r2 + j], o0, o1);
      qs[g * HD + j] = o0;
      qs[g * HD + j + r2] = o1;
    }
    if (start + len == npos) {
      // this chunk holds the position: append the rotated k and v (fp16)
      const size_t at = (size_t)bi * p.seq_stride + ((size_t)kvh * p.cap + pos) * HD;
      const float *kr = row + (size_t)(p.h + kvh) * HD, *vr = row + (size_t)(p.h + p.hk + kvh) * HD;
      if (t < (int)r2) {
        float o0, o1;
        rope_pair(kr[t], kr[t + r2], p.cos_t[(size_t)pos * r2 + t], p.sin_t[(size_t)pos * r2 + t], o0, o1);
        p.kw[at + t] = __float2half_rn(o0);
        p.kw[at + t + r2] = __float2half_rn(o1);
      }
      p.vw[at + t] = __float2half_rn(vr[t]);
    }
  } else {
    for (int i = t; i < G * HD; i += 128) qs[i] = p.q[((size_t)bi * p.h + h0) * HD + i];
  }
  // the appended k/v (generic stores) are read below by bulk copies (async proxy)
  asm volatile("fence.proxy.async;" ::: "memory");
  __syncthreads();

  float qr[G][4];
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int e = 0; e < 4; e++) qr[g][e] = qs[g * HD + 4 * lane + e];

  const size_t kvoff = (size_t)bi * p.seq_stride + ((size_t)kvh * p.cap + start) * HD;
  const __half *kb = p.kc + kvoff;
  const __half *vb = p.vc + kvoff;

  // K and V rows are staged in shared memory by bulk copies (a chunk's rows
  // of one kv head are contiguous): the whole chunk at once when it fits in
  // p.stage positions, else p.stage positions per round. The loops below
  // read shared memory only, so no global load waits on the previous
  // position's reductions. Every wait is bounded.
  uint32_t kv_phase = 0;
  auto stage_rows = [&](__half (*dst)[HD], const __half *src, uint32_t cnt) -> bool {
    __syncthreads();  // the previous round's rows are no longer read
    if (t == 0) {
      mbar_expect_tx(&kvbar, cnt * HD * 2);
      bulk_g2s(dst, src, cnt * HD * 2, &kvbar);
    }
    if (!mbar_wait(&kvbar, kv_phase & 1u, p.wait_ns)) kvfail = 1;
    kv_phase++;
    __syncthreads();
    if (kvfail && t == 0) atomicExch(p.err, 1u);
    return !kvfail;
  };
  if (one) {
    // K and V of the whole chunk: two bulk copies on one barrier phase
    if (t == 0) {
      mbar_expect_tx(&kvbar, 2 * len * HD * 2);
      bulk_g2s(kst, kb, len * HD * 2, &kvbar);
      bulk_g2s(vst, vb, len * HD * 2, &kvbar);
    }
    if (!mbar_wait(&kvbar, 0, p.wait_ns)) kvfail = 1;
    kv_phase = 1;
    __syncthreads();
    if (kvfail) {
      if (t == 0) atomicExch(p.err, 1u);
      return;
    }
  }
  // Scores: warp w takes positions w, w+4, ...; lane l holds dims 4l..4l+3.
  for (uint32_t s0 = 0; s0 < len; s0 += p.stage) {
    const uint32_t cnt = min(p.stage, len - s0);
    if (!one) {
      if (!stage_rows(kst, kb + (size_t)s0 * HD, cnt)) return;
    }
    __syncthreads();
    // positions i0, i0 + 4, i0 + 8, i0 + 12 per warp iteration: four
    // independent shuffle reductions per head in flight
    for (uint32_t i0 = warp; i0 < cnt; i0 += 16) {
      float part[4][G];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const uint32_t i = i0 + 4 * u;
        float2 k01 = make_float2(0.f, 0.f), k23 = k01;
        if (i < cnt) {
          uint2 raw = *reinterpret_cast<const uint2 *>(&kst[i][4 * lane]);
          k01 = __half22float2(*reinterpret_cast<__half2 *>(&raw.x));
          k23 = __half22float2(*reinterpret_cast<__half2 *>(&raw.y));
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
          float s = qr[g][0] * k01.x;
          s = fmaf(qr[g][1], k01.y, s);
          s = fmaf(qr[g][2], k23.x, s);
          s = fmaf(qr[g][3], k23.y, s);
          part[u][g] = s;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
          for (int g = 0; g < G; g++) part[u][g] += __shfl_xor_sync(0xffffffffu, part[u][g], o);
      if (lane == 0) {
#pragma unroll
        for (int u = 0; u < 4; u++)
          if (i0 + 4 * u < cnt) {
#pragma unroll
            for (int g = 0; g < G; g++) sc[g * chunk + s0 + i0 + 4 * u] = part[u][g] * p.inv_scale;
          }
      }
    }
  }
  __syncthreads();

  // Chunk softmax statistics; warp w handles heads w, w+4, ...
  for (int g = warp; g < G; g += 4) {
    float *s = sc + g * chunk;
    float m = -INFINITY;
    for (uint32_t i = lane; i < len; i += 32) m = fmaxf(m, s[i]);
    m = warp_max(m);
    float l = 0.f;
    for (uint32_t i = lane; i < len; i += 32) {
      float e = expf(s[i] - m);
      s[i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      mls[g][0] = m;
      mls[g][1] = l;
    }
  }
  __syncthreads();

  // Exp-weighted V: thread t covers dims 2*(t&63), +1 over every other position.
  const int dp = t & 63, sub = t >> 6;
  float acc[G][2];
#pragma unroll
  for (int g = 0; g < G; g++) acc[g][0] = acc[g][1] = 0.f;
  for (uint32_t s0 = 0; s0 < len; s0 += p.stage) {
    const uint32_t cnt = min(p.stage, len - s0);
    if (!one) {
      if (!stage_rows(vst, vb + (size_t)s0 * HD, cnt)) return;
    }
    for (uint32_t i = sub; i < cnt; i += 2) {
      float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&vst[i][2 * dp]));
#pragma unroll
      for (int g = 0; g < G; g++) {
        float e = sc[g * chunk + s0 + i];
        acc[g][0] = fmaf(e, v.x, acc[g][0]);
        acc[g][1] = fmaf(e, v.y, acc[g][1]);
      }
    }
    if (!one) __syncthreads();
  }
#pragma unroll
  for (int g = 0; g < G; g++) {
    red[sub][g][2 * dp] = acc[g][0];
    red[sub][g][2 * dp + 1] = acc[g][1];
  }
  __syncthreads();
  for (int i = t; i < G * HD; i += 128) {
    int g = i / HD, d = i % HD;
    size_t slot = ((size_t)bi * p.h + h0 + g) * p.nsplit + split;
    p.opart[slot * HD + d] = red[0][g][d] + red[1][g][d];
    if (d == 0) {
      p.ml[slot * 2] = mls[g][0];
      p.ml[slot * 2 + 1] = mls[g][1];
    }
  }
  if (!STEP) return;
  // the last chunk of this (sequence, kv head) to finish merges all chunks
  __threadfence();
  __syncthreads();
  const uint32_t ns = (npos + chunk - 1) / chunk;
  if (t == 0) ticket = atomicAdd(&p.cnt[bi * p.hk + kvh], 1u);
  __syncthreads();
  if (ticket != ns - 1) return;
  __threadfence();
  // Statistics of all G heads at once (warp w: heads w, w+4): the chunk
  // maxima, weights exp(m_s - M) and sums, then every thread (dimension t)
  // accumulates all heads with the loads of eight chunks in flight. Same
  // operations in the same order as merge_chunks, so the same bits.
  __shared__ float wsm[G][kMaxStepSplit], lsm[G][kMaxStepSplit], Ls[G];
  // the first eight chunks' outputs do not depend on the statistics: load them first
  float ov[G][8];
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int m = 0; m < 8; m++)
      if (m < (int)ns) ov[g][m] = __ldcg(&p.opart[(((size_t)bi * p.h + h0 + g) * p.nsplit + m) * HD + t]);
  for (int g = warp; g < G; g += 4) {
    const size_t base = ((size_t)bi * p.h + h0 + g) * p.nsplit;
    float M = -INFINITY;
    for (uint32_t s2 = lane; s2 < ns; s2 += 32) M = fmaxf(M, __ldcg(&p.ml[(base + s2) * 2]));
    M = warp_max(M);
    for (uint32_t s2 = lane; s2 < ns; s2 += 32) {
      wsm[g][s2] = expf(__ldcg(&p.ml[(base + s2) * 2]) - M);
      lsm[g][s2] = __ldcg(&p.ml[(base + s2) * 2 + 1]);
    }
    __syncwarp();
    if (lane == 0) {
      float L = 0.f;
      for (uint32_t s2 = 0; s2 < ns; s2++) L = fmaf(lsm[g][s2], wsm[g][s2], L);
      Ls[g] = L;
    }
  }
  __syncthreads();
  float o[G];
#pragma unroll
  for (int g = 0; g < G; g++) o[g] = 0.f;
  for (uint32_t s0 = 0; s0 < ns; s0 += 8) {
    if (s0 > 0) {
#pragma unroll
      for (int g = 0; g < G; g++)
#pragma unroll
        for (int m = 0; m < 8; m++)
          if (s0 + m < ns) ov[g][m] = __ldcg(&p.opart[(((size_t)bi * p.h + h0 + g) * p.nsplit + s0 + m) * HD + t]);
    }
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
      for (int m = 0; m < 8; m++)
        if (s0 + m < ns) o[g] = fmaf(ov[g][m], wsm[g][s0 + m], o[g]);
  }
#pragma unroll
  for (int g = 0; g < G; g++) {
    const float v = o[g] / Ls[g];
    p.out[((size_t)bi * p.h + h0 + g) * HD + t] = v;
    // head h0+g covers elements 128(h0+g).. of the attention output: warp w holds block 4(h0+g)+w
    if (p.xo.limbs) xq_store_block(p.xo, bi, (h0 + g) * 4 + warp, v);
  }
  if (t == 0) p.cnt[bi * p.hk + kvh] = 0;
}

__global__ void __launch_bounds__(128) k_attn_combine(AttnParams p) {
  pdl_trigger();
  pdl_wait();
  const uint32_t h = blockIdx.x, bi = blockIdx.y, d = threadIdx.x;
  const uint32_t npos = npos_of(p);
  const uint32_t chunk = chunk_of(p, npos);
  const uint32_t ns = (npos + chunk - 1) / chunk;
  __shared__ float sred[HD / 32];
  const float v = merge_chunks(p, bi, h, ns, d, sred);
  p.out[((size_t)bi * p.h + h) * HD + d] = v;
  // head h covers elements 128h..128h+127 of the attention output: warp w
  // holds block 4h+w
  if (p.xo.limbs) xq_store_block(p.xo, bi, h * 4 + (d >> 5), v);
}

// Prefill: one CTA per (position, head).
__global__ void __launch_bounds__(128) k_attention_f32(uint32_t h, uint32_t hk, uint32_t hd,
                                                       const float *__restrict__ q, const float *__restrict__ k,
                                                       const float *__restrict__ v, float *__restrict__ out) {
  extern __shared__ float sc[];  // [p+1]
  const uint32_t pos = blockIdx.x, hh = blockIdx.y;
  const uint32_t kvh = (hh * hk) / h;
  const uint32_t np = pos + 1;
  const float *qp = q + ((size_t)pos * h + hh) * hd;
  const float inv_scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  for (uint32_t i = threadIdx.x; i < np; i += blockDim.x) {
    const float *kp = k + ((size_t)i * hk + kvh) * hd;
    float dot = 0.0f;
    for (uint32_t d = 0; d < hd; d++) dot = __fadd_rn(dot, __fmul_rn(qp[d], kp[d]));
    sc[i] = __fmul_rn(dot, inv_scale);
  }
  __syncthreads();
  __shared__ float mx, sum;
  if (threadIdx.x == 0) {
    float m = sc[0];
    for (uint32_t i = 1; i < np; i++) m = sc[i] > m ? sc[i] : m;
    mx = m;
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < np; i += blockDim.x) sc[i] = expf(__fsub_rn(sc[i], mx));
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (uint32_t i = 0; i < np; i++) s = __fadd_rn(s, sc[i]);
    sum = s;
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < np; i += blockDim.x) sc[i] = __fdiv_rn(sc[i], sum);
  __syncthreads();
  for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.0f;
    for (uint32_t i = 0; i < np; i++) acc = __fadd_rn(acc, __fmul_rn(sc[i], v[((size_t)i * hk + kvh) * hd + d]));
    out[((size_t)pos * h + hh) * hd + d] = acc;
  }
}

template <int G, bool STEP = false>
pai_status_t launch_split(pai_b200_ctx_t *ctx, const AttnParams &p0, uint32_t batch) {
  AttnParams p = p0;
  // dynamic shared memory: q [G][HD] and scores [G][chunk] in fp32, then the
  // staged K and V rows; the whole chunk is staged at once when it fits
  // (up to kMaxStage positions), else kMaxStage-or-fewer positions per round
  const size_t base = (size_t)(G * HD + G * p.chunk) * sizeof(float);
  const size_t stat = (size_t)(2 * G * HD + 2 * G + (STEP ? 2 * G * kMaxStepSplit + G : 0)) * sizeof(float) + 64;
  const size_t cap = 200 * 1024, row2 = 2 * HD * sizeof(__half);  // K and V bytes per position
  if (base + stat + 32 * row2 > cap) return b200_fail(PAI_ERR_UNSUPPORTED, "attn_decode: chunk of %u positions", p.chunk);
  uint32_t stage = std::min<uint32_t>(p.chunk, kMaxStage);
  while (stage > 32 && base + stat + stage * row2 > cap) stage -= 32;
  p.stage = stage;
  const size_t smem = base + stage * row2;
  if (smem + stat > 48 * 1024) {
    static SmemOptIn opt;
    pai_status_t st = b200_cuda(opt.ensure(b200_ctx_device(ctx), smem,
                                           [](size_t b) {
                                             return cudaFuncSetAttribute(k_attn_split<G, STEP>,
                                                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                                         (int)b);
                                           }),
                                "k_attn_split smem attribute");
    if (st) return st;
  }
  b200_launch(ctx, k_attn_split<G, STEP>, dim3(p.hk, p.nsplit, batch), dim3(128), smem, p);
  return PAI_OK;
}

// Common set-up. With a device position (pos), nsplit is fixed here so that
// about two CTAs per SM work at the longest context and the kernels cut
// the current length into nsplit even chunks; with a host length, chunks
// are sized from it directly.
pai_status_t attn_setup(pai_b200_ctx_t *ctx, uint32_t batch, uint32_t h, uint32_t hk, uint32_t hd,
                        const int32_t *pos, uint64_t npos_host, uint64_t max_npos, uint64_t cap, uint64_t seq_stride,
                        float *out, const b200_xq_t *xq_out, AttnParams &p, uint32_t &G) {
  if (hd != HD) return b200_fail(PAI_ERR_UNSUPPORTED, "attn_decode: head_dim %u (this kernel takes 128)", hd);
  if (hk == 0 || h % hk) return b200_fail(PAI_ERR_INVALID_ARG, "attn_decode: heads %u / kv heads %u", h, hk);
  G = h / hk;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return b200_fail(PAI_ERR_UNSUPPORTED, "attn_decode: %u query heads per kv head", G);
  if (max_npos == 0 || max_npos > cap) return b200_fail(PAI_ERR_INVALID_ARG, "attn_decode: positions > cache");
  uint32_t chunk, nsplit;
  if (pos) {
    // chunks of at least 64 positions, about one CTA per SM at the longest
    // context: the fewer the chunks, the shorter the merge
    const uint64_t by_sms = (148 + (uint64_t)hk * batch - 1) / ((uint64_t)hk * batch);
    nsplit = (uint32_t)std::max<uint64_t>(
        1, std::min<uint64_t>(std::min<uint64_t>((max_npos + 63) / 64, by_sms), kMaxStepSplit));
    chunk = (uint32_t)std::max<uint64_t>(32, ((max_npos + nsplit - 1) / nsplit + 31) / 32 * 32);
  } else {
    const uint64_t want = (max_npos * hk * batch + 295) / 296;
    chunk = (uint32_t)std::min<uint64_t>(4096, std::max<uint64_t>(32, (want + 31) / 32 * 32));
    nsplit = (uint32_t)((max_npos + chunk - 1) / chunk);
  }
  p = AttnParams{};
  p.out = out;
  p.pos = pos;
  p.npos_host = (uint32_t)npos_host;
  p.h = h;
  p.hk = hk;
  p.chunk = chunk;
  p.nsplit = nsplit;
  p.cap = cap;
  p.seq_stride = seq_stride;
  p.inv_scale = 1.0f / sqrtf((float)hd);
  if (xq_out) p.xo = *xq_out;
  p.err = b200_ctx_errflag(ctx);
  p.wait_ns = b200_ctx_wait_ns(ctx);
  const uint64_t slots = (uint64_t)batch * h * nsplit;
  float *scratch;
  uint32_t *counters;
  pai_status_t st = b200_ctx_scratch(ctx, slots * (HD + 2), batch * hk, &scratch, &counters);
  if (st) return st;
  p.opart = scratch;
  p.ml = scratch + slots * HD;
  p.cnt = counters;
  return PAI_OK;
}

}  // namespace

extern "C" pai_status_t b200_launch_attn_decode(pai_b200_ctx_t *ctx, uint32_t batch, uint32_t h, uint32_t hk,
                                                uint32_t hd, const int32_t *pos, uint64_t npos_host,
                                                uint64_t max_npos, uint64_t cap, uint64_t seq_stride,
                                                const float *q, const uint16_t *kc, const uint16_t *vc,
                                                float *out, const b200_xq_t *xq_out) {
  AttnParams p;
  uint32_t G;
  pai_status_t st = attn_setup(ctx, batch, h, hk, hd, pos, npos_host, max_npos, cap, seq_stride, out, xq_out, p, G);
  if (st) return st;
  p.q = q;
  p.kc = (const __half *)kc;
  p.vc = (const __half *)vc;
  switch (G) {
    case 1: st = launch_split<1>(ctx, p, batch); break;
    case 2: st = launch_split<2>(ctx, p, batch); break;
    case 4: st = launch_split<4>(ctx, p, batch); break;
    default: st = launch_split<8>(ctx, p, batch); break;
  }
  if (st) return st;
  b200_launch(ctx, k_attn_combine, dim3(h, batch), dim3(HD), 0, p);
  return b200_launched(ctx, 2, "k_attn_decode");
}

extern "C" pai_status_t b200_launch_attn_step(pai_b200_ctx_t *ctx, uint32_t batch, uint32_t h, uint32_t hk,
                                              uint32_t hd, const int32_t *pos, uint64_t max_npos, uint64_t cap,
                                              uint64_t seq_stride, const float *qkv, const float *cos_t,
                                              const float *sin_t, uint16_t *kc, uint16_t *vc, float *out,
                                              const b200_xq_t *xq_out) {
  if (!pos || !qkv || !cos_t || !sin_t || !kc || !vc || !out)
    return b200_fail(PAI_ERR_INVALID_ARG, "attn_step: NULL pointer");
  AttnParams p;
  uint32_t G;
  pai_status_t st = attn_setup(ctx, batch, h, hk, hd, pos, 0, max_npos, cap, seq_stride, out, xq_out, p, G);
  if (st) return st;
  p.qkv = qkv;
  p.cos_t = cos_t;
  p.sin_t = sin_t;
  p.kc = (const __half *)kc;
  p.vc = (const __half *)vc;
  p.kw = (__half *)kc;
  p.vw = (__half *)vc;
  switch (G) {
    case 1: st = launch_split<1, true>(ctx, p, batch); break;
    case 2: st = launch_split<2, true>(ctx, p, batch); break;
    case 4: st = launch_split<4, true>(ctx, p, batch); break;
    default: st = launch_split<8, true>(ctx, p, batch); break;
  }
  if (st) return st;
  return b200_launched(ctx, 1, "k_attn_split(step)");
}

extern "C" pai_status_t pai_b200_attn_decode_f16kv(pai_b200_ctx_t *ctx, uint64_t h, uint64_t hk, uint64_t hd,
                                                   uint64_t npos, uint64_t cap, const float *q,
                                                   const uint16_t *kcache, const uint16_t *vcache, float *out) {
  if (!ctx || !q || !kcache || !vcache || !out) return b200_fail(PAI_ERR_INVALID_ARG, "attn_decode: NULL");
  if (((uintptr_t)kcache | (uintptr_t)vcache) & 15)
    return b200_fail(PAI_ERR_INVALID_ARG, "attn_decode: K/V caches must be 16-byte aligned");
  if (h == 0 || hk == 0 || npos == 0 || npos > cap || h > 4096 || cap > 0x7FFFFFFFull)
    return b200_fail(PAI_ERR_INVALID_ARG, "attn_decode: shape");
  return b200_launch_attn_decode(ctx, 1, (uint32_t)h, (uint32_t)hk, (uint32_t)hd, nullptr, npos, npos, cap, 0,
                                 q, kcache, vcache, out, nullptr);
}

extern "C" pai_status_t pai_b200_attention_f32(pai_b200_ctx_t *ctx, uint64_t h, uint64_t hk, uint64_t seq,
                                               uint64_t hd, const float *q, const float *k, const float *v,
                                               float *out) {
  // Argument rules of pai_ref_attention_f32 (ref_ops.c:298-301).
  if (!ctx || h == 0 || hk == 0 || seq == 0 || hd == 0 || h % hk != 0 || !q || !k || !v || !out)
    return b200_fail(PAI_ERR_INVALID_ARG, "attention: invalid arguments");
  size_t smem = seq * sizeof(float);
  if (smem > 200 * 1024 || h > 65535 || seq > 0x7FFFFFFFull)
    return b200_fail(PAI_ERR_UNSUPPORTED, "attention: seq %llu beyond the prefill kernel", (unsigned long long)seq);
  if (smem > 48 * 1024) {
    pai_status_t st = b200_cuda(
        cudaFuncSetAttribute(k_attention_f32, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
        "k_attention_f32 smem attribute");
    if (st) return st;
  }
  k_attention_f32<<<dim3((unsigned)seq, (unsigned)h), 128, smem, (cudaStream_t)b200_ctx_stream(ctx)>>>(
      (uint32_t)h, (uint32_t)hk, (uint32_t)hd, q, k, v, out);
  return b200_launched(ctx, 1, "k_attention_f32");
}

// ---- allocation-free decode attention ------------------------------------------------------
//
// pai_b200_attn_decode_f16kv keeps its chunk partials in the context's
// scratch buffer, which grows with cudaMalloc on first use. Callers that
// must not allocate device memory where they call attention -- a host
// runtime that reserved all of the GPU's memory up front for its own
// arena, code that runs while a CUDA graph is being captured, or a
// latency-critical loop where an allocation would synchronise the device
// -- use pai_b200_attn_decode_f16kv_noalloc instead. Its partials live in
// the fixed array below (4 MiB of device memory that every GPU loading
// this library holds until the process exits).
constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;
static __device__ __align__(256) float g_attn_noalloc_scratch[kNoAllocScratchFloats];

namespace {

// Device address of the array for `device`, looked up once per device with
// that device current (the host-side symbol is only a stand-in, not a
// device address).
pai_status_t noalloc_scratch(int device, float **out) {
  static std::mutex mu;
  static float *addr[64];
  if (device < 0 || device >= 64) return b200_fail(PAI_ERR_UNSUPPORTED, "attn_decode_noalloc: device %d", device);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device]) {
    int prev = 0;
    pai_status_t st = b200_cuda(cudaGetDevice(&prev), "cudaGetDevice");
    if (st) return st;
    st = b200_cuda(cudaSetDevice(device), "cudaSetDevice");
    if (st) return st;
    void *p = nullptr;
    st = b200_cuda(cudaGetSymbolAddress(&p, g_attn_noalloc_scratch), "cudaGetSymbolAddress");
    // the calling thread gets its own device back, or an error says it did not
    const pai_status_t back = b200_cuda(cudaSetDevice(prev), "cudaSetDevice (restoring the caller's device)");
    if (st) return st;
    if (back) return back;
    addr[device] = (float *)p;
  }
  *out = addr[device];
  return PAI_OK;
}

}  // namespace

extern "C" pai_status_t pai_b200_attn_decode_f16kv_noalloc(pai_b200_ctx_t *ctx, uint64_t h, uint64_t hk,
                                                           uint64_t hd, uint64_t npos, uint64_t cap,
                                                           const float *q, const uint16_t *kcache,
                                                           const uint16_t *vcache, float *out) {
  if (!ctx || !q || !kcache || !vcache || !out) return b200_fail(PAI_ERR_INVALID_ARG, "attn_decode_noalloc: NULL");
  if (((uintptr_t)kcache | (uintptr_t)vcache) & 15)
    return b200_fail(PAI_ERR_INVALID_ARG, "attn_decode_noalloc: K/V caches must be 16-byte aligned");
  if (h == 0 || hk == 0 || npos == 0 || npos > cap || h > 4096 || cap > 0x7FFFFFFFull)
    return b200_fail(PAI_ERR_INVALID_ARG, "attn_decode_noalloc: shape");
  if (hd != HD) return b200_fail(PAI_ERR_UNSUPPORTED, "attn_decode_noalloc: head_dim %llu (this kernel takes 128)",
                                 (unsigned long long)hd);
  if (h % hk) return b200_fail(PAI_ERR_INVALID_ARG, "attn_decode_noalloc: heads %llu / kv heads %llu",
                               (unsigned long long)h, (unsigned long long)hk);
  const uint64_t G = h / hk;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return b200_fail(PAI_ERR_UNSUPPORTED, "attn_decode_noalloc: %llu query heads per kv head", (unsigned long long)G);
  // Same position chunking as pai_b200_attn_decode_f16kv for one sequence.
  uint64_t want = (npos * hk + 295) / 296;
  uint32_t chunk = (uint32_t)(((want + 31) / 32) * 32);
  if (chunk < 32) chunk = 32;
  if (chunk > 4096) chunk = 4096;
  const uint32_t nsplit = (uint32_t)((npos + chunk - 1) / chunk);
  const uint64_t need = h * nsplit * (uint64_t)(HD + 2);
  if (need > kNoAllocScratchFloats)
    return b200_fail(PAI_ERR_UNSUPPORTED,
                     "attn_decode_noalloc: %llu heads x %u position chunks need %llu scratch floats; the fixed "
                     "array holds %llu (use pai_b200_attn_decode_f16kv)",
                     (unsigned long long)h, nsplit, (unsigned long long)need,
                     (unsigned long long)kNoAllocScratchFloats);
  float *scratch = nullptr;
  pai_status_t st = noalloc_scratch(b200_ctx_device(ctx), &scratch);
  if (st) return st;
  AttnParams p{};
  p.q = q;
  p.kc = (const __half *)kcache;
  p.vc = (const __half *)vcache;
  p.out = out;
  p.pos = nullptr;
  p.npos_host = (uint32_t)npos;
  p.h = (uint32_t)h;
  p.hk = (uint32_t)hk;
  p.chunk = chunk;
  p.nsplit = nsplit;
  p.cap = cap;
  p.seq_stride = 0;
  p.inv_scale = 1.0f / sqrtf((float)hd);
  p.opart = scratch;
  p.ml = scratch + h * nsplit * HD;
  p.err = b200_ctx_errflag(ctx);
  p.wait_ns = b200_ctx_wait_ns(ctx);
  switch (G) {
    case 1: st = launch_split<1>(ctx, p, 1); break;
    case 2: st = launch_split<2>(ctx, p, 1); break;
    case 4: st = launch_split<4>(ctx, p, 1); break;
    default: st = launch_split<8>(ctx, p, 1); break;
  }
  if (st) return st;
  b200_launch(ctx, k_attn_combine, dim3((unsigned)h, 1), dim3(HD), 0, p);
  return b200_launched(ctx, 2, "k_attn_decode_noalloc");
}
