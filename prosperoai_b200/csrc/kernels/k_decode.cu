// Host side of the persistent decode-step kernel (decode_kernel.cuh): checks
// a phase list against the kernel's limits, sizes the shared memory and the
// scratch the phases need, uploads the phases and launches the kernel
// instantiated for the layers' block type (k_decode_q4_0.cu, ...).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <new>

#include "decode_kernel.cuh"

struct b200_decode_plan {
  b200dec::Plan p;
};

namespace {

using b200dec::DPh;
using b200dec::kAttnSub;
using b200dec::kHD;
using b200dec::kStages;

// Bytes of the activation staging area of a GEMV phase for the largest CTA range.
size_t x_area_bytes(uint32_t nt, uint32_t batch, uint32_t xpu, uint64_t units, uint64_t max_range) {
  const uint64_t nent = std::min<uint64_t>(units, max_range);
  return (size_t)nt * nent * xpu * 1024 + 2 * (size_t)batch * nent * xpu * 16;
}

}  // namespace

extern "C" pai_status_t b200_decode_plan_create(pai_b200_ctx_t *ctx, uint32_t type, const b200_decode_args_t *a,
                                                const b200_phase_t *phases, uint32_t nphases,
                                                b200_decode_plan_t **out) {
  if (!ctx || !a || !phases || !out || nphases == 0) return b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: NULL");
  *out = nullptr;
  if (!b200_type_ok(type)) return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: block type %u", type);
  const uint32_t B = a->batch;
  if (B != 1 && B != 2 && B != 4 && B != 8) return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: batch %u", B);
  if (a->hd != kHD || a->hk == 0 || a->h % a->hk) return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: heads");
  const uint32_t G = a->h / a->hk;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: %u heads per kv head", G);
  if (!b200_type_ok(a->etype) || a->n_embd == 0 || a->n_embd % b200_blk_elems(a->etype))
    return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: embedding shape");
  if (a->nranks == 0 || a->nranks > B200_TP_MAX_RANKS || a->rank >= a->nranks)
    return b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: rank %u of %u", a->rank, a->nranks);
  for (uint32_t r = 0; a->nranks > 1 && r < a->nranks; r++)
    if (!a->land[r] || ((uintptr_t)a->land[r] & 255))
      return b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: landing buffer of rank %u", r);
  pai_status_t st = b200_ctx_use_device(ctx);
  if (st) return st;
  b200_decode_plan *plan = new (std::nothrow) b200_decode_plan();
  if (!plan) return b200_fail(PAI_ERR_NOMEM, "decode_plan: host allocation");
  b200dec::Plan *pl = &plan->p;
  pl->device = b200_ctx_device(ctx);
  pl->type = type;
  pl->nt = (int)((B + 1) / 2);
  pl->cons = b200dec::cons_for(pl->nt);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, pl->device);
  pl->grid = (uint32_t)sms;
  const uint32_t cons = (uint32_t)pl->cons, nthr = cons * 32;
  DPh *hp = (DPh *)calloc(nphases, sizeof(DPh));
  if (!hp) {
    delete plan;
    return b200_fail(PAI_ERR_NOMEM, "decode_plan: host allocation");
  }
  uint64_t partial_floats = 0, tiles = 0, groups4 = 0;
  uint32_t nx = 0;
  size_t area = 0;
  for (uint32_t i = 0; i < nphases && !st; i++) {
    const b200_phase_t &s = phases[i];
    DPh &d = hp[i];
    d.kind = s.kind;
    d.type = s.type;
    d.epi = s.epi;
    d.xsrc = s.xsrc;
    d.layer = s.layer;
    d.xi = s.xi;
    d.xf = s.xf;
    d.gamma = s.gamma;
    d.xo = s.xo;
    d.k = (uint32_t)s.k;
    if (s.kind == B200_PH_NORM) {
      if (!s.xf || !s.gamma || !s.xo.limbs || s.k == 0 || s.k % 32 || s.k > 0x7FFFFFFFull || s.xo.batch < B ||
          s.xo.k < s.k) {
        st = b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: phase %u (final norm) operands", i);
        break;
      }
      continue;
    }
    if (s.kind == B200_PH_EMBED || s.kind == B200_PH_ATTN) continue;
    if (s.kind == B200_PH_XCHG) {
      // the exchange adds every rank's rows [batch][n_embd] to y (= the hidden state)
      if (a->nranks < 2 || !s.y || s.n != a->n_embd || ((uintptr_t)s.y & 15) || s.xi != nx) {
        st = b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: phase %u (row exchange)", i);
        break;
      }
      d.n = (uint32_t)s.n;
      d.y = s.y;
      nx++;
      continue;
    }
    if (s.kind != B200_PH_GEMV) {
      st = b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: phase %u kind %u", i, s.kind);
      break;
    }
    if (s.type != type || !s.w || ((uintptr_t)s.w & 255) || s.n == 0 || s.k == 0 || s.k % b200_blk_elems(s.type) ||
        s.n > 0x7FFFFFF0ull || s.k > 0x7FFFFFFFull || !s.y) {
      st = b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: phase %u matrix", i);
      break;
    }
    if ((s.xsrc == B200_X_NORM && (!s.xf || !s.gamma || s.k % 32)) ||
        (s.xsrc == B200_X_XQ && (!s.xq.limbs || s.xq.batch < B || s.xq.k < s.k)) ||
        (s.epi == B200_EPI_RESIDUAL && !s.res) ||
        (s.epi == B200_EPI_PUSH && (a->nranks < 2 || s.n != a->n_embd || s.xi != nx)) ||
        (s.epi == B200_EPI_SILU_GLU && (s.n % 64 || (s.xo.limbs && (s.xo.batch < B || s.xo.k < s.n / 2))))) {
      st = b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: phase %u operands", i);
      break;
    }
    d.qs = (const uint8_t *)s.w;
    d.sc = d.qs + b200_sc_offset(s.type, s.n, s.k);
    d.n = (uint32_t)s.n;
    d.nout = (uint32_t)(s.n / 2);
    d.units = (uint32_t)b200_units(s.type, s.k);
    d.ntiles = (uint32_t)b200_ntiles(s.n);
    d.ngroups = (d.ntiles + cons - 1) / cons;
    d.npad = d.ntiles * 16;
    d.xq = s.xq;
    d.res = s.res;
    d.y = s.y;
    // the phase's work is split over gw = min(grid, total) CTAs (work_grid)
    const uint64_t total = (uint64_t)d.ngroups * d.units, gw = std::min<uint64_t>(pl->grid, total);
    const uint64_t share = total / gw, max_range = (total + gw - 1) / gw;
    // most CTAs one group meets: a CTA's share is at least floor(total/gw) >= 1
    d.maxseg = (uint32_t)std::min<uint64_t>(gw, (d.units + share - 1) / share + 1);
    if (d.maxseg > 1) partial_floats = std::max<uint64_t>(partial_floats, (uint64_t)d.maxseg * B * d.npad);
    tiles = std::max<uint64_t>(tiles, d.ntiles);
    groups4 = std::max<uint64_t>(groups4, (d.ntiles + 3) / 4);
    const uint32_t xpu = s.type == PAI_B200_Q4_K ? 2 : 1;
    area = std::max(area, x_area_bytes(pl->nt, B, xpu, d.units, max_range));
  }
  const uint32_t per_head = std::max<uint32_t>(1, pl->grid / (a->hk * B));
  area = std::max(area, (size_t)(G * kHD + G * kAttnSub + (nthr / 64) * G * kHD + G * 4) * sizeof(float));
  area = (area + 127) & ~(size_t)127;
  pl->smem = (size_t)kStages * cons * 2304u + area;  // ring (kStageBytes) + staging area
  if (!st && pl->smem > 220 * 1024)
    st = b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: %zu B of shared memory per CTA", pl->smem);
  // scratch: partials | attention partials | tile tickets | group tickets |
  // attention tickets | barrier words (256-byte aligned)
  const uint64_t attn_floats = (uint64_t)B * a->h * per_head * (kHD + 2);
  const uint64_t cnt_words = tiles + groups4 + (uint64_t)B * a->hk;
  const uint64_t bytes = (partial_floats + attn_floats) * 4 + cnt_words * 4 + 512;
  if (!st) st = b200_cuda(cudaMalloc(&pl->scratch, bytes), "decode scratch");
  if (!st) st = b200_cuda(cudaMemset(pl->scratch, 0, bytes), "decode scratch clear");
  if (!st) st = b200_cuda(cudaMalloc((void **)&pl->dph, nphases * sizeof(DPh)), "decode phases");
  if (!st) st = b200_cuda(cudaMemcpy(pl->dph, hp, nphases * sizeof(DPh), cudaMemcpyHostToDevice), "decode phases");
  free(hp);
  if (!st) {
    switch (type) {
      case PAI_B200_Q4_0: st = b200dec::attrs<PAI_B200_Q4_0>(pl); break;
      case PAI_B200_Q8_0: st = b200dec::attrs<PAI_B200_Q8_0>(pl); break;
      default: st = b200dec::attrs<PAI_B200_Q4_K>(pl); break;
    }
  }
  if (st) {
    b200_decode_plan_destroy(plan);
    return st;
  }
  b200dec::KP &k = pl->kp;
  k.ph = pl->dph;
  k.nph = nphases;
  k.batch = B;
  k.eps = a->eps == 0.0f ? 1e-5f : a->eps;
  k.etype = a->etype;
  k.n_embd = (uint32_t)a->n_embd;
  k.emb_qs = (const uint8_t *)a->emb;
  k.emb_sc = k.emb_qs + b200_sc_offset(a->etype, a->vocab, a->n_embd);
  k.emb_ntiles = b200_ntiles(a->vocab);
  k.tok_in = a->tok_in;
  k.x = a->x;
  k.h = a->h;
  k.hk = a->hk;
  k.per_head = per_head;
  k.pos = a->pos;
  k.cap = a->cap;
  k.seq_stride = a->seq_stride;
  k.layer_stride = a->layer_stride;
  k.kc = (__half *)a->kc;
  k.vc = (__half *)a->vc;
  k.cos_t = a->cos_t;
  k.sin_t = a->sin_t;
  k.qkv = a->qkv;
  k.att = a->att;
  k.xq_att = a->xq_att;
  k.inv_scale = 1.0f / sqrtf((float)kHD);
  uint8_t *sp = (uint8_t *)pl->scratch;
  k.partial = (float *)sp;
  sp += partial_floats * 4;
  k.apart = (float *)sp;
  sp += attn_floats * 4;
  k.tile_cnt = (uint32_t *)sp;
  sp += tiles * 4;
  k.grp_cnt = (uint32_t *)sp;
  sp += groups4 * 4;
  k.attn_cnt = (uint32_t *)sp;
  sp += (uint64_t)B * a->hk * 4;
  k.bar = (uint32_t *)(((uintptr_t)sp + 255) & ~(uintptr_t)255);
  k.err = b200_ctx_errflag(ctx);
  k.wait_ns = b200_ctx_wait_ns(ctx);
  k.rank = a->rank;
  k.nranks = a->nranks;
  for (uint32_t r = 0; r < a->nranks && a->nranks > 1; r++) k.land[r] = (uint8_t *)a->land[r];
  k.xrows = (uint32_t)(B * a->n_embd);
  k.nx = nx;
  *out = plan;
  return PAI_OK;
}

extern "C" pai_status_t b200_decode_launch(pai_b200_ctx_t *ctx, b200_decode_plan_t *plan) {
  if (!ctx || !plan) return b200_fail(PAI_ERR_INVALID_ARG, "decode_launch: NULL");
  b200dec::Plan *pl = &plan->p;
  pai_status_t st;
  switch (pl->type) {
    case PAI_B200_Q4_0: st = b200dec::launch<PAI_B200_Q4_0>(ctx, pl); break;
    case PAI_B200_Q8_0: st = b200dec::launch<PAI_B200_Q8_0>(ctx, pl); break;
    default: st = b200dec::launch<PAI_B200_Q4_K>(ctx, pl); break;
  }
  if (st) return st;
  return b200_launched(ctx, 1, "k_decode");
}

extern "C" void b200_decode_plan_destroy(b200_decode_plan_t *plan) {
  if (!plan) return;
  cudaSetDevice(plan->p.device);
  if (plan->p.scratch) cudaFree(plan->p.scratch);
  if (plan->p.dph) cudaFree(plan->p.dph);
  delete plan;
}
