// Host side of the persistent decode-step kernel (decode_kernel.cuh): checks
// the shapes against the kernel's limits, sizes the shared memory and the
// scratch, uploads the layer table and launches the kernel instantiated for
// the layers' block type (k_decode_q4_0.cu, ...).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <new>

#include "decode_kernel.cuh"

struct b200_decode_plan {
  b200dec::Plan p;
};

namespace {

using b200dec::kHD;
using b200dec::kStages;
using b200dec::Shape;

// Work split of an n x k matrix of type t over `grid` CTAs of `gt` tiles per
// row group (decode_kernel.cuh: phase_range, group_split).
Shape make_shape(uint32_t t, uint64_t n, uint64_t k, uint32_t gt, uint32_t grid, uint64_t &max_range) {
  Shape s{};
  s.n = (uint32_t)n;
  s.k = (uint32_t)k;
  s.units = (uint32_t)b200_units(t, k);
  s.ntiles = (uint32_t)b200_ntiles(n);
  s.ngroups = (s.ntiles + gt - 1) / gt;
  s.npad = s.ntiles * 16;
  s.gt = gt;
  s.sc_off = b200_sc_offset(t, n, k);
  const uint64_t total = (uint64_t)s.ngroups * s.units;
  s.gw = (uint32_t)std::min<uint64_t>(grid, total);
  const uint64_t share = total / s.gw;  // >= 1: a CTA's range is at least this long
  max_range = (total + s.gw - 1) / s.gw;
  s.maxseg = (uint32_t)std::min<uint64_t>(s.gw, (s.units + share - 1) / share + 1);
  return s;
}

}  // namespace

extern "C" pai_status_t b200_decode_plan_create(pai_b200_ctx_t *ctx, const b200_decode_args_t *a,
                                                const b200_decode_layer_t *layers, b200_decode_plan_t **out) {
  if (!ctx || !a || !layers || !out) return b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: NULL");
  *out = nullptr;
  const uint32_t T = a->type, B = a->batch;
  if (!b200_type_ok(T)) return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: block type %u", T);
  if (B != 1 && B != 2 && B != 4 && B != 8) return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: batch %u", B);
  if (a->hd != kHD || a->hk == 0 || a->h % a->hk || a->n_layer == 0)
    return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: heads");
  const uint32_t G = a->h / a->hk;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: %u heads per kv head", G);
  const uint64_t E = a->n_embd, el = b200_blk_elems(T);
  if (!b200_type_ok(a->etype) || E == 0 || E % b200_blk_elems(a->etype) || E % el || E % 128 || E > (1u << 20) ||
      a->k_o != (uint64_t)a->h * kHD || a->k_o % el || a->ffl % el || a->ffl % 32 ||
      a->n_qkv != (uint64_t)(a->h + 2 * a->hk) * kHD)
    return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: shapes");
  if (!a->x || !a->tok_in || !a->pos || !a->kc || !a->vc || !a->cos_t || !a->sin_t || !a->out_norm || !a->emb ||
      !a->xq_out.limbs || a->xq_out.batch < B || a->xq_out.k < E)
    return b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: NULL operand");
  if (a->nranks == 0 || a->nranks > B200_TP_MAX_RANKS || a->rank >= a->nranks)
    return b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: rank %u of %u", a->rank, a->nranks);
  for (uint32_t r = 0; a->nranks > 1 && r < a->nranks; r++)
    if (!a->land[r] || ((uintptr_t)a->land[r] & 255))
      return b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: landing buffer of rank %u", r);
  for (uint32_t l = 0; l < a->n_layer; l++) {
    const b200_decode_layer_t &L = layers[l];
    if (!L.wqkv || !L.wo || !L.wgu || !L.wdown || !L.attn_norm || !L.ffn_norm ||
        (((uintptr_t)L.wqkv | (uintptr_t)L.wo | (uintptr_t)L.wgu | (uintptr_t)L.wdown) & 255))
      return b200_fail(PAI_ERR_INVALID_ARG, "decode_plan: layer %u", l);
  }
  pai_status_t st = b200_ctx_use_device(ctx);
  if (st) return st;
  b200_decode_plan *plan = new (std::nothrow) b200_decode_plan();
  if (!plan) return b200_fail(PAI_ERR_NOMEM, "decode_plan: host allocation");
  b200dec::Plan *pl = &plan->p;
  pl->device = b200_ctx_device(ctx);
  pl->type = T;
  pl->nt = (int)((B + 1) / 2);
  pl->cons = b200dec::cons_for(pl->nt);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, pl->device);
  pl->grid = (uint32_t)sms;
  const uint32_t cons = (uint32_t)pl->cons, xpu = T == PAI_B200_Q4_K ? 2 : 1;
  b200dec::KP &k = pl->kp;
  const uint64_t dims[4][2] = {{a->n_qkv, E}, {E, a->k_o}, {2 * a->ffl, E}, {E, a->ffl}};
  uint64_t part_floats[2] = {0, 0};
  size_t area = 0;
  uint32_t tab = 0;
  for (int i = 0; i < 4; i++) {
    uint64_t max_range = 0;
    // tiles per consumer warp: decode_kernel.cuh's kTPW<T, NT>
    const uint32_t tpw = (T == PAI_B200_Q4_0 && pl->nt > 1) ? 2u : 1u;
    k.sh[i] = make_shape(T, dims[i][0], dims[i][1], cons * tpw, pl->grid, max_range);
    k.sh[i].tab = tab;
    tab += k.sh[i].ngroups;
    part_floats[i & 1] = std::max<uint64_t>(part_floats[i & 1], (uint64_t)k.sh[i].maxseg * B * k.sh[i].npad);
    // a staged operand holds at most min(units, longest range) entries
    area = std::max(area, b200dec::x_area_bytes(pl->nt, B, xpu, std::min<uint64_t>(k.sh[i].units, max_range)));
  }
  for (int i = 0; i < 4; i++)
    if ((uint64_t)k.sh[i].ngroups * k.sh[i].units >= (1ull << 31)) {
      delete plan;
      return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: matrix %d has too many (group, unit) pairs", i);
    }
  if (tab > b200dec::kTab) {
    delete plan;
    return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: %u row groups exceed the split table", tab);
  }
  // the stagings' per-warp scratch (128 floats) follows the largest staged operand
  k.scratch_off = (uint32_t)((area + 127) & ~(size_t)127);
  area = k.scratch_off + (size_t)cons * kHD * sizeof(float);
  // attention: q (padded quarter rows), k and v of one kv head, then the warps' partials
  area = std::max(area, ((size_t)G * 4 * b200dec::kQP + 2 * kHD + (size_t)cons * G * b200dec::kAS) * sizeof(float));
  area = (area + 127) & ~(size_t)127;
  pl->smem = (size_t)kStages * cons * 2304u + area;  // ring (kStageBytes) + staging area
  if (pl->smem > 220 * 1024) {
    delete plan;
    return b200_fail(PAI_ERR_UNSUPPORTED, "decode_plan: %zu B of shared memory per CTA", pl->smem);
  }
  // attention CTAs per (sequence, kv head): at most 16, the slots the o
  // GEMV's staging merges in one round of loads
  const uint32_t per_head = std::min<uint32_t>(b200dec::kMaxSlots, std::max<uint32_t>(1, pl->grid / (a->hk * B)));
  // scratch: partials [2] | attention partials | ssq (doubles) | xqn | xqa | xqh | barrier words
  // (xqa, xqh: the once-quantised o and down operands of batches of 3+)
  const uint64_t attn_floats = (uint64_t)B * a->h * per_head * b200dec::kAS;
  const uint64_t ssq_bytes = (uint64_t)B * (E / 32) * 8;
  const uint64_t xqn_bytes = b200_xq_bytes(B, E);
  const uint64_t off_p1 = b200_align256(part_floats[0] * 4), off_at = off_p1 + b200_align256(part_floats[1] * 4);
  const uint64_t off_ssq = off_at + b200_align256(attn_floats * 4), off_xqn = off_ssq + b200_align256(ssq_bytes);
  const uint64_t xqa_bytes = pl->nt > 1 ? b200_xq_bytes(B, a->k_o) : 0, xqh_bytes = pl->nt > 1 ? b200_xq_bytes(B, a->ffl) : 0;
  const uint64_t off_xqa = off_xqn + b200_align256(xqn_bytes), off_xqh = off_xqa + b200_align256(xqa_bytes);
  const uint64_t off_bar = off_xqh + b200_align256(xqh_bytes), bytes = off_bar + 256;
  st = b200_cuda(cudaMalloc(&pl->scratch, bytes), "decode scratch");
  if (!st) st = b200_cuda(cudaMemset(pl->scratch, 0, bytes), "decode scratch clear");
  b200dec::Layer *hl = st ? nullptr : (b200dec::Layer *)calloc(a->n_layer, sizeof(b200dec::Layer));
  if (!st && !hl) st = b200_fail(PAI_ERR_NOMEM, "decode_plan: host allocation");
  for (uint32_t l = 0; !st && l < a->n_layer; l++) {
    hl[l].w[0] = (const uint8_t *)layers[l].wqkv;
    hl[l].w[1] = (const uint8_t *)layers[l].wo;
    hl[l].w[2] = (const uint8_t *)layers[l].wgu;
    hl[l].w[3] = (const uint8_t *)layers[l].wdown;
    hl[l].attn_norm = layers[l].attn_norm;
    hl[l].ffn_norm = layers[l].ffn_norm;
  }
  if (!st) st = b200_cuda(cudaMalloc((void **)&pl->layers, a->n_layer * sizeof(b200dec::Layer)), "decode layers");
  if (!st)
    st = b200_cuda(cudaMemcpy(pl->layers, hl, a->n_layer * sizeof(b200dec::Layer), cudaMemcpyHostToDevice),
                   "decode layers");
  free(hl);
  if (!st) {
    switch (T) {
      case PAI_B200_Q4_0: st = b200dec::attrs<PAI_B200_Q4_0>(pl); break;
      case PAI_B200_Q8_0: st = b200dec::attrs<PAI_B200_Q8_0>(pl); break;
      default: st = b200dec::attrs<PAI_B200_Q4_K>(pl); break;
    }
  }
  if (st) {
    b200_decode_plan_destroy(plan);
    return st;
  }
  uint8_t *sp = (uint8_t *)pl->scratch;
  k.layers = pl->layers;
  k.n_layer = a->n_layer;
  k.batch = B;
  k.eps = a->eps == 0.0f ? 1e-5f : a->eps;
  k.etype = a->etype;
  k.n_embd = (uint32_t)E;
  k.emb_qs = (const uint8_t *)a->emb;
  k.emb_sc = k.emb_qs + b200_sc_offset(a->etype, a->vocab, E);
  k.emb_ntiles = b200_ntiles(a->vocab);
  k.tok_in = a->tok_in;
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
  k.inv_scale = 1.0f / sqrtf((float)kHD);
  k.x = a->x;
  k.xqn = b200_xq_view(sp + off_xqn, B, E);
  if (pl->nt > 1) {
    k.xqa = b200_xq_view(sp + off_xqa, B, a->k_o);
    k.xqh = b200_xq_view(sp + off_xqh, B, a->ffl);
  }
  k.ssq = (double *)(sp + off_ssq);
  k.xq_out = a->xq_out;
  k.out_norm = a->out_norm;
  k.part[0] = (float *)sp;
  k.part[1] = (float *)(sp + off_p1);
  k.apart = (float *)(sp + off_at);
  k.bar = (uint32_t *)(sp + off_bar);
  k.err = b200_ctx_errflag(ctx);
  k.wait_ns = b200_ctx_wait_ns(ctx);
  k.rank = a->rank;
  k.nranks = a->nranks;
  for (uint32_t r = 0; r < a->nranks && a->nranks > 1; r++) k.land[r] = (uint8_t *)a->land[r];
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
  if (plan->p.layers) cudaFree(plan->p.layers);
  delete plan;
}
