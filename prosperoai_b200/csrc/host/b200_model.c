/*
 * LLaMA-shaped decoder on the cuda-b200 backend: weight residency in one
 * device arena and the decode step, in the op order of the reference's
 * LLaMA graph (adapters/llama/llama.c:669-797):
 *
 *   x   = embed(token)                                   llama.c:510-522
 *   per layer:
 *     xn  = rmsnorm(x, attn_norm)                        :674-678
 *     q,k,v = xn.Wq, xn.Wk, xn.Wv    (one fused GEMV)    :680-697
 *     q,k = rope(q), rope(k); k,v -> fp16 cache          :713-724
 *     a   = attention(q, K, V)                           :725-730
 *     x   = x + a.Wo                 (residual fused)    :736-749
 *     xn  = rmsnorm(x, ffn_norm)                         :750-755
 *     h   = silu(xn.Wgate) * (xn.Wup) (one fused GEMV)   :756-781
 *     x   = x + h.Wdown              (residual fused)    :782-795
 *   logits = rmsnorm(x, output_norm).Wout; token = argmax :884-895
 *
 * The decode step runs every layer in one persistent cooperative kernel
 * (kernels/decode_kernel.cuh), then the lm head, the argmax and the token
 * feedback. With PAI_B200_PERSISTENT=0 (or a shape that kernel does not
 * take) a layer is 7 launches instead: each norm quantises x for the GEMV
 * that consumes it; RoPE, the cache append, attention and the chunk merge
 * are one kernel that also writes the o projection's quantised input; the
 * gate/up GEMV applies SiLU*up and quantises h for the down projection:
 * norm, qkv, attention, o (+x), norm, gate/up, down (+x).
 *
 * Host code only: every device step is a launcher from csrc/kernels.
 */
#include <stdlib.h>
#include <string.h>

#include "../b200_internal.h"

/* Row-offset sentinels understood by the pack kernel. */
#define ROW_ZERO (~0ull)
#define ROW_SKIP (~0ull - 1ull)

struct pai_b200_model {
  pai_b200_ctx_t *ctx;
  pai_b200_model_cfg_t cfg;
  uint32_t rank, tp;
  uint32_t hl, hkl, ffl, vl, v0; /* per-rank heads, kv heads, ffn rows, vocab rows, first vocab row */
  uint64_t n_qkv, k_o;           /* fused q|k|v rows; o input columns on this rank */
  uint8_t *arena;
  uint64_t arena_bytes;
  uint64_t sz_qkv, sz_o, sz_gu, sz_down, sz_emb, sz_out;
  uint8_t **wqkv, **wo, **wgu, **wdown;
  float **attn_norm, **ffn_norm;
  uint8_t *tok_embd, *output;
  float *output_norm;
  void *tmp_blocks, *tmp_f32, *tmp_off; /* load-time staging */
  void *tp_comm;                        /* tensor-parallel communicator */
  uint64_t tmp_blocks_bytes, tmp_f32_bytes, tmp_off_bytes;
};

static uint64_t a256(uint64_t v) { return (v + 255u) & ~(uint64_t)255u; }

pai_status_t pai_b200_model_create(pai_b200_ctx_t *ctx, const pai_b200_model_cfg_t *cfg, uint32_t tp_rank,
                                   uint32_t tp_size, pai_b200_model_t **out) {
  pai_b200_model_t *m;
  const pai_b200_model_cfg_t *c = cfg;
  uint64_t E, hd, off = 0;
  pai_status_t st;
  if (!ctx || !cfg || !out) {
    return b200_fail(PAI_ERR_INVALID_ARG, "model_create: NULL");
  }
  *out = NULL;
  if (tp_size == 0 || tp_rank >= tp_size) {
    return b200_fail(PAI_ERR_INVALID_ARG, "model_create: rank %u of %u", tp_rank, tp_size);
  }
  if (!b200_type_ok(c->wtype) || !b200_type_ok(c->etype)) {
    return b200_fail(PAI_ERR_UNSUPPORTED, "model_create: block types %u/%u", c->wtype, c->etype);
  }
  if (c->n_layer == 0 || c->n_embd == 0 || c->n_head == 0 || c->n_head_kv == 0 || c->head_dim != 128 ||
      c->n_ff == 0 || c->vocab == 0 || c->n_head % c->n_head_kv) {
    return b200_fail(PAI_ERR_UNSUPPORTED, "model_create: shape (head_dim must be 128, heads a multiple of kv heads)");
  }
  if (c->n_head_kv % tp_size || c->n_ff % (32u * tp_size) || c->vocab % tp_size) {
    return b200_fail(PAI_ERR_MISMATCH, "model_create: kv heads, ffn and vocab must split over %u ranks", tp_size);
  }
  E = c->n_embd;
  hd = c->head_dim;
  if (E % b200_blk_elems(c->wtype) || E % b200_blk_elems(c->etype) ||
      (c->n_head / tp_size * hd) % b200_blk_elems(c->wtype) || (c->n_ff / tp_size) % b200_blk_elems(c->wtype)) {
    return b200_fail(PAI_ERR_MISMATCH, "model_create: row lengths must be whole blocks on every rank");
  }
  m = (pai_b200_model_t *)calloc(1, sizeof(*m));
  if (!m) {
    return b200_fail(PAI_ERR_NOMEM, "model_create: host allocation");
  }
  m->ctx = ctx;
  m->cfg = *c;
  m->rank = tp_rank;
  m->tp = tp_size;
  m->hl = c->n_head / tp_size;
  m->hkl = c->n_head_kv / tp_size;
  m->ffl = c->n_ff / tp_size;
  m->vl = c->vocab / tp_size;
  m->v0 = m->vl * tp_rank;
  m->n_qkv = (uint64_t)(m->hl + 2 * m->hkl) * hd;
  m->k_o = (uint64_t)m->hl * hd;
  m->sz_qkv = a256(pai_b200_packed_bytes(c->wtype, m->n_qkv, E));
  m->sz_o = a256(pai_b200_packed_bytes(c->wtype, E, m->k_o));
  m->sz_gu = a256(pai_b200_packed_bytes(c->wtype, 2ull * m->ffl, E));
  m->sz_down = a256(pai_b200_packed_bytes(c->wtype, E, m->ffl));
  m->sz_emb = a256(pai_b200_packed_bytes(c->etype, c->vocab, E));
  m->sz_out = a256(pai_b200_packed_bytes(c->etype, m->vl, E));
  m->arena_bytes = (uint64_t)c->n_layer * (m->sz_qkv + m->sz_o + m->sz_gu + m->sz_down + 2 * a256(E * 4)) +
                   m->sz_emb + m->sz_out + a256(E * 4);
  m->wqkv = (uint8_t **)calloc(c->n_layer, sizeof(void *));
  m->wo = (uint8_t **)calloc(c->n_layer, sizeof(void *));
  m->wgu = (uint8_t **)calloc(c->n_layer, sizeof(void *));
  m->wdown = (uint8_t **)calloc(c->n_layer, sizeof(void *));
  m->attn_norm = (float **)calloc(c->n_layer, sizeof(void *));
  m->ffn_norm = (float **)calloc(c->n_layer, sizeof(void *));
  if (!m->wqkv || !m->wo || !m->wgu || !m->wdown || !m->attn_norm || !m->ffn_norm) {
    pai_b200_model_destroy(m);
    return b200_fail(PAI_ERR_NOMEM, "model_create: host allocation");
  }
  st = pai_b200_alloc(ctx, m->arena_bytes, (void **)&m->arena);
  if (st) {
    pai_b200_model_destroy(m);
    return st;
  }
  st = pai_b200_memset(ctx, m->arena, 0, m->arena_bytes);
  if (st) {
    pai_b200_model_destroy(m);
    return st;
  }
  for (uint32_t l = 0; l < c->n_layer; l++) {
    m->wqkv[l] = m->arena + off, off += m->sz_qkv;
    m->wo[l] = m->arena + off, off += m->sz_o;
    m->wgu[l] = m->arena + off, off += m->sz_gu;
    m->wdown[l] = m->arena + off, off += m->sz_down;
    m->attn_norm[l] = (float *)(m->arena + off), off += a256(E * 4);
    m->ffn_norm[l] = (float *)(m->arena + off), off += a256(E * 4);
  }
  m->tok_embd = m->arena + off, off += m->sz_emb;
  m->output = m->arena + off, off += m->sz_out;
  m->output_norm = (float *)(m->arena + off);
  *out = m;
  return PAI_OK;
}

pai_status_t pai_b200_model_destroy(pai_b200_model_t *m) {
  if (!m) {
    return PAI_OK;
  }
  if (m->arena) pai_b200_free(m->ctx, m->arena);
  if (m->tmp_blocks) pai_b200_free(m->ctx, m->tmp_blocks);
  if (m->tmp_f32) pai_b200_free(m->ctx, m->tmp_f32);
  if (m->tmp_off) pai_b200_free(m->ctx, m->tmp_off);
  free(m->wqkv);
  free(m->wo);
  free(m->wgu);
  free(m->wdown);
  free(m->attn_norm);
  free(m->ffn_norm);
  free(m);
  return PAI_OK;
}

uint64_t pai_b200_model_weight_bytes(const pai_b200_model_t *m) { return m ? m->arena_bytes : 0; }

uint64_t pai_b200_model_step_weight_bytes(const pai_b200_model_t *m) {
  const pai_b200_model_cfg_t *c;
  uint64_t E, per_layer;
  if (!m) return 0;
  c = &m->cfg;
  E = c->n_embd;
  per_layer = pai_b200_block_bytes(c->wtype, m->n_qkv * E) + pai_b200_block_bytes(c->wtype, E * m->k_o) +
              pai_b200_block_bytes(c->wtype, 2ull * m->ffl * E) + pai_b200_block_bytes(c->wtype, E * m->ffl);
  return c->n_layer * per_layer + pai_b200_block_bytes(c->etype, (uint64_t)m->vl * E) +
         pai_b200_block_bytes(c->etype, E);
}

/* ---- weight loading ----------------------------------------------------------------- */

static pai_status_t ensure_tmp(pai_b200_model_t *m, uint64_t blocks, uint64_t f32, uint64_t offs) {
  pai_status_t st = PAI_OK;
  if (blocks > m->tmp_blocks_bytes) {
    pai_b200_free(m->ctx, m->tmp_blocks);
    m->tmp_blocks = NULL;
    m->tmp_blocks_bytes = 0;
    st = pai_b200_alloc(m->ctx, blocks, &m->tmp_blocks);
    if (st) return st;
    m->tmp_blocks_bytes = blocks;
  }
  if (f32 > m->tmp_f32_bytes) {
    pai_b200_free(m->ctx, m->tmp_f32);
    m->tmp_f32 = NULL;
    m->tmp_f32_bytes = 0;
    st = pai_b200_alloc(m->ctx, f32, &m->tmp_f32);
    if (st) return st;
    m->tmp_f32_bytes = f32;
  }
  if (offs * 8 > m->tmp_off_bytes) {
    pai_b200_free(m->ctx, m->tmp_off);
    m->tmp_off = NULL;
    m->tmp_off_bytes = 0;
    st = pai_b200_alloc(m->ctx, offs * 8, &m->tmp_off);
    if (st) return st;
    m->tmp_off_bytes = offs * 8;
  }
  return st;
}

/* Source shape (rows x cols, block type) of a whole tensor kind. */
static int tensor_shape(const pai_b200_model_t *m, uint32_t kind, uint64_t *rows, uint64_t *cols,
                        uint32_t *type) {
  const pai_b200_model_cfg_t *c = &m->cfg;
  uint64_t E = c->n_embd, qd = (uint64_t)c->n_head * c->head_dim, kd = (uint64_t)c->n_head_kv * c->head_dim;
  *type = c->wtype;
  switch (kind) {
    case PAI_B200_T_TOK_EMBD:
    case PAI_B200_T_OUTPUT: *rows = c->vocab, *cols = E, *type = c->etype; return 1;
    case PAI_B200_T_WQ: *rows = qd, *cols = E; return 1;
    case PAI_B200_T_WK:
    case PAI_B200_T_WV: *rows = kd, *cols = E; return 1;
    case PAI_B200_T_WO: *rows = E, *cols = qd; return 1;
    case PAI_B200_T_WGATE:
    case PAI_B200_T_WUP: *rows = c->n_ff, *cols = E; return 1;
    case PAI_B200_T_WDOWN: *rows = E, *cols = c->n_ff; return 1;
    default: return 0;
  }
}

/* Pack this rank's share of a whole ggml tensor (already on the device
 * in m->tmp_blocks) into its place in the fused, sharded matrices. */
static pai_status_t pack_tensor(pai_b200_model_t *m, uint32_t kind, uint32_t layer) {
  const pai_b200_model_cfg_t *c = &m->cfg;
  uint64_t rows, cols, n_dst, k_dst, rb, hd = c->head_dim;
  uint32_t type;
  uint8_t *dst;
  uint64_t *off;
  pai_status_t st;
  tensor_shape(m, kind, &rows, &cols, &type);
  rb = pai_b200_block_bytes(type, cols);
  switch (kind) {
    case PAI_B200_T_WQ: case PAI_B200_T_WK: case PAI_B200_T_WV:
      dst = m->wqkv[layer], n_dst = m->n_qkv, k_dst = c->n_embd; break;
    case PAI_B200_T_WO: dst = m->wo[layer], n_dst = c->n_embd, k_dst = m->k_o; break;
    case PAI_B200_T_WGATE: case PAI_B200_T_WUP:
      dst = m->wgu[layer], n_dst = 2ull * m->ffl, k_dst = c->n_embd; break;
    case PAI_B200_T_WDOWN: dst = m->wdown[layer], n_dst = c->n_embd, k_dst = m->ffl; break;
    case PAI_B200_T_TOK_EMBD: dst = m->tok_embd, n_dst = c->vocab, k_dst = c->n_embd; break;
    default: dst = m->output, n_dst = m->vl, k_dst = c->n_embd; break;
  }
  off = (uint64_t *)malloc(n_dst * sizeof(uint64_t));
  if (!off) return b200_fail(PAI_ERR_NOMEM, "pack_tensor: host allocation");
  for (uint64_t r = 0; r < n_dst; r++) {
    uint64_t o = ROW_SKIP;
    uint64_t qrows = (uint64_t)m->hl * hd, krows = (uint64_t)m->hkl * hd;
    uint64_t g = r / 16, w = r % 16, i = g * 8 + (w % 8); /* gate/up tile: 8 gate then 8 up rows */
    switch (kind) {
      case PAI_B200_T_WQ:
        if (r < qrows) o = ((uint64_t)m->rank * qrows + r) * rb;
        break;
      case PAI_B200_T_WK:
        if (r >= qrows && r < qrows + krows) o = ((uint64_t)m->rank * krows + (r - qrows)) * rb;
        break;
      case PAI_B200_T_WV:
        if (r >= qrows + krows) o = ((uint64_t)m->rank * krows + (r - qrows - krows)) * rb;
        break;
      case PAI_B200_T_WO:
      case PAI_B200_T_WDOWN:
        o = r * rb + pai_b200_block_bytes(type, (uint64_t)m->rank * k_dst);
        break;
      case PAI_B200_T_WGATE:
        if (w < 8) o = ((uint64_t)m->rank * m->ffl + i) * rb;
        break;
      case PAI_B200_T_WUP:
        if (w >= 8) o = ((uint64_t)m->rank * m->ffl + i) * rb;
        break;
      case PAI_B200_T_TOK_EMBD: o = r * rb; break;
      default: o = ((uint64_t)m->v0 + r) * rb; break;
    }
    off[r] = o;
  }
  st = pai_b200_memcpy_h2d(m->ctx, m->tmp_off, off, n_dst * sizeof(uint64_t));
  if (!st) st = pai_b200_pack(m->ctx, type, n_dst, k_dst, m->tmp_blocks, (const uint64_t *)m->tmp_off, dst);
  if (!st) st = pai_b200_sync(m->ctx); /* the host offset table is freed next */
  free(off);
  return st;
}

/* Largest packed destination row count (size of the row-offset table). */
static uint64_t max_dst_rows(const pai_b200_model_t *m) {
  uint64_t v = m->n_qkv;
  if (2ull * m->ffl > v) v = 2ull * m->ffl;
  if (m->cfg.n_embd > v) v = m->cfg.n_embd;
  if (m->cfg.vocab > v) v = m->cfg.vocab;
  return v;
}

static float *norm_ptr(pai_b200_model_t *m, uint32_t kind, uint32_t layer) {
  if (kind == PAI_B200_T_OUTPUT_NORM) return m->output_norm;
  return kind == PAI_B200_T_ATTN_NORM ? m->attn_norm[layer] : m->ffn_norm[layer];
}

static int is_norm(uint32_t kind) {
  return kind == PAI_B200_T_OUTPUT_NORM || kind == PAI_B200_T_ATTN_NORM || kind == PAI_B200_T_FFN_NORM;
}

static int per_layer(uint32_t kind) {
  return kind != PAI_B200_T_TOK_EMBD && kind != PAI_B200_T_OUTPUT && kind != PAI_B200_T_OUTPUT_NORM;
}

pai_status_t pai_b200_model_set_tensor(pai_b200_model_t *m, uint32_t kind, uint32_t layer, const void *host) {
  uint64_t rows, cols, bytes;
  uint32_t type;
  pai_status_t st;
  if (!m || !host) return b200_fail(PAI_ERR_INVALID_ARG, "set_tensor: NULL");
  if (kind > PAI_B200_T_FFN_NORM) return b200_fail(PAI_ERR_INVALID_ARG, "set_tensor: kind %u", kind);
  if (per_layer(kind) && layer >= m->cfg.n_layer)
    return b200_fail(PAI_ERR_INVALID_ARG, "set_tensor: layer %u of %u", layer, m->cfg.n_layer);
  if (is_norm(kind)) {
    st = pai_b200_memcpy_h2d(m->ctx, norm_ptr(m, kind, layer), host, (uint64_t)m->cfg.n_embd * 4);
    return st ? st : pai_b200_sync(m->ctx);
  }
  tensor_shape(m, kind, &rows, &cols, &type);
  bytes = pai_b200_block_bytes(type, rows * cols);
  st = ensure_tmp(m, bytes, 0, max_dst_rows(m));
  if (!st) st = pai_b200_memcpy_h2d(m->ctx, m->tmp_blocks, host, bytes);
  if (!st) st = pack_tensor(m, kind, layer);
  return st;
}

uint64_t pai_b200_tensor_seed(uint64_t seed, uint32_t kind, uint32_t layer) {
  return seed * 0x100000001B3ull + ((uint64_t)layer << 8) + kind + 1u;
}

pai_status_t pai_b200_synth_blocks(pai_b200_ctx_t *ctx, uint32_t type, uint64_t rows, uint64_t cols,
                                   uint64_t seed, float stddev, float *tmp_f32, void *dst_blocks) {
  pai_status_t st;
  if (!ctx || !tmp_f32 || !dst_blocks) return b200_fail(PAI_ERR_INVALID_ARG, "synth_blocks: NULL");
  if (!b200_type_ok(type) || cols % b200_blk_elems(type))
    return b200_fail(PAI_ERR_MISMATCH, "synth_blocks: %llu columns of type %u", (unsigned long long)cols, type);
  st = b200_launch_synth_normal(ctx, tmp_f32, rows, cols, seed, stddev);
  if (!st) st = b200_launch_quantize(ctx, type, tmp_f32, rows * cols, dst_blocks);
  return st;
}

pai_status_t pai_b200_model_synthesize(pai_b200_model_t *m, uint64_t seed) {
  const pai_b200_model_cfg_t *c;
  uint64_t maxb = 0, maxf = 0, maxr = 0;
  pai_status_t st;
  static const uint32_t kinds[] = {PAI_B200_T_WQ, PAI_B200_T_WK, PAI_B200_T_WV, PAI_B200_T_WO,
                                   PAI_B200_T_WGATE, PAI_B200_T_WUP, PAI_B200_T_WDOWN};
  if (!m) return b200_fail(PAI_ERR_INVALID_ARG, "synthesize: NULL");
  c = &m->cfg;
  for (uint32_t kind = 0; kind <= PAI_B200_T_WDOWN; kind++) {
    uint64_t rows, cols;
    uint32_t type;
    if (!tensor_shape(m, kind, &rows, &cols, &type)) continue;
    if (pai_b200_block_bytes(type, rows * cols) > maxb) maxb = pai_b200_block_bytes(type, rows * cols);
    if (rows * cols * 4 > maxf) maxf = rows * cols * 4;
    if (rows > maxr) maxr = rows;
    if (cols > maxr) maxr = cols;
  }
  (void)maxr;
  st = ensure_tmp(m, maxb, maxf, max_dst_rows(m));
  if (st) return st;
  for (uint32_t l = 0; l < c->n_layer + 1; l++) {
    uint32_t nk = l < c->n_layer ? 7 : 2;
    for (uint32_t j = 0; j < nk; j++) {
      uint32_t kind = l < c->n_layer ? kinds[j] : (j == 0 ? PAI_B200_T_TOK_EMBD : PAI_B200_T_OUTPUT);
      uint32_t layer = l < c->n_layer ? l : 0;
      uint64_t rows, cols;
      uint32_t type;
      tensor_shape(m, kind, &rows, &cols, &type);
      st = pai_b200_synth_blocks(m->ctx, type, rows, cols, pai_b200_tensor_seed(seed, kind, layer), 0.02f,
                                 (float *)m->tmp_f32, m->tmp_blocks);
      if (!st) st = pack_tensor(m, kind, layer);
      if (st) return st;
    }
  }
  for (uint32_t l = 0; l < c->n_layer; l++) {
    st = b200_launch_fill(m->ctx, m->attn_norm[l], c->n_embd, 1.0f);
    if (!st) st = b200_launch_fill(m->ctx, m->ffn_norm[l], c->n_embd, 1.0f);
    if (st) return st;
  }
  st = b200_launch_fill(m->ctx, m->output_norm, c->n_embd, 1.0f);
  if (!st) st = pai_b200_sync(m->ctx);
  /* Release the staging buffers (up to a few GB for the embedding). */
  pai_b200_free(m->ctx, m->tmp_blocks);
  pai_b200_free(m->ctx, m->tmp_f32);
  m->tmp_blocks = m->tmp_f32 = NULL;
  m->tmp_blocks_bytes = m->tmp_f32_bytes = 0;
  return st;
}

/* ---- decode session ----------------------------------------------------------------- */

struct pai_b200_session {
  pai_b200_model_t *m;
  uint32_t batch, max_ctx, pos; /* max_ctx: capacity in positions, whole 128-position blocks */
  uint64_t kv_reservations;     /* pai_kv_cache_t.stats_blocks */
  int32_t *tok_in, *tok_out, *dpos; /* device */
  int32_t *htok;                    /* pinned host staging, 2*batch */
  float *x, *qkv, *att, *ox, *h, *logits, *cos_t, *sin_t;
  void *xq_buf;                   /* GEMV operands: */
  b200_xq_t xq_e, xq_o, xq_h;     /* normed x (fallback path), attention output, silu*up */
  uint16_t *kc, *vc; /* [layer][batch][hkl][max_ctx][hd] */
  uint64_t seq_stride, layer_stride;
  void *graph;
  uint32_t graph_kernels;
  b200_decode_plan_t *plan; /* persistent decode kernel of the layers (NULL: one launch per op) */
  void *land[B200_TP_MAX_RANKS]; /* tensor parallelism: every rank's landing buffer (persistent path) */
  int failed;               /* a bounded device wait ran out: the session refuses further work */
  int pf_gemm;              /* prefill layer matrices on the tensor-core GEMM (else the batched GEMV) */
  pai_b200_tp_t *tp; /* tensor-parallel communicator, NULL on one GPU */
  /* prefill scratch (allocated by the first prefill): rows of hidden state,
   * normed rows, q|k|v, attention output, gate|up, silu*up, o/down output,
   * token ids, and the GEMV operand of 8 rows */
  uint32_t pf_rows;
  float *pf_x, *pf_xn, *pf_qkv, *pf_att, *pf_gu, *pf_h, *pf_tmp;
  int32_t *pf_tok, *pf_htok;
  void *pf_xq_buf;
  b200_xq_t pf_xq;
};

/* Tensor-parallel hooks (csrc/host/b200_tp.c). */
void b200_tp_mark_failed(pai_b200_tp_t *tp);
pai_status_t b200_tp_land(pai_b200_tp_t *tp, uint64_t rows, void **out);
int b200_tp_failed(const pai_b200_tp_t *tp);
pai_status_t b200_tp_reserve(pai_b200_tp_t *tp, uint64_t cap);
float *b200_tp_slot(pai_b200_tp_t *tp, uint32_t slot);
pai_status_t b200_tp_allreduce_add(pai_b200_tp_t *tp, pai_b200_ctx_t *ctx, uint32_t slot, float *x, uint64_t n);
pai_status_t b200_tp_argmax(void *tp, pai_b200_ctx_t *ctx, uint32_t batch, uint32_t vl, uint32_t v0,
                            const float *logits, int32_t *tok_out);

/* y = W . rmsnorm_gamma(x): a many-CTA norm kernel quantises x once into
 * xq_e (it overlaps the GEMV's weight prefetch under programmatic
 * dependent launch), then the GEMV stages xq_e. The GEMV can also apply
 * the norm itself (b200_launch_gemv_norm), but then every CTA quantises
 * all of x, which costs more than this kernel at 4096-wide rows. */
static pai_status_t norm_gemv(pai_b200_session_t *s, uint32_t type, uint64_t n, const void *w, const float *gamma,
                              float *y, int epi, const b200_xq_t *xq_out) {
  pai_b200_model_t *m = s->m;
  const uint32_t B = s->batch, E = m->cfg.n_embd;
  pai_status_t st = b200_launch_rmsnorm_xq(m->ctx, B, E, s->x, gamma, m->cfg.eps, NULL, &s->xq_e);
  if (!st) st = b200_launch_gemv(m->ctx, type, B, n, E, w, &s->xq_e, NULL, y, epi, xq_out);
  return st;
}

/* The persistent decode kernel of the session: the layer table, the shapes
 * of this rank's shard, the cache and the lm head's operand (xq_e). Under
 * tensor parallelism it also maps every rank's landing buffer (collective). */
static pai_status_t make_plan(pai_b200_session_t *s) {
  pai_b200_model_t *m = s->m;
  const pai_b200_model_cfg_t *c = &m->cfg;
  b200_decode_layer_t *layers = (b200_decode_layer_t *)calloc(c->n_layer, sizeof(*layers));
  b200_decode_args_t a;
  pai_status_t st = PAI_OK;
  if (!layers) return b200_fail(PAI_ERR_NOMEM, "session_create: host allocation");
  for (uint32_t l = 0; l < c->n_layer; l++) {
    layers[l].wqkv = m->wqkv[l], layers[l].wo = m->wo[l], layers[l].wgu = m->wgu[l], layers[l].wdown = m->wdown[l];
    layers[l].attn_norm = m->attn_norm[l], layers[l].ffn_norm = m->ffn_norm[l];
  }
  memset(&a, 0, sizeof(a));
  a.type = c->wtype, a.batch = s->batch, a.n_layer = c->n_layer, a.eps = c->eps;
  a.etype = c->etype, a.emb = m->tok_embd, a.vocab = c->vocab, a.n_embd = c->n_embd, a.tok_in = s->tok_in;
  a.n_qkv = m->n_qkv, a.k_o = m->k_o, a.ffl = m->ffl;
  a.h = m->hl, a.hk = m->hkl, a.hd = c->head_dim, a.pos = s->dpos;
  a.cap = s->max_ctx, a.seq_stride = s->seq_stride, a.layer_stride = s->layer_stride;
  a.kc = s->kc, a.vc = s->vc, a.cos_t = s->cos_t, a.sin_t = s->sin_t;
  a.out_norm = m->output_norm, a.x = s->x, a.xq_out = s->xq_e;
  a.rank = m->rank, a.nranks = m->tp;
  if (m->tp > 1) st = b200_tp_land(s->tp, (uint64_t)s->batch * c->n_embd, s->land); /* collective */
  for (uint32_t r = 0; m->tp > 1 && r < m->tp; r++) a.land[r] = s->land[r];
  if (!st) st = b200_decode_plan_create(m->ctx, &a, layers, &s->plan);
  free(layers);
  return st;
}

static pai_status_t enqueue_step(pai_b200_session_t *s) {
  pai_b200_model_t *m = s->m;
  const pai_b200_model_cfg_t *c = &m->cfg;
  pai_b200_ctx_t *ctx = m->ctx;
  const uint32_t B = s->batch, E = c->n_embd, hd = c->head_dim;
  pai_status_t st;
  if (s->plan) {
    /* the layers in one persistent launch, then the lm head, the greedy
     * pick and the token feedback as separate launches; under tensor
     * parallelism the pick merges the ranks' pairs over peer memory and
     * feeds the token back itself (no collective library call) */
    st = b200_decode_launch(ctx, s->plan);
    b200_ctx_set_pdl(ctx, 1);
    if (!st) st = b200_launch_gemv(ctx, c->etype, B, m->vl, E, m->output, &s->xq_e, NULL, s->logits, B200_EPI_STORE, NULL);
    if (m->tp == 1) {
      if (!st) st = b200_launch_argmax(ctx, B, m->vl, s->logits, s->tok_out);
      if (!st) st = b200_launch_step_tail(ctx, B, s->tok_out, s->tok_in, s->dpos);
    } else if (!st) {
      st = b200_launch_argmax_peer(ctx, B, m->vl, m->v0, s->logits, s->land, (uint64_t)B * E, m->rank, m->tp,
                                   s->tok_out, s->tok_in, s->dpos);
    }
    b200_ctx_set_pdl(ctx, 0);
    return st;
  }
  b200_ctx_set_pdl(ctx, 1); /* every kernel of the step waits for its predecessor's writes */
  st = b200_launch_embed(ctx, c->etype, B, c->vocab, E, m->tok_embd, s->tok_in, s->x);
  for (uint32_t l = 0; !st && l < c->n_layer; l++) {
    uint16_t *kc = s->kc + (uint64_t)l * s->layer_stride, *vc = s->vc + (uint64_t)l * s->layer_stride;
    st = norm_gemv(s, c->wtype, m->n_qkv, m->wqkv[l], m->attn_norm[l], s->qkv, B200_EPI_STORE, NULL);
    if (!st)
      st = b200_launch_attn_step(ctx, B, m->hl, m->hkl, hd, s->dpos, s->max_ctx, s->max_ctx, s->seq_stride, s->qkv,
                                 s->cos_t, s->sin_t, kc, vc, s->att, &s->xq_o);
    if (m->tp == 1) {
      if (!st)
        st = b200_launch_gemv(ctx, c->wtype, B, E, m->k_o, m->wo[l], &s->xq_o, s->x, s->x, B200_EPI_RESIDUAL, NULL);
    } else {
      /* partial o output into exchange slot 0, then x += sum over ranks */
      if (!st)
        st = b200_launch_gemv(ctx, c->wtype, B, E, m->k_o, m->wo[l], &s->xq_o, NULL, b200_tp_slot(s->tp, 0),
                              B200_EPI_STORE, NULL);
      if (!st) st = b200_tp_allreduce_add(s->tp, ctx, 0, s->x, (uint64_t)B * E);
    }
    if (!st) st = norm_gemv(s, c->wtype, 2ull * m->ffl, m->wgu[l], m->ffn_norm[l], s->h, B200_EPI_SILU_GLU, &s->xq_h);
    if (m->tp == 1) {
      if (!st)
        st = b200_launch_gemv(ctx, c->wtype, B, E, m->ffl, m->wdown[l], &s->xq_h, s->x, s->x, B200_EPI_RESIDUAL, NULL);
    } else {
      if (!st)
        st = b200_launch_gemv(ctx, c->wtype, B, E, m->ffl, m->wdown[l], &s->xq_h, NULL, b200_tp_slot(s->tp, 1),
                              B200_EPI_STORE, NULL);
      if (!st) st = b200_tp_allreduce_add(s->tp, ctx, 1, s->x, (uint64_t)B * E);
    }
  }
  if (!st) st = norm_gemv(s, c->etype, m->vl, m->output, m->output_norm, s->logits, B200_EPI_STORE, NULL);
  if (!st) {
    st = m->tp == 1 ? b200_launch_argmax(ctx, B, m->vl, s->logits, s->tok_out)
                    : b200_tp_argmax(s->tp, ctx, B, m->vl, m->v0, s->logits, s->tok_out);
  }
  if (!st) st = b200_launch_step_tail(ctx, B, s->tok_out, s->tok_in, s->dpos);
  b200_ctx_set_pdl(ctx, 0);
  return st;
}

#define SALLOC(ptr, bytes)                                   \
  do {                                                       \
    if (!st) st = pai_b200_alloc(ctx, (bytes), (void **)&(ptr)); \
  } while (0)

pai_status_t pai_b200_model_set_tp(pai_b200_model_t *m, pai_b200_tp_t *tp) {
  if (!m) return b200_fail(PAI_ERR_INVALID_ARG, "model_set_tp: NULL model");
  if (tp && (pai_b200_tp_size(tp) != m->tp || pai_b200_tp_rank(tp) != m->rank))
    return b200_fail(PAI_ERR_MISMATCH, "model_set_tp: communicator rank %u of %u, model rank %u of %u",
                     pai_b200_tp_rank(tp), pai_b200_tp_size(tp), m->rank, m->tp);
  m->tp_comm = tp;
  return PAI_OK;
}

pai_status_t pai_b200_session_create(pai_b200_model_t *m, uint32_t batch, uint32_t max_ctx,
                                     pai_b200_session_t **out) {
  pai_b200_session_t *s;
  pai_b200_ctx_t *ctx;
  const pai_b200_model_cfg_t *c;
  pai_status_t st = PAI_OK;
  uint64_t kv;
  float *tab_c = NULL, *tab_s = NULL;
  if (!m || !out) return b200_fail(PAI_ERR_INVALID_ARG, "session_create: NULL");
  *out = NULL;
  if (batch != 1 && batch != 2 && batch != 4 && batch != 8)
    return b200_fail(PAI_ERR_UNSUPPORTED, "session_create: batch %u (1, 2, 4 or 8)", batch);
  if (max_ctx == 0) return b200_fail(PAI_ERR_INVALID_ARG, "session_create: max_ctx 0");
  if (max_ctx > 0x7FFFFFFFu - PAI_B200_KV_BLOCK_TOKENS)
    return b200_fail(PAI_ERR_UNSUPPORTED, "session_create: max_ctx %u", max_ctx);
  /* whole cache blocks (PAI_KV_BLOCK_TOKENS positions, cache/kv_cache.h:27) */
  max_ctx = (max_ctx + PAI_B200_KV_BLOCK_TOKENS - 1) / PAI_B200_KV_BLOCK_TOKENS * PAI_B200_KV_BLOCK_TOKENS;
  if (m->tp > 1 && !m->tp_comm) return b200_fail(PAI_ERR_INIT, "session_create: tensor-parallel model without a communicator");
  if (m->tp_comm && b200_tp_failed(m->tp_comm))
    return b200_fail(PAI_ERR_INIT, "session_create: the communicator's exchange timed out earlier; make a new one");
  ctx = m->ctx;
  c = &m->cfg;
  s = (pai_b200_session_t *)calloc(1, sizeof(*s));
  if (!s) return b200_fail(PAI_ERR_NOMEM, "session_create: host allocation");
  s->m = m;
  s->tp = m->tp_comm;
  if (s->tp) st = b200_tp_reserve(s->tp, (uint64_t)batch * c->n_embd); /* collective */
  s->batch = batch;
  s->max_ctx = max_ctx;
  s->seq_stride = (uint64_t)m->hkl * max_ctx * c->head_dim;
  s->layer_stride = s->seq_stride * batch;
  kv = s->layer_stride * c->n_layer * 2;
  SALLOC(s->tok_in, 64);
  SALLOC(s->tok_out, 64);
  SALLOC(s->dpos, 64);
  SALLOC(s->x, (uint64_t)batch * c->n_embd * 4);
  SALLOC(s->ox, (uint64_t)batch * c->n_embd * 4);
  SALLOC(s->qkv, (uint64_t)batch * m->n_qkv * 4);
  SALLOC(s->att, (uint64_t)batch * m->k_o * 4);
  {
    const uint64_t be = b200_xq_bytes(batch, c->n_embd), bo = b200_xq_bytes(batch, m->k_o);
    const uint64_t bh = b200_xq_bytes(batch, m->ffl);
    SALLOC(s->xq_buf, be + bo + bh);
    if (!st) st = pai_b200_memset(ctx, s->xq_buf, 0, be + bo + bh);
    if (!st) {
      s->xq_e = b200_xq_view(s->xq_buf, batch, c->n_embd);
      s->xq_o = b200_xq_view((uint8_t *)s->xq_buf + be, batch, m->k_o);
      s->xq_h = b200_xq_view((uint8_t *)s->xq_buf + be + bo, batch, m->ffl);
    }
  }
  SALLOC(s->h, (uint64_t)batch * m->ffl * 4);
  SALLOC(s->logits, (uint64_t)batch * m->vl * 4);
  SALLOC(s->cos_t, (uint64_t)max_ctx * c->head_dim / 2 * 4);
  SALLOC(s->sin_t, (uint64_t)max_ctx * c->head_dim / 2 * 4);
  SALLOC(s->kc, kv * 2); /* kv counts fp16 elements (K and V) */
  if (!st) s->vc = s->kc + s->layer_stride * c->n_layer;
  if (!st) st = pai_b200_host_alloc(ctx, 64, (void **)&s->htok);
  if (!st) st = pai_b200_memset(ctx, s->kc, 0, kv * 2);
  if (!st) st = pai_b200_memset(ctx, s->tok_in, 0, 64);
  if (!st) st = pai_b200_memset(ctx, s->dpos, 0, 64);
  if (!st) {
    tab_c = (float *)malloc((uint64_t)max_ctx * c->head_dim / 2 * 4);
    tab_s = (float *)malloc((uint64_t)max_ctx * c->head_dim / 2 * 4);
    if (!tab_c || !tab_s) st = b200_fail(PAI_ERR_NOMEM, "session_create: host tables");
  }
  if (!st) st = pai_b200_rope_cossin_f32(max_ctx, c->head_dim / 2, c->rope_theta, tab_c, tab_s);
  if (!st) st = pai_b200_memcpy_h2d(ctx, s->cos_t, tab_c, (uint64_t)max_ctx * c->head_dim / 2 * 4);
  if (!st) st = pai_b200_memcpy_h2d(ctx, s->sin_t, tab_s, (uint64_t)max_ctx * c->head_dim / 2 * 4);
  if (!st) st = pai_b200_sync(ctx);
  free(tab_c);
  free(tab_s);
  /* Prefill layer matrices run on the tensor-core GEMM (bf16 tiles) unless
   * PAI_B200_PREFILL_GEMM=0, which keeps the batched GEMV's per-row
   * arithmetic (the decode step's). */
  {
    const char *e = getenv("PAI_B200_PREFILL_GEMM");
    s->pf_gemm = !(e && e[0] == '0');
  }
  /* The layers of a step run as one persistent kernel unless
   * PAI_B200_PERSISTENT=0 (every rank of a tensor-parallel group must make
   * the same choice); with it, and for shapes the kernel does not take, one
   * launch per op. */
  if (!st) {
    const char *e = getenv("PAI_B200_PERSISTENT");
    if (!(e && e[0] == '0')) {
      st = make_plan(s);
      if (st == PAI_ERR_UNSUPPORTED) st = PAI_OK;
    }
  }
  /* One eager step sizes the shared scratch and sets kernel attributes,
   * then the step is captured once as a CUDA graph. The eager step wrote
   * only position 0 of the cache, which the first real step overwrites. */
  if (!st) st = enqueue_step(s);
  if (!st) st = pai_b200_sync(ctx);
  if (!st) st = pai_b200_memset(ctx, s->dpos, 0, 64);
  if (!st) st = pai_b200_memset(ctx, s->tok_in, 0, 64);
  if (!st) st = b200_graph_begin(ctx);
  if (!st) {
    pai_status_t st2 = enqueue_step(s);
    st = b200_graph_end(ctx, &s->graph, &s->graph_kernels);
    if (st2) st = st2;
  }
  if (!st) st = pai_b200_sync(ctx);
  if (st) {
    pai_b200_session_destroy(s);
    return st;
  }
  *out = s;
  return PAI_OK;
}

pai_status_t pai_b200_session_destroy(pai_b200_session_t *s) {
  pai_b200_ctx_t *ctx;
  if (!s) return PAI_OK;
  ctx = s->m->ctx;
  pai_b200_sync(ctx);
  b200_graph_destroy(s->graph);
  b200_decode_plan_destroy(s->plan);
  pai_b200_free(ctx, s->tok_in);
  pai_b200_free(ctx, s->tok_out);
  pai_b200_free(ctx, s->dpos);
  pai_b200_free(ctx, s->x);
  pai_b200_free(ctx, s->ox);
  pai_b200_free(ctx, s->qkv);
  pai_b200_free(ctx, s->att);
  pai_b200_free(ctx, s->xq_buf);
  pai_b200_free(ctx, s->h);
  pai_b200_free(ctx, s->logits);
  pai_b200_free(ctx, s->cos_t);
  pai_b200_free(ctx, s->sin_t);
  pai_b200_free(ctx, s->kc);
  pai_b200_host_free(ctx, s->htok);
  pai_b200_free(ctx, s->pf_x);
  pai_b200_free(ctx, s->pf_xn);
  pai_b200_free(ctx, s->pf_qkv);
  pai_b200_free(ctx, s->pf_att);
  pai_b200_free(ctx, s->pf_gu);
  pai_b200_free(ctx, s->pf_h);
  pai_b200_free(ctx, s->pf_tmp);
  pai_b200_free(ctx, s->pf_tok);
  pai_b200_free(ctx, s->pf_xq_buf);
  pai_b200_host_free(ctx, s->pf_htok);
  free(s);
  return PAI_OK;
}

uint32_t pai_b200_session_pos(const pai_b200_session_t *s) { return s ? s->pos : 0; }

/* Position accounting of pai_kv_cache_reserve (cache/kv_cache.c:125-152):
 * tokens == 0 is an invalid argument, positions beyond the capacity are
 * PAI_ERR_NOMEM; on success the first new position is returned and the
 * count advances. Host bookkeeping only: the caller moves the device
 * position (the decode graph advances it itself). */
static pai_status_t kv_take(pai_b200_session_t *s, uint32_t tokens, uint32_t *first) {
  if (tokens == 0) return b200_fail(PAI_ERR_INVALID_ARG, "kv_reserve: 0 tokens");
  if ((uint64_t)s->pos + tokens > s->max_ctx)
    return b200_fail(PAI_ERR_NOMEM, "kv_reserve: %u positions from %u exceed the %u-position cache", tokens, s->pos,
                     s->max_ctx);
  if (first) *first = s->pos;
  s->pos += tokens;
  s->kv_reservations++;
  return PAI_OK;
}

static pai_status_t set_device_pos(pai_b200_session_t *s) {
  int32_t p = (int32_t)s->pos;
  pai_status_t st = pai_b200_sync(s->m->ctx); /* the staging word may still feed an earlier copy */
  if (st) return st;
  memcpy(s->htok, &p, 4);
  st = pai_b200_memcpy_h2d(s->m->ctx, s->dpos, s->htok, 4);
  return st ? st : pai_b200_sync(s->m->ctx);
}

/* A wait that ran out inside a step leaves the tensor-parallel exchange
 * buffers out of step between ranks (a rank that timed out did not advance
 * its call counters; its peers may have): the session and its communicator
 * refuse further work until both are made again. On one GPU the session is
 * marked the same way, since the step's state is unknown. */
static pai_status_t seen(pai_b200_session_t *s, pai_status_t st) {
  if (st == PAI_ERR_TIMEOUT) {
    s->failed = 1;
    if (s->tp) b200_tp_mark_failed(s->tp);
  }
  return st;
}

static pai_status_t usable(const pai_b200_session_t *s) {
  if (s->failed)
    return b200_fail(PAI_ERR_INIT, "session: a device wait ran out in an earlier step; destroy the session%s and "
                                   "create it again", s->tp ? " and its tensor-parallel communicator" : "");
  return PAI_OK;
}

pai_status_t pai_b200_session_reset(pai_b200_session_t *s) {
  pai_status_t st;
  if (!s) return b200_fail(PAI_ERR_INVALID_ARG, "session_reset: NULL");
  st = pai_b200_memset(s->m->ctx, s->dpos, 0, 4);
  if (!st) {
    s->pos = 0;
    s->kv_reservations = 0;
  }
  return st;
}

pai_status_t pai_b200_session_kv_info(const pai_b200_session_t *s, pai_b200_kv_info_t *out) {
  if (!s || !out) return b200_fail(PAI_ERR_INVALID_ARG, "session_kv_info: NULL");
  memset(out, 0, sizeof(*out));
  out->capacity_tokens = s->max_ctx;
  out->positions = s->pos;
  out->block_tokens = PAI_B200_KV_BLOCK_TOKENS;
  out->n_layer = s->m->cfg.n_layer;
  out->batch = s->batch;
  out->kv_heads = s->m->hkl;
  out->head_dim = s->m->cfg.head_dim;
  out->layer_stride = s->layer_stride;
  out->seq_stride = s->seq_stride;
  out->head_stride = (uint64_t)s->max_ctx * s->m->cfg.head_dim;
  out->stats_blocks = s->kv_reservations;
  out->k = s->kc;
  out->v = s->vc;
  return PAI_OK;
}

pai_status_t pai_b200_session_kv_reserve(pai_b200_session_t *s, uint32_t tokens, uint32_t *out_pos) {
  pai_status_t st;
  if (!s || !out_pos) return b200_fail(PAI_ERR_INVALID_ARG, "session_kv_reserve: NULL");
  st = kv_take(s, tokens, out_pos);
  return st ? st : set_device_pos(s);
}

static pai_status_t check_tokens(const pai_b200_session_t *s, const int32_t *tokens) {
  for (uint32_t b = 0; b < s->batch; b++) {
    if (tokens[b] < 0 || (uint32_t)tokens[b] >= s->m->cfg.vocab)
      return b200_fail(PAI_ERR_INVALID_ARG, "token %d outside vocab %u", tokens[b], s->m->cfg.vocab);
  }
  return PAI_OK;
}

pai_status_t pai_b200_session_set_tokens(pai_b200_session_t *s, const int32_t *tokens) {
  pai_status_t st;
  if (!s || !tokens) return b200_fail(PAI_ERR_INVALID_ARG, "set_tokens: NULL");
  st = check_tokens(s, tokens);
  if (st) return st;
  memcpy(s->htok, tokens, s->batch * 4);
  return pai_b200_memcpy_h2d(s->m->ctx, s->tok_in, s->htok, s->batch * 4);
}

pai_status_t pai_b200_session_get_tokens(pai_b200_session_t *s, int32_t *tokens) {
  pai_status_t st;
  if (!s || !tokens) return b200_fail(PAI_ERR_INVALID_ARG, "get_tokens: NULL");
  st = pai_b200_memcpy_d2h(s->m->ctx, s->htok + s->batch, s->tok_out, s->batch * 4);
  if (!st) st = seen(s, pai_b200_sync(s->m->ctx));
  if (!st) memcpy(tokens, s->htok + s->batch, s->batch * 4);
  return st;
}

pai_status_t pai_b200_session_run(pai_b200_session_t *s, uint32_t steps) {
  pai_status_t st = PAI_OK;
  if (!s) return b200_fail(PAI_ERR_INVALID_ARG, "session_run: NULL");
  st = usable(s);
  if (st) return st;
  if ((uint64_t)s->pos + steps > s->max_ctx)
    return b200_fail(PAI_ERR_NOMEM, "session_run: %u steps from position %u exceed the %u-position cache", steps,
                     s->pos, s->max_ctx);
  /* one reservation of one position per step, as a stepped decode makes */
  for (uint32_t i = 0; i < steps && !st; i++) {
    st = b200_graph_launch(s->m->ctx, s->graph, s->graph_kernels);
    if (!st) st = kv_take(s, 1, NULL);
  }
  return st;
}

pai_status_t pai_b200_session_step(pai_b200_session_t *s, const int32_t *tokens, int32_t *next, float *logits) {
  pai_status_t st;
  if (!s || !tokens || !next) return b200_fail(PAI_ERR_INVALID_ARG, "session_step: NULL");
  st = pai_b200_session_set_tokens(s, tokens);
  if (!st) st = pai_b200_session_run(s, 1);
  if (!st && logits) {
    if (s->m->tp > 1) return b200_fail(PAI_ERR_UNSUPPORTED, "session_step: logits are sharded under tensor parallelism");
    st = pai_b200_memcpy_d2h(s->m->ctx, logits, s->logits, (uint64_t)s->batch * s->m->vl * 4);
  }
  if (!st) st = pai_b200_session_get_tokens(s, next);
  return st;
}

const float *pai_b200_session_hidden(const pai_b200_session_t *s) { return s ? s->x : NULL; }

uint32_t pai_b200_session_step_kernels(const pai_b200_session_t *s) { return s ? s->graph_kernels : 0; }

pai_status_t pai_b200_session_run_layers(pai_b200_session_t *s, uint32_t reps) {
  pai_status_t st;
  if (!s) return b200_fail(PAI_ERR_INVALID_ARG, "session_run_layers: NULL");
  if (!s->plan) return b200_fail(PAI_ERR_UNSUPPORTED, "session_run_layers: the session runs one launch per op");
  st = usable(s);
  for (uint32_t i = 0; i < reps && !st; i++) st = b200_decode_launch(s->m->ctx, s->plan);
  return st;
}

/* ---- prompt prefill ------------------------------------------------------------------ */

/* Rows of prompt positions per pass: the prefill scratch holds this many
 * rows (all sequences); a longer prompt runs in several passes, each
 * attending over the cache the earlier passes filled. */
#define PF_MAX_ROWS 2048u

static pai_status_t prefill_alloc(pai_b200_session_t *s) {
  pai_b200_model_t *m = s->m;
  pai_b200_ctx_t *ctx = m->ctx;
  const uint64_t R = PF_MAX_ROWS, E = m->cfg.n_embd;
  const uint64_t kmax = E > m->k_o ? (E > m->ffl ? E : m->ffl) : (m->k_o > m->ffl ? m->k_o : m->ffl);
  pai_status_t st = PAI_OK;
  if (s->pf_x) return PAI_OK;
  SALLOC(s->pf_x, R * E * 4);
  SALLOC(s->pf_xn, R * E * 4);
  SALLOC(s->pf_qkv, R * m->n_qkv * 4);
  SALLOC(s->pf_att, R * m->k_o * 4);
  SALLOC(s->pf_gu, R * 2 * m->ffl * 4);
  SALLOC(s->pf_h, R * m->ffl * 4);
  SALLOC(s->pf_tmp, R * E * 4);
  SALLOC(s->pf_tok, R * 4);
  SALLOC(s->pf_xq_buf, b200_xq_bytes(8, kmax));
  if (!st) st = pai_b200_host_alloc(ctx, R * 4, (void **)&s->pf_htok);
  if (!st) s->pf_rows = PF_MAX_ROWS;
  return st;
}

/* Y[rows][n] = X[rows][k] . W^T over a packed layer matrix: the tcgen05
 * GEMM (Q4_0, Q8_0, Q4_K), or with PAI_B200_PREFILL_GEMM=0 the GEMV in
 * groups of 8 rows (epi as in the
 * decode step; residual adds Y's old value when epi is B200_EPI_RESIDUAL,
 * SILU_GLU writes n/2 values per row). */
static pai_status_t rows_matmul(pai_b200_session_t *s, uint32_t type, uint32_t rows, uint64_t n, uint64_t k,
                                const void *w, const float *x, float *y, int epi) {
  pai_b200_model_t *m = s->m;
  pai_b200_ctx_t *ctx = m->ctx;
  pai_status_t st = PAI_OK;
  if (epi == B200_EPI_RESIDUAL && m->tp > 1) {
    /* row-parallel under tensor parallelism: this rank's partial rows, the
     * sum over ranks (NCCL all-reduce, the same bits on every rank), then
     * the residual add */
    st = rows_matmul(s, type, rows, n, k, w, x, s->pf_tmp, B200_EPI_STORE);
    if (!st) st = pai_b200_tp_allreduce_f32(s->tp, s->pf_tmp, (uint64_t)rows * n);
    if (!st) st = pai_b200_vecadd_f32(ctx, y, s->pf_tmp, y, (uint64_t)rows * n);
    return st;
  }
  if (s->pf_gemm) {
    float *dst = epi == B200_EPI_STORE ? y : (epi == B200_EPI_RESIDUAL ? s->pf_tmp : s->pf_gu);
    st = pai_b200_gemm_f32(ctx, type, rows, n, k, x, w, dst);
    if (!st && epi == B200_EPI_RESIDUAL) st = pai_b200_vecadd_f32(ctx, y, dst, y, (uint64_t)rows * n);
    if (!st && epi == B200_EPI_SILU_GLU) st = b200_launch_silu_glu_rows(ctx, rows, (uint32_t)(n / 2), dst, y);
    return st;
  }
  const uint64_t ystride = epi == B200_EPI_SILU_GLU ? n / 2 : n;
  for (uint32_t r0 = 0; r0 < rows && !st; r0 += 8) {
    const uint32_t b = rows - r0 < 8 ? rows - r0 : 8;
    b200_xq_t xq = b200_xq_view(s->pf_xq_buf, b, k);
    st = b200_launch_xprep(ctx, b, k, x + (uint64_t)r0 * k, &xq);
    if (!st)
      st = b200_launch_gemv(ctx, type, b, n, k, w, &xq, epi == B200_EPI_RESIDUAL ? y + (uint64_t)r0 * ystride : NULL,
                            y + (uint64_t)r0 * ystride, epi, NULL);
  }
  return st;
}

pai_status_t pai_b200_session_prefill(pai_b200_session_t *s, const int32_t *tokens, uint32_t n, int32_t *next) {
  if (!s || !tokens || !next || n == 0) return b200_fail(PAI_ERR_INVALID_ARG, "session_prefill: NULL or empty");
  pai_b200_model_t *m = s->m;
  pai_b200_ctx_t *ctx = m->ctx;
  const pai_b200_model_cfg_t *c = &m->cfg;
  const uint32_t B = s->batch, E = c->n_embd, hd = c->head_dim;
  if ((uint64_t)s->pos + n > s->max_ctx)
    return b200_fail(PAI_ERR_NOMEM, "session_prefill: %u positions from %u exceed the %u-position cache", n, s->pos,
                     s->max_ctx);
  for (uint64_t i = 0; i < (uint64_t)B * n; i++)
    if (tokens[i] < 0 || (uint32_t)tokens[i] >= c->vocab)
      return b200_fail(PAI_ERR_INVALID_ARG, "session_prefill: token %d outside vocab %u", tokens[i], c->vocab);
  pai_status_t st = usable(s);
  if (!st) st = prefill_alloc(s);
  const uint32_t per_pass = PF_MAX_ROWS / B;
  for (uint32_t done = 0; !st && done < n;) {
    const uint32_t mc = n - done < per_pass ? n - done : per_pass, rows = B * mc, p0 = s->pos;
    for (uint32_t b = 0; b < B; b++)
      memcpy(s->pf_htok + (uint64_t)b * mc, tokens + (uint64_t)b * n + done, (uint64_t)mc * 4);
    st = pai_b200_memcpy_h2d(ctx, s->pf_tok, s->pf_htok, (uint64_t)rows * 4);
    if (!st) st = b200_launch_embed(ctx, c->etype, rows, c->vocab, E, m->tok_embd, s->pf_tok, s->pf_x);
    for (uint32_t l = 0; !st && l < c->n_layer; l++) {
      uint16_t *kc = s->kc + (uint64_t)l * s->layer_stride, *vc = s->vc + (uint64_t)l * s->layer_stride;
      st = b200_launch_rmsnorm_xq(ctx, rows, E, s->pf_x, m->attn_norm[l], c->eps, s->pf_xn, NULL);
      if (!st) st = rows_matmul(s, c->wtype, rows, m->n_qkv, E, m->wqkv[l], s->pf_xn, s->pf_qkv, B200_EPI_STORE);
      if (!st)
        st = b200_launch_prefill_rope_append(ctx, rows, mc, p0, m->hl, m->hkl, hd, s->pf_qkv, s->cos_t, s->sin_t, kc,
                                             vc, s->max_ctx, s->seq_stride);
      if (!st)
        st = b200_launch_attn_prefill(ctx, rows, mc, p0, m->hl, m->hkl, hd, s->pf_qkv, kc, vc, s->max_ctx,
                                      s->seq_stride, s->pf_att);
      if (!st) st = rows_matmul(s, c->wtype, rows, E, m->k_o, m->wo[l], s->pf_att, s->pf_x, B200_EPI_RESIDUAL);
      if (!st) st = b200_launch_rmsnorm_xq(ctx, rows, E, s->pf_x, m->ffn_norm[l], c->eps, s->pf_xn, NULL);
      if (!st)
        st = rows_matmul(s, c->wtype, rows, 2ull * m->ffl, E, m->wgu[l], s->pf_xn, s->pf_h, B200_EPI_SILU_GLU);
      if (!st) st = rows_matmul(s, c->wtype, rows, E, m->ffl, m->wdown[l], s->pf_h, s->pf_x, B200_EPI_RESIDUAL);
    }
    /* the last position of each sequence becomes the decode state */
    for (uint32_t b = 0; !st && b < B; b++)
      st = pai_b200_memcpy_d2d(ctx, s->x + (uint64_t)b * E, s->pf_x + ((uint64_t)b * mc + mc - 1) * E,
                               (uint64_t)E * 4);
    if (!st) st = kv_take(s, mc, NULL);
    if (!st) done += mc;
  }
  /* logits of the last position, greedy token; it is also the next decode
   * step's input, and the device position follows the prompt */
  if (!st) st = norm_gemv(s, c->etype, m->vl, m->output, m->output_norm, s->logits, B200_EPI_STORE, NULL);
  if (!st) {
    st = m->tp == 1 ? b200_launch_argmax(ctx, B, m->vl, s->logits, s->tok_out)
                    : b200_tp_argmax(s->tp, ctx, B, m->vl, m->v0, s->logits, s->tok_out);
  }
  if (!st) st = pai_b200_memcpy_d2d(ctx, s->tok_in, s->tok_out, (uint64_t)B * 4);
  if (!st) {
    int32_t p = (int32_t)s->pos;
    memcpy(s->htok, &p, 4);
    st = pai_b200_memcpy_h2d(ctx, s->dpos, s->htok, 4);
    if (!st) st = seen(s, pai_b200_sync(ctx));
  }
  if (!st) st = pai_b200_session_get_tokens(s, next);
  return seen(s, st);
}
