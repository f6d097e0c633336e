/*
 * GGUF model import: a LLaMA-family GGUF file's ggml blocks become the
 * model's packed device weights directly, with no f32 dequantisation at
 * import and no file-size cap.
 *
 * The reference's importer (adapters/llama/llama.c:262-470) reads the file
 * into memory (at most 2 GiB, llama.c:279), parses it with
 * adapters/llama/gguf.c, takes the architecture, the hyperparameters and
 * the tensors below, dequantises every tensor to f32 and transposes the
 * matrices. This file maps the file instead (mmap), parses the same
 * container layout with the same validation rules, takes the same keys
 * and tensors, and hands each tensor's blocks, as stored, to
 * pai_b200_model_set_tensor, which packs this rank's shard on the device.
 *
 * Container layout read here (as adapters/llama/gguf.c reads it, for
 * versions 1-3): "GGUF", u32 version, u64 tensor count, u64 metadata count,
 * the metadata entries (u64-length key, u32 value type, value), the tensor
 * records (u64-length name, u32 dims, u64 extents, u32 ggml type, u64
 * offset), then the tensor data from the next multiple of
 * general.alignment (default 32).
 *
 * Keys (prefix = general.architecture, "llama" or "mistral"):
 *   {a}.block_count, .embedding_length, .feed_forward_length,
 *   .attention.head_count, .context_length             required
 *   {a}.attention.head_count_kv   default head_count
 *   {a}.rope.dimension_count      default head_dim
 *   {a}.rope.freq_base            default 10000
 *   tokenizer.ggml.tokens         array; its length is the vocabulary
 * Tensors: token_embd.weight, blk.L.{attn_norm, attn_q, attn_k, attn_v,
 * attn_output, ffn_norm, ffn_gate, ffn_up, ffn_down}.weight,
 * output_norm.weight, output.weight (absent: the lm head is the
 * embedding, llama.c:445-470). The RMSNorm epsilon is the executor's
 * default 1e-5, as in the reference's graph (no epsilon attribute,
 * llama.c:674, 756, 884).
 *
 * Status codes follow the reference: PAI_ERR_IO (file), PAI_ERR_PROTOCOL
 * (malformed container, tensor bytes outside the file), PAI_ERR_UNSUPPORTED
 * (version, architecture, more than 1024 tensors), PAI_ERR_MISMATCH
 * (absent key or tensor, inconsistent shape). Shapes the backend does not
 * run (head_dim other than 128, partial rotary dims, block types other than
 * Q4_0/Q8_0/Q4_K, mixed matrix types) are PAI_ERR_UNSUPPORTED.
 */
#define _GNU_SOURCE
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../b200_internal.h"

enum { GG_MAX_TENSORS = 1024, GG_NAME = 128 };
#define GG_MAX_EXTENT (1ull << 26)
enum { GV_U8 = 0, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STR, GV_ARR, GV_U64, GV_I64, GV_F64 };

typedef struct {
  const uint8_t *key;
  uint64_t key_len;
  uint32_t type;
  const uint8_t *val; /* the value's first byte */
} gg_kv;

typedef struct {
  char name[GG_NAME];
  uint32_t n_dims, type;
  uint64_t ne[4];
  uint64_t offset;
} gg_tensor;

typedef struct {
  const uint8_t *base;
  uint64_t size;
  uint32_t version;
  uint64_t n_kv, n_t;
  gg_kv *kv;
  gg_tensor *t;
  uint64_t data_off; /* aligned start of the tensor data */
} gg_file;

/* ---- little-endian reads with an explicit remaining-bytes check ---------------- */

static int take(const uint8_t **p, const uint8_t *end, uint64_t n) {
  if ((uint64_t)(end - *p) < n) return 0;
  *p += n;
  return 1;
}

static uint64_t le(const uint8_t *p, unsigned n) {
  uint64_t v = 0;
  for (unsigned i = 0; i < n; i++) v |= (uint64_t)p[i] << (8 * i);
  return v;
}

/* Width of a scalar value type, 0 for string/array/unknown. */
static unsigned scalar_width(uint32_t type) {
  switch (type) {
    case GV_U8: case GV_I8: case GV_BOOL: return 1;
    case GV_U16: case GV_I16: return 2;
    case GV_U32: case GV_I32: case GV_F32: return 4;
    case GV_U64: case GV_I64: case GV_F64: return 8;
    default: return 0;
  }
}

/* Advance over one value of `type`; 0 when it runs past the end or the
 * type is unknown. */
static int skip_value(const uint8_t **p, const uint8_t *end, uint32_t type) {
  unsigned w = scalar_width(type);
  if (w) return take(p, end, w);
  if (type == GV_STR) {
    const uint8_t *q = *p;
    if (!take(&q, end, 8)) return 0;
    if (!take(&q, end, le(*p, 8))) return 0;
    *p = q;
    return 1;
  }
  if (type == GV_ARR) {
    const uint8_t *q = *p;
    if (!take(&q, end, 12)) return 0;
    const uint32_t et = (uint32_t)le(*p, 4);
    const uint64_t count = le(*p + 4, 8);
    const unsigned ew = scalar_width(et);
    if (ew) {  /* fixed-width elements: one bounds check */
      if (count > (uint64_t)(end - q) / ew) return 0;
      q += count * ew;
    } else {
      for (uint64_t i = 0; i < count; i++)
        if (!skip_value(&q, end, et)) return 0;
    }
    *p = q;
    return 1;
  }
  return 0;
}

static void gg_close(gg_file *f) {
  free(f->kv);
  free(f->t);
  if (f->base) munmap((void *)f->base, f->size);
  memset(f, 0, sizeof(*f));
}

static const gg_kv *find_kv(const gg_file *f, const char *key) {
  const uint64_t n = strlen(key);
  for (uint64_t i = 0; i < f->n_kv; i++)
    if (f->kv[i].key_len == n && memcmp(f->kv[i].key, key, n) == 0) return &f->kv[i];
  return NULL;
}

/* Integer value of a scalar entry, any width (the reference's u32 getter
 * also takes the low bits of wider or float-typed entries). */
static pai_status_t kv_u32(const gg_file *f, const char *key, uint32_t *out) {
  const gg_kv *e = find_kv(f, key);
  if (!e || !scalar_width(e->type)) return PAI_ERR_MISMATCH;
  *out = (uint32_t)le(e->val, scalar_width(e->type));
  return PAI_OK;
}

static pai_status_t kv_f32(const gg_file *f, const char *key, float *out) {
  const gg_kv *e = find_kv(f, key);
  if (!e) return PAI_ERR_MISMATCH;
  if (e->type == GV_F32) {
    uint32_t b = (uint32_t)le(e->val, 4);
    memcpy(out, &b, 4);
    return PAI_OK;
  }
  if (e->type == GV_F64) {
    uint64_t b = le(e->val, 8);
    double d;
    memcpy(&d, &b, 8);
    *out = (float)d;
    return PAI_OK;
  }
  uint32_t u;
  pai_status_t st = kv_u32(f, key, &u);
  if (!st) *out = (float)u;
  return st;
}

static pai_status_t kv_str(const gg_file *f, const char *key, char *out, uint64_t cap) {
  const gg_kv *e = find_kv(f, key);
  if (!e || e->type != GV_STR) return PAI_ERR_MISMATCH;
  const uint64_t n = le(e->val, 8);
  if (n >= cap) return PAI_ERR_NOMEM;
  memcpy(out, e->val + 8, n);
  out[n] = 0;
  return PAI_OK;
}

static pai_status_t kv_array_len(const gg_file *f, const char *key, uint64_t *n) {
  const gg_kv *e = find_kv(f, key);
  if (!e || e->type != GV_ARR) return PAI_ERR_MISMATCH;
  *n = le(e->val + 4, 8);
  return PAI_OK;
}

static const gg_tensor *find_tensor(const gg_file *f, const char *name) {
  for (uint64_t i = 0; i < f->n_t; i++)
    if (strcmp(f->t[i].name, name) == 0) return &f->t[i];
  return NULL;
}

static pai_status_t gg_open(const char *path, gg_file *f) {
  memset(f, 0, sizeof(*f));
  int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return b200_fail(PAI_ERR_IO, "gguf: cannot open %s", path);
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size < 0) {
    close(fd);
    return b200_fail(PAI_ERR_IO, "gguf: cannot stat %s", path);
  }
  f->size = (uint64_t)sb.st_size;
  if (f->size < 24) {
    close(fd);
    return b200_fail(PAI_ERR_PROTOCOL, "gguf: %llu bytes is shorter than a header", (unsigned long long)f->size);
  }
  void *map = mmap(NULL, f->size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) return b200_fail(PAI_ERR_IO, "gguf: cannot map %s", path);
  f->base = (const uint8_t *)map;
  const uint8_t *p = f->base, *end = f->base + f->size;
  pai_status_t st = PAI_ERR_PROTOCOL;
  if (le(p, 4) != 0x46554747u) {
    b200_fail(st, "gguf: bad magic");
    goto fail;
  }
  f->version = (uint32_t)le(p + 4, 4);
  f->n_t = le(p + 8, 8);
  f->n_kv = le(p + 16, 8);
  p += 24;
  if (f->version < 1 || f->version > 3) {
    st = b200_fail(PAI_ERR_UNSUPPORTED, "gguf: version %u", f->version);
    goto fail;
  }
  if (f->n_t > GG_MAX_TENSORS) {
    st = b200_fail(PAI_ERR_UNSUPPORTED, "gguf: %llu tensors (at most %u)", (unsigned long long)f->n_t,
                   GG_MAX_TENSORS);
    goto fail;
  }
  /* each entry needs at least 12 bytes: the count cannot exceed that */
  if (f->n_kv > f->size / 12) {
    b200_fail(st, "gguf: metadata count %llu", (unsigned long long)f->n_kv);
    goto fail;
  }
  f->kv = (gg_kv *)calloc(f->n_kv ? f->n_kv : 1, sizeof(gg_kv));
  f->t = (gg_tensor *)calloc(f->n_t ? f->n_t : 1, sizeof(gg_tensor));
  if (!f->kv || !f->t) {
    st = b200_fail(PAI_ERR_NOMEM, "gguf: tables");
    goto fail;
  }
  for (uint64_t i = 0; i < f->n_kv; i++) {
    gg_kv *e = &f->kv[i];
    const uint8_t *q = p;
    if (!take(&q, end, 8)) goto bad;
    e->key_len = le(p, 8);
    e->key = q;
    if (!take(&q, end, e->key_len) || !take(&q, end, 4)) goto bad;
    e->type = (uint32_t)le(q - 4, 4);
    e->val = q;
    if (!skip_value(&q, end, e->type)) goto bad;
    p = q;
  }
  for (uint64_t i = 0; i < f->n_t; i++) {
    gg_tensor *t = &f->t[i];
    const uint8_t *q = p;
    if (!take(&q, end, 8)) goto bad;
    const uint64_t len = le(p, 8);
    if (len == 0 || len >= GG_NAME || !take(&q, end, len)) goto bad;
    memcpy(t->name, p + 8, len);
    t->name[len] = 0;
    const uint8_t *d = q;
    if (!take(&q, end, 4)) goto bad;
    t->n_dims = (uint32_t)le(d, 4);
    if (t->n_dims < 1 || t->n_dims > 4) goto bad;
    for (uint32_t j = 0; j < t->n_dims; j++) {
      d = q;
      if (!take(&q, end, 8)) goto bad;
      t->ne[j] = le(d, 8);
      if (t->ne[j] > GG_MAX_EXTENT) goto bad;
    }
    for (uint32_t j = t->n_dims; j < 4; j++) t->ne[j] = 1;
    d = q;
    if (!take(&q, end, 12)) goto bad;
    t->type = (uint32_t)le(d, 4);
    t->offset = le(d + 4, 8);
    p = q;
  }
  uint32_t align = 32;
  (void)kv_u32(f, "general.alignment", &align);
  if (align == 0 || (align & (align - 1)) || align > 4096) goto bad;
  f->data_off = ((uint64_t)(p - f->base) + align - 1) / align * align;
  if (f->data_off > f->size) goto bad;
  return PAI_OK;
bad:
  st = b200_fail(PAI_ERR_PROTOCOL, "gguf: malformed header, metadata or tensor table");
fail:
  gg_close(f);
  return st;
}

/* ---- the LLaMA view of a GGUF file ------------------------------------------------ */

static const char *const k_layer_names[9] = {"attn_norm", "attn_q",      "attn_k",   "attn_v",  "attn_output",
                                             "ffn_norm",  "ffn_gate",    "ffn_up",   "ffn_down"};
static const uint32_t k_layer_kinds[9] = {PAI_B200_T_ATTN_NORM, PAI_B200_T_WQ,    PAI_B200_T_WK,
                                          PAI_B200_T_WV,        PAI_B200_T_WO,    PAI_B200_T_FFN_NORM,
                                          PAI_B200_T_WGATE,     PAI_B200_T_WUP,   PAI_B200_T_WDOWN};

/* A tensor's ggml rows x cols (ne[1] x ne[0]) must be exactly as given. */
static pai_status_t want_shape(const gg_tensor *t, uint64_t rows, uint64_t cols) {
  const uint64_t r = t->n_dims >= 2 ? t->ne[1] : 1;
  if (t->ne[0] != cols || r != rows || t->ne[2] != 1 || t->ne[3] != 1)
    return b200_fail(PAI_ERR_MISMATCH, "gguf: %s is %llux%llu, expected %llux%llu", t->name,
                     (unsigned long long)r, (unsigned long long)t->ne[0], (unsigned long long)rows,
                     (unsigned long long)cols);
  return PAI_OK;
}

/* The tensor's bytes must lie inside the file. */
static pai_status_t tensor_bytes(const gg_file *f, const gg_tensor *t, uint64_t *bytes) {
  const uint64_t numel = t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3];
  const uint64_t b = t->type == 0 ? numel * 4 : pai_b200_block_bytes(t->type, numel);
  if (b == 0) return b200_fail(PAI_ERR_UNSUPPORTED, "gguf: %s has ggml type %u", t->name, t->type);
  if (t->offset > f->size - f->data_off || b > f->size - f->data_off - t->offset)
    return b200_fail(PAI_ERR_PROTOCOL, "gguf: %s lies outside the file", t->name);
  *bytes = b;
  return PAI_OK;
}

typedef struct {
  const gg_tensor *embd, *out, *onorm;
  const gg_tensor **layer; /* [n_layer][9] */
} gg_llama;

static pai_status_t llama_view(const gg_file *f, pai_b200_gguf_info_t *info, gg_llama *v) {
  char key[160];
  const char *a = info->architecture;
  uint32_t n_layer, n_embd, n_ff, n_head, n_kv, ctx, n_rot = 0;
  float theta = 10000.0f;
  uint64_t vocab;
  pai_status_t st;
  memset(v, 0, sizeof(*v));
  st = kv_str(f, "general.architecture", info->architecture, sizeof(info->architecture));
  if (st) return b200_fail(st, "gguf: general.architecture missing or too long");
  if (strcmp(a, "llama") != 0 && strcmp(a, "mistral") != 0)
    return b200_fail(PAI_ERR_UNSUPPORTED, "gguf: architecture %s (llama and mistral are read)", a);
#define REQ(suffix, dst)                                                          \
  snprintf(key, sizeof(key), "%s." suffix, a);                                   \
  if ((st = kv_u32(f, key, &dst)) != PAI_OK) return b200_fail(st, "gguf: %s missing", key);
  REQ("block_count", n_layer)
  REQ("embedding_length", n_embd)
  REQ("feed_forward_length", n_ff)
  REQ("attention.head_count", n_head)
#undef REQ
  snprintf(key, sizeof(key), "%s.attention.head_count_kv", a);
  if (kv_u32(f, key, &n_kv) != PAI_OK) n_kv = n_head;
  snprintf(key, sizeof(key), "%s.context_length", a);
  if ((st = kv_u32(f, key, &ctx)) != PAI_OK) return b200_fail(st, "gguf: %s missing", key);
  snprintf(key, sizeof(key), "%s.rope.dimension_count", a);
  (void)kv_u32(f, key, &n_rot);
  snprintf(key, sizeof(key), "%s.rope.freq_base", a);
  (void)kv_f32(f, key, &theta);
  if ((st = kv_array_len(f, "tokenizer.ggml.tokens", &vocab)) != PAI_OK)
    return b200_fail(st, "gguf: tokenizer.ggml.tokens missing");
  if (n_layer == 0 || n_embd == 0 || n_ff == 0 || n_head == 0 || ctx == 0 || vocab == 0 || vocab > 0xFFFFFFFFull ||
      n_embd % n_head || n_kv == 0 || n_head % n_kv)
    return b200_fail(PAI_ERR_MISMATCH, "gguf: inconsistent hyperparameters");
  const uint32_t hd = n_embd / n_head;
  if (n_rot == 0 || n_rot > hd || (n_rot & 1)) n_rot = hd;  /* the reference's fallback, llama.c:372-374 */
  info->version = f->version;
  info->tensor_count = f->n_t;
  info->context_length = ctx;
  info->n_rot = n_rot;
  pai_b200_model_cfg_t *c = &info->cfg;
  c->n_layer = n_layer;
  c->n_embd = n_embd;
  c->n_head = n_head;
  c->n_head_kv = n_kv;
  c->head_dim = hd;
  c->n_ff = n_ff;
  c->vocab = (uint32_t)vocab;
  c->eps = 1e-5f;
  c->rope_theta = theta;

  /* tensors: presence, shapes, byte ranges, types */
  v->layer = (const gg_tensor **)calloc((size_t)n_layer * 9, sizeof(*v->layer));
  if (!v->layer) return b200_fail(PAI_ERR_NOMEM, "gguf: tensor index");
  uint64_t used = 0, b;
  char name[GG_NAME + 32];
  if (!(v->embd = find_tensor(f, "token_embd.weight"))) return b200_fail(PAI_ERR_MISMATCH, "gguf: token_embd.weight missing");
  if (!(v->onorm = find_tensor(f, "output_norm.weight")))
    return b200_fail(PAI_ERR_MISMATCH, "gguf: output_norm.weight missing");
  v->out = find_tensor(f, "output.weight");
  info->tied_output = v->out == NULL;
  if (!v->out) v->out = v->embd;
  const uint32_t kvd = hd * n_kv;
  const uint64_t rows_of[9] = {1, n_embd, kvd, kvd, n_embd, 1, n_ff, n_ff, n_embd};
  const uint64_t cols_of[9] = {n_embd, n_embd, n_embd, n_embd, n_embd, n_embd, n_embd, n_embd, n_ff};
  uint32_t wtype = 0;
  for (uint32_t L = 0; L < n_layer; L++) {
    for (int i = 0; i < 9; i++) {
      snprintf(name, sizeof(name), "blk.%u.%s.weight", L, k_layer_names[i]);
      const gg_tensor *t = find_tensor(f, name);
      if (!t) return b200_fail(PAI_ERR_MISMATCH, "gguf: %s missing", name);
      if ((st = want_shape(t, rows_of[i], cols_of[i])) || (st = tensor_bytes(f, t, &b))) return st;
      const int norm = i == 0 || i == 5;
      if (norm && t->type != 0) return b200_fail(PAI_ERR_UNSUPPORTED, "gguf: %s is not f32", name);
      if (!norm) {
        if (!wtype) wtype = t->type;
        if (t->type != wtype || !b200_type_ok(t->type))
          return b200_fail(PAI_ERR_UNSUPPORTED, "gguf: %s has type %u (matrices must all be one of Q4_0/Q8_0/Q4_K)",
                           name, t->type);
      }
      v->layer[(size_t)L * 9 + i] = t;
      used += b;
    }
  }
  if ((st = want_shape(v->embd, vocab, n_embd)) || (st = tensor_bytes(f, v->embd, &b))) return st;
  used += b;
  if (!info->tied_output) {
    if ((st = want_shape(v->out, vocab, n_embd)) || (st = tensor_bytes(f, v->out, &b))) return st;
    used += b;
  }
  if ((st = want_shape(v->onorm, 1, n_embd)) || (st = tensor_bytes(f, v->onorm, &b))) return st;
  used += b;
  if (v->onorm->type != 0) return b200_fail(PAI_ERR_UNSUPPORTED, "gguf: output_norm.weight is not f32");
  if (v->embd->type != v->out->type || !b200_type_ok(v->embd->type))
    return b200_fail(PAI_ERR_UNSUPPORTED, "gguf: embedding/output types %u/%u (one of Q4_0/Q8_0/Q4_K, the same)",
                     v->embd->type, v->out->type);
  c->wtype = wtype;
  c->etype = v->embd->type;
  info->weight_bytes = used;
  if (hd != 128 || n_rot != hd)
    return b200_fail(PAI_ERR_UNSUPPORTED, "gguf: head_dim %u with %u rotary dims (the backend runs 128, fully rotated)",
                     hd, n_rot);
  return PAI_OK;
}

/* The tensors a LLaMA model uses, in load order (token_embd, output [unless
 * tied], output_norm, then blk.L.* per layer), as named views into the
 * mapped file; b200_gguf_release unmaps it. */
struct b200_gguf_view {
  gg_file f;
};

pai_status_t b200_gguf_llama_tensors(const char *path, pai_b200_gguf_info_t *info, b200_named_tensor_t **out,
                                     uint32_t *count, b200_gguf_view_t **view) {
  gg_llama v;
  b200_gguf_view_t *gv;
  pai_status_t st;
  if (!path || !info || !out || !count || !view) return b200_fail(PAI_ERR_INVALID_ARG, "gguf: NULL");
  *out = NULL;
  *count = 0;
  *view = NULL;
  memset(info, 0, sizeof(*info));
  gv = (b200_gguf_view_t *)calloc(1, sizeof(*gv));
  if (!gv) return b200_fail(PAI_ERR_NOMEM, "gguf: host allocation");
  st = gg_open(path, &gv->f);
  if (st) {
    free(gv);
    return st;
  }
  st = llama_view(&gv->f, info, &v);
  const uint32_t n = 3 + 9 * info->cfg.n_layer;
  b200_named_tensor_t *t = st ? NULL : (b200_named_tensor_t *)calloc(n, sizeof(*t));
  if (!st && !t) st = b200_fail(PAI_ERR_NOMEM, "gguf: host allocation");
  uint32_t k = 0;
  const uint8_t *data = gv->f.base + gv->f.data_off;
  const gg_tensor *top[3] = {v.embd, info->tied_output ? NULL : v.out, v.onorm};
  for (uint32_t i = 0; !st && i < 3 + 9 * info->cfg.n_layer; i++) {
    const gg_tensor *g = i < 3 ? top[i] : v.layer[i - 3];
    if (!g) continue;
    uint64_t b = 0;
    st = tensor_bytes(&gv->f, g, &b);
    if (st) break;
    snprintf(t[k].name, sizeof(t[k].name), "%s", g->name);
    t[k].type = g->type;
    t[k].rows = g->n_dims >= 2 ? g->ne[1] : 1;
    t[k].cols = g->ne[0];
    t[k].data = data + g->offset;
    t[k].bytes = b;
    k++;
  }
  free(v.layer);
  if (st) {
    free(t);
    gg_close(&gv->f);
    free(gv);
    return st;
  }
  *out = t;
  *count = k;
  *view = gv;
  return PAI_OK;
}

void b200_gguf_release(b200_gguf_view_t *view) {
  if (!view) return;
  gg_close(&view->f);
  free(view);
}

pai_status_t pai_b200_gguf_inspect(const char *path, pai_b200_gguf_info_t *info) {
  gg_file f;
  gg_llama v;
  if (!path || !info) return b200_fail(PAI_ERR_INVALID_ARG, "gguf_inspect: NULL");
  memset(info, 0, sizeof(*info));
  pai_status_t st = gg_open(path, &f);
  if (st) return st;
  st = llama_view(&f, info, &v);
  free(v.layer);
  gg_close(&f);
  return st;
}

pai_status_t pai_b200_model_load_gguf(pai_b200_ctx_t *ctx, const char *path, uint32_t tp_rank, uint32_t tp_size,
                                      pai_b200_model_t **out, pai_b200_gguf_info_t *info_out) {
  gg_file f;
  gg_llama v;
  pai_b200_gguf_info_t info;
  pai_b200_model_t *m = NULL;
  if (!ctx || !path || !out) return b200_fail(PAI_ERR_INVALID_ARG, "model_load_gguf: NULL");
  *out = NULL;
  memset(&info, 0, sizeof(info));
  pai_status_t st = gg_open(path, &f);
  if (st) return st;
  st = llama_view(&f, &info, &v);
  if (!st) st = pai_b200_model_create(ctx, &info.cfg, tp_rank, tp_size, &m);
  const uint8_t *data = f.base + f.data_off;
  if (!st) st = pai_b200_model_set_tensor(m, PAI_B200_T_TOK_EMBD, 0, data + v.embd->offset);
  if (!st) st = pai_b200_model_set_tensor(m, PAI_B200_T_OUTPUT, 0, data + v.out->offset);
  if (!st) st = pai_b200_model_set_tensor(m, PAI_B200_T_OUTPUT_NORM, 0, data + v.onorm->offset);
  for (uint32_t L = 0; !st && L < info.cfg.n_layer; L++)
    for (int i = 0; !st && i < 9; i++)
      st = pai_b200_model_set_tensor(m, k_layer_kinds[i], L, data + v.layer[(size_t)L * 9 + i]->offset);
  free(v.layer);
  gg_close(&f);
  if (st) {
    if (m) pai_b200_model_destroy(m);
    return st;
  }
  *out = m;
  if (info_out) *info_out = info;
  return PAI_OK;
}
