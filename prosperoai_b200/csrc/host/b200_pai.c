/*
 * Version-2 .pai containers that hold ggml blocks as stored (the format is
 * described in include/pai_b200.h): a converter from GGUF, a validating
 * reader, and the model loader. The reference's container (pai/pai.c,
 * models/container.c) has u32 offsets and stores only f32 or its own v0
 * grouped formats; this keeps its header, META payload and manifest entry
 * and widens what they can describe.
 *
 * Host code only; the blocks reach the device through
 * pai_b200_model_set_tensor, as for GGUF files.
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

#define PAIC_MAGIC 0x43494150u
#define SEC_META 1u
#define SEC_MANIFEST 2u
#define SEC_WEIGHTS 3u
#define META_BYTES 64u
#define HP_BYTES 52u
#define TABLE_ENTRY 24u
#define MAX_SECTIONS 8u
#define MAX_TENSORS 4096u
#define WEIGHT_ALIGN 256u
#define DTYPE_F32 0u /* pai/dtype.h:14 */
#define DTYPE_U8 8u  /* pai/dtype.h:22 */
#define QREPR_F16 1u /* ir/ir.h:81 */

/* ---- quantization descriptors ------------------------------------------------------- */

pai_status_t pai_b200_ir_quant_ggml(uint32_t t, pai_ir_quant_t *q) {
  if (!q) return b200_fail(PAI_ERR_INVALID_ARG, "ir_quant_ggml: NULL");
  if (!b200_type_ok(t)) return b200_fail(PAI_ERR_UNSUPPORTED, "ir_quant_ggml: ggml type %u", t);
  memset(q, 0, sizeof(*q));
  q->present = 1;
  q->bit_width = t == PAI_B200_Q8_0 ? 8 : 4;
  q->scale_repr = QREPR_F16;
  q->zero_point_repr = t == PAI_B200_Q4_K ? QREPR_F16 : 0; /* Q4_K: fp16 dmin per super-block */
  q->is_signed = t == PAI_B200_Q4_K ? 0 : 1;
  q->block_structure = PAI_IR_QUANT_BLOCK_GGML;
  q->group_size = (uint16_t)b200_blk_elems(t);
  return PAI_OK;
}

pai_status_t pai_b200_ir_quant_ggml_type(const pai_ir_quant_t *q, uint32_t *t) {
  if (!q || !t) return b200_fail(PAI_ERR_INVALID_ARG, "ir_quant_ggml_type: NULL");
  if (!q->present || q->block_structure != PAI_IR_QUANT_BLOCK_GGML)
    return b200_fail(PAI_ERR_UNSUPPORTED, "ir_quant: not a ggml block structure");
  if (q->bit_width == 4 && q->group_size == 32 && q->is_signed) {
    *t = PAI_B200_Q4_0;
  } else if (q->bit_width == 8 && q->group_size == 32 && q->is_signed) {
    *t = PAI_B200_Q8_0;
  } else if (q->bit_width == 4 && q->group_size == 256 && !q->is_signed) {
    *t = PAI_B200_Q4_K;
  } else {
    return b200_fail(PAI_ERR_UNSUPPORTED, "ir_quant: ggml blocks of %u bits x %u not read", q->bit_width,
                     q->group_size);
  }
  return PAI_OK;
}

/* ---- little-endian helpers and CRC-32 (IEEE, as the reference's protocol crc32) ------ */

static void put32(uint8_t *p, uint32_t v) {
  for (int i = 0; i < 4; i++) p[i] = (uint8_t)(v >> (8 * i));
}
static void put64(uint8_t *p, uint64_t v) {
  for (int i = 0; i < 8; i++) p[i] = (uint8_t)(v >> (8 * i));
}
static uint32_t get32(const uint8_t *p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static uint64_t get64(const uint8_t *p) { return (uint64_t)get32(p) | ((uint64_t)get32(p + 4) << 32); }

static uint32_t crc_update(uint32_t c, const uint8_t *p, uint64_t n) {
  static uint32_t table[256];
  static int ready = 0;
  if (!ready) {
    for (uint32_t i = 0; i < 256; i++) {
      uint32_t v = i;
      for (int k = 0; k < 8; k++) v = (v & 1) ? 0xEDB88320u ^ (v >> 1) : v >> 1;
      table[i] = v;
    }
    ready = 1;
  }
  for (uint64_t i = 0; i < n; i++) c = table[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
  return c;
}

/* ---- writer ------------------------------------------------------------------------- */

static uint64_t manifest_entry_bytes(const char *name) { return 2 + strlen(name) + 4 + 4 + 6 * 8 + 8 + 8 + 8; }

static pai_status_t write_all(FILE *fp, const void *p, uint64_t n, const char *path) {
  if (n && fwrite(p, 1, n, fp) != n) return b200_fail(PAI_ERR_IO, "pai: writing %s failed", path);
  return PAI_OK;
}

pai_status_t pai_b200_pai_from_gguf(const char *gguf_path, const char *pai_path) {
  pai_b200_gguf_info_t info;
  b200_named_tensor_t *t = NULL;
  b200_gguf_view_t *view = NULL;
  uint32_t n = 0;
  uint8_t *meta = NULL, *hp = NULL, *man = NULL;
  FILE *fp = NULL;
  if (!gguf_path || !pai_path) return b200_fail(PAI_ERR_INVALID_ARG, "pai_from_gguf: NULL");
  pai_status_t st = b200_gguf_llama_tensors(gguf_path, &info, &t, &n, &view);
  if (st) return st;
  const pai_b200_model_cfg_t *c = &info.cfg;
  /* payloads: META, HPARAMS, MANIFEST, WEIGHTS (offsets within WEIGHTS are
   * WEIGHT_ALIGN-aligned) */
  uint64_t man_bytes = 4, wbytes = 0;
  uint64_t *woff = (uint64_t *)calloc(n ? n : 1, sizeof(uint64_t));
  meta = (uint8_t *)calloc(1, META_BYTES);
  hp = (uint8_t *)calloc(1, HP_BYTES);
  if (!woff || !meta || !hp) st = b200_fail(PAI_ERR_NOMEM, "pai_from_gguf: host allocation");
  for (uint32_t i = 0; !st && i < n; i++) {
    man_bytes += manifest_entry_bytes(t[i].name);
    woff[i] = wbytes;
    wbytes += (t[i].bytes + WEIGHT_ALIGN - 1) / WEIGHT_ALIGN * WEIGHT_ALIGN;
  }
  if (!st) {
    man = (uint8_t *)calloc(1, man_bytes);
    if (!man) st = b200_fail(PAI_ERR_NOMEM, "pai_from_gguf: host allocation");
  }
  if (!st) {
    /* META (pai_pai_meta_t, pai/pai.h:51-63): name, family, context, layers,
     * kv bytes per token per layer (fp16 K and V), vocab */
    memcpy(meta, info.architecture, strnlen(info.architecture, 31)); /* name[32], NUL-terminated */
    put32(meta + 32, 1u);
    put32(meta + 36, info.context_length);
    put32(meta + 40, c->n_layer);
    put32(meta + 44, 2u * c->n_head_kv * c->head_dim * 2u);
    put32(meta + 48, c->vocab);
    const uint32_t hv[13] = {c->n_layer, c->n_embd, c->n_head, c->n_head_kv, c->head_dim, c->n_ff, c->vocab, 0, 0,
                             c->wtype,   c->etype,  info.n_rot, info.tied_output};
    for (int i = 0; i < 13; i++) put32(hp + 4 * i, hv[i]);
    memcpy(hp + 28, &c->eps, 4);
    memcpy(hp + 32, &c->rope_theta, 4);
    put32(man, n);
    uint8_t *p = man + 4;
    for (uint32_t i = 0; i < n; i++) {
      const uint32_t len = (uint32_t)strlen(t[i].name);
      const int blocked = t[i].type != 0;
      pai_ir_quant_t q;
      memset(&q, 0, sizeof(q));
      if (blocked && (st = pai_b200_ir_quant_ggml(t[i].type, &q))) break;
      p[0] = (uint8_t)len, p[1] = (uint8_t)(len >> 8), p += 2;
      memcpy(p, t[i].name, len), p += len;
      put32(p, i + 1), p += 4; /* value id */
      p[0] = (uint8_t)(blocked ? DTYPE_U8 : DTYPE_F32), p[1] = t[i].rows > 1 ? 2 : 1, p[2] = p[3] = 0, p += 4;
      const uint64_t shape[6] = {t[i].rows > 1 ? t[i].rows : t[i].cols, t[i].rows > 1 ? t[i].cols : 0, 0, 0, 0, 0};
      for (int d = 0; d < 6; d++) put64(p, shape[d]), p += 8;
      put64(p, woff[i]), p += 8;
      put64(p, t[i].bytes), p += 8;
      memcpy(p, &q, 8), p += 8;
    }
  }
  if (!st) {
    const uint32_t nsec = 4;
    const uint64_t sizes[4] = {META_BYTES, HP_BYTES, man_bytes, wbytes};
    const uint32_t types[4] = {SEC_META, PAI_B200_PAI_SEC_HPARAMS, SEC_MANIFEST, SEC_WEIGHTS};
    uint8_t head[16 + MAX_SECTIONS * TABLE_ENTRY];
    uint64_t off = 16 + (uint64_t)nsec * TABLE_ENTRY, offs[4];
    memset(head, 0, sizeof(head));
    for (uint32_t i = 0; i < nsec; i++) {
      if (types[i] == SEC_WEIGHTS) off = (off + WEIGHT_ALIGN - 1) / WEIGHT_ALIGN * WEIGHT_ALIGN;
      offs[i] = off;
      off += sizes[i];
    }
    put32(head, PAIC_MAGIC);
    head[4] = (uint8_t)PAI_B200_PAI_VERSION;
    put32(head + 8, nsec);
    for (uint32_t i = 0; i < nsec; i++) {
      uint8_t *e = head + 16 + i * TABLE_ENTRY;
      put32(e, types[i]);
      put32(e + 4, 0);
      put64(e + 8, offs[i]);
      put64(e + 16, sizes[i]);
    }
    uint32_t crc = 0xFFFFFFFFu;
    crc = crc_update(crc, head, 12);
    crc = crc_update(crc, head + 16, (uint64_t)nsec * TABLE_ENTRY);
    crc = crc_update(crc, meta, META_BYTES);
    crc = crc_update(crc, hp, HP_BYTES);
    crc = crc_update(crc, man, man_bytes);
    put32(head + 12, crc ^ 0xFFFFFFFFu);
    fp = fopen(pai_path, "wb");
    if (!fp) st = b200_fail(PAI_ERR_IO, "pai: cannot create %s", pai_path);
    if (!st) st = write_all(fp, head, 16 + (uint64_t)nsec * TABLE_ENTRY, pai_path);
    if (!st) st = write_all(fp, meta, META_BYTES, pai_path);
    if (!st) st = write_all(fp, hp, HP_BYTES, pai_path);
    if (!st) st = write_all(fp, man, man_bytes, pai_path);
    static const uint8_t zeros[WEIGHT_ALIGN];
    const uint64_t at = 16 + (uint64_t)nsec * TABLE_ENTRY + META_BYTES + HP_BYTES + man_bytes;
    if (!st) st = write_all(fp, zeros, offs[3] - at, pai_path);
    for (uint32_t i = 0; !st && i < n; i++) {
      st = write_all(fp, t[i].data, t[i].bytes, pai_path);
      const uint64_t pad = (WEIGHT_ALIGN - t[i].bytes % WEIGHT_ALIGN) % WEIGHT_ALIGN;
      if (!st) st = write_all(fp, zeros, pad, pai_path);
    }
    if (fp && fclose(fp) != 0 && !st) st = b200_fail(PAI_ERR_IO, "pai: writing %s failed", pai_path);
    fp = NULL;
  }
  free(woff);
  free(meta);
  free(hp);
  free(man);
  free(t);
  b200_gguf_release(view);
  return st;
}

/* ---- reader ------------------------------------------------------------------------- */

typedef struct {
  char name[128];
  uint32_t dtype, rank;
  uint64_t shape[6], offset, bytes;
  pai_ir_quant_t q;
} pai_entry;

typedef struct {
  uint8_t *base;
  uint64_t size;
  const uint8_t *weights;
  uint64_t weights_size;
  pai_entry *e;
  uint32_t n;
} pai_file;

static void pai_close(pai_file *f) {
  if (f->base) munmap(f->base, f->size);
  free(f->e);
  memset(f, 0, sizeof(*f));
}

#define BAD(...) (pai_close(f), b200_fail(PAI_ERR_PROTOCOL, __VA_ARGS__))

static pai_status_t pai_open(const char *path, pai_file *f, pai_b200_gguf_info_t *info) {
  struct stat sb;
  memset(f, 0, sizeof(*f));
  int fd = open(path, O_RDONLY);
  if (fd < 0) return b200_fail(PAI_ERR_IO, "pai: cannot open %s", path);
  if (fstat(fd, &sb) != 0 || sb.st_size < 16) {
    close(fd);
    return b200_fail(PAI_ERR_PROTOCOL, "pai: %s is too short", path);
  }
  f->size = (uint64_t)sb.st_size;
  void *m = mmap(NULL, f->size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return b200_fail(PAI_ERR_IO, "pai: cannot map %s", path);
  f->base = (uint8_t *)m;
  const uint8_t *b = f->base;
  if (get32(b) != PAIC_MAGIC) return BAD("pai: bad magic");
  const uint32_t version = (uint32_t)b[4] | ((uint32_t)b[5] << 8);
  if (version != PAI_B200_PAI_VERSION || b[6] || b[7]) {
    pai_close(f);
    return b200_fail(PAI_ERR_UNSUPPORTED, "pai: container version %u (this reader takes %u)", version,
                     PAI_B200_PAI_VERSION);
  }
  const uint32_t nsec = get32(b + 8);
  if (nsec == 0 || nsec > MAX_SECTIONS || 16 + (uint64_t)nsec * TABLE_ENTRY > f->size) return BAD("pai: section table");
  const uint8_t *meta = NULL, *hp = NULL, *man = NULL;
  uint64_t man_n = 0;
  uint32_t crc = crc_update(0xFFFFFFFFu, b, 12);
  crc = crc_update(crc, b + 16, (uint64_t)nsec * TABLE_ENTRY);
  for (uint32_t i = 0; i < nsec; i++) {
    const uint8_t *e = b + 16 + i * TABLE_ENTRY;
    const uint32_t type = get32(e);
    const uint64_t off = get64(e + 8), sz = get64(e + 16);
    if (off > f->size || sz > f->size - off) return BAD("pai: section %u outside the file", type);
    if (type != SEC_WEIGHTS) crc = crc_update(crc, b + off, sz);
    if (type == SEC_META && sz == META_BYTES) meta = b + off;
    if (type == PAI_B200_PAI_SEC_HPARAMS && sz == HP_BYTES) hp = b + off;
    if (type == SEC_MANIFEST) man = b + off, man_n = sz;
    if (type == SEC_WEIGHTS) f->weights = b + off, f->weights_size = sz;
  }
  if ((crc ^ 0xFFFFFFFFu) != get32(b + 12)) return BAD("pai: CRC mismatch");
  if (!meta || !hp || !man || !f->weights) {
    pai_close(f);
    return b200_fail(PAI_ERR_MISMATCH, "pai: META, HPARAMS, MANIFEST or WEIGHTS section missing");
  }
  /* HPARAMS */
  pai_b200_model_cfg_t *c = &info->cfg;
  memset(info, 0, sizeof(*info));
  c->n_layer = get32(hp), c->n_embd = get32(hp + 4), c->n_head = get32(hp + 8), c->n_head_kv = get32(hp + 12);
  c->head_dim = get32(hp + 16), c->n_ff = get32(hp + 20), c->vocab = get32(hp + 24);
  memcpy(&c->eps, hp + 28, 4);
  memcpy(&c->rope_theta, hp + 32, 4);
  c->wtype = get32(hp + 36), c->etype = get32(hp + 40);
  info->n_rot = get32(hp + 44), info->tied_output = get32(hp + 48);
  info->version = version;
  info->context_length = get32(meta + 36);
  memcpy(info->architecture, meta, 31);
  /* MANIFEST */
  if (man_n < 4) return BAD("pai: manifest");
  const uint32_t n = get32(man);
  if (n == 0 || n > MAX_TENSORS) return BAD("pai: %u manifest entries", n);
  f->e = (pai_entry *)calloc(n, sizeof(pai_entry));
  if (!f->e) {
    pai_close(f);
    return b200_fail(PAI_ERR_NOMEM, "pai: host allocation");
  }
  const uint8_t *p = man + 4, *end = man + man_n;
  for (uint32_t i = 0; i < n; i++) {
    if (end - p < 2) return BAD("pai: manifest entry %u", i);
    const uint32_t len = p[0] | ((uint32_t)p[1] << 8);
    if (len == 0 || len >= sizeof(f->e[i].name) || (uint64_t)(end - p) < 2 + (uint64_t)len + 80)
      return BAD("pai: manifest entry %u", i);
    pai_entry *e = &f->e[i];
    memcpy(e->name, p + 2, len);
    p += 2 + len + 4;
    e->dtype = p[0], e->rank = p[1], p += 4;
    for (int d = 0; d < 6; d++) e->shape[d] = get64(p), p += 8;
    e->offset = get64(p), e->bytes = get64(p + 8), p += 16;
    memcpy(&e->q, p, 8), p += 8;
    if (e->offset > f->weights_size || e->bytes > f->weights_size - e->offset)
      return BAD("pai: %s lies outside the weights", e->name);
  }
  f->n = n;
  info->tensor_count = n;
  return PAI_OK;
}

static const pai_entry *pai_find(const pai_file *f, const char *name) {
  for (uint32_t i = 0; i < f->n; i++)
    if (strcmp(f->e[i].name, name) == 0) return &f->e[i];
  return NULL;
}

/* The entry must hold rows x cols of the given ggml type (0: f32). */
static pai_status_t want(const pai_entry *e, const char *name, uint32_t type, uint64_t rows, uint64_t cols) {
  if (!e) return b200_fail(PAI_ERR_MISMATCH, "pai: %s missing", name);
  const uint64_t r = e->rank >= 2 ? e->shape[0] : 1, k = e->rank >= 2 ? e->shape[1] : e->shape[0];
  if (r != rows || k != cols)
    return b200_fail(PAI_ERR_MISMATCH, "pai: %s is %llux%llu, expected %llux%llu", name, (unsigned long long)r,
                     (unsigned long long)k, (unsigned long long)rows, (unsigned long long)cols);
  if (type == 0) {
    if (e->dtype != DTYPE_F32 || e->q.present || e->bytes != rows * cols * 4)
      return b200_fail(PAI_ERR_UNSUPPORTED, "pai: %s is not f32", name);
    return PAI_OK;
  }
  uint32_t gt = 0;
  pai_status_t st = pai_b200_ir_quant_ggml_type(&e->q, &gt);
  if (st) return st;
  if (e->dtype != DTYPE_U8 || gt != type || e->bytes != pai_b200_block_bytes(type, rows * cols))
    return b200_fail(PAI_ERR_MISMATCH, "pai: %s holds ggml type %u, expected %u", name, gt, type);
  return PAI_OK;
}

static const char *const k_layer[9] = {"attn_norm", "attn_q",   "attn_k",  "attn_v",  "attn_output",
                                       "ffn_norm",  "ffn_gate", "ffn_up",  "ffn_down"};
static const uint32_t k_kind[9] = {PAI_B200_T_ATTN_NORM, PAI_B200_T_WQ,       PAI_B200_T_WK,
                                   PAI_B200_T_WV,        PAI_B200_T_WO,       PAI_B200_T_FFN_NORM,
                                   PAI_B200_T_WGATE,     PAI_B200_T_WUP,      PAI_B200_T_WDOWN};

/* Check every tensor the model reads; views[i] receives its bytes (in
 * load order: token_embd, output, output_norm, then blk.L.*). */
static pai_status_t pai_llama(const pai_file *f, pai_b200_gguf_info_t *info, const uint8_t **views) {
  const pai_b200_model_cfg_t *c = &info->cfg;
  char name[160];
  pai_status_t st;
  uint64_t used = 0;
  if (c->n_layer == 0 || c->n_embd == 0 || c->n_head == 0 || c->n_head_kv == 0 || c->n_head % c->n_head_kv ||
      c->head_dim * c->n_head != c->n_embd || c->vocab == 0 || c->n_ff == 0 || !b200_type_ok(c->wtype) ||
      !b200_type_ok(c->etype))
    return b200_fail(PAI_ERR_MISMATCH, "pai: inconsistent hyperparameters");
  if (c->head_dim != 128 || info->n_rot != c->head_dim)
    return b200_fail(PAI_ERR_UNSUPPORTED, "pai: head_dim %u with %u rotary dims (the backend runs 128, fully rotated)",
                     c->head_dim, info->n_rot);
  const pai_entry *e = pai_find(f, "token_embd.weight");
  if ((st = want(e, "token_embd.weight", c->etype, c->vocab, c->n_embd))) return st;
  views[0] = f->weights + e->offset, used += e->bytes;
  const pai_entry *o = info->tied_output ? e : pai_find(f, "output.weight");
  if ((st = want(o, "output.weight", c->etype, c->vocab, c->n_embd))) return st;
  views[1] = f->weights + o->offset, used += info->tied_output ? 0 : o->bytes;
  e = pai_find(f, "output_norm.weight");
  if ((st = want(e, "output_norm.weight", 0, 1, c->n_embd))) return st;
  views[2] = f->weights + e->offset, used += e->bytes;
  const uint64_t kvd = (uint64_t)c->n_head_kv * c->head_dim;
  const uint64_t rows_of[9] = {1, c->n_embd, kvd, kvd, c->n_embd, 1, c->n_ff, c->n_ff, c->n_embd};
  const uint64_t cols_of[9] = {c->n_embd, c->n_embd, c->n_embd, c->n_embd, c->n_embd,
                               c->n_embd, c->n_embd, c->n_embd, c->n_ff};
  for (uint32_t L = 0; L < c->n_layer; L++) {
    for (int i = 0; i < 9; i++) {
      snprintf(name, sizeof(name), "blk.%u.%s.weight", L, k_layer[i]);
      e = pai_find(f, name);
      if ((st = want(e, name, (i == 0 || i == 5) ? 0 : c->wtype, rows_of[i], cols_of[i]))) return st;
      views[3 + (size_t)L * 9 + i] = f->weights + e->offset, used += e->bytes;
    }
  }
  info->weight_bytes = used;
  return PAI_OK;
}

pai_status_t pai_b200_pai_inspect(const char *path, pai_b200_gguf_info_t *info) {
  pai_file f;
  if (!path || !info) return b200_fail(PAI_ERR_INVALID_ARG, "pai_inspect: NULL");
  pai_status_t st = pai_open(path, &f, info);
  if (st) return st;
  const uint8_t **views = (const uint8_t **)calloc(3 + (size_t)info->cfg.n_layer * 9, sizeof(*views));
  st = views ? pai_llama(&f, info, views) : b200_fail(PAI_ERR_NOMEM, "pai_inspect: host allocation");
  free(views);
  pai_close(&f);
  return st;
}

pai_status_t pai_b200_model_load_pai(pai_b200_ctx_t *ctx, const char *path, uint32_t tp_rank, uint32_t tp_size,
                                     pai_b200_model_t **out, pai_b200_gguf_info_t *info_out) {
  pai_file f;
  pai_b200_gguf_info_t info;
  pai_b200_model_t *m = NULL;
  if (!ctx || !path || !out) return b200_fail(PAI_ERR_INVALID_ARG, "model_load_pai: NULL");
  *out = NULL;
  pai_status_t st = pai_open(path, &f, &info);
  if (st) return st;
  const uint8_t **views = (const uint8_t **)calloc(3 + (size_t)info.cfg.n_layer * 9, sizeof(*views));
  st = views ? pai_llama(&f, &info, views) : b200_fail(PAI_ERR_NOMEM, "model_load_pai: host allocation");
  if (!st) st = pai_b200_model_create(ctx, &info.cfg, tp_rank, tp_size, &m);
  if (!st) st = pai_b200_model_set_tensor(m, PAI_B200_T_TOK_EMBD, 0, views[0]);
  if (!st) st = pai_b200_model_set_tensor(m, PAI_B200_T_OUTPUT, 0, views[1]);
  if (!st) st = pai_b200_model_set_tensor(m, PAI_B200_T_OUTPUT_NORM, 0, views[2]);
  for (uint32_t L = 0; !st && L < info.cfg.n_layer; L++)
    for (int i = 0; !st && i < 9; i++) st = pai_b200_model_set_tensor(m, k_kind[i], L, views[3 + (size_t)L * 9 + i]);
  free(views);
  pai_close(&f);
  if (st) {
    if (m) pai_b200_model_destroy(m);
    return st;
  }
  *out = m;
  if (info_out) *info_out = info;
  return PAI_OK;
}
