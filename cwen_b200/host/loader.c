/* Model loading for the C host: GGUF files and the seeded synthetic model.
 *
 * The GGUF reader follows the checks of the reference's load_gguf
 * (run.c:3230-3303): version 2 or 3, at most 4 dims, no zero or int-overflowing
 * dims, every tensor extent inside the mapping, 32-byte aligned data section
 * (or general.alignment when the file declares it).  Unlike the reference it
 * derives the model geometry from the tensor shapes instead of compiling it
 * in, and hands each tensor to the engine's upload call.
 */
#define _GNU_SOURCE
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <errno.h>

#include "cwen_host.h"
#include "host_err.h"
#include "synth.h"

#define GG_MAX_TENSORS 4096

typedef struct {
  char name[96];
  int type;
  int n_dims;
  uint64_t ne[4];
  uint64_t off;
  const uint8_t *data;
} gg_tensor;

typedef struct {
  const uint8_t *p, *end;
  int bad;
  char why[160];
} gg_cur;

static void gg_fail(gg_cur *c, const char *why) {
  if (!c->bad) snprintf(c->why, sizeof c->why, "%s", why);
  c->bad = 1;
}
static const uint8_t *gg_take(gg_cur *c, uint64_t n) {
  if (c->bad || (uint64_t)(c->end - c->p) < n) {
    gg_fail(c, "truncated");
    return NULL;
  }
  const uint8_t *q = c->p;
  c->p += n;
  return q;
}
static uint64_t gg_u64(gg_cur *c) {
  const uint8_t *q = gg_take(c, 8);
  uint64_t v = 0;
  if (q) memcpy(&v, q, 8);
  return v;
}
static uint32_t gg_u32(gg_cur *c) {
  const uint8_t *q = gg_take(c, 4);
  uint32_t v = 0;
  if (q) memcpy(&v, q, 4);
  return v;
}
static void gg_str(gg_cur *c, char *buf, size_t cap) {
  uint64_t n = gg_u64(c);
  if (c->bad) return;
  if (n >= cap) {
    gg_fail(c, "string too long");
    return;
  }
  const uint8_t *q = gg_take(c, n);
  if (!q) return;
  memcpy(buf, q, n);
  buf[n] = 0;
}
/* Skip one KV value; returns the value when it is a u32/i32 (alignment). */
static uint64_t gg_skip(gg_cur *c, uint32_t t, int depth) {
  if (depth > 64) {
    gg_fail(c, "kv nesting too deep");
    return 0;
  }
  uint64_t v = 0;
  switch (t) {
    case 0: case 1: case 7: gg_take(c, 1); break;
    case 2: case 3: gg_take(c, 2); break;
    case 4: case 5: v = gg_u32(c); break;
    case 6: gg_take(c, 4); break;
    case 8: { uint64_t n = gg_u64(c); gg_take(c, n); } break;
    case 9: {
      uint32_t at = gg_u32(c);
      uint64_t n = gg_u64(c);
      for (uint64_t i = 0; i < n && !c->bad; i++) gg_skip(c, at, depth + 1);
    } break;
    case 10: case 11: case 12: gg_take(c, 8); break;
    default: gg_fail(c, "unknown kv type");
  }
  return v;
}

static size_t gg_nbytes(int type, uint64_t ne0, uint64_t rows) {
  switch (type) {
    case CWEN_T_F32: return (size_t)(ne0 * rows * 4);
    case CWEN_T_Q4_0: return (size_t)(ne0 / 32 * 18 * rows);
    case CWEN_T_Q8_0: return (size_t)(ne0 / 32 * 34 * rows);
    default: return 0;
  }
}

static const gg_tensor *gg_find(const gg_tensor *t, int n, const char *name) {
  for (int i = 0; i < n; i++)
    if (!strcmp(t[i].name, name)) return &t[i];
  return NULL;
}

/* Geometry from shapes: see the file comment. */
static int gg_dims(const gg_tensor *t, int n, cwen_dims *d, char *why, size_t wl) {
  memset(d, 0, sizeof *d);
  d->head_dim = 256; d->n_rot = 64; d->ssm_d = 128; d->conv_k = 4;
  const gg_tensor *e = gg_find(t, n, "token_embd.weight");
  if (!e) { snprintf(why, wl, "missing token_embd.weight"); return -1; }
  d->n_embd = (int)e->ne[0];
  d->n_vocab = (int)e->ne[1];
  int mtp_layer = -1, max_layer = -1, first_full = -1;
  for (int i = 0; i < n; i++) {
    int l = -1, off = 0;
    if (sscanf(t[i].name, "blk.%d.%n", &l, &off) != 1 || off == 0) continue;
    if (!strcmp(t[i].name + off, "nextn.eh_proj.weight")) mtp_layer = l;
    if (!strcmp(t[i].name + off, "ffn_gate.weight") && l > max_layer) max_layer = l;
  }
  if (max_layer < 0) { snprintf(why, wl, "no blk.*.ffn_gate.weight"); return -1; }
  d->n_layer = mtp_layer == max_layer ? max_layer : max_layer + 1;
  d->has_mtp = mtp_layer == d->n_layer;
  char nm[96];
  for (int l = 0; l < d->n_layer; l++) {
    snprintf(nm, sizeof nm, "blk.%d.attn_q.weight", l);
    const gg_tensor *q = gg_find(t, n, nm);
    if (q && first_full < 0) {
      first_full = l;
      d->n_head = (int)(q->ne[1] / 512);
      snprintf(nm, sizeof nm, "blk.%d.attn_k.weight", l);
      const gg_tensor *k = gg_find(t, n, nm);
      d->n_head_kv = k ? (int)(k->ne[1] / 256) : 0;
    }
  }
  d->full_interval = first_full >= 0 ? first_full + 1 : d->n_layer + 1;
  snprintf(nm, sizeof nm, "blk.0.ffn_gate.weight");
  const gg_tensor *g = gg_find(t, n, nm);
  d->n_ff = g ? (int)g->ne[1] : 0;
  for (int l = 0; l < d->n_layer; l++) {
    snprintf(nm, sizeof nm, "blk.%d.attn_gate.weight", l);
    const gg_tensor *z = gg_find(t, n, nm);
    snprintf(nm, sizeof nm, "blk.%d.attn_qkv.weight", l);
    const gg_tensor *qkv = gg_find(t, n, nm);
    if (z && qkv) {
      d->ssm_n_vh = (int)(z->ne[1] / 128);
      d->ssm_n_kh = (int)((qkv->ne[1] / 128 - (uint64_t)d->ssm_n_vh) / 2);
      break;
    }
  }
  if (!d->n_head) { d->n_head = 1; d->n_head_kv = 1; }
  if (!d->ssm_n_vh) { d->ssm_n_vh = 1; d->ssm_n_kh = 1; }
  return 0;
}

/* A mapped and parsed GGUF file. */
typedef struct {
  uint8_t *map;
  size_t len;
  gg_tensor *t;
  int nt;
} gg_file;

static void gg_close(gg_file *g) {
  free(g->t);
  if (g->map) munmap(g->map, g->len);
  memset(g, 0, sizeof *g);
}

/* Map and parse a GGUF file: header, key/values (general.alignment), the
 * tensor table, every tensor's extent inside the file.  On failure the
 * message goes to cwen_cuda_last_error() and the code is returned. */
static int gg_open(const char *path, gg_file *g) {
  memset(g, 0, sizeof *g);
  int fd = open(path, O_RDONLY);
  if (fd < 0) return host_fail(CWEN_EINVAL, "gguf: %s: %s", path, strerror(errno));
  struct stat st;
  if (fstat(fd, &st) || !S_ISREG(st.st_mode) || st.st_size < 24) {
    close(fd);
    return host_fail(CWEN_EINVAL, "gguf: %s: not a gguf file", path);
  }
  g->len = (size_t)st.st_size;
  uint8_t *map = (uint8_t *)mmap(NULL, g->len, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) {
    g->len = 0;
    return host_fail(CWEN_ENOMEM, "gguf: %s: mmap: %s", path, strerror(errno));
  }
  g->map = map;
  gg_cur c = {map, map + g->len, 0, {0}};
  const uint8_t *magic = gg_take(&c, 4);
  if (!magic || memcmp(magic, "GGUF", 4)) gg_fail(&c, "bad magic");
  uint32_t ver = gg_u32(&c);
  if (!c.bad && (ver < 2 || ver > 3)) gg_fail(&c, "unsupported gguf version");
  uint64_t n_t = gg_u64(&c), n_kv = gg_u64(&c);
  if (!c.bad && n_t > GG_MAX_TENSORS) gg_fail(&c, "too many tensors");
  uint64_t align = 32;
  for (uint64_t i = 0; i < n_kv && !c.bad; i++) {
    char key[256];
    gg_str(&c, key, sizeof key);
    uint32_t ty = gg_u32(&c);
    uint64_t v = gg_skip(&c, ty, 0);
    if (!c.bad && !strcmp(key, "general.alignment") && (ty == 4 || ty == 5)) align = v;
  }
  if (!c.bad && (align == 0 || (align & (align - 1)))) gg_fail(&c, "bad general.alignment");
  if (!c.bad) {
    g->t = (gg_tensor *)calloc(n_t ? n_t : 1, sizeof *g->t);
    if (!g->t) {
      gg_close(g);
      return host_fail(CWEN_ENOMEM, "gguf: %s: out of host memory", path);
    }
    g->nt = (int)n_t;
  }
  for (int i = 0; i < g->nt && !c.bad; i++) {
    gg_tensor *x = &g->t[i];
    gg_str(&c, x->name, sizeof x->name);
    uint32_t nd = gg_u32(&c);
    if (c.bad) break;
    if (nd < 1 || nd > 4) { gg_fail(&c, "n_dims outside 1..4"); break; }
    x->n_dims = (int)nd;
    x->ne[0] = x->ne[1] = x->ne[2] = x->ne[3] = 1;
    for (uint32_t k = 0; k < nd && !c.bad; k++) {
      x->ne[k] = gg_u64(&c);
      if (!c.bad && (x->ne[k] == 0 || x->ne[k] > 0x7fffffffull)) gg_fail(&c, "dim zero or beyond INT_MAX");
    }
    x->type = (int)gg_u32(&c);
    x->off = gg_u64(&c);
    /* rows = ne1*ne2*ne3, checked after each product (each factor < 2^31) */
    uint64_t rows = 1;
    for (int k = 1; k < 4 && !c.bad; k++) {
      rows *= x->ne[k];
      if (rows > 0x7fffffffull) gg_fail(&c, "tensor rows beyond INT_MAX");
    }
    if (!c.bad && (x->type == CWEN_T_Q4_0 || x->type == CWEN_T_Q8_0) && x->ne[0] % 32)
      gg_fail(&c, "quantized row length not a multiple of 32");
  }
  if (!c.bad) {
    uint64_t data_off = (uint64_t)(c.p - map);
    data_off = (data_off + align - 1) & ~(align - 1);
    for (int i = 0; i < g->nt && !c.bad; i++) {
      gg_tensor *x = &g->t[i];
      if (data_off >= g->len || x->off >= g->len - data_off) {
        snprintf(c.why, sizeof c.why, "%s: tensor offset out of file", x->name);
        c.bad = 1;
        break;
      }
      x->data = map + data_off + x->off;
      const size_t nb = gg_nbytes(x->type, x->ne[0], x->ne[1] * x->ne[2] * x->ne[3]);
      if (nb && nb > g->len - data_off - x->off) {
        snprintf(c.why, sizeof c.why, "%s: extent beyond file", x->name);
        c.bad = 1;
      }
    }
  }
  if (c.bad) {
    gg_close(g);
    return host_fail(CWEN_EINVAL, "gguf: %s: %s", path, c.why);
  }
  return CWEN_OK;
}

/* ---- CWENR sidecar (load_cwenr, run.c:3305-3643) ----
 *
 * The reference can take its Q4_0 weights from an offline sidecar written by
 * its repack tool (format: tools/repack_q4.py:1-30).  Header, 32 bytes:
 * "CWENR001", u32 version (2, 3 or 4), u32 entry count, u64 data base, and a
 * stamp {u32 "CWEN", u32 size of the source GGUF in 4 KiB pages} (zeros: an
 * unstamped sidecar).  Then one 128-byte entry per tensor: name[96], i32 ne0,
 * i32 rows, u64 off_a, u64 off_b, u32 flags.  v2 entries point at packed
 * 20-byte blocks {qs[16], f32 d} (off_a, off_b = byte count); v3 entries at a
 * qs stream (16 B per block) and an f16 scale stream; v4 adds interleaved
 * pairs (ffn_gate + ffn_up, attn_k + attn_v) that share one qs stream
 * (qsA|qsB per block) and one scale stream (dA|dB), flags 1 and 2 naming the
 * side (any other flag value is a solo v3 entry).
 *
 * The engine lays Q4_0 weights out for its own kernels when they are
 * uploaded, so a sidecar only decides the bytes: a bound tensor's blocks are
 * put back into GGUF block form (f16 d, qs[16]; a v2 f32 scale rounded to
 * f16, nearest-even) on the host and uploaded like GGUF bytes.  What binds,
 * and what makes the whole sidecar ignored, follows the reference:
 *  - path: CWEN_REPACK when set and non-empty, else the GGUF path with
 *    ".gguf" replaced by ".cwenr", else the GGUF path + ".cwenr"; no file
 *    there means no sidecar;
 *  - ignored: shorter than 32 bytes, bad magic, a stamp whose page count
 *    is not the GGUF's (stale), version outside 2..4, more than 1024
 *    entries, a data base outside the file or a directory past its end, or
 *    no entry that binds;
 *  - an entry is skipped when its name is not a Q4_0 tensor of the GGUF, its
 *    shape differs, its streams reach past the end of the file (checked as
 *    remainders, so offsets cannot wrap), or (v2) its byte count is not
 *    20 B per block. */
#define CR_ENT 128
#define CR_MAX_ENT 1024
#define CR_STAMP_TAG 0x4e455743u /* "CWEN" */

typedef struct {
  int ver;           /* 0: not bound; 2, 3 or 4 */
  int side;          /* interleaved pair: 0 (flags 1) or 1 (flags 2); -1 solo */
  const uint8_t *qs; /* v2: packed blocks; v3/v4: qs stream */
  const uint8_t *sc; /* v3/v4: f16 scale stream */
} cr_bind;

typedef struct {
  uint8_t *map;
  size_t len;
  cr_bind *b; /* one per GGUF tensor */
  int bound, n_il;
} cr_file;

static void cr_close(cr_file *r) {
  free(r->b);
  if (r->map) munmap(r->map, r->len);
  memset(r, 0, sizeof *r);
}

/* The sidecar path for a GGUF path (cwenr_path_for, run.c:3310-3325): 0, or
 * -1 when it does not fit in cap. */
static int cr_path(const char *gguf, char *out, size_t cap) {
  const char *env = getenv("CWEN_REPACK");
  if (env && env[0]) {
    int k = snprintf(out, cap, "%s", env);
    return k < 0 || (size_t)k >= cap ? -1 : 0;
  }
  const size_t n = strlen(gguf);
  if (n > 5 && !strcmp(gguf + n - 5, ".gguf")) {
    if (n + 1 >= cap) return -1; /* ".cwenr" is one byte longer than ".gguf" */
    memcpy(out, gguf, n - 5);
    memcpy(out + n - 5, ".cwenr", 7);
    return 0;
  }
  int k = snprintf(out, cap, "%s.cwenr", gguf);
  return k < 0 || (size_t)k >= cap ? -1 : 0;
}

/* Map the sidecar of the GGUF at gguf_path and bind its entries to g's
 * tensors.  Never an error: an absent or unusable sidecar leaves r empty (the
 * GGUF bytes are used), with the reason on stderr like the reference. */
static void cr_open(const char *gguf_path, const gg_file *g, cr_file *r) {
  memset(r, 0, sizeof *r);
  char path[4096];
  if (cr_path(gguf_path, path, sizeof path)) {
    fprintf(stderr, "cwenr: sidecar path for %s does not fit; skipping sidecar\n", gguf_path);
    return;
  }
  int fd = open(path, O_RDONLY);
  if (fd < 0) return; /* optional */
  struct stat st;
  if (fstat(fd, &st) || !S_ISREG(st.st_mode) || st.st_size < 32) {
    fprintf(stderr, "cwenr: %s: unusable, ignoring sidecar\n", path);
    close(fd);
    return;
  }
  r->len = (size_t)st.st_size;
  void *m = mmap(NULL, r->len, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) {
    fprintf(stderr, "cwenr: %s: mmap: %s\n", path, strerror(errno));
    r->len = 0;
    return;
  }
  r->map = (uint8_t *)m;
  const uint8_t *p = r->map;
  const char *why = NULL;
  uint32_t ver = 0, n = 0, tag = 0, pages = 0;
  uint64_t base = 0;
  memcpy(&ver, p + 8, 4);
  memcpy(&n, p + 12, 4);
  memcpy(&base, p + 16, 8);
  memcpy(&tag, p + 24, 4);
  memcpy(&pages, p + 28, 4);
  struct stat gs;
  if (memcmp(p, "CWENR001", 8))
    why = "bad magic";
  else if (tag == CR_STAMP_TAG &&
           (uint64_t)pages != (stat(gguf_path, &gs) == 0 ? ((uint64_t)gs.st_size + 4095) / 4096 : 0))
    why = "stale sidecar (the GGUF changed since the repack)";
  else if ((ver != 2 && ver != 3 && ver != 4) || n > CR_MAX_ENT || base >= r->len ||
           32u + (size_t)n * CR_ENT > r->len)
    why = "bad header";
  if (!why) {
    r->b = (cr_bind *)calloc(g->nt ? (size_t)g->nt : 1, sizeof *r->b);
    if (!r->b) why = "out of host memory";
  }
  const size_t rem = r->len - (size_t)base; /* bytes from the data base on */
  for (uint32_t i = 0; !why && i < n; i++) {
    const uint8_t *e = p + 32 + (size_t)i * CR_ENT;
    char name[96];
    memcpy(name, e, 96);
    name[95] = 0;
    int32_t ne0, ne1;
    uint64_t oa, ob;
    uint32_t flags = 0;
    memcpy(&ne0, e + 96, 4);
    memcpy(&ne1, e + 100, 4);
    memcpy(&oa, e + 104, 8);
    memcpy(&ob, e + 112, 8);
    if (ver >= 3) memcpy(&flags, e + 120, 4);
    int ti = -1;
    for (int k = 0; k < g->nt; k++)
      if (!strcmp(g->t[k].name, name)) { ti = k; break; }
    if (ti < 0) { fprintf(stderr, "cwenr: unknown %s\n", name); continue; }
    const gg_tensor *x = &g->t[ti];
    if (x->type != CWEN_T_Q4_0) { fprintf(stderr, "cwenr: skip non-Q4_0 %s\n", name); continue; }
    const uint64_t rows = x->ne[1] * x->ne[2] * x->ne[3];
    if ((uint64_t)(int64_t)ne0 != x->ne[0] || (uint64_t)(int64_t)ne1 != rows) {
      fprintf(stderr, "cwenr: shape %s\n", name);
      continue;
    }
    const uint64_t nblk = x->ne[0] / 32 * rows;
    cr_bind b = {(int)ver, -1, NULL, NULL};
    if (ver == 2) {
      if (oa > rem || ob > rem - oa) { fprintf(stderr, "cwenr: OOB %s\n", name); continue; }
      if (ob != nblk * 20) { fprintf(stderr, "cwenr: size %s\n", name); continue; }
      b.qs = p + base + oa;
    } else {
      const int il = flags == 1 || flags == 2;
      const uint64_t qsb = nblk * (il ? 32u : 16u), scb = nblk * (il ? 4u : 2u);
      if (oa > rem || ob > rem || qsb > rem - oa || scb > rem - ob) {
        fprintf(stderr, "cwenr: OOB %s\n", name);
        continue;
      }
      b.side = il ? (int)flags - 1 : -1;
      b.qs = p + base + oa;
      b.sc = p + base + ob;
      r->n_il += il;
    }
    r->b[ti] = b;
    r->bound++;
  }
  if (!why && !r->bound) why = "no usable entries";
  if (why) {
    fprintf(stderr, "cwenr: %s: %s; ignoring sidecar\n", path, why);
    cr_close(r);
    return;
  }
  fprintf(stderr, "cwenr: v%u bound %d Q4 tensors (il=%d) from %s\n", ver, r->bound, r->n_il, path);
}

/* f32 -> f16 bits, round to nearest even (the conversion the reference
 * applies to v2 scales, run.c:3623). */
static uint16_t cr_f16(float f) {
  _Float16 h = (_Float16)f;
  uint16_t u;
  memcpy(&u, &h, 2);
  return u;
}

/* nblk blocks of a bound tensor in GGUF Q4_0 form {f16 d, qs[16]}. */
static void cr_blocks(const cr_bind *b, uint64_t nblk, uint8_t *dst) {
  for (uint64_t k = 0; k < nblk; k++, dst += 18) {
    if (b->ver == 2) {
      const uint8_t *s = b->qs + k * 20;
      float d;
      memcpy(&d, s + 16, 4);
      const uint16_t h = cr_f16(d);
      memcpy(dst, &h, 2);
      memcpy(dst + 2, s, 16);
    } else if (b->side >= 0) {
      memcpy(dst, b->sc + k * 4 + (size_t)b->side * 2, 2);
      memcpy(dst + 2, b->qs + k * 32 + (size_t)b->side * 16, 16);
    } else {
      memcpy(dst, b->sc + k * 2, 2);
      memcpy(dst + 2, b->qs + k * 16, 16);
    }
  }
}

int cwen_gguf_tensor_bytes(const char *path, const char *name, void *out, size_t cap, int *from_sidecar) {
  if (!path || !name) return host_fail(CWEN_EINVAL, "cwen_gguf_tensor_bytes: null argument");
  gg_file g;
  int rc = gg_open(path, &g);
  if (rc) return rc;
  int ti = -1;
  for (int k = 0; k < g.nt; k++)
    if (!strcmp(g.t[k].name, name)) { ti = k; break; }
  if (ti < 0) {
    gg_close(&g);
    return host_fail(CWEN_EINVAL, "gguf: %s: no tensor %s", path, name);
  }
  const gg_tensor *x = &g.t[ti];
  const uint64_t rows = x->ne[1] * x->ne[2] * x->ne[3];
  const size_t nb = gg_nbytes(x->type, x->ne[0], rows);
  if (!nb || nb > 0x7fffffffull) {
    gg_close(&g);
    return host_fail(CWEN_EINVAL, "gguf: %s: %s: type %d not readable here", path, name, x->type);
  }
  cr_file r;
  cr_open(path, &g, &r);
  const int side = r.b && r.b[ti].ver;
  if (from_sidecar) *from_sidecar = side;
  if (out) {
    if (cap < nb) {
      rc = host_fail(CWEN_EINVAL, "cwen_gguf_tensor_bytes: %s needs %zu bytes", name, nb);
    } else if (side) {
      cr_blocks(&r.b[ti], x->ne[0] / 32 * rows, (uint8_t *)out);
    } else {
      memcpy(out, x->data, nb);
    }
  }
  cr_close(&r);
  gg_close(&g);
  return rc ? rc : (int)nb;
}

int cwen_gguf_dims(const char *path, cwen_dims *out) {
  if (!path || !out) return host_fail(CWEN_EINVAL, "cwen_gguf_dims: null argument");
  gg_file g;
  int rc = gg_open(path, &g);
  if (rc) return rc;
  char why[160];
  if (gg_dims(g.t, g.nt, out, why, sizeof why)) rc = host_fail(CWEN_EINVAL, "gguf: %s: %s", path, why);
  gg_close(&g);
  return rc;
}

int cwen_load_gguf(const char *path) {
  if (!path) return host_fail(CWEN_EINVAL, "cwen_load_gguf: null path");
  gg_file g;
  int rc = gg_open(path, &g);
  if (rc) return rc;
  cwen_dims d;
  char why[160];
  if (gg_dims(g.t, g.nt, &d, why, sizeof why)) {
    rc = host_fail(CWEN_EINVAL, "gguf: %s: %s", path, why);
    goto out;
  }
  rc = cwen_cuda_model_config(&d);
  cr_file r;
  cr_open(path, &g, &r);
  uint8_t *buf = NULL; /* GGUF-form blocks of one sidecar-bound tensor */
  size_t buf_len = 0;
  for (int i = 0; i < g.nt && !rc; i++) {
    const gg_tensor *x = &g.t[i];
    if (x->type != CWEN_T_F32 && x->type != CWEN_T_Q4_0 && x->type != CWEN_T_Q8_0) continue;
    const uint64_t rows = x->ne[1] * x->ne[2] * x->ne[3];
    const void *src = x->data;
    if (r.b && r.b[i].ver) {
      const size_t nb = gg_nbytes(x->type, x->ne[0], rows);
      if (nb > buf_len) {
        free(buf);
        buf = (uint8_t *)malloc(nb);
        buf_len = buf ? nb : 0;
        if (!buf) {
          rc = host_fail(CWEN_ENOMEM, "cwenr: out of host memory for %s", x->name);
          break;
        }
      }
      cr_blocks(&r.b[i], x->ne[0] / 32 * rows, buf);
      src = buf;
    }
    rc = cwen_cuda_upload(x->name, x->type, src, (int)x->ne[0], (int)rows);
  }
  free(buf);
  cr_close(&r);
  if (!rc) rc = cwen_cuda_model_finalize();
out:
  gg_close(&g);
  return rc;
}

int cwen_write_synth_gguf(const char *path, const cwen_dims *dims, uint64_t seed, int threads) {
  if (!path || !dims) return host_fail(CWEN_EINVAL, "cwen_write_synth_gguf: null argument");
  cw_dims d;
  memcpy(&d, dims, sizeof d);
  if (d.n_layer < 1 || d.full_interval < 1 || d.n_embd < 32 || d.n_embd % 32 || d.n_ff % 32 || d.n_vocab < 1)
    return host_fail(CWEN_EINVAL, "cwen_write_synth_gguf: geometry out of range");
  if (cw_write_gguf(path, &d, seed, threads)) return host_fail(CWEN_EINVAL, "cwen_write_synth_gguf: cannot write %s", path);
  return CWEN_OK;
}

void cwen_dims_reference(cwen_dims *d) {
  if (!d) return;
  cw_dims s;
  cw_dims_full(&s);
  memcpy(d, &s, sizeof *d);
}
void cwen_dims_small(cwen_dims *d) {
  if (!d) return;
  cw_dims s;
  cw_dims_tiny(&s);
  memcpy(d, &s, sizeof *d);
}

int cwen_load_synth(uint64_t seed, const cwen_dims *dims, int threads) {
  if (!dims) return host_fail(CWEN_EINVAL, "cwen_load_synth: dims is NULL");
  cw_dims d;
  memcpy(&d, dims, sizeof d);
  int rc = cwen_cuda_model_config(dims);
  if (rc) return rc;
  const int n = cw_model_tensor_count(&d);
  size_t cap = 0;
  for (int i = 0; i < n; i++) {
    cw_tensor_desc td;
    cw_model_tensor_desc(&d, i, &td);
    size_t nb = cw_tensor_nbytes(td.type, td.ne0, td.ne1);
    if (nb > cap) cap = nb;
  }
  void *buf = malloc(cap);
  if (!buf) return CWEN_ENOMEM;
  for (int i = 0; i < n && !rc; i++) {
    cw_tensor_desc td;
    cw_model_tensor_desc(&d, i, &td);
    /* a row-sharded matrix: only the rows this GPU keeps are generated */
    int r0 = 0, r1 = td.ne1;
    cwen_cuda_shard_rows_for(td.name, td.ne1, &r0, &r1);
    cw_synth_tensor_rows(seed, &td, buf, threads, r0, r1);
    rc = cwen_cuda_upload(td.name, td.type, buf, td.ne0, td.ne1);
  }
  free(buf);
  if (rc) return rc;
  return cwen_cuda_model_finalize();
}
