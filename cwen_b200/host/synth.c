/* Seeded synthetic model generator (see synth.h). */
#define _GNU_SOURCE
#include "synth.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ---- half precision ---- */
float cw_f16_to_f32(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) & 1u, e = (uint32_t)(h >> 10) & 0x1fu, f = h & 0x3ffu, u;
  if (e == 0) {
    float x = ldexpf((float)f, -24);
    return s ? -x : x;
  }
  if (e == 31) return f ? NAN : (s ? -INFINITY : INFINITY);
  u = (s << 31) | ((e - 15 + 127) << 23) | (f << 13);
  float r;
  memcpy(&r, &u, 4);
  return r;
}

uint16_t cw_f32_to_f16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  uint32_t sign = (u >> 16) & 0x8000u, rest = u & 0x7fffffffu;
  if (rest >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (rest > 0x7f800000u ? 0x200u : 0));
  if (rest < 0x33000000u) return (uint16_t)sign;
  uint32_t e = rest >> 23, m = rest & 0x7fffffu;
  if (e < 113) { /* subnormal half */
    uint32_t t = 0x800000u | m, sh = 126u - e, half = 1u << (sh - 1);
    uint32_t r = t >> sh, rem = t & ((half << 1) - 1u);
    if (rem > half || (rem == half && (r & 1u))) r++;
    return (uint16_t)(sign + r);
  }
  uint32_t he = e - 112u, r = m >> 13, rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) {
    if (++r == 0x400u) { r = 0; he++; }
  }
  if (he >= 31u) return (uint16_t)(sign | 0x7c00u);
  return (uint16_t)(sign | (he << 10) | r);
}

/* ---- counter-based RNG ---- */
static inline uint64_t mix64(uint64_t x) {
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
/* i-th output of the splitmix64 sequence seeded by `key`. */
static inline uint64_t rnd_at(uint64_t key, uint64_t i) { return mix64(key + (i + 1) * 0x9E3779B97F4A7C15ull); }
static uint64_t stream_key(uint64_t seed, const char *name) {
  uint64_t h = 1469598103934665603ull;
  for (const unsigned char *p = (const unsigned char *)name; *p; p++) { h ^= *p; h *= 1099511628211ull; }
  return mix64(h ^ mix64(seed));
}
static inline double u01(uint64_t r) { return ((double)(r >> 11) + 1.0) * (1.0 / 9007199254740992.0); } /* (0,1] */
/* Standard normal from two draws (Box-Muller, cosine branch). */
static inline double normal_at(uint64_t key, uint64_t i) {
  double a = u01(rnd_at(key, 2 * i)), b = u01(rnd_at(key, 2 * i + 1));
  return sqrt(-2.0 * log(a)) * cos(6.283185307179586 * b);
}

/* ---- geometry ---- */
void cw_dims_full(cw_dims *d) {
  d->n_embd = 5120; d->n_ff = 17408; d->n_vocab = 248320; d->n_layer = 64;
  d->n_head = 24; d->n_head_kv = 4; d->head_dim = 256; d->n_rot = 64;
  d->ssm_n_kh = 16; d->ssm_n_vh = 48; d->ssm_d = 128; d->conv_k = 4;
  d->full_interval = 4; d->has_mtp = 0;
}
void cw_dims_tiny(cw_dims *d) {
  d->n_embd = 512; d->n_ff = 1024; d->n_vocab = 2048; d->n_layer = 4;
  d->n_head = 4; d->n_head_kv = 2; d->head_dim = 256; d->n_rot = 64;
  d->ssm_n_kh = 2; d->ssm_n_vh = 4; d->ssm_d = 128; d->conv_k = 4;
  d->full_interval = 4; d->has_mtp = 0;
}

size_t cw_tensor_nbytes(int type, int ne0, int ne1) {
  switch (type) {
    case CW_T_F32: return (size_t)ne0 * (size_t)ne1 * 4u;
    case CW_T_Q4_0: return (size_t)(ne0 / 32) * 18u * (size_t)ne1;
    case CW_T_Q8_0: return (size_t)(ne0 / 32) * 34u * (size_t)ne1;
    default: return 0;
  }
}

enum { PER_LIN = 14, PER_FULL = 11, N_MTP = 15 };

static void set_desc(cw_tensor_desc *o, const char *name, int type, int ne0, int ne1, int kind) {
  snprintf(o->name, sizeof o->name, "%s", name);
  o->type = type; o->ne0 = ne0; o->ne1 = ne1; o->kind = kind;
}

int cw_model_tensor_count(const cw_dims *d) {
  int n = 3;
  for (int l = 0; l < d->n_layer; l++) n += cw_is_linear(d, l) ? PER_LIN : PER_FULL;
  if (d->has_mtp) n += N_MTP;
  return n;
}

int cw_model_tensor_desc(const cw_dims *d, int i, cw_tensor_desc *o) {
  const int H = d->n_embd, I = d->n_ff, V = d->n_vocab;
  const int QKV = cw_qkv_dim(d), Z = d->ssm_n_vh * d->ssm_d, LVH = d->ssm_n_vh;
  const int QO = d->n_head * d->head_dim, KO = d->n_head_kv * d->head_dim, HD = d->head_dim;
  char n[96];
  if (i < 0) return -1;
  if (i == 0) { set_desc(o, "token_embd.weight", CW_T_Q4_0, H, V, CW_GEN_QMAT); return 0; }
  if (i == 1) { set_desc(o, "output_norm.weight", CW_T_F32, H, 1, CW_GEN_ONES); return 0; }
  if (i == 2) { set_desc(o, "output.weight", CW_T_Q4_0, H, V, CW_GEN_QMAT); return 0; }
  i -= 3;
  for (int l = 0; l < d->n_layer; l++) {
    int lin = cw_is_linear(d, l), cnt = lin ? PER_LIN : PER_FULL;
    if (i >= cnt) { i -= cnt; continue; }
#define T(suf, ty, a, b, k) do { snprintf(n, sizeof n, "blk.%d." suf, l); set_desc(o, n, ty, a, b, k); return 0; } while (0)
    switch (i) {
      case 0: T("attn_norm.weight", CW_T_F32, H, 1, CW_GEN_ONES);
      case 1: T("post_attention_norm.weight", CW_T_F32, H, 1, CW_GEN_ONES);
      case 2: T("ffn_gate.weight", CW_T_Q4_0, H, I, CW_GEN_QMAT);
      case 3: T("ffn_up.weight", CW_T_Q4_0, H, I, CW_GEN_QMAT);
      case 4: T("ffn_down.weight", CW_T_Q4_0, I, H, CW_GEN_QMAT);
      default: break;
    }
    if (lin) {
      switch (i) {
        case 5: T("attn_qkv.weight", CW_T_Q4_0, H, QKV, CW_GEN_QMAT);
        case 6: T("attn_gate.weight", CW_T_Q4_0, H, Z, CW_GEN_QMAT);
        case 7: T("ssm_a", CW_T_F32, LVH, 1, CW_GEN_NEG1);
        case 8: T("ssm_dt.bias", CW_T_F32, LVH, 1, CW_GEN_ZERO);
        case 9: T("ssm_alpha.weight", CW_T_Q4_0, H, LVH, CW_GEN_QMAT);
        case 10: T("ssm_beta.weight", CW_T_Q4_0, H, LVH, CW_GEN_QMAT);
        case 11: T("ssm_conv1d.weight", CW_T_F32, d->conv_k, QKV, CW_GEN_CONV);
        case 12: T("ssm_norm.weight", CW_T_F32, d->ssm_d, 1, CW_GEN_ONES);
        case 13: T("ssm_out.weight", CW_T_Q4_0, Z, H, CW_GEN_QMAT);
        default: return -1;
      }
    } else {
      switch (i) {
        case 5: T("attn_q.weight", CW_T_Q4_0, H, QO * 2, CW_GEN_QMAT);
        case 6: T("attn_k.weight", CW_T_Q4_0, H, KO, CW_GEN_QMAT);
        case 7: T("attn_v.weight", CW_T_Q4_0, H, KO, CW_GEN_QMAT);
        case 8: T("attn_output.weight", CW_T_Q4_0, QO, H, CW_GEN_QMAT);
        case 9: T("attn_q_norm.weight", CW_T_F32, HD, 1, CW_GEN_ONES);
        case 10: T("attn_k_norm.weight", CW_T_F32, HD, 1, CW_GEN_ONES);
        default: return -1;
      }
    }
#undef T
  }
  if (!d->has_mtp || i >= N_MTP) return -1;
  {
    int l = d->n_layer;
#define M(suf, ty, a, b, k) do { snprintf(n, sizeof n, "blk.%d." suf, l); set_desc(o, n, ty, a, b, k); return 0; } while (0)
    switch (i) {
      case 0: M("attn_norm.weight", CW_T_F32, H, 1, CW_GEN_ONES);
      case 1: M("post_attention_norm.weight", CW_T_F32, H, 1, CW_GEN_ONES);
      case 2: M("attn_q.weight", CW_T_Q8_0, H, QO * 2, CW_GEN_QMAT);
      case 3: M("attn_k.weight", CW_T_Q8_0, H, KO, CW_GEN_QMAT);
      case 4: M("attn_v.weight", CW_T_Q8_0, H, KO, CW_GEN_QMAT);
      case 5: M("attn_output.weight", CW_T_Q8_0, QO, H, CW_GEN_QMAT);
      case 6: M("attn_q_norm.weight", CW_T_F32, HD, 1, CW_GEN_ONES);
      case 7: M("attn_k_norm.weight", CW_T_F32, HD, 1, CW_GEN_ONES);
      case 8: M("ffn_gate.weight", CW_T_Q8_0, H, I, CW_GEN_QMAT);
      case 9: M("ffn_up.weight", CW_T_Q8_0, H, I, CW_GEN_QMAT);
      case 10: M("ffn_down.weight", CW_T_Q8_0, I, H, CW_GEN_QMAT);
      case 11: M("nextn.eh_proj.weight", CW_T_Q8_0, 2 * H, H, CW_GEN_QMAT);
      case 12: M("nextn.enorm.weight", CW_T_F32, H, 1, CW_GEN_ONES);
      case 13: M("nextn.hnorm.weight", CW_T_F32, H, 1, CW_GEN_ONES);
      case 14: M("nextn.shared_head_norm.weight", CW_T_F32, H, 1, CW_GEN_ONES);
      default: return -1;
    }
#undef M
  }
}

/* ---- threaded fills ---- */
typedef struct {
  uint64_t key;
  int type;
  size_t nblk, b0, b1;
  uint8_t *dst;
} fill_job;

static void fill_q4_range(uint64_t key, uint8_t *dst, size_t b0, size_t b1) {
  for (size_t b = b0; b < b1; b++) {
    uint8_t *blk = dst + b * 18u;
    uint16_t d = cw_f32_to_f16((float)fabs(0.01 * normal_at(key, b)));
    memcpy(blk, &d, 2);
    uint64_t r0 = rnd_at(key ^ 0x51ull, 2 * b), r1 = rnd_at(key ^ 0x51ull, 2 * b + 1);
    memcpy(blk + 2, &r0, 8);
    memcpy(blk + 10, &r1, 8);
  }
}
static void fill_q8_range(uint64_t key, uint8_t *dst, size_t b0, size_t b1) {
  for (size_t b = b0; b < b1; b++) {
    uint8_t *blk = dst + b * 34u;
    uint16_t d = cw_f32_to_f16((float)fabs(0.01 * normal_at(key, b)));
    memcpy(blk, &d, 2);
    for (int j = 0; j < 32; j++) {
      uint64_t r = rnd_at(key ^ 0x88ull, 32 * b + (uint64_t)j);
      blk[2 + j] = (uint8_t)(int8_t)((int)(r % 255u) - 127);
    }
  }
}
static void *fill_worker(void *arg) {
  fill_job *j = (fill_job *)arg;
  if (j->type == CW_T_Q4_0) fill_q4_range(j->key, j->dst, j->b0, j->b1);
  else fill_q8_range(j->key, j->dst, j->b0, j->b1);
  return NULL;
}
static int n_threads(int want) {
  if (want > 0) return want;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n < 1 ? 1 : (n > 64 ? 64 : (int)n);
}
/* Blocks [lo, hi) of a quantized tensor (each written at its own offset of dst). */
static void fill_quant_range(uint64_t key, int type, size_t lo, size_t hi, uint8_t *dst, int threads) {
  int nt = n_threads(threads);
  const size_t nblk = hi - lo;
  if (nblk < 65536 || nt == 1) {
    fill_job j = {key, type, nblk, lo, hi, dst};
    fill_worker(&j);
    return;
  }
  pthread_t tid[64];
  fill_job jobs[64];
  size_t per = (nblk + (size_t)nt - 1) / (size_t)nt;
  int launched = 0;
  for (int t = 0; t < nt; t++) {
    size_t b0 = lo + (size_t)t * per, b1 = b0 + per < hi ? b0 + per : hi;
    if (b0 >= b1) break;
    jobs[t] = (fill_job){key, type, nblk, b0, b1, dst};
    if (pthread_create(&tid[t], NULL, fill_worker, &jobs[t])) { fill_worker(&jobs[t]); tid[t] = 0; }
    launched = t + 1;
  }
  for (int t = 0; t < launched; t++)
    if (tid[t]) pthread_join(tid[t], NULL);
}

void cw_synth_q4_0(uint64_t seed, const char *stream, int ne0, int ne1, void *dst, int threads) {
  fill_quant_range(stream_key(seed, stream), CW_T_Q4_0, 0, (size_t)(ne0 / 32) * (size_t)ne1, (uint8_t *)dst, threads);
}
void cw_synth_q8_0(uint64_t seed, const char *stream, int ne0, int ne1, void *dst, int threads) {
  fill_quant_range(stream_key(seed, stream), CW_T_Q8_0, 0, (size_t)(ne0 / 32) * (size_t)ne1, (uint8_t *)dst, threads);
}
void cw_synth_normal(uint64_t seed, const char *stream, float mean, float std, float *dst, size_t n) {
  uint64_t key = stream_key(seed, stream);
  for (size_t i = 0; i < n; i++) dst[i] = (float)(mean + std * normal_at(key, i));
}
void cw_synth_ids(uint64_t seed, const char *stream, int hi, int32_t *dst, size_t n) {
  uint64_t key = stream_key(seed, stream);
  for (size_t i = 0; i < n; i++) dst[i] = (int32_t)(rnd_at(key, i) % (uint64_t)hi);
}

void cw_synth_tensor_rows(uint64_t seed, const cw_tensor_desc *t, void *dst, int threads, int r0, int r1) {
  if (t->kind != CW_GEN_QMAT) {
    cw_synth_tensor(seed, t, dst, threads);
    return;
  }
  const size_t nb = (size_t)(t->ne0 / 32);
  fill_quant_range(stream_key(seed, t->name), t->type, (size_t)r0 * nb, (size_t)r1 * nb, (uint8_t *)dst, threads);
}

void cw_synth_tensor(uint64_t seed, const cw_tensor_desc *t, void *dst, int threads) {
  size_t n = (size_t)t->ne0 * (size_t)t->ne1;
  float *f = (float *)dst;
  switch (t->kind) {
    case CW_GEN_QMAT:
      if (t->type == CW_T_Q4_0) cw_synth_q4_0(seed, t->name, t->ne0, t->ne1, dst, threads);
      else cw_synth_q8_0(seed, t->name, t->ne0, t->ne1, dst, threads);
      break;
    case CW_GEN_ONES: for (size_t i = 0; i < n; i++) f[i] = 1.0f; break;
    case CW_GEN_ZERO: for (size_t i = 0; i < n; i++) f[i] = 0.0f; break;
    case CW_GEN_NEG1: for (size_t i = 0; i < n; i++) f[i] = -1.0f; break;
    case CW_GEN_CONV: cw_synth_normal(seed, t->name, 0.0f, 0.1f, f, n); break;
    default: break;
  }
}

/* ---- GGUF v3 writer ---- */
static int wr(FILE *f, const void *p, size_t n) { return fwrite(p, 1, n, f) == n ? 0 : -1; }
static int wr_u32(FILE *f, uint32_t v) { return wr(f, &v, 4); }
static int wr_u64(FILE *f, uint64_t v) { return wr(f, &v, 8); }
static int wr_str(FILE *f, const char *s) { uint64_t n = strlen(s); return wr_u64(f, n) || wr(f, s, n); }

int cw_write_gguf(const char *path, const cw_dims *d, uint64_t seed, int threads) {
  FILE *f = fopen(path, "wb");
  if (!f) return -1;
  int nt = cw_model_tensor_count(d), rc = 0;
  rc |= wr(f, "GGUF", 4);
  rc |= wr_u32(f, 3);
  rc |= wr_u64(f, (uint64_t)nt);
  rc |= wr_u64(f, 1); /* one kv: general.architecture */
  rc |= wr_str(f, "general.architecture");
  rc |= wr_u32(f, 8); /* string */
  rc |= wr_str(f, "qwen35");
  uint64_t off = 0;
  for (int i = 0; i < nt && !rc; i++) {
    cw_tensor_desc t;
    cw_model_tensor_desc(d, i, &t);
    rc |= wr_str(f, t.name);
    int nd = t.ne1 > 1 ? 2 : 1;
    rc |= wr_u32(f, (uint32_t)nd);
    rc |= wr_u64(f, (uint64_t)t.ne0);
    if (nd == 2) rc |= wr_u64(f, (uint64_t)t.ne1);
    rc |= wr_u32(f, (uint32_t)t.type);
    rc |= wr_u64(f, off);
    off += (cw_tensor_nbytes(t.type, t.ne0, t.ne1) + 31u) & ~(size_t)31u;
  }
  long pos = ftell(f);
  static const char zeros[32] = {0};
  if (pos < 0) rc = -1;
  else if (pos % 32) rc |= wr(f, zeros, (size_t)(32 - pos % 32));
  for (int i = 0; i < nt && !rc; i++) {
    cw_tensor_desc t;
    cw_model_tensor_desc(d, i, &t);
    size_t nb = cw_tensor_nbytes(t.type, t.ne0, t.ne1);
    void *buf = malloc(nb ? nb : 1);
    if (!buf) { rc = -1; break; }
    cw_synth_tensor(seed, &t, buf, threads);
    rc |= wr(f, buf, nb);
    free(buf);
    if (nb % 32) rc |= wr(f, zeros, 32 - nb % 32);
  }
  if (fclose(f)) rc = -1;
  return rc;
}
