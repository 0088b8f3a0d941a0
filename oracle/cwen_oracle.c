/* TEST INFRASTRUCTURE ONLY: CPU oracle for the cwen verify-decode path.
 * Never linked into the product; the product fails loudly without its CUDA
 * library instead of falling back here.
 *
 * Each function restates the reference (maci0/cwen run.c) along its scalar
 * (non-SIMD) code path, with the same operation order.  The reference itself
 * only builds with AVX2 or AVX-512 (dot_q8s, run.c:1335-1359, is AVX2-only),
 * whose kernels reassociate the fp32 sums, so the oracle agrees with the
 * compiled reference to fp32 rounding, not bit for bit; tests/test_oracle_pin.py
 * pins it against oracle/_ref and the committed golden vectors.
 * Build: -std=c11 -O2 -ffp-contract=off (no FMA contraction).
 */
#include "cwen_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static const float OR_EPS = 1e-6f;      /* RMS_EPS, run.c:89 */
static const float OR_THETA = 1e7f;     /* ROPE_THETA, run.c:90 */

/* rmsnorm, scalar branch of run.c:346-367. */
void or_rmsnorm(float *o, const float *x, const float *w, int n) {
  float ss = 0;
  for (int i = 0; i < n; i++) ss += x[i] * x[i];
  float s = 1.f / sqrtf(ss / n + OR_EPS);
  for (int i = 0; i < n; i++) o[i] = w[i] * x[i] * s;
}
static inline float or_silu(float x) { return x * (1.f / (1.f + expf(-x))); } /* run.c:378-384 */
static inline float or_softplus(float x) { return x > 20.f ? x : logf(1.f + expf(x)); } /* run.c:393 */
static inline float or_sigmoid(float x) { return 1.f / (1.f + expf(-x)); } /* run.c:394-400 */
/* l2norm_rows, scalar branch of run.c:401-423. */
static void or_l2norm_rows(float *x, int rows, int dim) {
  for (int r = 0; r < rows; r++) {
    float *p = x + (size_t)r * dim, ss = 0;
    for (int i = 0; i < dim; i++) ss += p[i] * p[i];
    float s = 1.f / sqrtf(ss + OR_EPS);
    for (int i = 0; i < dim; i++) p[i] *= s;
  }
}

/* Q4_0 row dot: dot_q4_0 scalar branch (run.c:1018-1022) over dot_nib16
   (run.c:432-437): per 32-block, low nibble j pairs with x[j], high nibble
   with x[j+16], both offset by 8, scaled by the block's f16 scale. */
static float or_dot_q4_0(const uint8_t *row, const float *y, int K) {
  int nb = K / 32;
  float sum = 0;
  for (int i = 0; i < nb; i++) {
    const uint8_t *blk = row + (size_t)i * 18;
    uint16_t dh;
    memcpy(&dh, blk, 2);
    float d = cw_f16_to_f32(dh);
    const uint8_t *q = blk + 2;
    const float *yy = y + (size_t)i * 32;
    float s = 0;
    for (int j = 0; j < 16; j++)
      s += ((int)(q[j] & 0xF) - 8) * d * yy[j] + ((int)(q[j] >> 4) - 8) * d * yy[j + 16];
    sum += s;
  }
  return sum;
}
/* Q8_0 row dot: dot_q8_0 scalar branch (run.c:1267-1272), one running sum. */
static float or_dot_q8_0(const uint8_t *row, const float *y, int K) {
  int nb = K / 32;
  float sum = 0;
  for (int i = 0; i < nb; i++) {
    const uint8_t *blk = row + (size_t)i * 34;
    uint16_t dh;
    memcpy(&dh, blk, 2);
    float d = cw_f16_to_f32(dh);
    const int8_t *q = (const int8_t *)(blk + 2);
    const float *yy = y + (size_t)i * 32;
    for (int j = 0; j < 32; j++) sum += (float)q[j] * d * yy[j];
  }
  return sum;
}
static float or_row_dot(int type, const void *W, int K, int i, const float *x) {
  size_t rb = cw_tensor_nbytes(type, K, 1);
  const uint8_t *row = (const uint8_t *)W + (size_t)i * rb;
  return type == CW_T_Q8_0 ? or_dot_q8_0(row, x, K) : or_dot_q4_0(row, x, K);
}
/* Operand rounding of the GPU engine, a test-only switch (off by default; not
   part of the reference).  The engine's tensor-core GEMV scales each X column
   by a power of two that puts its largest |x| in [2^14, 2^15) and splits it
   into f16 hi + lo parts: 22 significant bits instead of fp32's 24.  With the
   switch on, or_gemv and or_gemvb round X that way before the reference's dot
   products, so a test can measure how far that operand precision alone moves
   a forward pass from the reference. */
static int or_xround = 0;
void or_set_xround(int on) { or_xround = on; }
static void or_round_x(const float *x, int K, float *out) {
  float mx = 0.f;
  for (int k = 0; k < K; k++) mx = fmaxf(mx, fabsf(x[k]));
  if (!(mx > 0.f) || !isfinite(mx)) {
    memcpy(out, x, (size_t)K * sizeof(float));
    return;
  }
  int e;
  frexpf(mx, &e); /* mx in [2^(e-1), 2^e) */
  const int sh = 15 - e;
  for (int k = 0; k < K; k++) {
    const float xs = ldexpf(x[k], sh);
    const float hi = (float)(_Float16)xs;
    const float lo = (float)(_Float16)(xs - hi);
    out[k] = ldexpf(hi + lo, -sh);
  }
}
/* gemv (run.c:1419): y[i] = row i . x */
void or_gemv(int type, const void *W, int K, int M, const float *x, float *y) {
  float *xr = NULL;
  if (or_xround) {
    xr = (float *)malloc((size_t)K * sizeof(float));
    or_round_x(x, K, xr);
    x = xr;
  }
#pragma omp parallel for schedule(static)
  for (int i = 0; i < M; i++) y[i] = or_row_dot(type, W, K, i, x);
  free(xr);
}
/* gemvb (run.c:1577) on the GGUF Q4_0/Q8_0 path: B independent column dots
   per row (run.c:1666-1679). */
void or_gemvb(int type, const void *W, int K, int M, const float *X, int xs, float *Y, int ys, int B) {
  float *xr = NULL;
  if (or_xround) {
    xr = (float *)malloc((size_t)B * K * sizeof(float));
    for (int b = 0; b < B; b++) or_round_x(X + (size_t)b * xs, K, xr + (size_t)b * K);
    X = xr;
    xs = K;
  }
#pragma omp parallel for schedule(static)
  for (int i = 0; i < M; i++)
    for (int b = 0; b < B; b++) Y[(size_t)b * ys + i] = or_row_dot(type, W, K, i, X + (size_t)b * xs);
  free(xr);
}
/* embed_token_to, Q4_0 branch (run.c:1873-1881). */
void or_embed_q4_0(const void *W, int K, int token, float *dst) {
  const uint8_t *row = (const uint8_t *)W + (size_t)token * (size_t)(K / 32) * 18;
  for (int i = 0; i < K / 32; i++) {
    const uint8_t *blk = row + (size_t)i * 18;
    uint16_t dh;
    memcpy(&dh, blk, 2);
    float d = cw_f16_to_f32(dh);
    for (int j = 0; j < 16; j++) {
      dst[i * 32 + j] = (float)((blk[2 + j] & 0xF) - 8) * d;
      dst[i * 32 + j + 16] = (float)((blk[2 + j] >> 4) - 8) * d;
    }
  }
}
/* conv1d_update (run.c:2183-2200): depthwise causal conv, kernel stored
   [channel][4], state [channel][3] oldest first, then SiLU. */
void or_conv1d_update(float *qkv, float *cs, const float *kw, int qkv_dim) {
  for (int c = 0; c < qkv_dim; c++) {
    const float *w = kw + (size_t)c * 4;
    float *st = cs + (size_t)c * 3;
    float cur = qkv[c];
    qkv[c] = st[0] * w[0] + st[1] * w[1] + st[2] * w[2] + cur * w[3];
    st[0] = st[1]; st[1] = st[2]; st[2] = cur;
  }
  for (int c = 0; c < qkv_dim; c++) qkv[c] = or_silu(qkv[c]);
}
/* gdn_step, scalar branches of run.c:2014-2180.  S[hv][i][j]: i indexes the
   key dim, j the value dim.  qkv = [q nkh*D | k nkh*D | v nvh*D]; value head
   hv reads key head hv % nkh. */
void or_gdn_step(const cw_dims *d, float *S, float *qkv, const float *z, const float *decay,
                 const float *beta, const float *wn, float *out) {
  const int D = d->ssm_d, NKH = d->ssm_n_kh, NVH = d->ssm_n_vh;
  float scale = 1.f / sqrtf((float)D);
  float *q0 = qkv, *k0 = qkv + (size_t)NKH * D, *v0 = qkv + (size_t)2 * NKH * D;
  or_l2norm_rows(q0, NKH, D);
  or_l2norm_rows(k0, NKH, D);
  float *sk = (float *)malloc((size_t)D * 2 * sizeof(float)), *delta = sk + D;
  for (int hv = 0; hv < NVH; hv++) {
    int hk = hv % NKH;
    const float *q = q0 + (size_t)hk * D, *k = k0 + (size_t)hk * D, *v = v0 + (size_t)hv * D;
    float *Sh = S + (size_t)hv * D * D;
    float g = expf(decay[hv]), bh = beta[hv];
    for (int i = 0; i < D * D; i++) Sh[i] *= g;
    for (int j = 0; j < D; j++) {
      float s = 0;
      for (int i = 0; i < D; i++) s += Sh[i * D + j] * k[i];
      sk[j] = s;
    }
    for (int j = 0; j < D; j++) delta[j] = bh * (v[j] - sk[j]);
    for (int i = 0; i < D; i++) {
      float ki = k[i];
      for (int j = 0; j < D; j++) Sh[i * D + j] += ki * delta[j];
    }
    float *o = out + (size_t)hv * D;
    for (int j = 0; j < D; j++) {
      float s = 0;
      for (int i = 0; i < D; i++) s += Sh[i * D + j] * q[i];
      o[j] = s * scale;
    }
  }
  free(sk);
  for (int hv = 0; hv < NVH; hv++) {
    float *o = out + (size_t)hv * D;
    const float *zz = z + (size_t)hv * D;
    float ss = 0;
    for (int i = 0; i < D; i++) ss += o[i] * o[i];
    float s = 1.f / sqrtf(ss / D + OR_EPS);
    for (int i = 0; i < D; i++) {
      float gz = zz[i] * (1.f / (1.f + expf(-zz[i])));
      o[i] = wn[i] * o[i] * s * gz;
    }
  }
}
/* rope_tables + rope_apply (run.c:1903-1948), YaRN off: 32 adjacent pairs
   (2i, 2i+1) of the first 64 dims, frequency theta^(-i/64). */
void or_rope(float *q, int n_heads, int head_dim, int pos) {
  float C[32], S[32];
  for (int idx = 0; idx < 32; idx++) {
    float freq = 1.f / powf(OR_THETA, (float)(idx) / (float)64);
    float ang = (float)pos * freq;
    C[idx] = cosf(ang);
    S[idx] = sinf(ang);
  }
  for (int h = 0; h < n_heads; h++) {
    float *v = q + (size_t)h * head_dim;
    for (int idx = 0; idx < 32; idx++) {
      float a = v[2 * idx], b = v[2 * idx + 1];
      v[2 * idx] = a * C[idx] - b * S[idx];
      v[2 * idx + 1] = a * S[idx] + b * C[idx];
    }
  }
}
/* attention_heads_kv, scalar branches (run.c:2362-2409): per q head h (kv head
   h / (NH/NKV)), scores q.k / sqrt(HD) over slots t0..pos, fp32 softmax
   (max-subtract, exp, one reciprocal), t-ascending weighted V sum, then the
   sigmoid gate. */
void or_attention(const cw_dims *d, const float *Kb, const float *Vb, int t0, int pos,
                  const float *q, const float *gate, float *y) {
  const int HD = d->head_dim, NH = d->n_head, NKV = d->n_head_kv, kv_mul = NH / NKV;
  float scale = 1.f / sqrtf((float)HD);
  float *at = (float *)malloc((size_t)(pos + 1) * sizeof(float));
  memset(y, 0, (size_t)NH * HD * sizeof(float));
  for (int h = 0; h < NH; h++) {
    int hkv = h / kv_mul;
    const float *qh = q + (size_t)h * HD;
    for (int t = t0; t <= pos; t++) {
      const float *k = Kb + ((size_t)t * NKV + hkv) * HD;
      float s = 0;
      for (int i = 0; i < HD; i++) s += qh[i] * k[i];
      at[t] = s * scale;
    }
    float mx = at[t0];
    for (int t = t0 + 1; t <= pos; t++) if (at[t] > mx) mx = at[t];
    float sum = 0;
    for (int t = t0; t <= pos; t++) { at[t] = expf(at[t] - mx); sum += at[t]; }
    float inv = 1.f / sum;
    for (int t = t0; t <= pos; t++) at[t] *= inv;
    float *o = y + (size_t)h * HD;
    for (int t = t0; t <= pos; t++) {
      const float *vv = Vb + ((size_t)t * NKV + hkv) * HD;
      for (int i = 0; i < HD; i++) o[i] += at[t] * vv[i];
    }
    for (int i = 0; i < HD; i++) o[i] *= or_sigmoid(gate[(size_t)h * HD + i]);
  }
  free(at);
}
/* argmax_of (run.c:2647-2669): first maximum, strict '>'. */
int or_argmax(const float *lg, int n) {
  int bi = 0;
  float bv = lg[0];
  for (int i = 1; i < n; i++) if (lg[i] > bv) { bv = lg[i]; bi = i; }
  return bi;
}

/* ---- model ---- */
typedef struct {
  const void *attn_norm, *post_norm, *ffn_gate, *ffn_up, *ffn_down;
  const void *qkv, *gate_z, *ssm_a, *ssm_dt, *ssm_alpha, *ssm_beta, *ssm_conv, *ssm_norm, *ssm_out;
  const void *wq, *wk, *wv, *wo, *q_norm, *k_norm;
  int t_gate, t_up, t_down, t_qkv, t_gz, t_al, t_be, t_out, t_q, t_k, t_v, t_o;
} or_layer;

/* the nextn (MTP) block, blk.<n_layer> (run.c:3098-3131) */
typedef struct {
  const void *eh_proj, *enorm, *hnorm, *shn;
  int t_eh, t_q, t_k, t_v, t_o, t_gate, t_up, t_down;
  float *K, *V;                 /* own KV cache [ctx][n_head_kv * head_dim] */
  float *hprev;                 /* NHprev: parked normed hidden */
  int hpos;                     /* mtp_hpos */
  float *emb, *cat, *resid, *ln, *qfull, *qh, *gq, *kh, *vh, *ao, *op, *ffg, *ffu, *oh, *lg;
} or_mtp;

struct or_model {
  cw_dims d;
  int ctx;
  or_mtp mtp;
  void *blobs[2048];
  int nblobs;
  const void *tok_embd, *output, *output_norm;
  or_layer *L;
  float *S, *conv, *K, *V;      /* per linear / full layer */
  int *lin_idx, *full_idx;
  float *x, *xb, *xb2, *hb, *hb2, *qkvb, *zb, *ab, *bb, *qfull, *qh, *gq, *kh, *vh, *yatt, *logits;
  float *layer_out;
};

static void *or_alloc(or_model *m, size_t n) {
  void *p = calloc(1, n ? n : 1);
  if (p) m->blobs[m->nblobs++] = p;
  return p;
}

or_model *or_model_synth(const cw_dims *d, uint64_t seed, int ctx, int threads) {
  or_model *m = (or_model *)calloc(1, sizeof *m);
  if (!m) return NULL;
  m->d = *d;
  m->ctx = ctx;
  const int H = d->n_embd, I = d->n_ff, V = d->n_vocab, QKV = cw_qkv_dim(d);
  const int Z = d->ssm_n_vh * d->ssm_d, QO = d->n_head * d->head_dim, KO = d->n_head_kv * d->head_dim;
  m->L = (or_layer *)or_alloc(m, sizeof(or_layer) * (size_t)(d->n_layer + 1));  /* + the MTP block */
  m->lin_idx = (int *)or_alloc(m, sizeof(int) * (size_t)d->n_layer);
  m->full_idx = (int *)or_alloc(m, sizeof(int) * (size_t)d->n_layer);
  int nlin = 0, nfull = 0;
  for (int l = 0; l < d->n_layer; l++) {
    if (cw_is_linear(d, l)) m->lin_idx[l] = nlin++; else m->full_idx[l] = nfull++;
  }
  int nt = cw_model_tensor_count(&m->d);
  for (int i = 0; i < nt; i++) {
    cw_tensor_desc t;
    cw_model_tensor_desc(&m->d, i, &t);
    void *buf = or_alloc(m, cw_tensor_nbytes(t.type, t.ne0, t.ne1));
    cw_synth_tensor(seed, &t, buf, threads);
    int l = -1;
    char suf[96] = {0};
    if (sscanf(t.name, "blk.%d.%95s", &l, suf) != 2) l = -1;
    if (l < 0) {
      if (!strcmp(t.name, "token_embd.weight")) m->tok_embd = buf;
      else if (!strcmp(t.name, "output.weight")) m->output = buf;
      else if (!strcmp(t.name, "output_norm.weight")) m->output_norm = buf;
      continue;
    }
    or_layer *w = &m->L[l];
#define B(nm, f) else if (!strcmp(suf, nm)) w->f = buf
    if (0) {}
    B("attn_norm.weight", attn_norm); B("post_attention_norm.weight", post_norm);
    B("ffn_gate.weight", ffn_gate); B("ffn_up.weight", ffn_up); B("ffn_down.weight", ffn_down);
    B("attn_qkv.weight", qkv); B("attn_gate.weight", gate_z); B("ssm_a", ssm_a); B("ssm_dt.bias", ssm_dt);
    B("ssm_alpha.weight", ssm_alpha); B("ssm_beta.weight", ssm_beta); B("ssm_conv1d.weight", ssm_conv);
    B("ssm_norm.weight", ssm_norm); B("ssm_out.weight", ssm_out);
    B("attn_q.weight", wq); B("attn_k.weight", wk); B("attn_v.weight", wv); B("attn_output.weight", wo);
    B("attn_q_norm.weight", q_norm); B("attn_k_norm.weight", k_norm);
#undef B
    if (l == d->n_layer) {
      or_mtp *n = &m->mtp;
      if (!strcmp(suf, "nextn.eh_proj.weight")) { n->eh_proj = buf; n->t_eh = t.type; }
      else if (!strcmp(suf, "nextn.enorm.weight")) n->enorm = buf;
      else if (!strcmp(suf, "nextn.hnorm.weight")) n->hnorm = buf;
      else if (!strcmp(suf, "nextn.shared_head_norm.weight")) n->shn = buf;
      else if (!strcmp(suf, "attn_q.weight")) n->t_q = t.type;
      else if (!strcmp(suf, "attn_k.weight")) n->t_k = t.type;
      else if (!strcmp(suf, "attn_v.weight")) n->t_v = t.type;
      else if (!strcmp(suf, "attn_output.weight")) n->t_o = t.type;
      else if (!strcmp(suf, "ffn_gate.weight")) n->t_gate = t.type;
      else if (!strcmp(suf, "ffn_up.weight")) n->t_up = t.type;
      else if (!strcmp(suf, "ffn_down.weight")) n->t_down = t.type;
    }
  }
  if (d->has_mtp) {
    or_mtp *n = &m->mtp;
    n->K = (float *)or_alloc(m, sizeof(float) * (size_t)ctx * KO);
    n->V = (float *)or_alloc(m, sizeof(float) * (size_t)ctx * KO);
#define A_(f, cnt) n->f = (float *)or_alloc(m, sizeof(float) * (size_t)(cnt))
    A_(hprev, H); A_(emb, H); A_(cat, 2 * H); A_(resid, H); A_(ln, H); A_(qfull, 2 * QO); A_(qh, QO);
    A_(gq, QO); A_(kh, KO); A_(vh, KO); A_(ao, QO); A_(op, H); A_(ffg, I); A_(ffu, I); A_(oh, H); A_(lg, V);
#undef A_
    n->hpos = -1;
  }
  m->S = (float *)or_alloc(m, sizeof(float) * (size_t)nlin * d->ssm_n_vh * d->ssm_d * d->ssm_d);
  m->conv = (float *)or_alloc(m, sizeof(float) * (size_t)nlin * QKV * 3);
  m->K = (float *)or_alloc(m, sizeof(float) * (size_t)(nfull ? nfull : 1) * ctx * KO);
  m->V = (float *)or_alloc(m, sizeof(float) * (size_t)(nfull ? nfull : 1) * ctx * KO);
  m->x = (float *)or_alloc(m, 4u * H); m->xb = (float *)or_alloc(m, 4u * H);
  m->xb2 = (float *)or_alloc(m, 4u * H); m->hb = (float *)or_alloc(m, 4u * (size_t)(I > Z ? I : Z));
  m->hb2 = (float *)or_alloc(m, 4u * I); m->qkvb = (float *)or_alloc(m, 4u * QKV);
  m->zb = (float *)or_alloc(m, 4u * Z); m->ab = (float *)or_alloc(m, 4u * d->ssm_n_vh);
  m->bb = (float *)or_alloc(m, 4u * d->ssm_n_vh); m->qfull = (float *)or_alloc(m, 8u * QO);
  m->qh = (float *)or_alloc(m, 4u * QO); m->gq = (float *)or_alloc(m, 4u * QO);
  m->kh = (float *)or_alloc(m, 4u * KO); m->vh = (float *)or_alloc(m, 4u * KO);
  m->yatt = (float *)or_alloc(m, 4u * QO); m->logits = (float *)or_alloc(m, 4u * (size_t)V);
  m->layer_out = (float *)or_alloc(m, 4u * (size_t)H * d->n_layer);
  return m;
}

void or_model_free(or_model *m) {
  if (!m) return;
  for (int i = 0; i < m->nblobs; i++) free(m->blobs[i]);
  free(m);
}

void or_reset(or_model *m) {
  const cw_dims *d = &m->d;
  m->mtp.hpos = -1;
  int nlin = 0;
  for (int l = 0; l < d->n_layer; l++) nlin += cw_is_linear(d, l);
  memset(m->S, 0, sizeof(float) * (size_t)nlin * d->ssm_n_vh * d->ssm_d * d->ssm_d);
  memset(m->conv, 0, sizeof(float) * (size_t)nlin * cw_qkv_dim(d) * 3);
}

static void or_resadd(float *x, const float *dlt, int n) { for (int i = 0; i < n; i++) x[i] += dlt[i]; }

/* mlp (run.c:2205, unfused semantics): gate, up, silu(gate)*up, down, residual. */
static void or_mlp(or_model *m, const or_layer *w) {
  const cw_dims *d = &m->d;
  or_gemv(CW_T_Q4_0, w->ffn_gate, d->n_embd, d->n_ff, m->xb, m->hb);
  or_gemv(CW_T_Q4_0, w->ffn_up, d->n_embd, d->n_ff, m->xb, m->hb2);
  for (int i = 0; i < d->n_ff; i++) m->hb[i] = or_silu(m->hb[i]) * m->hb2[i];
  or_gemv(CW_T_Q4_0, w->ffn_down, d->n_ff, d->n_embd, m->hb, m->xb2);
  or_resadd(m->x, m->xb2, d->n_embd);
}
/* layer_linear (run.c:2323-2350). */
static void or_layer_linear(or_model *m, int l) {
  const cw_dims *d = &m->d;
  const or_layer *w = &m->L[l];
  const int H = d->n_embd, NVH = d->ssm_n_vh, QKV = cw_qkv_dim(d), Z = NVH * d->ssm_d;
  int li = m->lin_idx[l];
  or_rmsnorm(m->xb, m->x, (const float *)w->attn_norm, H);
  or_gemv(CW_T_Q4_0, w->qkv, H, QKV, m->xb, m->qkvb);
  or_gemv(CW_T_Q4_0, w->gate_z, H, Z, m->xb, m->zb);
  or_gemv(CW_T_Q4_0, w->ssm_alpha, H, NVH, m->xb, m->ab);
  or_gemv(CW_T_Q4_0, w->ssm_beta, H, NVH, m->xb, m->bb);
  const float *dt = (const float *)w->ssm_dt, *A = (const float *)w->ssm_a;
  for (int i = 0; i < NVH; i++) {
    m->ab[i] = A[i] * or_softplus(m->ab[i] + dt[i]);
    m->bb[i] = or_sigmoid(m->bb[i]);
  }
  or_conv1d_update(m->qkvb, m->conv + (size_t)li * QKV * 3, (const float *)w->ssm_conv, QKV);
  or_gdn_step(d, m->S + (size_t)li * NVH * d->ssm_d * d->ssm_d, m->qkvb, m->zb, m->ab, m->bb,
              (const float *)w->ssm_norm, m->hb);
  or_gemv(CW_T_Q4_0, w->ssm_out, Z, H, m->hb, m->xb2);
  or_resadd(m->x, m->xb2, H);
  or_rmsnorm(m->xb, m->x, (const float *)w->post_norm, H);
  or_mlp(m, w);
}
/* layer_full (run.c:2417-2458). */
static void or_layer_full(or_model *m, int l, int pos) {
  const cw_dims *d = &m->d;
  const or_layer *w = &m->L[l];
  const int H = d->n_embd, HD = d->head_dim, NH = d->n_head, NKV = d->n_head_kv;
  const int QO = NH * HD, KO = NKV * HD;
  int fi = m->full_idx[l];
  or_rmsnorm(m->xb, m->x, (const float *)w->attn_norm, H);
  or_gemv(CW_T_Q4_0, w->wq, H, 2 * QO, m->xb, m->qfull);
  for (int h = 0; h < NH; h++) {
    memcpy(m->qh + (size_t)h * HD, m->qfull + (size_t)h * HD * 2, HD * sizeof(float));
    memcpy(m->gq + (size_t)h * HD, m->qfull + (size_t)h * HD * 2 + HD, HD * sizeof(float));
  }
  or_gemv(CW_T_Q4_0, w->wk, H, KO, m->xb, m->kh);
  or_gemv(CW_T_Q4_0, w->wv, H, KO, m->xb, m->vh);
  for (int h = 0; h < NH; h++) or_rmsnorm(m->qh + (size_t)h * HD, m->qh + (size_t)h * HD, (const float *)w->q_norm, HD);
  for (int h = 0; h < NKV; h++) or_rmsnorm(m->kh + (size_t)h * HD, m->kh + (size_t)h * HD, (const float *)w->k_norm, HD);
  or_rope(m->qh, NH, HD, pos);
  or_rope(m->kh, NKV, HD, pos);
  float *Kb = m->K + (size_t)fi * m->ctx * KO, *Vb = m->V + (size_t)fi * m->ctx * KO;
  memcpy(Kb + (size_t)pos * KO, m->kh, KO * sizeof(float));
  memcpy(Vb + (size_t)pos * KO, m->vh, KO * sizeof(float));
  or_attention(d, Kb, Vb, 0, pos, m->qh, m->gq, m->yatt);
  or_gemv(CW_T_Q4_0, w->wo, QO, H, m->yatt, m->xb2);
  or_resadd(m->x, m->xb2, H);
  or_rmsnorm(m->xb, m->x, (const float *)w->post_norm, H);
  or_mlp(m, w);
}
/* forward_ex (run.c:2594-2645) without dumps; the per-layer residual stream is
   kept in layer_out (the CWEN_DUMP layerNN files). */
void or_forward(or_model *m, int token, int pos, int need_logits) {
  const cw_dims *d = &m->d;
  or_embed_q4_0(m->tok_embd, d->n_embd, token, m->x);
  for (int l = 0; l < d->n_layer; l++) {
    if (cw_is_linear(d, l)) or_layer_linear(m, l);
    else or_layer_full(m, l, pos);
    memcpy(m->layer_out + (size_t)l * d->n_embd, m->x, sizeof(float) * d->n_embd);
  }
  if (!need_logits) return;
  or_rmsnorm(m->xb, m->x, (const float *)m->output_norm, d->n_embd);
  or_gemv(CW_T_Q4_0, m->output, d->n_embd, d->n_vocab, m->xb, m->logits);
}
const float *or_logits(const or_model *m) { return m->logits; }
const float *or_hidden(const or_model *m) { return m->x; }
const float *or_layer_out(const or_model *m, int l) { return m->layer_out + (size_t)l * m->d.n_embd; }
const float *or_gdn_state(const or_model *m, int layer) {
  return m->S + (size_t)m->lin_idx[layer] * m->d.ssm_n_vh * m->d.ssm_d * m->d.ssm_d;
}
/* ---- MTP (nextn) drafter ---- */
/* mtp_step (run.c:3098-3131): one nextn step at slot pos with input token and
   predecessor hidden h_target; writes K/V at pos of the nextn cache and the
   shared-head-normed hidden into out_h. */
void or_mtp_step(or_model *m, int token, int pos, const float *h_target, float *out_h) {
  const cw_dims *d = &m->d;
  or_mtp *n = &m->mtp;
  const or_layer *w = &m->L[d->n_layer];
  const int H = d->n_embd, I = d->n_ff, HD = d->head_dim, NH = d->n_head, NKV = d->n_head_kv;
  const int QO = NH * HD, KO = NKV * HD;
  or_embed_q4_0(m->tok_embd, H, token, n->emb);
  or_rmsnorm(n->cat, n->emb, (const float *)n->enorm, H);
  or_rmsnorm(n->cat + H, h_target, (const float *)n->hnorm, H);
  or_gemv(n->t_eh, n->eh_proj, 2 * H, H, n->cat, n->resid);
  or_rmsnorm(n->ln, n->resid, (const float *)w->attn_norm, H);
  or_gemv(n->t_q, w->wq, H, 2 * QO, n->ln, n->qfull);
  for (int h = 0; h < NH; h++) {
    memcpy(n->qh + (size_t)h * HD, n->qfull + (size_t)h * HD * 2, HD * sizeof(float));
    memcpy(n->gq + (size_t)h * HD, n->qfull + (size_t)h * HD * 2 + HD, HD * sizeof(float));
  }
  or_gemv(n->t_k, w->wk, H, KO, n->ln, n->kh);
  or_gemv(n->t_v, w->wv, H, KO, n->ln, n->vh);
  for (int h = 0; h < NH; h++) or_rmsnorm(n->qh + (size_t)h * HD, n->qh + (size_t)h * HD, (const float *)w->q_norm, HD);
  for (int h = 0; h < NKV; h++) or_rmsnorm(n->kh + (size_t)h * HD, n->kh + (size_t)h * HD, (const float *)w->k_norm, HD);
  or_rope(n->qh, NH, HD, pos);
  or_rope(n->kh, NKV, HD, pos);
  memcpy(n->K + (size_t)pos * KO, n->kh, KO * sizeof(float));
  memcpy(n->V + (size_t)pos * KO, n->vh, KO * sizeof(float));
  or_attention(d, n->K, n->V, 1, pos, n->qh, n->gq, n->ao);   /* the nextn stream starts at slot 1 */
  or_gemv(n->t_o, w->wo, QO, H, n->ao, n->op);
  or_resadd(n->resid, n->op, H);
  or_rmsnorm(n->ln, n->resid, (const float *)w->post_norm, H);
  or_gemv(n->t_gate, w->ffn_gate, H, I, n->ln, n->ffg);
  or_gemv(n->t_up, w->ffn_up, H, I, n->ln, n->ffu);
  for (int i = 0; i < I; i++) n->ffg[i] = or_silu(n->ffg[i]) * n->ffu[i];
  or_gemv(n->t_down, w->ffn_down, I, H, n->ffg, n->op);
  or_resadd(n->resid, n->op, H);
  or_rmsnorm(out_h, n->resid, (const float *)n->shn, H);
}
/* mtp_commit (run.c:3147-3159): fold the token scored at pos into the nextn
   stream (a step at pos when the previous position was parked), then park
   rmsnorm(x_pre, output_norm) for the next slot. */
void or_mtp_commit(or_model *m, int pos, int token, const float *x_pre) {
  or_mtp *n = &m->mtp;
  if (!m->d.has_mtp) return;
  if (pos >= 1 && n->hpos == pos - 1) or_mtp_step(m, token, pos, n->hprev, n->oh);
  or_rmsnorm(n->hprev, x_pre, (const float *)m->output_norm, m->d.n_embd);
  n->hpos = pos;
}
/* mtp_draft (run.c:3166-3187) after the last committed slot pos_n: chain of
   nextn steps from the pending token, each scored by the shared lm_head. */
int or_mtp_draft(or_model *m, int pos_n, int pend, int32_t *out, int max_d) {
  or_mtp *n = &m->mtp;
  const int H = m->d.n_embd, V = m->d.n_vocab;
  if (!m->d.has_mtp || n->hpos != pos_n || max_d <= 0) return 0;
  int cnt = max_d;
  if (pos_n + cnt >= m->ctx) cnt = m->ctx - 1 - pos_n;
  if (cnt <= 0) return 0;
  float *hprev = (float *)malloc(sizeof(float) * (size_t)H);
  memcpy(hprev, n->hprev, sizeof(float) * (size_t)H);
  int tok = pend;
  for (int t = 0; t < cnt; t++) {
    or_mtp_step(m, tok, pos_n + 1 + t, hprev, n->oh);
    or_gemv(CW_T_Q4_0, m->output, H, V, n->oh, n->lg);
    out[t] = or_argmax(n->lg, V);
    tok = out[t];
    memcpy(hprev, n->oh, sizeof(float) * (size_t)H);
  }
  free(hprev);
  return cnt;
}
const float *or_mtp_hprev(const or_model *m) { return m->mtp.hprev; }
const float *or_mtp_logits(const or_model *m) { return m->mtp.lg; }

/* Serial greedy decode (generate_tokens, run.c:5027-5045): token g is the
   argmax after the prompt and the g previous tokens. */
int or_generate(or_model *m, const int32_t *tokens, int n_tok, int n_gen, int32_t *out) {
  or_reset(m);
  int pos = 0;
  for (int i = 0; i < n_tok; i++) { or_forward(m, tokens[i], pos, i + 1 == n_tok); if (i + 1 < n_tok) pos++; }
  int n = 0;
  for (int g = 0; g < n_gen; g++) {
    if (pos + 1 >= m->ctx) break;
    int next = or_argmax(m->logits, m->d.n_vocab);
    out[n++] = next;
    if (g + 1 == n_gen) break;
    pos++;
    or_forward(m, next, pos, 1);
  }
  return n;
}
