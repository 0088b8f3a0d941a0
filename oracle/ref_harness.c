/* TEST INFRASTRUCTURE ONLY -- never linked into the product.
 *
 * Builds the reference engine (run.c of maci0/cwen, compiled where it lies,
 * unmodified) into a library with a small C surface so that tests, the
 * golden-fixture script and the CPU baseline of bench.py can call the
 * reference's own kernels and forward passes on seeded synthetic weights.
 *
 * The reference's `main` is renamed so that every static function of the
 * translation unit (gemvb run.c:1577, gdn_step run.c:2014, conv1d_update
 * run.c:2183, attention_heads_kv run.c:2362, forward_ex run.c:2594,
 * forward_block run.c:2752, generate_tokens run.c:5027, ...) is reachable
 * from the wrappers below.  Weights are bound through the reference's own
 * tensor table and validator (rebind_layers_from_tens, run.c:3366), so the
 * shapes the reference enforces are the shapes this harness feeds it.
 */
#define main cwen_reference_cli_main
#include "run.c"
#undef main

#include "synth.h"

#define CWREF_API __attribute__((visibility("default")))

/* ---- kernels on caller buffers ---- */
static Tensor mk_tensor(int type, const void *data, int ne0, int ne1) {
  Tensor t;
  memset(&t, 0, sizeof t);
  t.data = data; t.type = type; t.ne0 = ne0; t.ne1 = ne1;
  return t;
}

/* Y[b*ys + i] = row i of W (GGUF Q4_0 or Q8_0, ne0=K, ne1=M) . X[b*xs ...] */
CWREF_API void cwref_gemvb(int type, const void *W, int K, int M, const float *X, int xs, float *Y, int ys, int B) {
  Tensor t = mk_tensor(type, W, K, M);
  gemvb(&t, X, xs, Y, ys, B);
}
CWREF_API void cwref_gemv(int type, const void *W, int K, int M, const float *x, float *y) {
  Tensor t = mk_tensor(type, W, K, M);
  gemv(&t, x, y);
}
/* Split layout T_Q4_0RS (run.c:98): qs[16*nb*M] contiguous + f16 scales [nb*M].
   qs must be 16-byte aligned (dot_q4_bcol uses aligned loads). */
CWREF_API void cwref_split_q4_0(const void *W, int K, int M, uint8_t *qs, uint16_t *sc) {
  const block_q4_0 *b = (const block_q4_0 *)W;
  size_t nb = (size_t)K / 32;
  for (size_t i = 0; i < nb * (size_t)M; i++) {
    memcpy(qs + i * 16, b[i].qs, 16);
    sc[i] = b[i].d;
  }
}
CWREF_API void cwref_gemvb_split(const uint8_t *qs, const uint16_t *sc, int K, int M, const float *X, int xs, float *Y, int ys, int B) {
  Tensor t = mk_tensor(T_Q4_0RS, qs, K, M);
  t.scales = sc;
  gemvb(&t, X, xs, Y, ys, B);
}

CWREF_API void cwref_rmsnorm(float *o, const float *x, const float *w, int n) { rmsnorm(o, x, w, n); }
CWREF_API void cwref_rope(float *q, int n_heads, int pos) { rope_apply(q, n_heads, pos); }
CWREF_API void cwref_attention(const float *Kb, const float *Vb, int t0, int pos, const float *q, const float *gate, float *y) {
  attention_heads_kv(Kb, Vb, t0, pos, q, gate, y);
}
CWREF_API int cwref_argmax(const float *lg) { return argmax_of(lg); }

/* One GDN layer step on caller-owned state: conv1d_update then gdn_step
   (the order layer_linear uses, run.c:2345-2346).  S [48][128][128],
   conv state [10240][3], conv weight [10240][4], ssm_norm [128]. */
CWREF_API void cwref_gdn_step(float *S, float *conv_state, const float *conv_w, const float *norm_w,
                              float *qkv, float *z, float *decay, float *beta, float *out) {
  float *saveS = Srec, *saveC = Cstate;
  Tensor sc = W[0].ssm_conv, sn = W[0].ssm_norm;
  Srec = S; Cstate = conv_state;
  W[0].ssm_conv = mk_tensor(T_F32, conv_w, CONV_K, QKV_DIM);
  W[0].ssm_norm = mk_tensor(T_F32, norm_w, LSD, 1);
  conv1d_update(0, qkv);
  gdn_step(0, qkv, z, decay, beta, out);
  Srec = saveS; Cstate = saveC; W[0].ssm_conv = sc; W[0].ssm_norm = sn;
}
/* ---- n-gram drafters ---- */
/* Prompt-lookup scan (ngram_draft, run.c:4533). */
CWREF_API int cwref_ngram_draft(const int *h, int hn, int *out, int n_key, int max_d) {
  return ngram_draft(h, hn, out, n_key, max_d);
}
/* A fresh, empty counted map with key length n_key: the allocation of
   alloc_state (run.c:3972-3978), eviction hand back at slot 0. */
CWREF_API int cwref_ngmap_init(int n_key) {
  free(NGM.keys); free(NGM.tok); free(NGM.cnt); free(NGM.used);
  memset(&NGM, 0, sizeof NGM);
  NG_evict_hand = 0;
  Scfg_n_key = n_key;
  NGM.cap = NG_CAP;
  NGM.keys = malloc(sizeof(int) * NG_CAP * (size_t)n_key);
  NGM.tok = malloc(sizeof(int) * NG_CAP);
  NGM.cnt = calloc(NG_CAP, sizeof(int));
  NGM.used = calloc(NG_CAP, 1);
  return (NGM.keys && NGM.tok && NGM.cnt && NGM.used) ? 0 : -1;
}
CWREF_API void cwref_ng_update_range(const int *h, int a, int b) { ng_update_range(h, a, b); }
/* The n-gram branch of a speculative cycle as generate_tokens_spec runs it
   (run.c:4925-4930): map lookups, then the scan when it proposes more. */
CWREF_API int cwref_ng_propose(const int *h, int hn, int *out, int cap) {
  int scan[256];
  if (cap > 256) cap = 256;
  int E = ng_draft_map(h, hn, out, cap);
  int esc = ngram_draft(h, hn, scan, Scfg_n_key, cap);
  if (esc > E) { E = esc; memcpy(out, scan, (size_t)E * sizeof(int)); }
  return E;
}

/* NGC2 persistence of the counted map (ng_save / ng_load, run.c:4656-4716). */
CWREF_API void cwref_ng_save(const char *path) { ng_save(path); }
CWREF_API void cwref_ng_load(const char *path) { ng_load(path); }
CWREF_API long long cwref_ng_used(void) { return (long long)NGM.used_n; }

/* decay/beta transform of layer_linear (run.c:2339-2344). */
CWREF_API void cwref_decay_beta(const float *A, const float *dt, float *ab, float *bb, int n) {
  for (int i = 0; i < n; i++) { ab[i] = A[i] * softplus(ab[i] + dt[i]); bb[i] = sigmoid(bb[i]); }
}

/* ---- whole model on seeded weights ---- */
static void *g_model_blobs[1024];
static int g_model_nblobs;

/* Generate the seeded model (synth.h, reference geometry) in host memory and
   bind it through the reference's tensor table + validator. */
CWREF_API int cwref_load_synth(uint64_t seed, int has_mtp, int threads) {
  cw_dims d;
  cw_dims_full(&d);
  d.has_mtp = has_mtp;
  int nt = cw_model_tensor_count(&d);
  if (nt > (int)(sizeof Tens / sizeof Tens[0]) || nt > (int)(sizeof g_model_blobs / sizeof g_model_blobs[0])) return -1;
  /* a second model in the same process replaces the first */
  for (int i = 0; i < g_model_nblobs; i++) free(g_model_blobs[i]);
  g_model_nblobs = 0;
  Ntens = 0;
  for (int i = 0; i < nt; i++) {
    cw_tensor_desc t;
    cw_model_tensor_desc(&d, i, &t);
    size_t nb = cw_tensor_nbytes(t.type, t.ne0, t.ne1);
    void *buf = aligned_alloc(64, (nb + 63) & ~(size_t)63);
    if (!buf) return -2;
    cw_synth_tensor(seed, &t, buf, threads);
    g_model_blobs[g_model_nblobs++] = buf;
    snprintf(Tnames[Ntens], sizeof Tnames[0], "%s", t.name);
    Tens[Ntens] = mk_tensor(t.type, buf, t.ne0, t.ne1);
    Ntens++;
  }
  rebind_layers_from_tens();
  return 0;
}
/* The tensor blobs cwref_load_synth generated, in descriptor order (returns
   their count), so that another build of this harness in the same process,
   or the engine's upload, can use the same bytes instead of generating them
   again. */
CWREF_API int cwref_blobs(void **out, int cap) {
  int n = g_model_nblobs < cap ? g_model_nblobs : cap;
  for (int i = 0; i < n; i++) out[i] = g_model_blobs[i];
  return g_model_nblobs;
}
/* Bind blobs made by cwref_load_synth of another build (same seed and
   geometry, descriptor order) through the reference's validator. */
CWREF_API int cwref_bind_blobs(void *const *blobs, int n, int has_mtp) {
  cw_dims d;
  cw_dims_full(&d);
  d.has_mtp = has_mtp;
  int nt = cw_model_tensor_count(&d);
  if (nt != n || nt > (int)(sizeof Tens / sizeof Tens[0])) return -1;
  Ntens = 0;
  for (int i = 0; i < nt; i++) {
    cw_tensor_desc t;
    cw_model_tensor_desc(&d, i, &t);
    snprintf(Tnames[Ntens], sizeof Tnames[0], "%s", t.name);
    Tens[Ntens] = mk_tensor(t.type, blobs[i], t.ne0, t.ne1);
    Ntens++;
  }
  rebind_layers_from_tens();
  return 0;
}
/* alloc_state (run.c:3928) after choosing context / speculation / MTP use. */
CWREF_API void cwref_alloc_state(int ctx, int spec, int use_mtp) {
  g_ctx = ctx;
  spec_enabled = spec;
  mtp_use = use_mtp && mtp_on;
  alloc_state();
}
CWREF_API void cwref_reset_state(void) { reset_state(); }
CWREF_API int cwref_pos(void) { return pos_n; }
CWREF_API void cwref_set_pos(int p) { pos_n = p; }
CWREF_API void cwref_forward_ex(int token, int need_logits) { forward_ex(token, need_logits); }
CWREF_API void cwref_forward_block(const int *toks, int B, int nlogits) { forward_block(toks, B, nlogits); }
CWREF_API void cwref_get_logits(float *out) { memcpy(out, logits, (size_t)V * sizeof(float)); }
CWREF_API void cwref_get_blogits(int b, float *out) { memcpy(out, Blogits + (size_t)b * V, (size_t)V * sizeof(float)); }
CWREF_API void cwref_get_x(float *out) { memcpy(out, x, (size_t)H * sizeof(float)); }
CWREF_API void cwref_get_bx(int b, float *out) { memcpy(out, BXres + (size_t)b * H, (size_t)H * sizeof(float)); }
CWREF_API void cwref_get_gdn_state(int layer, float *S_out, float *conv_out) {
  if (S_out) memcpy(S_out, Srec + (size_t)layer * LVH * LSD * LSD, (size_t)LVH * LSD * LSD * 4);
  if (conv_out) memcpy(conv_out, Cstate + (size_t)layer * QKV_DIM * (CONV_K - 1), (size_t)QKV_DIM * (CONV_K - 1) * 4);
}
CWREF_API void cwref_snap_save(void) { snap_save(); }
CWREF_API void cwref_snap_load(void) { snap_load(); }
CWREF_API void cwref_mtp_commit(int pos, int token, const float *x_pre) { mtp_commit(pos, token, x_pre); }
CWREF_API int cwref_mtp_draft(int pend, int *out, int max_d) { return mtp_draft(pend, out, max_d); }

/* The reference's own decode drivers (generate_tokens run.c:5027, which
   routes to generate_tokens_spec run.c:4882 when speculation is on). */
typedef struct { int32_t *out; int n, cap; } ref_sink;
static void ref_sink_fn(int token, int idx, void *ud) {
  (void)idx;
  ref_sink *s = (ref_sink *)ud;
  if (s->n < s->cap) s->out[s->n++] = token;
}
/* forward_ex (run.c:2594-2645) at the current slot with the residual stream
   after every layer copied to layers_out[l*H] -- what CWEN_DUMP writes to
   layerNN_posMM.bin (run.c:2624-2628) -- and the logits to logits_out, without
   the file I/O, so that dumps can start at any slot of a block-prefilled
   context (the reference fixes its dump choice at its first forward). */
CWREF_API void cwref_forward_layers(int token, float *layers_out, float *logits_out) {
  embed_token_to(token, x);
  for (int l = 0; l < L; l++) {
    if (W[l].is_linear) layer_linear(l);
    else layer_full(l);
    memcpy(layers_out + (size_t)l * H, x, (size_t)H * sizeof(float));
  }
  rmsnorm(xb, x, (const float *)output_norm.data, H);
  gemv(&output, xb, logits);
  memcpy(logits_out, logits, (size_t)V * sizeof(float));
}
/* One iteration of generate_tokens' loop (run.c:5033-5041) after a prefill:
   the next slot, forward_ex of the token, the argmax of its logits. */
CWREF_API int cwref_decode_step(int token) {
  pos_n++;
  forward_ex(token, 1);
  return argmax_logits();
}
CWREF_API int cwref_generate(const int32_t *tokens, int n_tok, int n_gen, int32_t *out) {
  ref_sink s = {out, 0, n_gen};
  reset_state();
  return generate_tokens(tokens, n_tok, n_gen, ref_sink_fn, &s);
}
/* Speculation knobs (spec_config_init run.c:4021 semantics). */
CWREF_API void cwref_spec_config(int max_draft, int min_draft, int n_key, int cooldown) {
  Scfg_max_draft = max_draft; Scfg_min_draft = min_draft; Scfg_n_key = n_key; Scfg_cooldown = cooldown;
}
CWREF_API int cwref_dims(int *out16) {
  int v[16] = {H, I, V, L, NH, NKV, HD, NROT, LKH, LVH, LSD, CONV_K, QKV_DIM, FULL_INT, MAX_SEQ, SPEC_BMAX};
  memcpy(out16, v, sizeof v);
  return 16;
}
CWREF_API int cwref_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
