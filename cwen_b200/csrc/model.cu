// Model binding (by GGUF tensor name), decode state and the block forward
// pass.  Replaces rebind_layers_from_tens (run.c:3366-3408), alloc_state /
// reset_state (run.c:3928-4016), forward_ex (run.c:2594) and forward_block
// (run.c:2752-2779) of the reference.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include "attn.cuh"
#include "engine.cuh"
#include "model.cuh"
#include "rowops.cuh"
#include "shard.cuh"

namespace cw {

int alloc_qmat(QMat &m, int type, int K, int rows, bool pair);
int upload_qmat_rows(int type, const void *host, int ne0, int ne1, QMat &m, int rows_off, int stride, int phase);

static Model g_model;
Model &model() { return g_model; }

static inline int rup16(int x) { return (x + 15) & ~15; }

enum {
  LB_ATTN_NORM = 1 << 0, LB_POST_NORM = 1 << 1, LB_GATE = 1 << 2, LB_UP = 1 << 3, LB_DOWN = 1 << 4,
  LB_QKV = 1 << 5, LB_Z = 1 << 6, LB_A = 1 << 7, LB_DT = 1 << 8, LB_ALPHA = 1 << 9, LB_BETA = 1 << 10,
  LB_CONV = 1 << 11, LB_SSM_NORM = 1 << 12, LB_SSM_OUT = 1 << 13,
  LB_Q = 1 << 14, LB_K = 1 << 15, LB_V = 1 << 16, LB_O = 1 << 17, LB_QN = 1 << 18, LB_KN = 1 << 19,
};
static const uint32_t LB_COMMON = LB_ATTN_NORM | LB_POST_NORM | LB_GATE | LB_UP | LB_DOWN;
static const uint32_t LB_LINEAR = LB_COMMON | LB_QKV | LB_Z | LB_A | LB_DT | LB_ALPHA | LB_BETA | LB_CONV |
                                  LB_SSM_NORM | LB_SSM_OUT;
static const uint32_t LB_FULL = LB_COMMON | LB_Q | LB_K | LB_V | LB_O | LB_QN | LB_KN;
enum { GB_EMB = 1, GB_OUT = 2, GB_ONORM = 4 };
enum {
  MB_ATTN_NORM = 1 << 0, MB_POST_NORM = 1 << 1, MB_Q = 1 << 2, MB_K = 1 << 3, MB_V = 1 << 4, MB_O = 1 << 5,
  MB_QN = 1 << 6, MB_KN = 1 << 7, MB_GATE = 1 << 8, MB_UP = 1 << 9, MB_DOWN = 1 << 10, MB_EH = 1 << 11,
  MB_EN = 1 << 12, MB_HN = 1 << 13, MB_SHN = 1 << 14,
};
static const uint32_t MB_ALL = (1u << 15) - 1;

static void free_qmat(QMat &m) {
  if (m.w) cudaFree(m.w);
  m = QMat();
}

void model_free() {
  Model &M = g_model;
  auto F = [](void *p) {
    if (p) cudaFree(p);
  };
  for (auto &l : M.L) {
    F(l.attn_norm); F(l.post_norm); free_qmat(l.in_proj); free_qmat(l.out_proj); free_qmat(l.gate_up);
    free_qmat(l.down); F(l.ssm_a); F(l.ssm_dt); F(l.conv_w); F(l.ssm_norm); F(l.q_norm); F(l.k_norm);
  }
  F(M.tok_embd); free_qmat(M.lm_head); F(M.output_norm);
  MtpW &T = M.mtp;
  F(T.attn_norm); F(T.post_norm); F(T.q_norm); F(T.k_norm); F(T.enorm); F(T.hnorm); F(T.shared_head_norm);
  free_qmat(T.eh_proj); free_qmat(T.in_proj); free_qmat(T.out_proj); free_qmat(T.gate_up); free_qmat(T.down);
  F(M.x); F(M.proj); F(M.gdn_out); F(M.h); F(M.qbuf); F(M.attn_part); F(M.logits); F(M.best); F(M.walk);
  F(M.attn_o);
  F(M.toks); F(M.err); F(M.rope); F(M.dump); F(M.replay[0]); F(M.replay[1]);
  for (int i = 0; i < 2; i++) {
    for (auto p : M.S[i]) F(p);
    for (auto p : M.conv[i]) F(p);
  }
  for (auto p : M.gin) F(p);
  for (auto p : M.craw) F(p);
  for (auto p : M.delta) F(p);
  for (auto p : M.Kc) F(p);
  for (auto p : M.Vc) F(p);
  F(M.mtp_K); F(M.mtp_V); F(M.mtp_hprev); F(M.mtp_x); F(M.mtp_cat); F(M.mtp_out); F(M.mtp_draft);
  F(M.mtp_emb); F(M.mtp_hin);
  if (M.h_walk) cudaFreeHost(M.h_walk);
  if (M.h_toks) cudaFreeHost(M.h_toks);
  if (M.h_draft) cudaFreeHost(M.h_draft);
  M = Model();
}

static int dev_f32(float *&p, const void *host, size_t n) {
  if (!p) CW_CHECK(cudaMalloc(&p, n * sizeof(float)));
  CW_CHECK(cudaMemcpy(p, host, n * sizeof(float), cudaMemcpyHostToDevice));
  return CWEN_OK;
}

static int shape_err(const char *name, int ne0, int ne1, int want0, int want1) {
  set_error("cwen_cuda_upload: %s: shape (%d,%d), need (%d,%d)", name, ne0, ne1, want0, want1);
  return CWEN_EINVAL;
}

// Bind one matrix into a (fused) QMat.  `rows_off` is its first output row.
static int bind_mat(const char *name, int type, const void *host, int ne0, int ne1, int want0, int want1,
                    QMat &m, int total_rows, int rows_off, int stride_mt, int mt_phase) {
  if (ne0 != want0 || ne1 != want1) return shape_err(name, ne0, ne1, want0, want1);
  if (type != CWEN_T_Q4_0 && type != CWEN_T_Q8_0) {
    set_error("cwen_cuda_upload: %s: type %d, need Q4_0 or Q8_0", name, type);
    return CWEN_EINVAL;
  }
  if (!m.w) {
    int rc = alloc_qmat(m, type, ne0, total_rows, stride_mt == 2);
    if (rc) return rc;
  } else if (m.type != type) {
    set_error("cwen_cuda_upload: %s: all parts of a fused matrix must share one type", name);
    return CWEN_EINVAL;
  }
  return upload_qmat_rows(type, host, ne0, ne1, m, rows_off, stride_mt, mt_phase);
}

// A row-sharded matrix (the FFN and lm_head under a shard group): the full
// GGUF shape is checked, this GPU's rows [r0, r1) of it are uploaded.
static int bind_mat_shard(const char *name, int type, const void *host, int ne0, int ne1, int want0, int want1,
                          QMat &m, int stride_mt, int mt_phase) {
  if (ne0 != want0 || ne1 != want1) return shape_err(name, ne0, ne1, want0, want1);
  int r0, r1;
  shard_rows(want1, 16, r0, r1);
  const size_t rb = (size_t)(ne0 / 32) * (type == CWEN_T_Q8_0 ? 34 : 18);
  return bind_mat(name, type, (const uint8_t *)host + (size_t)r0 * rb, ne0, r1 - r0, want0, r1 - r0, m,
                  (r1 - r0) * stride_mt, 0, stride_mt, mt_phase);
}

static int bind_vec(const char *name, int type, const void *host, int ne0, int ne1, int n, float *&dst) {
  if (type != CWEN_T_F32) {
    set_error("cwen_cuda_upload: %s: type %d, need F32", name, type);
    return CWEN_EINVAL;
  }
  if ((long long)ne0 * ne1 < n) return shape_err(name, ne0, ne1, n, 1);
  return dev_f32(dst, host, (size_t)n);
}

static int upload_layer(int l, const char *suf, int type, const void *host, int ne0, int ne1, const char *name) {
  Model &M = g_model;
  const cwen_dims &d = M.d;
  const int H = d.n_embd, I = d.n_ff;
  LayerW &w = M.L[l];
  int rc = CWEN_OK;
  uint32_t bit = 0;
  if (!strcmp(suf, "attn_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, H, w.attn_norm); bit = LB_ATTN_NORM; }
  else if (!strcmp(suf, "post_attention_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, H, w.post_norm); bit = LB_POST_NORM; }
  // the FFN: this GPU's output rows under a shard group (all of them otherwise)
  else if (!strcmp(suf, "ffn_gate.weight")) { rc = bind_mat_shard(name, type, host, ne0, ne1, H, I, w.gate_up, 2, 0); bit = LB_GATE; }
  else if (!strcmp(suf, "ffn_up.weight")) { rc = bind_mat_shard(name, type, host, ne0, ne1, H, I, w.gate_up, 2, 1); bit = LB_UP; }
  else if (!strcmp(suf, "ffn_down.weight")) { rc = bind_mat_shard(name, type, host, ne0, ne1, I, H, w.down, 1, 0); bit = LB_DOWN; }
  else if (w.linear) {
    const int NVH = d.ssm_n_vh;
    if (!strcmp(suf, "attn_qkv.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, M.QKV, w.in_proj, M.ps_lin, 0, 1, 0); bit = LB_QKV; }
    else if (!strcmp(suf, "attn_gate.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, M.Z, w.in_proj, M.ps_lin, M.QKV, 1, 0); bit = LB_Z; }
    else if (!strcmp(suf, "ssm_alpha.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, NVH, w.in_proj, M.ps_lin, M.a_off, 1, 0); bit = LB_ALPHA; }
    else if (!strcmp(suf, "ssm_beta.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, NVH, w.in_proj, M.ps_lin, M.b_off, 1, 0); bit = LB_BETA; }
    else if (!strcmp(suf, "ssm_a")) { rc = bind_vec(name, type, host, ne0, ne1, NVH, w.ssm_a); bit = LB_A; }
    else if (!strcmp(suf, "ssm_dt.bias")) { rc = bind_vec(name, type, host, ne0, ne1, NVH, w.ssm_dt); bit = LB_DT; }
    else if (!strcmp(suf, "ssm_conv1d.weight")) { rc = bind_vec(name, type, host, ne0, ne1, 4 * M.QKV, w.conv_w); bit = LB_CONV; }
    else if (!strcmp(suf, "ssm_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, d.ssm_d, w.ssm_norm); bit = LB_SSM_NORM; }
    else if (!strcmp(suf, "ssm_out.weight")) { rc = bind_mat(name, type, host, ne0, ne1, M.Z, H, w.out_proj, H, 0, 1, 0); bit = LB_SSM_OUT; }
  } else {
    const int QO = d.n_head * d.head_dim, KO = d.n_head_kv * d.head_dim;
    if (!strcmp(suf, "attn_q.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, 2 * QO, w.in_proj, M.ps_full, 0, 1, 0); bit = LB_Q; }
    else if (!strcmp(suf, "attn_k.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, KO, w.in_proj, M.ps_full, 2 * QO, 1, 0); bit = LB_K; }
    else if (!strcmp(suf, "attn_v.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, KO, w.in_proj, M.ps_full, 2 * QO + KO, 1, 0); bit = LB_V; }
    else if (!strcmp(suf, "attn_output.weight")) { rc = bind_mat(name, type, host, ne0, ne1, QO, H, w.out_proj, H, 0, 1, 0); bit = LB_O; }
    else if (!strcmp(suf, "attn_q_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, d.head_dim, w.q_norm); bit = LB_QN; }
    else if (!strcmp(suf, "attn_k_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, d.head_dim, w.k_norm); bit = LB_KN; }
  }
  if (rc == CWEN_OK) w.bound |= bit;
  return rc;
}

static int upload_mtp(const char *suf, int type, const void *host, int ne0, int ne1, const char *name) {
  Model &M = g_model;
  const cwen_dims &d = M.d;
  const int H = d.n_embd, I = d.n_ff, QO = d.n_head * d.head_dim, KO = d.n_head_kv * d.head_dim;
  MtpW &w = M.mtp;
  int rc = CWEN_OK;
  uint32_t bit = 0;
  if (!strcmp(suf, "attn_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, H, w.attn_norm); bit = MB_ATTN_NORM; }
  else if (!strcmp(suf, "post_attention_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, H, w.post_norm); bit = MB_POST_NORM; }
  else if (!strcmp(suf, "attn_q.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, 2 * QO, w.in_proj, M.ps_full, 0, 1, 0); bit = MB_Q; }
  else if (!strcmp(suf, "attn_k.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, KO, w.in_proj, M.ps_full, 2 * QO, 1, 0); bit = MB_K; }
  else if (!strcmp(suf, "attn_v.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, KO, w.in_proj, M.ps_full, 2 * QO + KO, 1, 0); bit = MB_V; }
  else if (!strcmp(suf, "attn_output.weight")) { rc = bind_mat(name, type, host, ne0, ne1, QO, H, w.out_proj, H, 0, 1, 0); bit = MB_O; }
  else if (!strcmp(suf, "attn_q_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, d.head_dim, w.q_norm); bit = MB_QN; }
  else if (!strcmp(suf, "attn_k_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, d.head_dim, w.k_norm); bit = MB_KN; }
  else if (!strcmp(suf, "ffn_gate.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, I, w.gate_up, 2 * I, 0, 2, 0); bit = MB_GATE; }
  else if (!strcmp(suf, "ffn_up.weight")) { rc = bind_mat(name, type, host, ne0, ne1, H, I, w.gate_up, 2 * I, 0, 2, 1); bit = MB_UP; }
  else if (!strcmp(suf, "ffn_down.weight")) { rc = bind_mat(name, type, host, ne0, ne1, I, H, w.down, H, 0, 1, 0); bit = MB_DOWN; }
  else if (!strcmp(suf, "nextn.eh_proj.weight")) { rc = bind_mat(name, type, host, ne0, ne1, 2 * H, H, w.eh_proj, H, 0, 1, 0); bit = MB_EH; }
  else if (!strcmp(suf, "nextn.enorm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, H, w.enorm); bit = MB_EN; }
  else if (!strcmp(suf, "nextn.hnorm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, H, w.hnorm); bit = MB_HN; }
  else if (!strcmp(suf, "nextn.shared_head_norm.weight")) { rc = bind_vec(name, type, host, ne0, ne1, H, w.shared_head_norm); bit = MB_SHN; }
  if (rc == CWEN_OK) w.bound |= bit;
  return rc;
}

// host: rope cos/sin tables with the reference's float formula (run.c:1903-1931,
// YaRN off): freq_i = 1/powf(1e7, i/64), angle = (float)pos * freq_i.
static int build_rope(int ctx) {
  Model &M = g_model;
  std::vector<float2> t((size_t)ctx * 32);
  for (int p = 0; p < ctx; p++)
    for (int i = 0; i < 32; i++) {
      const float freq = 1.f / powf(1e7f, (float)i / 64.f);
      const float ang = (float)p * freq;
      t[(size_t)p * 32 + i] = make_float2(cosf(ang), sinf(ang));
    }
  CW_CHECK(cudaMalloc(&M.rope, t.size() * sizeof(float2)));
  CW_CHECK(cudaMemcpy(M.rope, t.data(), t.size() * sizeof(float2), cudaMemcpyHostToDevice));
  return CWEN_OK;
}

static int alloc_state() {
  Model &M = g_model;
  Engine &E = engine();
  const cwen_dims &d = M.d;
  const int H = d.n_embd, I = d.n_ff, V = d.n_vocab, bm = E.bmax, ctx = E.ctx;
  const int NVH = d.ssm_n_vh, KO = d.n_head_kv * d.head_dim;
  auto A = [](float *&p, size_t n) -> int {
    CW_CHECK(cudaMalloc(&p, n * sizeof(float)));
    CW_CHECK(cudaMemset(p, 0, n * sizeof(float)));
    return CWEN_OK;
  };
  int rc;
  if ((rc = A(M.x, (size_t)bm * H)) || (rc = A(M.proj, (size_t)bm * M.PS)) ||
      (rc = A(M.gdn_out, (size_t)bm * M.Z)) || (rc = A(M.h, (size_t)bm * I)) ||
      (rc = A(M.qbuf, (size_t)bm * d.n_head * d.head_dim)) || (rc = A(M.logits, (size_t)bm * V)))
    return rc;
  M.nch_max = attn_splits_max(ctx);
  if ((rc = A(M.attn_part, attn_part_floats(bm, d.n_head, M.nch_max)))) return rc;
  if ((rc = A(M.attn_o, (size_t)bm * d.n_head * 256))) return rc;
  CW_CHECK(cudaMalloc(&M.best, argmax_part_bytes(bm)));
  CW_CHECK(cudaMemset(M.best, 0, argmax_part_bytes(bm)));
  CW_CHECK(cudaMalloc(&M.walk, (size_t)(bm + 2) * sizeof(int)));
  CW_CHECK(cudaMalloc(&M.toks, (size_t)bm * sizeof(int)));
  CW_CHECK(cudaMalloc(&M.err, sizeof(int)));
  CW_CHECK(cudaMemset(M.err, 0, sizeof(int)));
  CW_CHECK(cudaMallocHost(&M.h_walk, (size_t)(bm + 2) * sizeof(int)));
  CW_CHECK(cudaMallocHost(&M.h_toks, (size_t)bm * sizeof(int)));
  const int GS = M.QKV + 2 * NVH;
  for (int i = 0; i < 2; i++) {
    M.S[i].assign(M.n_lin, nullptr);
    M.conv[i].assign(M.n_lin, nullptr);
  }
  M.gin.assign(M.n_lin, nullptr);
  M.craw.assign(M.n_lin, nullptr);
  M.delta.assign(M.n_lin, nullptr);
  for (int li = 0; li < M.n_lin; li++) {
    for (int i = 0; i < 2; i++) {
      if ((rc = A(M.S[i][li], (size_t)NVH * 128 * 128)) || (rc = A(M.conv[i][li], (size_t)M.QKV * 3))) return rc;
    }
    if ((rc = A(M.gin[li], (size_t)bm * GS)) || (rc = A(M.craw[li], (size_t)bm * M.QKV)) ||
        (rc = A(M.delta[li], (size_t)bm * M.Z)))
      return rc;
  }
  M.Kc.assign(M.n_full, nullptr);
  M.Vc.assign(M.n_full, nullptr);
  for (int fi = 0; fi < M.n_full; fi++) {
    // slots past the committed prefix are always written before they are read
    CW_CHECK(cudaMalloc(&M.Kc[fi], (size_t)ctx * KO * sizeof(float)));
    CW_CHECK(cudaMalloc(&M.Vc[fi], (size_t)ctx * KO * sizeof(float)));
  }
  for (int i = 0; i < 2; i++) {
    std::vector<GdnLayerPtrs> p(M.n_lin);
    for (int li = 0; li < M.n_lin; li++) p[li] = {M.S[i][li], M.conv[i][li], M.gin[li], M.craw[li], M.delta[li]};
    CW_CHECK(cudaMalloc(&M.replay[i], sizeof(GdnLayerPtrs) * (M.n_lin ? M.n_lin : 1)));
    if (M.n_lin)
      CW_CHECK(cudaMemcpy(M.replay[i], p.data(), sizeof(GdnLayerPtrs) * M.n_lin, cudaMemcpyHostToDevice));
  }
  if ((rc = build_rope(ctx))) return rc;
  if (M.mtp_on) {
    CW_CHECK(cudaMalloc(&M.mtp_K, (size_t)ctx * KO * sizeof(float)));
    CW_CHECK(cudaMalloc(&M.mtp_V, (size_t)ctx * KO * sizeof(float)));
    if ((rc = A(M.mtp_hprev, (size_t)H)) || (rc = A(M.mtp_x, (size_t)bm * H)) || (rc = A(M.mtp_cat, (size_t)bm * 2 * H)) ||
        (rc = A(M.mtp_out, (size_t)bm * H)) || (rc = A(M.mtp_emb, (size_t)bm * H)) || (rc = A(M.mtp_hin, (size_t)bm * H)))
      return rc;
    CW_CHECK(cudaMalloc(&M.mtp_draft, (size_t)3 * (bm + 1) * sizeof(int)));  // walk results per draft step
    CW_CHECK(cudaMallocHost(&M.h_draft, (size_t)(bm + 1) * sizeof(int)));
  }
  return CWEN_OK;
}

// The lm_head GEMV into the logits of rows 0..B-1 (row-sharded under a
// shard group: every GPU then holds all logits after the barrier).
// X: the rows (raw fp32, RMSNorm(X) * norm_w when norm_w is set) for an
// engine whose kernel takes raw X; otherwise the prepared fragments are used.
static cudaError_t lm_head_gemv(int B, const float *X, const float *norm_w, cudaStream_t st) {
  Model &M = g_model;
  Engine &E = engine();
  const int V = M.d.n_vocab, H = M.d.n_embd;
  const bool raw = gemv_raw_x(E.gs);
  auto run = [&]() {
    return raw ? timed_gemv(M.lm_head, B, M.logits, V, EPI_STORE, st, X, H, norm_w)
               : timed_gemv(M.lm_head, B, M.logits, V, EPI_STORE, st);
  };
  if (!shard().on()) return run();
  int r0, r1;
  shard_rows(V, 16, r0, r1);
  shard_target(E.gs, M.logits, r0);
  const cudaError_t e = run();
  shard_untarget(E.gs);
  if (e != cudaSuccess) return e;
  return shard_barrier(st);
}

// ---- the forward pass ----
static int run_layer_block(int l, int B, int pos0, cudaStream_t st) {
  Model &M = g_model;
  Engine &E = engine();
  const cwen_dims &d = M.d;
  LayerW &w = M.L[l];
  const int H = d.n_embd, I = d.n_ff;
  long long &nl = E.prof.launches;
  // attn_norm: inside the in_proj GEMV when the previous ffn_down left the
  // rows' sums of squares (gemv_run_xn), else a row kernel first
  if (w.linear) {
    const int li = w.idx, nxt = M.cur ^ 1;
    CW_CHECK(timed_gemv(w.in_proj, B, M.proj, M.PS, EPI_STORE, st, M.x, H, w.attn_norm));
    GdnLayerArgs g;
    g.proj = M.proj; g.ps = M.PS; g.B = B; g.nkh = d.ssm_n_kh; g.nvh = d.ssm_n_vh;
    g.a_off = M.a_off; g.b_off = M.b_off;
    g.convw = w.conv_w; g.cstate_in = M.conv[M.cur][li]; g.cstate_out = M.conv[nxt][li];
    g.craw = M.craw[li]; g.A = w.ssm_a; g.dt = w.ssm_dt; g.gin = M.gin[li];
    g.S_in = M.S[M.cur][li]; g.S_out = M.S[nxt][li]; g.out = M.gdn_out; g.delta = M.delta[li];
    g.z = M.proj + M.QKV; g.wn = w.ssm_norm;  // gated norm of the head outputs, in the recurrence kernel
    CW_CHECK(launch_gdn_layer(g, st));
    nl += gdn_fusable(d.ssm_n_kh, d.ssm_n_vh) ? 1 : 2;
  } else {
    const int fi = w.idx;
    CW_CHECK(timed_gemv(w.in_proj, B, M.proj, M.PS, EPI_STORE, st, M.x, H, w.attn_norm));
    AttnArgs a;
    a.proj = M.proj; a.ps = M.PS; a.nh = d.n_head; a.nkv = d.n_head_kv; a.B = B;
    a.qn = w.q_norm; a.kn = w.k_norm; a.rope = M.rope; a.pos0 = pos0; a.t0 = 0;
    a.qbuf = M.qbuf; a.Kc = M.Kc[fi]; a.Vc = M.Vc[fi]; a.part = M.attn_part; a.nch_max = M.nch_max; a.out = M.attn_o;
    CW_CHECK(launch_attention(a, E.gs, st));
    nl += 3;
  }
  // ssm_out reads the gated-norm rows raw, wo the attention combine's rows
  // (with the new residual rows' sums of squares for the gate/up GEMV's norm)
  if (w.linear) CW_CHECK(timed_gemv(w.out_proj, B, M.x, H, EPI_ADD, st, M.gdn_out, M.Z, nullptr, true));
  else CW_CHECK(timed_gemv(w.out_proj, B, M.x, H, EPI_ADD, st, M.attn_o, d.n_head * 256, nullptr, true));
  const bool sh = shard().on();
  int r0, r1;
  if (sh) {
    shard_rows(I, 16, r0, r1);
    shard_target(E.gs, M.h, r0);
  }
  // post_attention_norm inside the gate/up GEMV when its shape allows local
  // X, else a row kernel first (gemv_run_xn decides; the launch count follows)
  cudaError_t ge = timed_gemv(w.gate_up, B, M.h, I, EPI_SWIGLU, st, M.x, H, w.post_norm);
  if (sh) {
    shard_untarget(E.gs);
    if (ge == cudaSuccess) ge = shard_barrier(st);
  }
  CW_CHECK(ge);
  // the SwiGLU rows, raw; the new residual's sums of squares for the next
  // layer's attn_norm (sharded: each GPU sees only its rows, so the next
  // layer normalises in a row kernel instead)
  if (sh) {
    shard_rows(H, 16, r0, r1);
    shard_target(E.gs, M.x, r0);
  }
  ge = timed_gemv(w.down, B, M.x, H, EPI_ADD, st, M.h, I, nullptr, !sh && l + 1 < d.n_layer);
  if (sh) {
    shard_untarget(E.gs);
    if (ge == cudaSuccess) ge = shard_barrier(st);
  }
  CW_CHECK(ge);
  if (M.dump_on)
    CW_CHECK(cudaMemcpyAsync(M.dump + (size_t)l * E.bmax * H, M.x, (size_t)B * H * sizeof(float),
                             cudaMemcpyDeviceToDevice, st));
  return CWEN_OK;
}

// ---- MTP (nextn) drafter ----
// nextn steps (mtp_step, run.c:3098-3131) for B consecutive slots pos0.. at
// once: row j takes token toks.t[j] (or, for a single row, the device int at
// dtok) and the predecessor hidden hin + j*H (device); each row writes K/V at
// its slot of the nextn cache and its shared-head-normed hidden to hout + j*H,
// and hout stays the pending GEMV input (for the shared lm_head of a draft).
// Row j attends slots [1, pos0 + j] -- the rows before it in the same call
// included -- so B rows give the bits of B single-row steps in order.
static int mtp_step_dev(int pos0, int B, const Toks16 &toks, const int *dtok, const float *hin, float *hout,
                        cudaStream_t st) {
  Model &M = g_model;
  Engine &E = engine();
  const cwen_dims &d = M.d;
  MtpW &w = M.mtp;
  const int H = d.n_embd, I = d.n_ff;
  const bool raw = gemv_raw_x(E.gs);
  CW_CHECK(launch_embed(M.tok_embd, H, d.n_vocab, toks, B, M.mtp_emb, M.err, st, dtok));
  CW_CHECK(launch_cat_norm_prep(M.mtp_emb, hin, w.enorm, w.hnorm, H, B, E.gs, st, raw ? M.mtp_cat : nullptr));
  if (raw) {
    CW_CHECK(timed_gemv(w.eh_proj, B, M.mtp_x, H, EPI_STORE, st, M.mtp_cat, 2 * H));
    CW_CHECK(timed_gemv(w.in_proj, B, M.proj, M.PS, EPI_STORE, st, M.mtp_x, H, w.attn_norm));
  } else {
    CW_CHECK(timed_gemv(w.eh_proj, B, M.mtp_x, H, EPI_STORE, st));
    CW_CHECK(launch_norm_prep(M.mtp_x, w.attn_norm, H, B, E.gs, nullptr, st));
    CW_CHECK(timed_gemv(w.in_proj, B, M.proj, M.PS, EPI_STORE, st));
  }
  AttnArgs a;
  a.proj = M.proj; a.ps = M.PS; a.nh = d.n_head; a.nkv = d.n_head_kv; a.B = B;
  a.qn = w.q_norm; a.kn = w.k_norm; a.rope = M.rope; a.pos0 = pos0; a.t0 = 1;  // the nextn stream starts at slot 1
  a.qbuf = M.qbuf; a.Kc = M.mtp_K; a.Vc = M.mtp_V; a.part = M.attn_part; a.nch_max = M.nch_max; a.out = M.attn_o;
  CW_CHECK(launch_attention(a, E.gs, st));
  CW_CHECK(timed_gemv(w.out_proj, B, M.mtp_x, H, EPI_ADD, st, M.attn_o, d.n_head * 256));
  if (raw) {
    CW_CHECK(timed_gemv(w.gate_up, B, M.h, I, EPI_SWIGLU, st, M.mtp_x, H, w.post_norm));
  } else {
    CW_CHECK(launch_norm_prep(M.mtp_x, w.post_norm, H, B, E.gs, nullptr, st));
    CW_CHECK(timed_gemv(w.gate_up, B, M.h, I, EPI_SWIGLU, st));
  }
  CW_CHECK(timed_gemv(w.down, B, M.mtp_x, H, EPI_ADD, st, M.h, I));
  CW_CHECK(launch_norm_prep(M.mtp_x, w.shared_head_norm, H, B, E.gs, hout, st));
  // embed, cat_norm_prep, the norm_preps, attention prep/split/combine; the
  // GEMVs (and any X preparation of theirs) are counted by timed_gemv
  E.prof.launches += raw ? 6 : 8;
  return CWEN_OK;
}

static int check_ready(const char *fn) {
  if (!engine().live || !g_model.finalized) {
    set_error("%s: model not finalised (cwen_cuda_init, cwen_cuda_model_config, uploads, "
              "cwen_cuda_model_finalize)", fn);
    return CWEN_ESTATE;
  }
  return CWEN_OK;
}

int forward_block_impl(const int *toks, int B, int nlogits) {
  Model &M = g_model;
  Engine &E = engine();
  const cwen_dims &d = M.d;
  int rc = check_ready("cwen_cuda_forward_block");
  if (rc) return rc;
  if (M.pending) {
    set_error("cwen_cuda_forward_block: previous block not committed (cwen_cuda_commit)");
    return CWEN_ESTATE;
  }
  if (shard().configured && !shard().opened) {
    set_error("cwen_cuda_forward_block: shard group configured but not opened (cwen_cuda_shard_open)");
    return CWEN_ESTATE;
  }
  if (B < 1 || B > E.bmax || nlogits < -1 || nlogits > B) {
    set_error("cwen_cuda_forward_block: need 1 <= B <= %d and -1 <= nlogits <= B", E.bmax);
    return CWEN_EINVAL;
  }
  if (M.n_past + B > E.ctx) {
    set_error("cwen_cuda_forward_block: context full (%d + %d > ctx %d)", M.n_past, B, E.ctx);
    return CWEN_ERANGE;
  }
  for (int b = 0; b < B; b++)
    if (toks[b] < 0 || toks[b] >= d.n_vocab) {
      set_error("token id %d out of range [0,%d)", toks[b], d.n_vocab);
      return CWEN_ERANGE;
    }
  cudaStream_t st = E.stream;
  Toks16 tk;
  memset(&tk, 0, sizeof tk);
  memcpy(tk.t, toks, (size_t)B * sizeof(int));
  CW_CHECK(launch_embed(M.tok_embd, d.n_embd, d.n_vocab, tk, B, M.x, M.err, st));
  E.prof.launches++;
  const int pos0 = M.n_past;
  for (int l = 0; l < d.n_layer; l++) {
    rc = run_layer_block(l, B, pos0, st);
    if (rc) return rc;
  }
  M.pending_nlog = 0;
  if (nlogits != 0) {
    const int r0 = nlogits == -1 ? B - 1 : 0, nr = nlogits == -1 ? 1 : nlogits;
    const float *xr = M.x + (size_t)r0 * d.n_embd;
    if (!gemv_raw_x(E.gs)) {
      CW_CHECK(launch_norm_prep(xr, M.output_norm, d.n_embd, nr, E.gs, nullptr, st));
      E.prof.launches++;
    }
    CW_CHECK(lm_head_gemv(nr, xr, M.output_norm, st));
    // blk = toks of the block: row j's argmax is checked against toks[j+1]
    Toks16 blk;
    memset(&blk, 0, sizeof blk);
    memcpy(blk.t, toks + r0, (size_t)(B - r0) * sizeof(int));
    CW_CHECK(launch_argmax_walk(M.logits, d.n_vocab, d.n_vocab, nr, nlogits == -1 ? 0 : nr - 1, blk, M.best,
                                M.walk, st));
    E.prof.launches += 1;
    CW_CHECK(cudaMemcpyAsync(M.h_walk, M.walk, (size_t)(nr + 2) * sizeof(int), cudaMemcpyDeviceToHost, st));
    M.pending_nlog = nr;
  }
  M.pending = B;
  return CWEN_OK;
}

int commit_impl(int k) {
  Model &M = g_model;
  Engine &E = engine();
  if (!M.pending || k < 0 || k >= M.pending) {
    set_error("cwen_cuda_commit: k=%d outside the pending block of %d rows", k, M.pending);
    return M.pending ? CWEN_EINVAL : CWEN_ESTATE;
  }
  if (k == M.pending - 1) {
    M.cur ^= 1;  // every row kept: the block's final state becomes committed
  } else if (M.n_lin) {
    CW_CHECK(launch_gdn_replay(M.replay[M.cur], M.n_lin, k, M.d.ssm_n_kh, M.d.ssm_n_vh, E.stream));
    E.prof.launches++;
  }
  M.n_past += k + 1;
  M.pending = 0;
  return CWEN_OK;
}

}  // namespace cw

using namespace cw;

extern "C" {

int cwen_cuda_model_config(const cwen_dims *dims) {
  Engine &E = engine();
  Model &M = g_model;
  if (!E.live) {
    set_error("cwen_cuda_model_config: engine not initialised");
    return CWEN_ESTATE;
  }
  if (M.configured) {
    set_error("cwen_cuda_model_config: model already configured");
    return CWEN_ESTATE;
  }
  const cwen_dims &d = *dims;
  if (d.head_dim != 256 || d.n_rot != 64 || d.ssm_d != 128 || d.conv_k != 4 || d.n_embd % 512 ||
      d.n_ff % 512 || d.n_vocab < 1 || d.n_layer < 1 || d.n_head < 1 || d.n_head_kv < 1 ||
      d.n_head % d.n_head_kv || d.ssm_n_kh < 1 || d.ssm_n_vh % d.ssm_n_kh || d.full_interval < 1 ||
      (d.n_head * 256) % 64 || (d.ssm_n_vh * 128) % 64 || d.n_embd > E.gs.kmax || d.n_ff > E.gs.kmax) {
    set_error("cwen_cuda_model_config: unsupported geometry (head_dim 256, n_rot 64, ssm_d 128, conv_k 4, "
              "n_embd and n_ff multiples of 512, value heads a multiple of key heads)");
    return CWEN_EINVAL;
  }
  if (shard().configured && d.n_ff % (16 * shard().world)) {
    set_error("cwen_cuda_model_config: n_ff %d is not a multiple of 16 x %d GPUs", d.n_ff, shard().world);
    return CWEN_EINVAL;
  }
  M.d = d;
  M.QKV = (2 * d.ssm_n_kh + d.ssm_n_vh) * 128;
  M.Z = d.ssm_n_vh * 128;
  M.a_off = M.QKV + M.Z;
  M.b_off = M.a_off + rup16(d.ssm_n_vh);
  M.ps_lin = M.b_off + rup16(d.ssm_n_vh);
  M.ps_full = 2 * d.n_head * 256 + 2 * d.n_head_kv * 256;
  M.PS = M.ps_lin > M.ps_full ? M.ps_lin : M.ps_full;
  M.L.assign(d.n_layer, LayerW());
  M.n_lin = M.n_full = 0;
  for (int l = 0; l < d.n_layer; l++) {
    M.L[l].linear = ((l + 1) % d.full_interval) != 0;
    M.L[l].idx = M.L[l].linear ? M.n_lin++ : M.n_full++;
  }
  M.configured = true;
  return CWEN_OK;
}

int cwen_cuda_upload(const char *name, int type, const void *host, int ne0, int ne1) {
  Model &M = g_model;
  if (!engine().live || !M.configured || M.finalized) {
    set_error("cwen_cuda_upload: call after cwen_cuda_model_config and before cwen_cuda_model_finalize");
    return CWEN_ESTATE;
  }
  if (!name || !host || ne0 <= 0 || ne1 <= 0) {
    set_error("cwen_cuda_upload: bad arguments");
    return CWEN_EINVAL;
  }
  const cwen_dims &d = M.d;
  int rc = CWEN_OK;
  if (!strcmp(name, "token_embd.weight")) {
    if (type != CWEN_T_Q4_0) {
      set_error("cwen_cuda_upload: token_embd.weight: type %d, need Q4_0", type);
      return CWEN_EINVAL;
    }
    if (ne0 != d.n_embd || ne1 != d.n_vocab) return shape_err(name, ne0, ne1, d.n_embd, d.n_vocab);
    const size_t bytes = (size_t)(ne0 / 32) * 18 * ne1;
    if (!M.tok_embd) CW_CHECK(cudaMalloc(&M.tok_embd, bytes));
    CW_CHECK(cudaMemcpy(M.tok_embd, host, bytes, cudaMemcpyHostToDevice));
    M.gbound |= GB_EMB;
    return CWEN_OK;
  }
  if (!strcmp(name, "output.weight")) {
    rc = bind_mat_shard(name, type, host, ne0, ne1, d.n_embd, d.n_vocab, M.lm_head, 1, 0);
    if (!rc) M.gbound |= GB_OUT;
    return rc;
  }
  if (!strcmp(name, "output_norm.weight")) {
    rc = bind_vec(name, type, host, ne0, ne1, d.n_embd, M.output_norm);
    if (!rc) M.gbound |= GB_ONORM;
    return rc;
  }
  int l = -1, n = 0;
  if (sscanf(name, "blk.%d.%n", &l, &n) == 1 && n > 0 && l >= 0) {
    if (l < d.n_layer) return upload_layer(l, name + n, type, host, ne0, ne1, name);
    if (l == d.n_layer) {
      rc = upload_mtp(name + n, type, host, ne0, ne1, name);
      return rc;
    }
  }
  return CWEN_OK;  // tensors the path does not use are ignored, like the reference's lookups
}

int cwen_cuda_model_finalize(void) {
  Model &M = g_model;
  if (!engine().live || !M.configured || M.finalized) {
    set_error("cwen_cuda_model_finalize: out of order");
    return CWEN_ESTATE;
  }
  if ((M.gbound & (GB_EMB | GB_ONORM)) != (GB_EMB | GB_ONORM)) {
    set_error("gguf: missing token_embd.weight or output_norm.weight");
    return CWEN_EINVAL;
  }
  if (!(M.gbound & GB_OUT)) {
    set_error("gguf: missing output.weight (tied embeddings are not supported by this engine)");
    return CWEN_EINVAL;
  }
  for (int l = 0; l < M.d.n_layer; l++) {
    const uint32_t need = M.L[l].linear ? LB_LINEAR : LB_FULL;
    if ((M.L[l].bound & need) != need) {
      set_error("gguf: layer %d incomplete (bound mask 0x%x, need 0x%x)", l, M.L[l].bound, need);
      return CWEN_EINVAL;
    }
  }
  M.mtp_on = M.mtp.bound == MB_ALL;
  if (M.mtp.bound && !M.mtp_on) {
    set_error("gguf: blk.%d (MTP) partially present (mask 0x%x)", M.d.n_layer, M.mtp.bound);
    return CWEN_EINVAL;
  }
  int rc = alloc_state();
  if (rc) return rc;
  if ((rc = shard_alloc_local())) return rc;
  CW_CHECK(cudaDeviceSynchronize());
  M.finalized = true;
  return CWEN_OK;
}

int cwen_cuda_reset(void) {
  Model &M = g_model;
  int rc = check_ready("cwen_cuda_reset");
  if (rc) return rc;
  cudaStream_t st = engine().stream;
  for (int li = 0; li < M.n_lin; li++) {
    CW_CHECK(cudaMemsetAsync(M.S[M.cur][li], 0, (size_t)M.Z * 128 * sizeof(float), st));
    CW_CHECK(cudaMemsetAsync(M.conv[M.cur][li], 0, (size_t)M.QKV * 3 * sizeof(float), st));
  }
  M.n_past = 0;
  M.pending = 0;
  M.mtp_hpos = -1;
  return CWEN_OK;
}

int cwen_cuda_n_past(void) { return g_model.n_past; }

int cwen_cuda_model_dims(cwen_dims *out) {
  if (!out) {
    set_error("cwen_cuda_model_dims: out is NULL");
    return CWEN_EINVAL;
  }
  if (!g_model.configured) {
    set_error("cwen_cuda_model_dims: no model configured");
    return CWEN_ESTATE;
  }
  *out = g_model.d;
  return CWEN_OK;
}

int cwen_cuda_forward_block(const int *toks, int B, int nlogits) {
  if (!toks) {
    set_error("cwen_cuda_forward_block: toks is NULL");
    return CWEN_EINVAL;
  }
  return forward_block_impl(toks, B, nlogits);
}

int cwen_cuda_accept(int *k_out, int *ustar_out, int *argmax_out) {
  Model &M = g_model;
  int rc = check_ready("cwen_cuda_accept");
  if (rc) return rc;
  if (!M.pending || !M.pending_nlog) {
    set_error("cwen_cuda_accept: no pending block with logits");
    return CWEN_ESTATE;
  }
  CW_CHECK(cudaStreamSynchronize(engine().stream));
  int err = 0;
  CW_CHECK(cudaMemcpy(&err, M.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) {
    set_error("device reported a token id out of range");
    return CWEN_ERANGE;
  }
  rc = gemv_status();
  if (rc) return rc;
  if ((rc = shard_status())) return rc;
  if (k_out) *k_out = M.h_walk[0];
  if (ustar_out) *ustar_out = M.h_walk[1];
  if (argmax_out) memcpy(argmax_out, M.h_walk + 2, (size_t)M.pending_nlog * sizeof(int));
  return CWEN_OK;
}

int cwen_cuda_commit(int k) {
  int rc = check_ready("cwen_cuda_commit");
  if (rc) return rc;
  return commit_impl(k);
}

int cwen_cuda_forward_serial(int token, int need_logits, int *argmax_out) {
  int rc = forward_block_impl(&token, 1, need_logits ? 1 : 0);
  if (rc) return rc;
  if (need_logits) {
    rc = cwen_cuda_accept(nullptr, argmax_out, nullptr);
    if (rc) return rc;
  }
  return commit_impl(0);
}

int cwen_cuda_logits(int row, float *host) {
  Model &M = g_model;
  int rc = check_ready("cwen_cuda_logits");
  if (rc) return rc;
  if (row < 0 || row >= engine().bmax || !host) {
    set_error("cwen_cuda_logits: bad row");
    return CWEN_EINVAL;
  }
  CW_CHECK(cudaStreamSynchronize(engine().stream));
  CW_CHECK(cudaMemcpy(host, M.logits + (size_t)row * M.d.n_vocab, (size_t)M.d.n_vocab * sizeof(float),
                      cudaMemcpyDeviceToHost));
  return CWEN_OK;
}

int cwen_cuda_hidden(int row, float *host) {
  Model &M = g_model;
  int rc = check_ready("cwen_cuda_hidden");
  if (rc) return rc;
  if (row < 0 || row >= engine().bmax || !host) {
    set_error("cwen_cuda_hidden: bad row");
    return CWEN_EINVAL;
  }
  CW_CHECK(cudaStreamSynchronize(engine().stream));
  CW_CHECK(cudaMemcpy(host, M.x + (size_t)row * M.d.n_embd, (size_t)M.d.n_embd * sizeof(float),
                      cudaMemcpyDeviceToHost));
  return CWEN_OK;
}

int cwen_cuda_dump_layers(int on) {
  Model &M = g_model;
  int rc = check_ready("cwen_cuda_dump_layers");
  if (rc) return rc;
  if (on && !M.dump)
    CW_CHECK(cudaMalloc(&M.dump, (size_t)M.d.n_layer * engine().bmax * M.d.n_embd * sizeof(float)));
  M.dump_on = on != 0;
  return CWEN_OK;
}

int cwen_cuda_dump_read(int layer, int row, float *host) {
  Model &M = g_model;
  int rc = check_ready("cwen_cuda_dump_read");
  if (rc) return rc;
  if (!M.dump || layer < 0 || layer >= M.d.n_layer || row < 0 || row >= engine().bmax || !host) {
    set_error("cwen_cuda_dump_read: dumps off or bad layer/row");
    return CWEN_EINVAL;
  }
  CW_CHECK(cudaStreamSynchronize(engine().stream));
  CW_CHECK(cudaMemcpy(host, M.dump + ((size_t)layer * engine().bmax + row) * M.d.n_embd,
                      (size_t)M.d.n_embd * sizeof(float), cudaMemcpyDeviceToHost));
  return CWEN_OK;
}

int cwen_cuda_mtp_ready(void) { return engine().live && g_model.finalized && g_model.mtp_on ? 1 : 0; }

int cwen_cuda_mtp_commit(int pos, int token, int row) {
  Model &M = g_model;
  Engine &E = engine();
  int rc = check_ready("cwen_cuda_mtp_commit");
  if (rc) return rc;
  if (!M.mtp_on) {
    set_error("cwen_cuda_mtp_commit: the model has no MTP block (blk.%d.nextn.*)", M.d.n_layer);
    return CWEN_ESTATE;
  }
  if (row < 0 || row >= E.bmax || pos < 0 || pos >= E.ctx) {
    set_error("cwen_cuda_mtp_commit: need 0 <= row < %d and 0 <= pos < ctx %d", E.bmax, E.ctx);
    return CWEN_EINVAL;
  }
  if (token < 0 || token >= M.d.n_vocab) {
    set_error("token id %d out of range [0,%d)", token, M.d.n_vocab);
    return CWEN_ERANGE;
  }
  const int H = M.d.n_embd;
  cudaStream_t st = E.stream;
  // a step at pos when pos-1 is parked; its output is not needed
  if (pos >= 1 && M.mtp_hpos == pos - 1) {
    Toks16 tk;
    memset(&tk, 0, sizeof tk);
    tk.t[0] = token;
    rc = mtp_step_dev(pos, 1, tk, nullptr, M.mtp_hprev, M.mtp_out, st);
    if (rc) return rc;
  }
  CW_CHECK(launch_norm_prep(M.x + (size_t)row * H, M.output_norm, H, 1, E.gs, M.mtp_hprev, st));
  E.prof.launches++;
  M.mtp_hpos = pos;
  return CWEN_OK;
}

int cwen_cuda_mtp_commit_block(int pos0, const int *toks, int n) {
  Model &M = g_model;
  Engine &E = engine();
  int rc = check_ready("cwen_cuda_mtp_commit_block");
  if (rc) return rc;
  if (!M.mtp_on) {
    set_error("cwen_cuda_mtp_commit_block: the model has no MTP block (blk.%d.nextn.*)", M.d.n_layer);
    return CWEN_ESTATE;
  }
  if (!toks || n < 1 || n > E.bmax || pos0 < 0 || pos0 + n > E.ctx) {
    set_error("cwen_cuda_mtp_commit_block: need 1 <= n <= %d rows inside the context", E.bmax);
    return CWEN_EINVAL;
  }
  for (int j = 0; j < n; j++)
    if (toks[j] < 0 || toks[j] >= M.d.n_vocab) {
      set_error("token id %d out of range [0,%d)", toks[j], M.d.n_vocab);
      return CWEN_ERANGE;
    }
  if (pos0 >= 1 && M.mtp_hpos != pos0 - 1) {
    // not contiguous with the parked slot: fold row by row (steps where the reference steps)
    for (int j = 0; j < n; j++) {
      rc = cwen_cuda_mtp_commit(pos0 + j, toks[j], j);
      if (rc) return rc;
    }
    return CWEN_OK;
  }
  const int H = M.d.n_embd;
  cudaStream_t st = E.stream;
  // predecessor hiddens: slot pos0 + j steps on rmsnorm(x_pre of slot pos0 + j - 1)
  // -- the parked one for j = 0, row j - 1 of the last forward otherwise
  const int j0 = pos0 == 0 ? 1 : 0;  // slot 0 only parks (no attendable slot yet)
  if (n > 1) {
    CW_CHECK(launch_norm_prep(M.x, M.output_norm, H, n - 1, E.gs, M.mtp_hin + H, st));
    E.prof.launches++;
  }
  if (j0 == 0) CW_CHECK(cudaMemcpyAsync(M.mtp_hin, M.mtp_hprev, (size_t)H * sizeof(float), cudaMemcpyDeviceToDevice, st));
  if (n > j0) {
    Toks16 tk;
    memset(&tk, 0, sizeof tk);
    for (int j = j0; j < n; j++) tk.t[j - j0] = toks[j];
    rc = mtp_step_dev(pos0 + j0, n - j0, tk, nullptr, M.mtp_hin + (size_t)j0 * H, M.mtp_out, st);
    if (rc) return rc;
  }
  CW_CHECK(launch_norm_prep(M.x + (size_t)(n - 1) * H, M.output_norm, H, 1, E.gs, M.mtp_hprev, st));
  E.prof.launches++;
  M.mtp_hpos = pos0 + n - 1;
  return CWEN_OK;
}

int cwen_cuda_mtp_draft(int pend, int *out, int max_d) {
  Model &M = g_model;
  Engine &E = engine();
  int rc = check_ready("cwen_cuda_mtp_draft");
  if (rc) return rc;
  const int pos_n = M.n_past - 1;
  if (!M.mtp_on || M.mtp_hpos != pos_n || max_d <= 0 || M.pending) return 0;
  if (!out || pend < 0 || pend >= M.d.n_vocab) {
    set_error("cwen_cuda_mtp_draft: need out and a pending token in [0,%d)", M.d.n_vocab);
    return CWEN_EINVAL;
  }
  int n = max_d < E.bmax ? max_d : E.bmax;
  if (pos_n + n >= E.ctx) n = E.ctx - 1 - pos_n;
  if (n <= 0) return 0;
  const int H = M.d.n_embd, V = M.d.n_vocab;
  cudaStream_t st = E.stream;
  const float *hin = M.mtp_hprev;
  Toks16 none;
  memset(&none, 0, sizeof none);
  for (int t = 0; t < n; t++) {
    float *hout = M.mtp_out + (size_t)(t & 1) * H;
    Toks16 tk;
    memset(&tk, 0, sizeof tk);
    tk.t[0] = pend;
    rc = mtp_step_dev(pos_n + 1 + t, 1, tk, t ? M.mtp_draft + 3 * (t - 1) + 1 : nullptr, hin, hout, st);
    if (rc) return rc;
    CW_CHECK(lm_head_gemv(1, hout, nullptr, st));
    CW_CHECK(launch_argmax_walk(M.logits, V, V, 1, 0, none, M.best, M.mtp_draft + 3 * t, st));
    E.prof.launches += 1;
    hin = hout;
  }
  int res[3 * 16];
  CW_CHECK(cudaMemcpyAsync(res, M.mtp_draft, (size_t)3 * n * sizeof(int), cudaMemcpyDeviceToHost, st));
  CW_CHECK(cudaStreamSynchronize(st));
  int err = 0;
  CW_CHECK(cudaMemcpy(&err, M.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) {
    set_error("device reported a token id out of range");
    return CWEN_ERANGE;
  }
  rc = gemv_status();
  if (rc) return rc;
  for (int t = 0; t < n; t++) out[t] = res[3 * t + 1];
  return n;
}

// Hidden-state slots of the nextn stream seen by cwen_cuda_mtp_step.
static float *mtp_slot(int slot) {
  Model &M = g_model;
  const int H = M.d.n_embd;
  if (slot == CWEN_MTP_PARKED) return M.mtp_hprev;
  if (slot == CWEN_MTP_OUT0) return M.mtp_out;
  if (slot == CWEN_MTP_OUT1) return M.mtp_out + H;
  return nullptr;
}

int cwen_cuda_mtp_step(int tok, int pos, int src, int dst) {
  Model &M = g_model;
  Engine &E = engine();
  int rc = check_ready("cwen_cuda_mtp_step");
  if (rc) return rc;
  if (!M.mtp_on) {
    set_error("cwen_cuda_mtp_step: the model has no MTP block (blk.%d.nextn.*)", M.d.n_layer);
    return CWEN_ESTATE;
  }
  if (pos < 1 || pos >= E.ctx || !mtp_slot(src) || (dst != CWEN_MTP_OUT0 && dst != CWEN_MTP_OUT1) || E.bmax < 2) {
    set_error("cwen_cuda_mtp_step: need 1 <= pos < ctx %d, a source slot 0..2 and an output slot 1..2", E.ctx);
    return CWEN_EINVAL;
  }
  if (tok < 0 || tok >= M.d.n_vocab) {
    set_error("token id %d out of range [0,%d)", tok, M.d.n_vocab);
    return CWEN_ERANGE;
  }
  Toks16 tk;
  memset(&tk, 0, sizeof tk);
  tk.t[0] = tok;
  rc = mtp_step_dev(pos, 1, tk, nullptr, mtp_slot(src), mtp_slot(dst), E.stream);
  if (rc) return rc;
  CW_CHECK(cudaStreamSynchronize(E.stream));
  int err = 0;
  CW_CHECK(cudaMemcpy(&err, M.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) {
    set_error("device reported a token id out of range");
    return CWEN_ERANGE;
  }
  return gemv_status();
}

int cwen_cuda_mtp_read(int slot, float *host) {
  Model &M = g_model;
  int rc = check_ready("cwen_cuda_mtp_read");
  if (rc) return rc;
  if (!M.mtp_on || !mtp_slot(slot) || !host) {
    set_error("cwen_cuda_mtp_read: need an MTP model, a slot 0..2 and a host buffer");
    return CWEN_EINVAL;
  }
  CW_CHECK(cudaStreamSynchronize(engine().stream));
  CW_CHECK(cudaMemcpy(host, mtp_slot(slot), (size_t)M.d.n_embd * sizeof(float), cudaMemcpyDeviceToHost));
  return CWEN_OK;
}

int cwen_cuda_gdn_state(int layer, float *S_host, float *conv_host) {
  Model &M = g_model;
  int rc = check_ready("cwen_cuda_gdn_state");
  if (rc) return rc;
  if (layer < 0 || layer >= M.d.n_layer || !M.L[layer].linear) {
    set_error("cwen_cuda_gdn_state: layer %d is not a GDN layer", layer);
    return CWEN_EINVAL;
  }
  const int li = M.L[layer].idx;
  CW_CHECK(cudaStreamSynchronize(engine().stream));
  if (S_host)
    CW_CHECK(cudaMemcpy(S_host, M.S[M.cur][li], (size_t)M.Z * 128 * sizeof(float), cudaMemcpyDeviceToHost));
  if (conv_host)
    CW_CHECK(cudaMemcpy(conv_host, M.conv[M.cur][li], (size_t)M.QKV * 3 * sizeof(float), cudaMemcpyDeviceToHost));
  return CWEN_OK;
}

}  // extern "C"
