// Model weights, decode state and the block forward pass on one GPU.
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "../../include/cwen_cuda.h"
#include "gdn.cuh"
#include "qgemv.cuh"

namespace cw {

struct LayerW {
  bool linear = true;
  int idx = 0;                      // index among linear / full layers
  float *attn_norm = nullptr, *post_norm = nullptr;
  QMat in_proj;                     // GDN: qkv|gate|alpha|beta, attention: q|k|v
  QMat out_proj;                    // ssm_out / attn_output
  QMat gate_up;                     // ffn_gate / ffn_up, 16-row groups interleaved
  QMat down;
  float *ssm_a = nullptr, *ssm_dt = nullptr, *conv_w = nullptr, *ssm_norm = nullptr;
  float *q_norm = nullptr, *k_norm = nullptr;
  uint32_t bound = 0;               // bit per required tensor
};

struct MtpW {
  float *attn_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  float *enorm = nullptr, *hnorm = nullptr, *shared_head_norm = nullptr;
  QMat eh_proj, in_proj, out_proj, gate_up, down;
  uint32_t bound = 0;
};

struct Model {
  cwen_dims d{};
  bool configured = false, finalized = false;
  int QKV = 0, Z = 0, a_off = 0, b_off = 0, ps_lin = 0, ps_full = 0, PS = 0;
  std::vector<LayerW> L;
  int n_lin = 0, n_full = 0;
  uint8_t *tok_embd = nullptr;       // GGUF Q4_0 rows [V][H/32 blocks]
  QMat lm_head;
  float *output_norm = nullptr;
  uint32_t gbound = 0;
  MtpW mtp;
  bool mtp_on = false;

  // decode state
  int n_past = 0;      // tokens in the committed state
  int cur = 0;         // which GDN buffer holds the committed state
  int pending = 0;     // rows of the last block not yet committed
  int pending_nlog = 0;
  float *x = nullptr, *proj = nullptr, *gdn_out = nullptr, *h = nullptr, *qbuf = nullptr;
  float *attn_part = nullptr;
  float *attn_o = nullptr;  // gated attention output rows [bmax][n_head*256]
  int nch_max = 0;
  float *logits = nullptr;
  void *best = nullptr;  // argmax + walk scratch (launch_argmax_walk)
  int *walk = nullptr, *toks = nullptr, *err = nullptr;
  int *h_walk = nullptr, *h_toks = nullptr;  // pinned host mirrors
  float2 *rope = nullptr;
  std::vector<float *> S[2], conv[2], gin, craw, delta;
  GdnLayerPtrs *replay[2] = {nullptr, nullptr};
  std::vector<float *> Kc, Vc;
  float *dump = nullptr;
  bool dump_on = false;
  // MTP stream
  float *mtp_K = nullptr, *mtp_V = nullptr;
  float *mtp_hprev = nullptr;   // parked normed hidden [H]
  int mtp_hpos = -1;
  float *mtp_x = nullptr, *mtp_cat = nullptr, *mtp_out = nullptr;
  float *mtp_emb = nullptr, *mtp_hin = nullptr;  // [bmax][H]: embeddings and predecessor hiddens of a block
  int *mtp_draft = nullptr, *h_draft = nullptr;
};

Model &model();
void model_free();

}  // namespace cw
