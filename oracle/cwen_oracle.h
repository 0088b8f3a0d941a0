/* TEST INFRASTRUCTURE ONLY: the CPU oracle for the cwen verify-decode path.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it.
 *
 * A scalar C restatement of the reference's algorithm (maci0/cwen run.c),
 * written to follow the reference's non-SIMD code paths operation for
 * operation.  Unlike the reference the geometry is a runtime parameter
 * (cw_dims), so the same code also runs a small model.
 */
#ifndef CWEN_ORACLE_H
#define CWEN_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#include "synth.h"
#ifdef __cplusplus
extern "C" {
#endif

/* ---- kernels ---- */
void or_rmsnorm(float *o, const float *x, const float *w, int n);
void or_gemv(int type, const void *W, int K, int M, const float *x, float *y);
void or_gemvb(int type, const void *W, int K, int M, const float *X, int xs, float *Y, int ys, int B);
/* Test-only: round every GEMV's X to the GPU engine's operand precision
   (f16 hi + lo after a power-of-two column scale) while on != 0. */
void or_set_xround(int on);
void or_embed_q4_0(const void *W, int K, int token, float *dst);
void or_conv1d_update(float *qkv, float *conv_state, const float *conv_w, int qkv_dim);
void or_gdn_step(const cw_dims *d, float *S, float *qkv, const float *z, const float *decay,
                 const float *beta, const float *norm_w, float *out);
void or_rope(float *q, int n_heads, int head_dim, int pos);
void or_attention(const cw_dims *d, const float *Kb, const float *Vb, int t0, int pos,
                  const float *q, const float *gate, float *y);
int or_argmax(const float *lg, int n);

/* ---- model ---- */
typedef struct or_model or_model;
/* Seeded model (synth.h) with geometry d, KV cache for ctx positions. */
or_model *or_model_synth(const cw_dims *d, uint64_t seed, int ctx, int threads);
void or_model_free(or_model *m);
void or_reset(or_model *m);
/* Serial forward of one token at slot pos (forward_ex semantics). */
void or_forward(or_model *m, int token, int pos, int need_logits);
const float *or_logits(const or_model *m);
const float *or_hidden(const or_model *m);
/* Residual stream after layer l of the last or_forward (per-layer dump). */
const float *or_layer_out(const or_model *m, int l);
const float *or_gdn_state(const or_model *m, int layer);
/* MTP (nextn) drafter of a model with d.has_mtp (run.c:3098-3187). */
void or_mtp_step(or_model *m, int token, int pos, const float *h_target, float *out_h);
void or_mtp_commit(or_model *m, int pos, int token, const float *x_pre);
int or_mtp_draft(or_model *m, int pos_n, int pend, int32_t *out, int max_d);
const float *or_mtp_hprev(const or_model *m);
/* logits of the last draft step */
const float *or_mtp_logits(const or_model *m);
/* Serial greedy decode: prefill tokens[0..n_tok), then n_gen argmax tokens. */
int or_generate(or_model *m, const int32_t *tokens, int n_tok, int n_gen, int32_t *out);

#ifdef __cplusplus
}
#endif
#endif
