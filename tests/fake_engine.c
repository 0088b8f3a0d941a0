/* TEST INFRASTRUCTURE ONLY: a stand-in for the GPU engine, i.e. the
 * cwen_cuda_* calls the C host driver (cwen_b200/host/driver.c) makes, over a
 * deterministic toy model whose argmax after token t at slot p is
 * fake_next(t, p).  Linked with driver.c into a test library (see
 * tests/test_driver.py), it runs the serial and speculative drivers on the
 * CPU so their control flow can be compared with a restatement of the
 * reference's loops.  The conventions are the engine's (include/cwen_cuda.h):
 * a block scores rows at slots n_past.., accept walks the drafts, commit(k)
 * keeps rows 0..k. */
#include <stdio.h>
#include <string.h>

#include "cwen_cuda.h"

#define FAKE_BMAX 16

static int g_V = 50, g_P = 7, g_Q = 3, g_ctx = 4096;
static int g_np, g_pending, g_nlog;
static int g_am[FAKE_BMAX], g_blk[FAKE_BMAX];
static long long g_blocks, g_serial;
static char g_err[256] = "no error";

/* vocabulary V; at slots p with p % P == Q the toy model's answer shifts by one
 * (P <= 0: never), so drafted repeats are sometimes rejected */
int fake_config(int V, int P, int Q, int ctx) {
  if (V < 2 || ctx < 1) return -1;
  g_V = V;
  g_P = P;
  g_Q = Q;
  g_ctx = ctx;
  g_np = g_pending = 0;
  g_blocks = g_serial = 0;
  return 0;
}
int fake_next(int t, int p) { return (int)(((long long)t * 7 + 3 + (g_P > 0 && p % g_P == g_Q)) % g_V); }
long long fake_blocks(void) { return g_blocks; }
long long fake_serial(void) { return g_serial; }

const char *cwen_cuda_last_error(void) { return g_err; }
void cwen_host_set_error(const char *msg) { snprintf(g_err, sizeof g_err, "%s", msg ? msg : "?"); }
int cwen_cuda_ctx(void) { return g_ctx; }
int cwen_cuda_n_past(void) { return g_np; }
/* A toy nextn head: it drafts the toy model's answer without the shift, so
 * its drafts are rejected exactly at the shifted slots.  It drafts only when
 * every committed slot has been folded into its stream, in order (the
 * mtp_commit contract, run.c:3143-3159); a fold out of order is counted. */
static int g_mtp, g_mtp_hpos = -1, g_mtp_bad;
int fake_config_mtp(int on) {
  g_mtp = on;
  g_mtp_hpos = -1;
  g_mtp_bad = 0;
  return 0;
}
int fake_mtp_bad(void) { return g_mtp_bad; }
int fake_guess(int t, int p) {
  (void)p;
  return (int)(((long long)t * 7 + 3) % g_V);
}
int cwen_cuda_mtp_ready(void) { return g_mtp; }
int cwen_cuda_mtp_commit_block(int pos0, const int *toks, int n) {
  if (!g_mtp) return CWEN_ESTATE;
  if (!toks || n < 1 || pos0 != g_mtp_hpos + 1 || pos0 + n > g_np) {
    g_mtp_bad++;
    cwen_host_set_error("fake mtp_commit_block: fold out of order");
    return CWEN_EINVAL;
  }
  g_mtp_hpos = pos0 + n - 1;
  return CWEN_OK;
}
int cwen_cuda_mtp_draft(int pend, int *out, int max_d) {
  const int pos_n = g_np - 1;
  if (!g_mtp || g_mtp_hpos != pos_n || max_d <= 0 || g_pending) return 0;
  int n = max_d < FAKE_BMAX ? max_d : FAKE_BMAX;
  if (pos_n + n >= g_ctx) n = g_ctx - 1 - pos_n;
  if (n <= 0) return 0;
  int t = pend;
  for (int i = 0; i < n; i++) {
    t = fake_guess(t, pos_n + 1 + i);
    out[i] = t;
  }
  return n;
}
/* the loader's engine calls: no engine here (the host code's own paths end
 * at these with CWEN_ESTATE, as on a machine without a GPU) */
int cwen_cuda_model_config(const cwen_dims *dims) {
  (void)dims;
  return CWEN_ESTATE;
}
int cwen_cuda_upload(const char *name, int type, const void *host, int ne0, int ne1) {
  (void)name;
  (void)type;
  (void)host;
  (void)ne0;
  (void)ne1;
  return CWEN_ESTATE;
}
int cwen_cuda_model_finalize(void) { return CWEN_ESTATE; }
int cwen_cuda_shard_rows_for(const char *name, int ne1, int *r0, int *r1) {
  (void)name;
  *r0 = 0;
  *r1 = ne1;  /* no shard group: every row */
  return CWEN_OK;
}
int cwen_cuda_model_dims(cwen_dims *d) {
  memset(d, 0, sizeof *d);
  d->n_vocab = g_V;
  return CWEN_OK;
}
int cwen_cuda_reset(void) {
  g_np = 0;
  g_pending = 0;
  g_mtp_hpos = -1;
  return CWEN_OK;
}
int cwen_cuda_forward_block(const int *toks, int B, int nlogits) {
  if (g_pending || !toks || B < 1 || B > FAKE_BMAX || nlogits < -1 || nlogits > B || g_np + B > g_ctx) {
    cwen_host_set_error("fake forward_block: bad call");
    return CWEN_EINVAL;
  }
  for (int j = 0; j < B; j++) {
    if (toks[j] < 0 || toks[j] >= g_V) return CWEN_ERANGE;
    g_blk[j] = toks[j];
    g_am[j] = fake_next(toks[j], g_np + j);
  }
  g_pending = B;
  g_nlog = nlogits;
  g_blocks++;
  return CWEN_OK;
}
int cwen_cuda_accept(int *k_out, int *ustar_out, int *argmax_out) {
  if (!g_pending || g_nlog == 0) return CWEN_ESTATE;
  int k = 0, ustar;
  if (g_nlog == -1) {
    ustar = g_am[g_pending - 1];
  } else {
    while (k < g_nlog - 1 && g_am[k] == g_blk[k + 1]) k++;
    ustar = g_am[k];
  }
  if (k_out) *k_out = k;
  if (ustar_out) *ustar_out = ustar;
  if (argmax_out && g_nlog > 0) memcpy(argmax_out, g_am, (size_t)g_nlog * sizeof(int));
  return CWEN_OK;
}
int cwen_cuda_commit(int k) {
  if (!g_pending || k < 0 || k >= g_pending) return CWEN_EINVAL;
  g_np += k + 1;
  g_pending = 0;
  return CWEN_OK;
}
int cwen_cuda_forward_serial(int token, int need_logits, int *argmax_out) {
  (void)need_logits;
  if (g_pending || g_np >= g_ctx) return CWEN_ESTATE;
  if (token < 0 || token >= g_V) return CWEN_ERANGE;
  if (argmax_out) *argmax_out = fake_next(token, g_np);
  g_np++;
  g_serial++;
  return CWEN_OK;
}
