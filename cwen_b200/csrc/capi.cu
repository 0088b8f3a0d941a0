// C ABI entry points (include/cwen_cuda.h): engine lifetime and the
// stand-alone verify GEMV.
#include <stdlib.h>
#include <string.h>

#include "engine.cuh"
#include "attn.cuh"
#include "gdn.cuh"
#include "model.cuh"
#include "qmv.cuh"
#include "rowops.cuh"
#include "shard.cuh"

namespace cw {

static Engine g_engine;
static char g_err[512] = "no error";

Engine &engine() { return g_engine; }

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
}

int cuda_fail(cudaError_t e, const char *what) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? CWEN_ENOMEM : CWEN_ECUDA;
}

int ensure_staging(size_t bytes) {
  Engine &E = engine();
  if (E.staging_bytes >= bytes) return CWEN_OK;
  if (E.staging) cudaFree(E.staging);
  E.staging = nullptr;
  E.staging_bytes = 0;
  CW_CHECK(cudaMalloc(&E.staging, bytes));
  E.staging_bytes = bytes;
  return CWEN_OK;
}

int ensure_io(size_t floats) {
  Engine &E = engine();
  if (E.io_floats >= floats) return CWEN_OK;
  if (E.io) cudaFree(E.io);
  E.io = nullptr;
  E.io_floats = 0;
  CW_CHECK(cudaMalloc(&E.io, floats * sizeof(float)));
  E.io_floats = floats;
  return CWEN_OK;
}

// Source row r of the tensor becomes row rows_off + r of the fused matrix;
// with stride 2 (interleaved gate/up) its 8-row group (qmv) or 16-row group
// (the other kernels) lands in every second slot, phase 0 or 1.
int upload_qmat_rows(int type, const void *host, int ne0, int ne1, QMat &m, int rows_off, int stride, int phase) {
  Engine &E = engine();
  const size_t rb = (size_t)(ne0 / 32) * (type == CWEN_T_Q8_0 ? 34 : 18);
  const size_t bytes = rb * (size_t)ne1;
  // Chunk by whole 16-row groups so each repack sees complete m-tiles.
  const size_t max_chunk = (size_t)256 << 20;
  size_t rows_per = (max_chunk / rb) / 16 * 16;
  if (rows_per < 16) rows_per = 16;
  int rc = ensure_staging(rows_per * rb < bytes ? rows_per * rb : bytes);
  if (rc) return rc;
  for (size_t r0 = 0; r0 < (size_t)ne1; r0 += rows_per) {
    const size_t nr = (size_t)ne1 - r0 < rows_per ? (size_t)ne1 - r0 : rows_per;
    CW_CHECK(cudaMemcpyAsync(E.staging, (const uint8_t *)host + r0 * rb, nr * rb, cudaMemcpyHostToDevice, E.stream));
    if (m.kern == GK_QMV)
      CW_CHECK(qmv_repack(m, E.staging, (int)nr, (long long)r0, rows_off / 8 * stride + phase, stride, E.stream));
    else
      CW_CHECK(qmat_repack(m, E.staging, (int)nr, rows_off / 16 * stride + phase + (int)(r0 / 16) * stride, stride,
                           E.stream));
    CW_CHECK(cudaStreamSynchronize(E.stream));
  }
  return CWEN_OK;
}

cudaError_t timed_gemv(const QMat &m, int B, float *Y, int ys, int epi, cudaStream_t st, const float *X, int xs,
                       const float *norm_w, bool want_stats) {
  Engine &E = engine();
  Prof &P = E.prof;
  if (!X) E.prof.launches += 1;
  else if (norm_w) E.prof.launches += gemv_norm_fused(m, X, xs, B, E.gs) ? 1 : 2;
  else E.prof.launches += gemv_uses_local_x(m, X, xs, E.gs) ? 1 : 2;
  auto run = [&]() {
    if (!X) return gemv_run(m, B, Y, ys, epi, E.gs, st);
    if (norm_w) return gemv_run_xn(m, X, xs, norm_w, B, Y, ys, epi, E.gs, st);
    return gemv_run_x(m, X, xs, B, Y, ys, epi, E.gs, st, want_stats);
  };
  if (!P.on) return run();
  if (P.used + 2 > P.ev.size()) {
    for (int i = 0; i < 256; i++) {
      cudaEvent_t e;
      cudaError_t r = cudaEventCreate(&e);
      if (r != cudaSuccess) return r;
      P.ev.push_back(e);
    }
  }
  cudaEvent_t a = P.ev[P.used], b = P.ev[P.used + 1];
  cudaEventRecord(a, st);
  cudaError_t r = run();
  cudaEventRecord(b, st);
  P.used += 2;
  const double wbytes = (double)(m.K / 32) * (m.type == 8 ? 34 : 18) * (double)m.M;
  P.bytes.push_back(wbytes + 4.0 * B * m.K + 4.0 * B * m.M);
  return r;
}

// Error flag of the GEMV's bounded waits; read after a synchronize.  A set
// flag means a kernel gave up on a wait (the arrival counters may be stale,
// so they are cleared too).
int gemv_status() {
  Engine &E = engine();
  int err = 0;
  CW_CHECK(cudaMemcpy(&err, E.gs.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (!err) return CWEN_OK;
  CW_CHECK(cudaMemset(E.gs.err, 0, sizeof(int)));
  CW_CHECK(cudaMemset(E.gs.cnt, 0, (size_t)E.gs.max_tiles * sizeof(int)));
  set_error("verify GEMV: a bounded device wait gave up (code %d)", err);
  return CWEN_ETIMEOUT;
}

int alloc_qmat(QMat &m, int type, int K, int rows, bool pair) {
  Engine &E = engine();
  m.kern = E.gs.kern;  // the layout of the engine's GEMV kernel
  m.tc = m.kern == GK_TC;
  m.type = type;
  m.K = K;
  m.n_mt = (rows + 15) / 16;
  m.M = rows;
  m.pair = pair;
  m.n_ht = (rows + 7) / 8;
  m.G = E.n_sm;
  m.bytes = m.kern == GK_QMV ? qmv_bytes(type, K, m.n_ht) : qmat_bytes(type, K, m.n_mt);
  CW_CHECK(cudaMalloc(&m.w, m.bytes));
  CW_CHECK(cudaMemsetAsync(m.w, 0, m.bytes, engine().stream));
  return CWEN_OK;
}

}  // namespace cw

using namespace cw;

extern "C" {

const char *cwen_cuda_last_error(void) { return g_err; }

// Host-side (C) failures record their message here too (host/host_err.h).
void cwen_host_set_error(const char *msg) { set_error("%s", msg ? msg : "unknown host error"); }

int cwen_cuda_init(int device, int ctx, int bmax) {
  Engine &E = engine();
  if (E.live) {
    set_error("cwen_cuda_init: already initialised");
    return CWEN_ESTATE;
  }
  if (bmax < 1 || bmax > QG_MAXB || ctx < 1) {
    set_error("cwen_cuda_init: bmax must be in [1,%d] and ctx >= 1", QG_MAXB);
    return CWEN_EINVAL;
  }
  CW_CHECK(cudaSetDevice(device));
  CW_CHECK(qgemv_configure());
  CW_CHECK(rowops_configure());
  CW_CHECK(attn_configure());
  CW_CHECK(gdn_configure());
  E.device = device;
  E.ctx = ctx;
  E.bmax = bmax;
  CW_CHECK(cudaDeviceGetAttribute(&E.n_sm, cudaDevAttrMultiProcessorCount, device));
  CW_CHECK(cudaStreamCreateWithFlags(&E.stream, cudaStreamNonBlocking));
  GemvScratch &s = E.gs;
  // the verify-GEMV kernel of this engine: mma.sync (default), CWEN_GEMV=qmv or tcgen05
  const char *gk = getenv("CWEN_GEMV");
  s.kern = gk && !strcmp(gk, "tcgen05") ? GK_TC : (gk && !strcmp(gk, "qmv") ? GK_QMV : GK_MMA);
  s.tc = s.kern == GK_TC;
  s.kmax = 32768;
  s.G = E.n_sm;  // one persistent CTA per SM
  s.max_tiles = 1 << 16;
  CW_CHECK(cudaMalloc(&s.xf, (size_t)(s.kmax / 32) * 128 * sizeof(uint4)));
  CW_CHECK(cudaMemset(s.xf, 0, (size_t)(s.kmax / 32) * 128 * sizeof(uint4)));  // padding columns stay finite
  CW_CHECK(cudaMalloc(&s.xexp, QG_MAXB * sizeof(int)));
  CW_CHECK(cudaMalloc(&s.qx, qmv_xbuf_bytes(s.kmax)));
  CW_CHECK(cudaMalloc(&s.qflag, (size_t)qmv_nflags(s.kmax) * sizeof(int)));
  CW_CHECK(cudaMemset(s.qflag, 0, (size_t)qmv_nflags(s.kmax) * sizeof(int)));
  CW_CHECK(cudaMalloc(&s.ws, gemv_scratch_ws_floats(s.G) * sizeof(float)));
  CW_CHECK(cudaMalloc(&s.cnt, (size_t)s.max_tiles * sizeof(int)));
  CW_CHECK(cudaMemset(s.cnt, 0, (size_t)s.max_tiles * sizeof(int)));
  CW_CHECK(cudaMalloc(&s.err, sizeof(int)));
  CW_CHECK(cudaMemset(s.err, 0, sizeof(int)));
  CW_CHECK(cudaMalloc(&s.stat, (size_t)160 * QG_STAT_COLS * sizeof(float)));
  CW_CHECK(cudaMalloc(&s.stat_next, (size_t)160 * QG_STAT_COLS * sizeof(float)));
  CW_CHECK(cudaMalloc(&E.aw, argmax_part_bytes(QG_MAXB)));
  CW_CHECK(cudaMemset(E.aw, 0, argmax_part_bytes(QG_MAXB)));
  CW_CHECK(cudaMalloc(&E.aw_res, (2 + QG_MAXB) * sizeof(int)));
  E.live = true;
  return CWEN_OK;
}

int cwen_cuda_ctx(void) { return engine().live ? engine().ctx : 0; }
void *cwen_cuda_stream(void) { return engine().live ? (void *)engine().stream : nullptr; }

void cwen_cuda_shutdown(void) {
  Engine &E = engine();
  if (!E.live) return;
  cudaStreamSynchronize(E.stream);
  shard_free();
  model_free();
  gdn_verify_free();
  for (auto &m : E.mats) cudaFree(m.w);
  E.mats.clear();
  for (auto e : E.prof.ev) cudaEventDestroy(e);
  cudaFree(E.gs.xf);
  cudaFree(E.gs.xexp);
  cudaFree(E.gs.qx);
  cudaFree(E.gs.qflag);
  cudaFree(E.gs.ws);
  cudaFree(E.gs.cnt);
  cudaFree(E.gs.err);
  cudaFree(E.gs.stat);
  cudaFree(E.gs.stat_next);
  cudaFree(E.aw);
  cudaFree(E.aw_res);
  if (E.staging) cudaFree(E.staging);
  if (E.io) cudaFree(E.io);
  cudaStreamDestroy(E.stream);
  E = Engine();
}

int cwen_cuda_weight_upload(int type, const void *host, int ne0, int ne1, int *wid) {
  Engine &E = engine();
  if (!E.live) {
    set_error("cwen_cuda_weight_upload: engine not initialised");
    return CWEN_ESTATE;
  }
  if ((type != CWEN_T_Q4_0 && type != CWEN_T_Q8_0) || !host || !wid || ne0 <= 0 || ne1 <= 0 || ne0 % 64 ||
      ne0 > E.gs.kmax) {
    set_error("cwen_cuda_weight_upload: need Q4_0/Q8_0, ne0 a positive multiple of 64 <= %d, ne1 > 0", E.gs.kmax);
    return CWEN_EINVAL;
  }
  QMat m;
  int rc = alloc_qmat(m, type, ne0, ne1, false);
  if (rc) return rc;
  rc = upload_qmat_rows(type, host, ne0, ne1, m, 0, 1, 0);
  if (rc) {
    cudaFree(m.w);
    return rc;
  }
  E.mats.push_back(m);
  *wid = (int)E.mats.size() - 1;
  return CWEN_OK;
}

int cwen_cuda_gemvb(int wid, const float *dX, int xs, float *dY, int ys, int B, void *stream) {
  Engine &E = engine();
  if (!E.live || wid < 0 || wid >= (int)E.mats.size()) {
    set_error("cwen_cuda_gemvb: bad weight handle %d", wid);
    return E.live ? CWEN_EINVAL : CWEN_ESTATE;
  }
  const QMat &m = E.mats[wid];
  if (B < 1 || B > E.bmax || !dX || !dY || xs < m.K || ys < m.M) {
    set_error("cwen_cuda_gemvb: need 1 <= B <= %d, xs >= K, ys >= M", E.bmax);
    return CWEN_EINVAL;
  }
  cudaStream_t st = stream ? (cudaStream_t)stream : E.stream;
  CW_CHECK(timed_gemv(m, B, dY, ys, EPI_STORE, st, dX, xs));
  return CWEN_OK;
}

int cwen_cuda_accept_logits(const float *dlogits, int n, int ldl, int B, const int *blk, int E_drafts, int *res,
                            void *stream) {
  Engine &E = engine();
  if (!E.live) {
    set_error("cwen_cuda_accept_logits: engine not initialised");
    return CWEN_ESTATE;
  }
  if (!dlogits || !res || n < 1 || ldl < n || B < 1 || B > QG_MAXB || E_drafts < 0 || E_drafts >= B ||
      (E_drafts > 0 && !blk)) {
    set_error("cwen_cuda_accept_logits: need logits, 1 <= B <= %d, 0 <= E < B, n <= ldl, blk when E > 0", QG_MAXB);
    return CWEN_EINVAL;
  }
  Toks16 tk;
  memset(&tk, 0, sizeof tk);
  if (E_drafts > 0) memcpy(tk.t, blk, (size_t)(E_drafts + 1) * sizeof(int));
  cudaStream_t st = stream ? (cudaStream_t)stream : E.stream;
  CW_CHECK(launch_argmax_walk(dlogits, n, ldl, B, E_drafts, tk, E.aw, E.aw_res, st));
  E.prof.launches++;
  CW_CHECK(cudaMemcpyAsync(res, E.aw_res, (size_t)(2 + B) * sizeof(int), cudaMemcpyDeviceToHost, st));
  CW_CHECK(cudaStreamSynchronize(st));
  return CWEN_OK;
}

int cwen_cuda_profile(int on) {
  Engine &E = engine();
  if (!E.live) {
    set_error("cwen_cuda_profile: engine not initialised");
    return CWEN_ESTATE;
  }
  CW_CHECK(cudaStreamSynchronize(E.stream));
  E.prof.on = on != 0;
  E.prof.used = 0;
  E.prof.bytes.clear();
  E.prof.launches = 0;
  return CWEN_OK;
}

int cwen_cuda_profile_read(double *gemv_ms, double *gemv_bytes, long long *gemv_calls, long long *launches) {
  Engine &E = engine();
  if (!E.live) {
    set_error("cwen_cuda_profile_read: engine not initialised");
    return CWEN_ESTATE;
  }
  Prof &P = E.prof;
  double ms = 0, by = 0;
  for (size_t i = 0; i + 1 < P.used; i += 2) {
    CW_CHECK(cudaEventSynchronize(P.ev[i + 1]));
    float t = 0;
    CW_CHECK(cudaEventElapsedTime(&t, P.ev[i], P.ev[i + 1]));
    ms += t;
    by += P.bytes[i / 2];
  }
  if (gemv_ms) *gemv_ms = ms;
  if (gemv_bytes) *gemv_bytes = by;
  if (gemv_calls) *gemv_calls = (long long)(P.used / 2);
  if (launches) *launches = P.launches;
  return CWEN_OK;
}

int cwen_cuda_gemvb_host(int wid, const float *hX, int xs, float *hY, int ys, int B) {
  Engine &E = engine();
  if (!E.live || wid < 0 || wid >= (int)E.mats.size()) {
    set_error("cwen_cuda_gemvb_host: bad weight handle %d", wid);
    return E.live ? CWEN_EINVAL : CWEN_ESTATE;
  }
  const QMat &m = E.mats[wid];
  if (B < 1 || B > E.bmax || !hX || !hY || xs < m.K || ys < m.M) {
    set_error("cwen_cuda_gemvb_host: need 1 <= B <= %d, xs >= K, ys >= M", E.bmax);
    return CWEN_EINVAL;
  }
  const size_t nx = (size_t)B * xs, ny = (size_t)B * ys;
  int rc = ensure_io(nx + ny);
  if (rc) return rc;
  float *dX = E.io, *dY = E.io + nx;
  CW_CHECK(cudaMemcpyAsync(dX, hX, nx * sizeof(float), cudaMemcpyHostToDevice, E.stream));
  rc = cwen_cuda_gemvb(wid, dX, xs, dY, ys, B, E.stream);
  if (rc) return rc;
  CW_CHECK(cudaMemcpyAsync(hY, dY, ny * sizeof(float), cudaMemcpyDeviceToHost, E.stream));
  CW_CHECK(cudaStreamSynchronize(E.stream));
  return gemv_status();
}

}  // extern "C"
