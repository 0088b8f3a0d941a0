// Stand-alone GatedDeltaNet verify step with rollback on caller device
// buffers (cwen_cuda_gdn_verify, include/cwen_cuda.h): the kernels of the
// engine's linear-attention layers (gdn.cu) on one layer whose state the
// caller owns.  The per-block scratch the engine keeps per layer (the state
// after the last row, the rows' rank-1 records, the raw conv inputs) is held
// here and grown on demand.
#include "engine.cuh"
#include "gdn.cuh"

namespace cw {

namespace {
struct GdnVerifyScratch {
  float *ws = nullptr;  // S after the block | conv state after the block | craw | gin | delta
  size_t floats = 0;
  cudaStream_t last_stream = nullptr;
};
GdnVerifyScratch g_vs;
}  // namespace

void gdn_verify_free() {
  if (g_vs.ws) cudaFree(g_vs.ws);
  g_vs = GdnVerifyScratch();
}

}  // namespace cw

using namespace cw;

extern "C" int cwen_cuda_gdn_verify(int nkh, int nvh, int B, const float *proj, int ps, const float *convw,
                                    const float *A, const float *dt, const float *wn, float *S, float *conv,
                                    int keep, float *out, void *stream) {
  Engine &E = engine();
  if (!E.live) {
    set_error("cwen_cuda_gdn_verify: engine not initialised");
    return CWEN_ESTATE;
  }
  if (nkh < 1 || nkh > 64 || nvh < 1 || nvh > 256 || B < 1 || B > GDN_MAXB || keep < 0 || keep > B) {
    set_error("cwen_cuda_gdn_verify: need 1 <= nkh <= 64, 1 <= nvh <= 256, 1 <= B <= %d, 0 <= keep <= B", GDN_MAXB);
    return CWEN_EINVAL;
  }
  const int QKV = (2 * nkh + nvh) * 128, Z = nvh * 128, GS = QKV + 2 * nvh;
  if (ps < QKV + Z + 2 * nvh || !proj || !convw || !A || !dt || !wn || !S || !conv || !out) {
    set_error("cwen_cuda_gdn_verify: need ps >= %d (q|k|v|z|alpha|beta) and non-null buffers", QKV + Z + 2 * nvh);
    return CWEN_EINVAL;
  }
  cudaStream_t st = stream ? (cudaStream_t)stream : E.stream;
  if (gdn_fusable(nkh, nvh)) {
    // one launch: the block's rows and the rollback to row keep - 1 on the
    // caller's state in place (no scratch, no copy, no replay)
    GdnLayerArgs g = {};
    g.proj = proj; g.ps = ps; g.B = B; g.nkh = nkh; g.nvh = nvh;
    g.a_off = QKV + Z; g.b_off = QKV + Z + nvh;
    g.convw = convw; g.cstate_in = conv; g.cstate_out = conv;
    g.A = A; g.dt = dt; g.S_in = S; g.S_out = S; g.out = out; g.z = proj + QKV; g.wn = wn;
    CW_CHECK(launch_gdn_fused(g, keep, st));
    return CWEN_OK;
  }
  const size_t nS = (size_t)nvh * 128 * 128;
  const size_t need = nS + (size_t)QKV * 3 + (size_t)GDN_MAXB * ((size_t)QKV + GS + Z);
  if (g_vs.floats < need) {
    // the previous scratch may still be read by work queued on the stream
    CW_CHECK(cudaStreamSynchronize(g_vs.last_stream ? g_vs.last_stream : st));
    if (g_vs.ws) cudaFree(g_vs.ws);
    g_vs.ws = nullptr;
    g_vs.floats = 0;
    CW_CHECK(cudaMalloc(&g_vs.ws, need * sizeof(float)));
    g_vs.floats = need;
  }
  float *S_out = g_vs.ws, *c_out = S_out + nS, *craw = c_out + (size_t)QKV * 3;
  float *gin = craw + (size_t)GDN_MAXB * QKV, *delta = gin + (size_t)GDN_MAXB * GS;

  GdnLayerArgs g;
  g.proj = proj; g.ps = ps; g.B = B; g.nkh = nkh; g.nvh = nvh;
  g.a_off = QKV + Z; g.b_off = QKV + Z + nvh;
  g.convw = convw; g.cstate_in = conv; g.cstate_out = c_out; g.craw = craw;
  g.A = A; g.dt = dt; g.gin = gin;
  g.S_in = S; g.S_out = S_out; g.out = out; g.delta = delta;
  g.z = proj + QKV; g.wn = wn;
  CW_CHECK(launch_gdn_layer(g, st));
  if (keep == B) {
    // every row kept: the block's final state becomes the committed one
    CW_CHECK(cudaMemcpyAsync(S, S_out, nS * sizeof(float), cudaMemcpyDeviceToDevice, st));
    CW_CHECK(cudaMemcpyAsync(conv, c_out, (size_t)QKV * 3 * sizeof(float), cudaMemcpyDeviceToDevice, st));
  } else if (keep > 0) {
    // rows 0..keep-1 replayed onto the committed state in place
    GdnLayerPtrs p;
    p.S = S; p.cstate = conv; p.gin = gin; p.craw = craw; p.delta = delta;
    CW_CHECK(launch_gdn_replay1(p, keep - 1, nkh, nvh, st));
  }
  g_vs.last_stream = st;
  return CWEN_OK;
}
