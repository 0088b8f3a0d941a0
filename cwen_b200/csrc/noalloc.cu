// Verify GEMV whose scratch lives in statically allocated device memory.
//
// cwen_cuda_gemvb needs scratch of the engine, which cwen_cuda_init
// allocates: for the default kernel the buffer its X operands are converted
// into and the per-phase flags that publish them; for the earlier kernels the
// split-K partials, the per-tile arrival counters and the prepared X tiles.
// This variant runs the same kernels, chosen by the same shape rule, on
// file-scope __device__ arrays instead, so that a call allocates nothing and
// gives the same bits.  It is
// meant for callers that must not call cudaMalloc on their per-call path: a
// host framework whose caching allocator already reserved the device memory
// (a cudaMalloc there fails or fragments its pool), and latency-critical
// loops where cudaMalloc / cudaFree would synchronize the device and stall
// the other streams.
//
// Limits (the arrays are sized for them; every GPU that loads the library
// holds NA_STATIC_BYTES, about 24 MiB, of them until the process exits):
//   K <= 32768, B <= 16, at most 2048 tiles of 512 rows (M <= 1,048,576),
//   at most 320 CTAs of split-K partials.
#include "engine.cuh"
#include "qgemv.cuh"
#include "qmv.cuh"

namespace cw {
namespace {

constexpr int NA_KMAX = 32768;
constexpr int NA_MAX_CTAS = 320;
constexpr int NA_MAX_TILES = 2048;
constexpr int NA_MAX_DEVICES = 64;
constexpr size_t NA_XF_UINT4 = (size_t)(NA_KMAX / 32) * 128;  // X operands for K <= NA_KMAX (2 KB per 32-block)
constexpr size_t NA_WS_FLOATS = (size_t)NA_MAX_CTAS * 2 * WS_TILE_FLOATS;

static __device__ __align__(256) uint4 g_na_xf[NA_XF_UINT4];
static __device__ __align__(256) int g_na_xexp[QG_MAXB];
static __device__ __align__(256) float g_na_ws[NA_WS_FLOATS];
static __device__ __align__(256) int g_na_cnt[NA_MAX_TILES];
static __device__ __align__(256) int g_na_err[1];
// the default kernel's X operands (per K phase of 512: a 128-byte header and
// 16 blocks x 4 n-tiles x 512 bytes) and its phase flags (zero at load)
constexpr int NA_PHASES = NA_KMAX / 512;
static __device__ __align__(256) uint8_t g_na_qx[(size_t)NA_PHASES * (128 + 16 * 4 * 512)];
static __device__ __align__(256) int g_na_qflag[NA_PHASES];
constexpr size_t NA_STATIC_BYTES = sizeof(g_na_xf) + sizeof(g_na_xexp) + sizeof(g_na_ws) + sizeof(g_na_cnt) +
                                   sizeof(g_na_err) + sizeof(g_na_qx) + sizeof(g_na_qflag);
static_assert(NA_STATIC_BYTES > (23u << 20) && NA_STATIC_BYTES < (25u << 20), "documented as about 24 MiB");

struct NaDevice {
  bool ready = false;
  GemvScratch s;
};
NaDevice g_na[NA_MAX_DEVICES];

// Device addresses of the static arrays, looked up once per device with that
// device current.  The array names are host-side stand-ins in host code; only
// these addresses may be handed to kernels.
int na_setup(int device, int n_sm) {
  NaDevice &D = g_na[device];
  if (D.ready) return CWEN_OK;
  int cur = -1;
  CW_CHECK(cudaGetDevice(&cur));
  if (cur != device) CW_CHECK(cudaSetDevice(device));
  GemvScratch s;
  // the first failing lookup is reported after the caller's device is current again
  cudaError_t e = cudaGetSymbolAddress((void **)&s.xf, g_na_xf);
  if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&s.xexp, g_na_xexp);
  if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&s.ws, g_na_ws);
  if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&s.cnt, g_na_cnt);
  if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&s.err, g_na_err);
  if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&s.qx, g_na_qx);
  if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&s.qflag, g_na_qflag);
  if (cur != device) {
    const cudaError_t e2 = cudaSetDevice(cur);
    if (e == cudaSuccess) e = e2;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cwen_cuda_gemvb_static: static scratch lookup");
  s.kmax = NA_KMAX;
  if (qmv_xbuf_bytes(NA_KMAX) > sizeof(g_na_qx) || qmv_nflags(NA_KMAX) > NA_PHASES) {
    set_error("cwen_cuda_gemvb_static: static X operand buffer too small");
    return CWEN_EINVAL;
  }
  s.G = n_sm < NA_MAX_CTAS ? n_sm : NA_MAX_CTAS;  // the engine's grid when it fits
  s.max_tiles = NA_MAX_TILES;
  D.s = s;
  D.ready = true;
  return CWEN_OK;
}

}  // namespace
}  // namespace cw

using namespace cw;

extern "C" int cwen_cuda_gemvb_static(int wid, const float *dX, int xs, float *dY, int ys, int B, void *stream) {
  Engine &E = engine();
  if (!E.live) {
    set_error("cwen_cuda_gemvb_static: engine not initialised");
    return CWEN_ESTATE;
  }
  if (wid < 0 || wid >= (int)E.mats.size()) {
    set_error("cwen_cuda_gemvb_static: bad weight handle %d", wid);
    return CWEN_EINVAL;
  }
  const QMat &m = E.mats[wid];
  if (B < 1 || B > QG_MAXB || !dX || !dY || xs < m.K || ys < m.M) {
    set_error("cwen_cuda_gemvb_static: need 1 <= B <= %d, xs >= K, ys >= M, non-null X and Y", QG_MAXB);
    return CWEN_EINVAL;
  }
  const int n_tiles = (m.n_mt + QG_TILE_MT - 1) / QG_TILE_MT;
  if (m.K > NA_KMAX || n_tiles > NA_MAX_TILES) {
    set_error("cwen_cuda_gemvb_static: K=%d, M=%d exceed the static scratch (K <= %d, M <= %d)", m.K, m.M, NA_KMAX,
              NA_MAX_TILES * QG_TILE_MT * 16);
    return CWEN_EINVAL;
  }
  if (E.device < 0 || E.device >= NA_MAX_DEVICES) {
    set_error("cwen_cuda_gemvb_static: device %d beyond %d", E.device, NA_MAX_DEVICES);
    return CWEN_EINVAL;
  }
  const int rc = na_setup(E.device, E.n_sm);
  if (rc) return rc;
  GemvScratch &s = g_na[E.device].s;
  s.kern = E.gs.kern;
  s.tc = E.gs.tc;  // the engine's kernel (its weights are in that kernel's layout)
  cudaStream_t st = stream ? (cudaStream_t)stream : E.stream;
  // Clear the split-K sync words this call can use (arrival counters per
  // tile, or partial flags per CTA slot) in case an earlier call stopped
  // part-way or an earlier engine left flag values behind.  The wait-timeout
  // flag is left alone: cwen_cuda_gemvb_static_status reads and clears it.
  const int nsync = n_tiles > 2 * s.G ? n_tiles : 2 * s.G;
  CW_CHECK(cudaMemsetAsync(s.cnt, 0, (size_t)nsync * sizeof(int), st));
  // the same path as cwen_cuda_gemvb (local X for the shapes that allow it,
  // else X preparation + GEMV), so both give the same bits
  CW_CHECK(gemv_run_x(m, dX, xs, B, dY, ys, EPI_STORE, s, st, false));
  return CWEN_OK;
}

extern "C" int cwen_cuda_gemvb_static_status(void *stream) {
  Engine &E = engine();
  if (!E.live) {
    set_error("cwen_cuda_gemvb_static_status: engine not initialised");
    return CWEN_ESTATE;
  }
  if (E.device < 0 || E.device >= NA_MAX_DEVICES || !g_na[E.device].ready) return CWEN_OK;  // no call yet
  GemvScratch &s = g_na[E.device].s;
  CW_CHECK(cudaStreamSynchronize(stream ? (cudaStream_t)stream : E.stream));
  int err = 0;
  CW_CHECK(cudaMemcpy(&err, s.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (!err) return CWEN_OK;
  CW_CHECK(cudaMemset(s.err, 0, sizeof(int)));
  CW_CHECK(cudaMemset(s.cnt, 0, (size_t)s.max_tiles * sizeof(int)));
  set_error("cwen_cuda_gemvb_static: a bounded device wait gave up (code %d); the output of the calls since the "
            "last status check is not valid", err);
  return CWEN_ETIMEOUT;
}
