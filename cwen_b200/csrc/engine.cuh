// Engine state shared by the C ABI and the model code.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <vector>

#include "../../include/cwen_cuda.h"
#include "qgemv.cuh"

namespace cw {

// Optional device-side timing of the GEMV launches (CUDA events on the
// launching stream), read back by cwen_cuda_profile_read.
struct Prof {
  bool on = false;
  std::vector<cudaEvent_t> ev;  // pairs: [2i] before, [2i+1] after launch i
  std::vector<double> bytes;    // algorithmic bytes of launch i
  size_t used = 0;
  long long launches = 0;       // every kernel this engine launched
};

struct Engine {
  bool live = false;
  int device = -1;
  int ctx = 0, bmax = 0;
  int n_sm = 0;
  cudaStream_t stream = nullptr;
  GemvScratch gs;
  std::vector<QMat> mats;  // stand-alone GEMV weights (cwen_cuda_weight_upload)
  uint8_t *staging = nullptr;  // device staging for GGUF uploads
  size_t staging_bytes = 0;
  void *aw = nullptr;    // argmax + walk scratch of cwen_cuda_accept_logits
  int *aw_res = nullptr; // its result row [2 + 16]
  float *io = nullptr;  // device buffers for the host-buffer entry points
  size_t io_floats = 0;
  Prof prof;
};

// GEMV over already-prepared X with optional event timing + launch counting.
// X != nullptr: raw fp32 X [B][xs] (gemv_run_x), RMSNorm(X) * norm_w with
// norm_w (gemv_run_xn); otherwise prepared fragments.  want_stats: leave the
// output rows' sums of squares for the next GEMV's RMSNorm.
cudaError_t timed_gemv(const QMat &m, int B, float *Y, int ys, int epi, cudaStream_t st, const float *X = nullptr,
                       int xs = 0, const float *norm_w = nullptr, bool want_stats = false);

Engine &engine();
// CWEN_OK, or CWEN_ETIMEOUT when a GEMV gave up on a bounded wait (synchronous).
int gemv_status();
void set_error(const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);

#define CW_CHECK(expr)                                   \
  do {                                                   \
    cudaError_t _e = (expr);                             \
    if (_e != cudaSuccess) return cw::cuda_fail(_e, #expr); \
  } while (0)

// Upload `bytes` of host data to a device buffer through the staging area and
// run `fn(device_src)` on it; used by the repacking uploads.
int ensure_staging(size_t bytes);
int ensure_io(size_t floats);

}  // namespace cw
