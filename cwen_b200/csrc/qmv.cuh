// The qmv verify GEMV (qmv.cu, selected with CWEN_GEMV=qmv): launch arguments
// and host entry points.  Raw fp32 X in, optional RMSNorm weight folded in;
// the X operands are converted once per call into a phase buffer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "qgemv.cuh"

namespace cw {

struct QmvArgs {
  const uint8_t *w;  // repacked weights [CTA][32-block][half-tile]
  int K, nblk, n_ht, M;
  bool pair;         // gate/up interleaved by half-tile: SwiGLU output rows
  int G, wm;         // CTAs of the layout, row groups of the warp grid
  const float *x;    // column b at x + b * xs
  int xs, xal;       // xal: rows 16-byte aligned (vector loads)
  const float *xw;   // != nullptr: X = rmsnorm(x) * xw, the row scale applied to the outputs
  int B;
  float *y;
  int ys, epi;
  // row-sharded matrix: rows row0.. of the full output, np > 0 copies of Y
  int row0, np;
  float *yp[QG_MAX_PEERS];
  int *err;
  uint8_t *xg;  // X operands of the call, per phase [header | 16 blocks x NT x 512 B]
  int *flags;   // per phase: the epoch of the call that published it
  int epoch;
};

// Device bytes of a matrix of n_ht half-tiles (8 rows) in this kernel's layout.
size_t qmv_bytes(int type, int K, int n_ht);
// Repack `nrows` GGUF rows at src (device): row a0 + r of the tensor lands in
// half-tile ht_base + ((a0 + r) / 8) * ht_stride, row (a0 + r) % 8.
cudaError_t qmv_repack(const QMat &m, const uint8_t *src, int nrows, long long a0, int ht_base, int ht_stride,
                       cudaStream_t st);
// Y = W * X (epi: store, add into Y, or SiLU(gate) * up of an interleaved
// gate/up matrix), X fp32 rows [B][xs]; with norm_w, X = rmsnorm(x) * norm_w.
cudaError_t qmv_run(const QMat &m, const float *X, int xs, const float *norm_w, int B, float *Y, int ys, int epi,
                    GemvScratch &s, cudaStream_t st);
// Scratch of the X conversion for rows up to kmax long: the operand buffer
// (bytes) and the per-phase flags (ints, zero before the first call).
size_t qmv_xbuf_bytes(int kmax);
int qmv_nflags(int kmax);
cudaError_t qmv_configure();

}  // namespace cw
