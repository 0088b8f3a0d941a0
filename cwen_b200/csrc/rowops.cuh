// Host launchers of the row-wise kernels (rowops.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "qgemv.cuh"

namespace cw {

// Up to 16 token ids passed by value in the kernel parameters, so a launch
// never depends on a host staging buffer outliving it.
struct Toks16 {
  int t[16];
};

cudaError_t launch_embed(const uint8_t *emb, int H, int V, const Toks16 &toks, int B, float *x, int *err,
                         cudaStream_t st, const int *dtok = nullptr);
// MTP input rows b < B: [rmsnorm(e_b, we) | rmsnorm(h_b, wh)] (2H) -> GEMV input column b,
// or, with out, the fp32 rows out [B][2H] (for a kernel that takes raw X).
cudaError_t launch_cat_norm_prep(const float *e, const float *h, const float *we, const float *wh, int H, int B,
                                 GemvScratch &s, cudaStream_t st, float *out = nullptr);
// x [B][H] -> rmsnorm(x) * w as GEMV input (and optionally into out [B][H]).
cudaError_t launch_norm_prep(const float *x, const float *w, int H, int B, GemvScratch &s, float *out,
                             cudaStream_t st);
// rows x [B][xs], first K values -> GEMV input.
cudaError_t launch_row_prep(const float *x, int xs, int K, int B, GemvScratch &s, cudaStream_t st);
// First-max argmax of B <= 16 rows of logits (row stride ldl) and the greedy
// walk against blk[0..E], E < B, in one launch: res = [k, ustar, argmax rows...].
// scratch: argmax_part_bytes(B) bytes of device memory whose first word is
// zero before the first launch (the kernel leaves it zero again).
size_t argmax_part_bytes(int bmax);
cudaError_t launch_argmax_walk(const float *lg, int n, int ldl, int B, int E, const Toks16 &blk, void *scratch,
                               int *res, cudaStream_t st);

// Kernel attributes set once per process (shared-memory carveout).
cudaError_t rowops_configure();

}  // namespace cw
