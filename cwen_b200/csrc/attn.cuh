// Gated GQA attention -- host interface (attn.cu).
#pragma once
#include <cuda_runtime.h>

#include "qgemv.cuh"

namespace cw {

struct AttnArgs {
  const float *proj;  // [B][ps]: per q head [q 256 | gate 256] x nh | k nkv*256 | v nkv*256
  int ps, nh, nkv, B;
  const float *qn, *kn;  // attn_q_norm / attn_k_norm [256]
  const float2 *rope;    // (cos, sin) [ctx][32]
  int pos0;              // slot of row 0
  int t0;                // first attendable slot (1 for the MTP stream)
  float *qbuf;           // [B][nh][256]
  float *Kc, *Vc;        // this layer's cache [ctx][nkv][256]
  float *part;           // split partials [B][nh][nch_max][4 + 256]
  int nch_max;           // partial slots per (row, head): attn_splits_max(ctx)
  float *out;            // gated attention output [B][nh*256] (the wo GEMV's raw rows)
};

// Prep + split attention + combine into a.out.
cudaError_t launch_attention(const AttnArgs &a, GemvScratch &s, cudaStream_t st);
int attn_splits_max(int ctx);
size_t attn_part_floats(int bmax, int nh, int nch_max);

// Kernel attributes set once per process (shared-memory carveout).
cudaError_t attn_configure();

}  // namespace cw
