// Row-wise producers of verify-GEMV inputs and the reductions they share.
//
// A GEMV input row (one per verify position b) is produced by one CTA, or by
// a thread-block cluster whose CTAs each hold a slice of the row in shared
// memory and exchange the row-wide sums and maxima through distributed shared
// memory, so the norm that precedes a GEMV in the reference (rmsnorm
// run.c:346, the MTP input norms run.c:3100-3102) fuses with the conversion
// of the row into the GEMV's f16 hi/lo fragments.
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"

namespace cw {

constexpr int PREP_THREADS = 512;

// Block-wide max / sum over PREP_THREADS threads (red: >= 32 floats smem).
CW_DEV float block_max(float v, float *red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
  return warp_max(v);
}
// Deterministic block sum: fixed per-thread strided order, fixed tree.
CW_DEV float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
  return warp_sum(v);
}

// Exponent of a column whose largest magnitude is mx: max|x| * 2^e in
// [2^14, 2^15), so that the f16 hi part holds 11 bits and the lo part the next 11.
CW_DEV int xfrag_exponent(float mx) {
  int e = 0;
  if (mx > 0.f && mx <= 3.0e38f) {
    int p;
    frexpf(mx, &p);
    e = 15 - p;
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
  }
  return e;
}

// Emit the GEMV's X operands of column b for the 32-blocks [kb0, kb0 + nkb)
// from v (v[0] is element 32*kb0 of the column); the power-of-two `scale` is
// applied here.  Per 32-block 2 KB (128 uint4): two k16 steps x (hi tile,
// lo tile), a tile 16 columns x 16 K, K-major without swizzle (column n,
// 8-K chunk c at byte (n % 8) * 16 + (n / 8) * 256 + c * 128): the B operand
// layout of the tensor cores.
CW_DEV void emit_xfrag_blocks(const float *v, int kb0, int nkb, int b, uint4 *__restrict__ xf, float scale,
                              bool live) {
  for (int item = threadIdx.x; item < nkb * 4; item += blockDim.x) {
    const int kbl = item >> 2, c = item & 3;
    const float *r = v + kbl * 32 + c * 8;
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float v0 = live ? r[2 * i] * scale : 0.f, v1 = live ? r[2 * i + 1] * scale : 0.f;
      const half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
      const half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
      hi[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      lo[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    uint4 *o = xf + (size_t)(kb0 + kbl) * 128 + (c >> 1) * 64 + (b >> 3) * 16 + (c & 1) * 8 + (b & 7);
    o[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);   // hi tile
    o[32] = make_uint4(lo[0], lo[1], lo[2], lo[3]);  // lo tile, 512 bytes on
  }
}

// The same for the mma.sync kernel (qgemv_mma.cu): per (32-block, n-tile of
// 4 columns) 32 uint4; column b is B-operand column b % 4 (hi parts) and
// b % 4 + 4 (lo parts) of n-tile b / 4, lane (column, t) holding (x[4t],
// x[4t+2]) (x[4t+1], x[4t+3]) (x[4t+16], x[4t+18]) (x[4t+17], x[4t+19]), the
// K order of that kernel's A fragments; nt n-tiles.
CW_DEV void emit_xfrag_blocks_mma(const float *v, int kb0, int nkb, int b, int nt, uint4 *__restrict__ xf,
                                  float scale, bool live) {
  const int g = b & 3, n = b >> 2;
  for (int item = threadIdx.x; item < nkb * 4; item += blockDim.x) {
    const int kbl = item >> 2, t = item & 3;
    const float *r = v + kbl * 32;
    const int js[8] = {4 * t, 4 * t + 2, 4 * t + 1, 4 * t + 3, 4 * t + 16, 4 * t + 18, 4 * t + 17, 4 * t + 19};
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float v0 = live ? r[js[2 * i]] * scale : 0.f, v1 = live ? r[js[2 * i + 1]] * scale : 0.f;
      const half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
      const half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
      hi[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      lo[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    uint4 *o = xf + (size_t)((kb0 + kbl) * nt + n) * 32;
    o[g * 4 + t] = make_uint4(hi[0], hi[1], hi[2], hi[3]);        // B column g: hi part
    o[(g + 4) * 4 + t] = make_uint4(lo[0], lo[1], lo[2], lo[3]);  // B column g + 4: lo part
  }
}
// One of the two: mma_nt == 0 the tcgen05 layout, else the mma.sync layout
// with mma_nt n-tiles.
CW_DEV void emit_xops(const float *v, int kb0, int nkb, int b, int mma_nt, uint4 *__restrict__ xf, float scale,
                      bool live) {
  if (mma_nt) emit_xfrag_blocks_mma(v, kb0, nkb, b, mma_nt, xf, scale, live);
  else emit_xfrag_blocks(v, kb0, nkb, b, xf, scale, live);
}

// Emit the X operands for column b from v[0..K) in shared memory (one CTA
// holds the whole column).
CW_DEV void emit_xfrag(const float *v, int K, int b, int mma_nt, uint4 *__restrict__ xf, int *__restrict__ xexp,
                       float *red, bool live) {
  float mx = 0.f;
  if (live)
    for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(v[k]));
  mx = block_max(mx, red);
  const int e = xfrag_exponent(mx);
  if (threadIdx.x == 0) xexp[b] = e;
  emit_xops(v, 0, K / 32, b, mma_nt, xf, __int_as_float((127 + e) << 23), live);
}

// One float per CTA reduced over the thread-block cluster (<= 32 CTAs)
// through distributed shared memory; every CTA gets the result.  Each warp
// reads the CTAs' slots in parallel (lane i <- rank i) and reduces them with a
// fixed xor tree, so the result is deterministic and the same in every CTA.
// `slot` is one float of this CTA's shared memory.
template <bool MAX>
CW_DEV float cluster_reduce(float v, float *slot) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  if (threadIdx.x == 0) *slot = v;
  cl.sync();
  const unsigned l = threadIdx.x & 31;
  float o = l < cl.num_blocks() ? *cl.map_shared_rank(slot, l) : 0.f;  // 0: identity of the sum and of the max of |.|
  o = MAX ? warp_max(o) : warp_sum(o);
  cl.sync();  // every CTA has read every slot before any slot is reused
  return o;
}

// Block-wide (sum, max) pair in one exchange (red: >= 64 floats smem).
CW_DEV float2 block_sum_max(float v, float m, float *red) {
  v = warp_sum(v);
  m = warp_max(m);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    red[w] = v;
    red[32 + w] = m;
  }
  __syncthreads();
  const bool in = l < (int)(blockDim.x >> 5);
  return make_float2(warp_sum(in ? red[l] : 0.f), warp_max(in ? red[32 + l] : 0.f));
}

// (sum, max) pair per CTA reduced over the thread-block cluster in one
// exchange, like cluster_reduce.  `slot` is one float2 of this CTA's shared memory.
CW_DEV float2 cluster_reduce_sum_max(float2 v, float2 *slot) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  if (threadIdx.x == 0) *slot = v;
  cl.sync();
  const unsigned l = threadIdx.x & 31;
  const float2 o = l < cl.num_blocks() ? *cl.map_shared_rank(slot, l) : make_float2(0.f, 0.f);
  const float2 r = make_float2(warp_sum(o.x), warp_max(o.y));
  cl.sync();  // every CTA has read every slot before any CTA leaves
  return r;
}

CW_DEV float silu_dev(float x) { return x * (1.f / (1.f + expf(-x))); }
CW_DEV float sigmoid_dev(float x) { return 1.f / (1.f + expf(-x)); }

}  // namespace cw
