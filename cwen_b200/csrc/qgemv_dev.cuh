// Device-side pieces shared by the two verify-GEMV kernels (qgemv.cu on the
// 5th-generation tensor cores, qgemv_mma.cu on warp-level mma.sync): the
// launch arguments, the exact nibble / int8 -> f16 unpack, and the epilogue
// of a reduced split tile.
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"
#include "qgemv.cuh"

namespace cw {

// ---- nibble / int8 -> f16 (exact) ----
// Q4: word w = qs bytes [4t..4t+3] of one row's block.  Returns half2s:
//   s0 = (lo(b0), lo(b2))  t0 = (lo(b1), lo(b3))  s1 = (hi(b0), hi(b2))  t1 = (hi(b1), hi(b3))
// each value (nibble - 8), via the 0x6400 (=1024.0) exponent trick.
CW_DEV void q4_to_f16(uint32_t w, uint32_t &s0, uint32_t &t0, uint32_t &s1, uint32_t &t1) {
  constexpr uint32_t MAGIC = 0x64006400u;
  constexpr int AND_OR = (0xF0 & 0xCC) | 0xAA;
  const uint32_t lo0 = lop3<AND_OR>(w, 0x000F000Fu, MAGIC);
  const uint32_t hi0 = lop3<AND_OR>(w, 0x00F000F0u, MAGIC);
  const uint32_t w2 = w >> 8;
  const uint32_t lo1 = lop3<AND_OR>(w2, 0x000F000Fu, MAGIC);
  const uint32_t hi1 = lop3<AND_OR>(w2, 0x00F000F0u, MAGIC);
  const half2 k1032 = __halves2half2(__ushort_as_half(0xE408u), __ushort_as_half(0xE408u));  // -1032
  const half2 k16th = __halves2half2(__ushort_as_half(0x2C00u), __ushort_as_half(0x2C00u));  // 1/16
  const half2 k72 = __halves2half2(__ushort_as_half(0xD480u), __ushort_as_half(0xD480u));    // -72
  half2 r;
  r = __hadd2(*reinterpret_cast<const half2 *>(&lo0), k1032); s0 = *reinterpret_cast<uint32_t *>(&r);
  r = __hadd2(*reinterpret_cast<const half2 *>(&lo1), k1032); t0 = *reinterpret_cast<uint32_t *>(&r);
  r = __hfma2(*reinterpret_cast<const half2 *>(&hi0), k16th, k72); s1 = *reinterpret_cast<uint32_t *>(&r);
  r = __hfma2(*reinterpret_cast<const half2 *>(&hi1), k16th, k72); t1 = *reinterpret_cast<uint32_t *>(&r);
}
// Q8: word of 4 int8 (b0..b3) -> (b0, b2), (b1, b3) as half2, exact.
CW_DEV void q8_to_f16(uint32_t w, uint32_t &s, uint32_t &t) {
  const uint32_t u = w ^ 0x80808080u;  // int8 -> uint8 + 128
  uint32_t a, b;
  asm("prmt.b32 %0, %1, %2, 0x4240;" : "=r"(a) : "r"(u), "r"(0x64646464u));
  asm("prmt.b32 %0, %1, %2, 0x4341;" : "=r"(b) : "r"(u), "r"(0x64646464u));
  const half2 k1152 = __halves2half2(__ushort_as_half(0xE480u), __ushort_as_half(0xE480u));  // -1152
  half2 r;
  r = __hadd2(*reinterpret_cast<const half2 *>(&a), k1152); s = *reinterpret_cast<uint32_t *>(&r);
  r = __hadd2(*reinterpret_cast<const half2 *>(&b), k1152); t = *reinterpret_cast<uint32_t *>(&r);
}

// ---- the GEMV ----
struct GemvArgs {
  const uint8_t *w;
  int n_mt, kp, M;
  const uint4 *xf;
  const int *xexp;
  int B;
  float *y;
  int ys, epi;
  float *ws;
  int *cnt;
  int *err;
  int G;
  long long units;
  int cl;  // > 1: the contributors of each split tile form one thread-block cluster of cl CTAs
  // local-X variant: raw fp32 rows X (column b at xr + b*xrs), turned into
  // fragments by each CTA for its own k-range with its own column exponents
  const float *xr;
  int xrs;
  const float *xw;     // != nullptr: X = RMSNorm(xr) * xw (run.c:346), scale from st_in
  const float *st_in;  // sums of squares of the rows, [st_g][16] per-CTA partials of the GEMV that wrote them
  int st_g;
  float *st_out;       // != nullptr: this GEMV's per-CTA sums of squares of its output rows [G][16]
  // Row-sharded matrix (rows row0.. of the full output): np > 0 copies of Y,
  // one per GPU of the shard group (the local one included), all written.
  int row0, np;
  float *yp[QG_MAX_PEERS];
  // mma kernel, global split-K mode: this launch's value of the partial flags
  int epoch;
};

// Offset in Y of local row `row` (row0 + row of the full output), column col.
CW_DEV size_t y_off(const GemvArgs &a, int col, int row) { return (size_t)col * a.ys + a.row0 + row; }
// Store an output element -- into every GPU's copy of Y for a sharded matrix
// (posted NVLink stores; the launcher's cross-GPU barrier follows the GEMV).
CW_DEV void y_put(const GemvArgs &a, size_t off, float v) {
  if (a.np == 0) {
    a.y[off] = v;
  } else {
    for (int p = 0; p < a.np; p++) a.yp[p][off] = v;
  }
}
// The GEMV's own output element (EPI_STORE, or EPI_ADD onto the local copy).
CW_DEV void y_out(const GemvArgs &a, int col, int row, float v) {
  const size_t off = y_off(a, col, row);
  y_put(a, off, a.epi == EPI_ADD ? a.y[off] + v : v);
}
// Before a sharded GEMV's threads retire: their peer stores are performed
// system-wide before the barrier kernel that follows signals the other GPUs.
CW_DEV void y_fence(const GemvArgs &a) {
  if (a.np) __threadfence_system();
}

CW_DEV float silu_f(float x) { return x * (1.f / (1.f + expf(-x))); }

// Thread-block cluster barrier (every thread of every CTA of the cluster),
// release / acquire at cluster scope.
CW_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Power-of-two unscale of column col: the global exponent of prepared
// fragments, or (local-X variant) 1 for partials already unscaled by the CTA
// that computed them.
CW_DEV float split_unscale(const GemvArgs &a, int col) {
  return a.xr ? 1.f : __int_as_float((127 - __ldg(a.xexp + col)) << 23);
}

// Epilogue of a reduced split-tile share: lane (mt, row) holds row `row` of
// m-tile mt0 + mt, four columns per float4 (NC4 of them).  The whole warp
// calls it (the SwiGLU pairs gate and up rows across the warp's halves).
template <int NC4>
CW_DEV void split_epilogue(const GemvArgs &a, int mt0, int mt, int row, bool live, const float4 (&sum)[NC4],
                           float *wst, const float *ypre = nullptr) {
#pragma unroll
  for (int n = 0; n < NC4; n++) {
    const float e4[4] = {sum[n].x, sum[n].y, sum[n].z, sum[n].w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int col = n * 4 + j;
      if (col >= a.B) continue;
      if (a.st_out && a.epi == EPI_ADD) {  // sums of squares of the new rows (warp order, then CTA order)
        float v2 = 0.f;
        const int grow = (mt0 + mt) * 16 + row;
        if (live && grow < a.M) {
          const float v = (ypre ? ypre[col] : a.y[y_off(a, col, grow)]) + e4[j] * split_unscale(a, col);
          v2 = v * v;
        }
        v2 = warp_sum(v2);
        if ((threadIdx.x & 31) == 0) wst[col] += v2;
      }
      const float sc = split_unscale(a, col);
      if (a.epi == EPI_SWIGLU) {
        const float up = __shfl_down_sync(0xffffffffu, e4[j], 16);
        if (live && mt == 0) {
          const int orow = (mt0 >> 1) * 16 + row;
          if (orow * 2 < a.M) y_put(a, y_off(a, col, orow), silu_f(e4[j] * sc) * (up * sc));
        }
      } else if (live) {
        const int grow = (mt0 + mt) * 16 + row;
        if (grow < a.M) {
          if (ypre && a.epi == EPI_ADD)
            y_put(a, y_off(a, col, grow), ypre[col] + e4[j] * sc);
          else
            y_out(a, col, grow, e4[j] * sc);
        }
      }
    }
  }
}

// The warp-level mma.sync kernel (qgemv_mma.cu): its weight repack, its
// launch for the arguments gemv_launch prepared, its one-time attributes.
namespace mma {
cudaError_t repack(const QMat &dst, const uint8_t *src, int M, int mt_off, int mt_stride, cudaStream_t st);
cudaError_t launch(const GemvArgs &a, int type, bool xl, cudaStream_t st);
cudaError_t configure();
}  // namespace mma

}  // namespace cw
