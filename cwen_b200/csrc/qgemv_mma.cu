// Batched Q4_0 / Q8_0 verify GEMV on warp-level tensor-core MMAs
// (mma.sync m16n8k16), the engine's default kernel; the work split of the
// tcgen05 kernel of qgemv.cu, with its own weight and X layouts.
//
// Replaces the reference's gemvb()/gemv() (run.c:1577-1680, 1419-1527) and
// the row dots under them (dot_q4_0 run.c:1009-1025, dot_nib16 run.c:432,
// dot_q8_0 run.c:1248-1274).
//
// Arithmetic.  Columns come in n-tiles of 4: B-operand columns 0..3 hold the
// f16 hi parts of the 4 columns and 4..7 their lo parts.  Per 16 rows x 32
// weights and n-tile two chained m16n8k16 MMAs (k 0..15, k 16..31; products
// exact, fp32 accumulate) give the block partials of the hi and the lo
// halves; one FFMA per element applies the block's f16 scale, acc = fma(d,
// c, acc), and the hi and lo sums are added at the end of the tile.  (q - 8)
// is exact in f16.  Two MMAs per 16 x 32 weights at B <= 4 (one column per
// decode step), 4 at B <= 8, 6 at a 9-row verify block.
//
// Weight layout.  Rows in 16-row m-tiles, m-tiles in 512-row tiles of 32; per
// (m-tile, pair of 32-blocks) one 576-byte chunk [512 B nibbles in mma
// A-fragment order | 64 B f16 scales] (Q8_0: 1088 B [1024 B int8 | 64 B
// scales]), stored [tile][k-pair][m-tile] so that one (tile, k-pair) is one
// contiguous 18 KB / 34 KB stage -- the same stage size as the tcgen05 layout.
//
// X operands.  Per (32-block, n-tile of 4 columns) 32 uint4; lane (g, t) of
// the B operand holds, of column 4n + g % 4 (hi parts for g < 4, lo parts for
// g >= 4),
//   (x[4t], x[4t+2]) (x[4t+1], x[4t+3]) (x[4t+16], x[4t+18]) (x[4t+17], x[4t+19]).
//
// Work split, pipeline and the split-tile reduction: as in qgemv.cu (bulk-copy
// ring with two producer threads, 16 consumer warps with two m-tiles each,
// stream-K over (tile, k-pair) units, cluster or global split-K reduction).
#include <utility>

#include "common.cuh"
#include "qgemv.cuh"
#include "qgemv_dev.cuh"
#include "rowprep.cuh"
#include "sm100.cuh"

namespace cw {
namespace mma {

constexpr int QGM_THREADS = (QG_CONS_WARPS + 2) * 32;  // 16 consumer warps + two producer warps

// ---- weight repack: GGUF rows -> fragment-ordered chunks ----
// One thread per (m-tile, k-pair, lane); each writes its lane's qs bytes and
// lanes 0..7 also the scale words of row pair (g, g+8).
template <int TYPE>
__global__ void repack_kernel(uint8_t *dst, int dst_kp, const uint8_t *src, int M, int K, int mt_off,
                              int mt_stride) {
  const int nb = K / 32, kp = K / 64;
  const int src_mt = (M + 15) / 16;
  const long long total = (long long)src_mt * kp * 32;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int lane = (int)(idx % 32);
    const int p = (int)((idx / 32) % kp);
    const int smt = (int)(idx / 32 / kp);
    const int g = lane >> 2, t = lane & 3;
    const int dmt = mt_off + smt * mt_stride;
    const size_t chunk = (size_t)(TYPE == 8 ? 1088 : 576);
    // [tile][k-pair][m-tile within tile]: one (tile, k-pair) is contiguous
    uint8_t *c = dst + (((size_t)(dmt / QG_TILE_MT) * dst_kp + p) * QG_TILE_MT + dmt % QG_TILE_MT) * chunk;
    const int r0 = smt * 16 + g, r1 = r0 + 8;
    uint32_t words[8];
    uint16_t sc[4];
    for (int kbi = 0; kbi < 2; kbi++) {
      const int kb = 2 * p + kbi;
      for (int ri = 0; ri < 2; ri++) {
        const int r = ri ? r1 : r0;
        uint16_t d = 0;
        uint32_t wa = 0, wb = 0;
        if (r < M) {
          if (TYPE == 8) {
            const uint8_t *blk = src + ((size_t)r * nb + kb) * 34;
            d = (uint16_t)(blk[0] | (blk[1] << 8));
            const uint8_t *q = blk + 2;
            wa = q[4 * t] | (q[4 * t + 1] << 8) | (q[4 * t + 2] << 16) | ((uint32_t)q[4 * t + 3] << 24);
            wb = q[16 + 4 * t] | (q[16 + 4 * t + 1] << 8) | (q[16 + 4 * t + 2] << 16) |
                 ((uint32_t)q[16 + 4 * t + 3] << 24);
          } else {
            const uint8_t *blk = src + ((size_t)r * nb + kb) * 18;
            d = (uint16_t)(blk[0] | (blk[1] << 8));
            const uint8_t *q = blk + 2;
            wa = q[4 * t] | (q[4 * t + 1] << 8) | (q[4 * t + 2] << 16) | ((uint32_t)q[4 * t + 3] << 24);
          }
        }
        if (TYPE == 8) {
          words[kbi * 4 + ri * 2 + 0] = wa;
          words[kbi * 4 + ri * 2 + 1] = wb;
        } else {
          words[kbi * 2 + ri] = wa;
        }
        sc[kbi * 2 + ri] = d;
      }
    }
    if (TYPE == 8) {
      uint4 *o = reinterpret_cast<uint4 *>(c + lane * 32);
      o[0] = make_uint4(words[0], words[1], words[2], words[3]);
      o[1] = make_uint4(words[4], words[5], words[6], words[7]);
    } else {
      *reinterpret_cast<uint4 *>(c + lane * 16) = make_uint4(words[0], words[1], words[2], words[3]);
    }
    if (t == 0) {
      const size_t qbytes = TYPE == 8 ? 1024 : 512;
      uint2 s;
      s.x = (uint32_t)sc[0] | ((uint32_t)sc[1] << 16);  // kb0: (d_g, d_g8)
      s.y = (uint32_t)sc[2] | ((uint32_t)sc[3] << 16);  // kb1
      *reinterpret_cast<uint2 *>(c + qbytes + g * 8) = s;
    }
  }
}

cudaError_t repack(const QMat &dst, const uint8_t *src, int M, int mt_off, int mt_stride, cudaStream_t st) {
  const int src_mt = (M + 15) / 16;
  if (dst.K % 64 || mt_off < 0 || mt_stride < 1 || mt_off + (src_mt - 1) * mt_stride >= dst.n_mt)
    return cudaErrorInvalidValue;
  const long long total = (long long)src_mt * (dst.K / 64) * 32;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  const int grid = (int)(blocks < 65535 ? blocks : 65535);
  if (dst.type == 8)
    repack_kernel<8><<<grid, threads, 0, st>>>(dst.w, dst.K / 64, src, M, dst.K, mt_off, mt_stride);
  else
    repack_kernel<2><<<grid, threads, 0, st>>>(dst.w, dst.K / 64, src, M, dst.K, mt_off, mt_stride);
  return cudaGetLastError();
}

// Fold the lo-part accumulators into the hi-part ones: lane (g, t < 2) holds
// B columns 2t, 2t+1 (hi parts), lane (g, t + 2) the same columns' lo parts.
// Afterwards lanes t < 2 hold the sums (hi + lo, in that order).
template <int NT>
CW_DEV void fold_lo(float (&acc)[2][NT][4]) {
#pragma unroll
  for (int mt = 0; mt < 2; mt++)
#pragma unroll
    for (int n = 0; n < NT; n++)
#pragma unroll
      for (int i = 0; i < 4; i++) acc[mt][n][i] += __shfl_xor_sync(0xffffffffu, acc[mt][n][i], 2);
}

// Apply the epilogue for one warp's folded accumulators (rows of m-tiles
// mt0, mt0+1; lanes t < 2 carry the columns n*4 + 2t + {0, 1}).
template <int NT>
CW_DEV void gemv_epilogue(const GemvArgs &a, int mt0, bool has1, const float (&acc)[2][NT][4], int g, int t,
                          const float *xun) {
  if (t >= 2) return;
#pragma unroll
  for (int n = 0; n < NT; n++) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int col = n * 4 + 2 * t + (i & 1);
      if (col >= a.B) continue;
      const float sc = xun ? xun[col] : __int_as_float((127 - __ldg(a.xexp + col)) << 23);
      const int rr = g + ((i >> 1) << 3);
      if (a.epi == EPI_SWIGLU) {
        const int row = (mt0 >> 1) * 16 + rr;
        if (row * 2 < a.M) {
          const float gt = acc[0][n][i] * sc, up = acc[1][n][i] * sc;
          y_put(a, y_off(a, col, row), silu_f(gt) * up);
        }
      } else {
#pragma unroll
        for (int mt = 0; mt < 2; mt++) {
          if (mt == 1 && !has1) continue;
          const int row = (mt0 + mt) * 16 + rr;
          if (row >= a.M) continue;
          y_out(a, col, row, acc[mt][n][i] * sc);
        }
      }
    }
  }
}


template <int TYPE, int NT, bool XL = false>
struct QgLayout {
  static constexpr int CHUNK = TYPE == 8 ? 1088 : 576;       // one m-tile x one k-pair
  static constexpr int QB = TYPE == 8 ? 1024 : 512;          // its quant bytes (scales follow)
  static constexpr int WB = QG_TILE_MT * CHUNK;              // weights of one (tile, k-pair)
  static constexpr int XB = XL ? 0 : NT * 1024;              // X fragments of one k-pair (streamed)
  static constexpr int STAGE = WB + XB;
  // local-X variant: the CTA's k-range of X fragments, resident (<= QG_XL_KP_MMA k-pairs x NT n-tiles)
  static constexpr int XL_BYTES = XL ? QG_XL_KP_MMA * NT * 1024 : 0;
  // per column: 2^-e [16] floats, per-warp sums [16][16] floats, prologue maxima [16] ints and scales [16] floats
  static constexpr int XE_BYTES = XL ? 64 + 16 * 16 * 4 + 128 : 0;
  // ring depth: 8 stages, fewer when the resident X needs the room (the
  // depth changes only the overlap, never the arithmetic)
  static constexpr int FIT = (227 * 1024 - 256 - XL_BYTES - XE_BYTES) / STAGE;
  static constexpr int STAGES = TYPE == 8 ? 5 : (FIT < 8 ? FIT : 8);
  static constexpr int BAR_OFF = STAGES * STAGE;
  static constexpr int XL_OFF = BAR_OFF + 256;
  static constexpr int XE_OFF = XL_OFF + XL_BYTES;
  static constexpr int SMEM = XE_OFF + XE_BYTES;
  static_assert(STAGES >= 3, "ring depth");
  static constexpr int XL_AHEAD = STAGES > 5 ? 4 : 2;  // weight stages issued before the local-X prologue ends
  static_assert(WB % 16 == 0 && XB % 16 == 0 && STAGE % 16 == 0, "bulk copies need 16-byte multiples");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// Persistent stream-K GEMV: warps 0..15 consume (warp w owns m-tiles 2w, 2w+1
// of the current 512-row tile); lane 0 of warp 16 streams the weights and
// lane 0 of warp 17 the X fragments.
// Local X (run by the 16 consumer warps once, after pdl_wait): the CTA's
// k-range [64*ka0, 64*(ka0+nkp)) of every column of the raw rows X becomes
// f16 hi/lo fragments in shared memory, scaled by the CTA's own power of two
// 2^e (max |x| over the range in [2^14, 2^15)); xun[col] = 2^-e unscales the
// CTA's results.  The fragments hold the same values and layout gemv_prep_x
// emits, except for the exponent's range.  The work is spread over all 512
// threads: an item is (column b, 32-block kb, lane quarter t), the 8 values
// one B-operand lane holds; every load of the prologue is issued in one
// round (items, row norm partials), the column maxima meet in shared memory
// (an integer max of non-negative floats: order-free), and the second pass
// converts from registers (the first KEEP items of a thread: every item of
// up to 8 columns x 40 k-pairs) or reloads.
// cm: [16] int column maxima, ssc: [16] float row scales (shared memory).
template <int NT>
CW_DEV void x_local_prologue(const GemvArgs &a, uint4 *xl, float *xun, int *cm, float *ssc, int ka0, int nkp) {
  constexpr int NTH = QG_CONS_WARPS * 32, KEEP = NT == 1 ? 2 : 3;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nblk = 2 * nkp, nitem = a.B * nblk * 4;
  if (tid < 16) cm[tid] = 0;
  // RMSNorm: the row's sum of squares from the per-CTA partials of the GEMV
  // that wrote it, in slot order then a fixed xor tree (warp b, column b)
  float ss = 0.f;
  if (a.xw && warp < a.B)
#pragma unroll
    for (int i = 0; i < 5; i++)
      if (lane + 32 * i < a.st_g) ss += __ldcg(a.st_in + (size_t)(lane + 32 * i) * QG_STAT_COLS + warp);
  // item it -> column b = it / (nblk * 4), block kb, quarter t: elements
  // 4t..4t+3 and 16+4t..16+4t+3 of the block
  auto item_ptr = [&](int it, int &b, int &kb, int &t) {
    b = it / (nblk * 4);
    const int r = it - b * nblk * 4;
    kb = r >> 2;
    t = r & 3;
  };
  float4 kv[KEEP][2];
  named_bar(1, NTH);  // cm cleared
#pragma unroll
  for (int j = 0; j < KEEP; j++) {
    const int it = tid + j * NTH;
    if (it < nitem) {
      int b, kb, t;
      item_ptr(it, b, kb, t);
      const float *x = a.xr + (size_t)b * a.xrs + (size_t)ka0 * 64 + kb * 32 + 4 * t;
      float4 u0 = __ldg(reinterpret_cast<const float4 *>(x)), u1 = __ldg(reinterpret_cast<const float4 *>(x + 16));
      if (a.xw) {
        const float *w = a.xw + (size_t)ka0 * 64 + kb * 32 + 4 * t;
        const float4 w0 = __ldg(reinterpret_cast<const float4 *>(w)), w1 = __ldg(reinterpret_cast<const float4 *>(w + 16));
        u0 = make_float4(w0.x * u0.x, w0.y * u0.y, w0.z * u0.z, w0.w * u0.w);
        u1 = make_float4(w1.x * u1.x, w1.y * u1.y, w1.z * u1.z, w1.w * u1.w);
      }
      kv[j][0] = u0;
      kv[j][1] = u1;
      const float mi = fmaxf(fmaxf(fmaxf(fabsf(u0.x), fabsf(u0.y)), fmaxf(fabsf(u0.z), fabsf(u0.w))),
                             fmaxf(fmaxf(fabsf(u1.x), fabsf(u1.y)), fmaxf(fabsf(u1.z), fabsf(u1.w))));
      atomicMax(cm + b, __float_as_int(mi));
    }
  }
  for (int it = tid + KEEP * NTH; it < nitem; it += NTH) {
    int b, kb, t;
    item_ptr(it, b, kb, t);
    const float *x = a.xr + (size_t)b * a.xrs + (size_t)ka0 * 64 + kb * 32 + 4 * t;
    float4 u0 = __ldg(reinterpret_cast<const float4 *>(x)), u1 = __ldg(reinterpret_cast<const float4 *>(x + 16));
    if (a.xw) {
      const float *w = a.xw + (size_t)ka0 * 64 + kb * 32 + 4 * t;
      const float4 w0 = __ldg(reinterpret_cast<const float4 *>(w)), w1 = __ldg(reinterpret_cast<const float4 *>(w + 16));
      u0 = make_float4(w0.x * u0.x, w0.y * u0.y, w0.z * u0.z, w0.w * u0.w);
      u1 = make_float4(w1.x * u1.x, w1.y * u1.y, w1.z * u1.z, w1.w * u1.w);
    }
    const float mi = fmaxf(fmaxf(fmaxf(fabsf(u0.x), fabsf(u0.y)), fmaxf(fabsf(u0.z), fabsf(u0.w))),
                           fmaxf(fmaxf(fabsf(u1.x), fabsf(u1.y)), fmaxf(fabsf(u1.z), fabsf(u1.w))));
    atomicMax(cm + b, __float_as_int(mi));
  }
  if (a.xw && warp < a.B) {
    ss = warp_sum(ss);
    if (lane == 0) ssc[warp] = 1.f / sqrtf(ss / (float)(a.kp * 64) + 1e-6f);
  }
  named_bar(1, NTH);  // column maxima and row scales complete
  if (tid < 16) {
    if (tid < a.B) {
      float mx = __int_as_float(cm[tid]);
      const float s = a.xw ? ssc[tid] : 1.f;
      mx *= s;  // max |(w x) s| = max |w x| * s: s > 0 and rounding is monotonic
      const int e = xfrag_exponent(mx);
      xun[tid] = __int_as_float((127 - e) << 23);
      // ((w x) s) 2^e == (w x) (s 2^e) exactly: 2^e only shifts the exponent
      ssc[tid] = s * __int_as_float((127 + e) << 23);
    } else {
      xun[tid] = 1.f;  // padding column
    }
  }
  named_bar(1, NTH);  // per-column scales ready
  // item it -> its 8 values as hi / lo fragments (u0: x[4t..4t+3], u1: x[4t+16..4t+19])
  auto emit = [&](int it, const float4 &u0, const float4 &u1) {
    int b, kb, t;
    item_ptr(it, b, kb, t);
    float r[8];
    r[0] = u0.x; r[1] = u0.y; r[2] = u0.z; r[3] = u0.w;
    r[4] = u1.x; r[5] = u1.y; r[6] = u1.z; r[7] = u1.w;
    const float sc = ssc[b];
    // B operand lane (col & 3, t): (x[4t], x[4t+2]) (x[4t+1], x[4t+3]) (x[4t+16], x[4t+18]) (x[4t+17], x[4t+19])
    // r[] holds x[4t..4t+3] then x[4t+16..4t+19]
    const int js[8] = {0, 2, 1, 3, 4, 6, 5, 7};
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float v0 = r[js[2 * i]] * sc, v1 = r[js[2 * i + 1]] * sc;
      const half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
      const half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
      hw[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      lw[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    uint4 *o = xl + ((size_t)kb * NT + (b >> 2)) * 32 + (b & 3) * 4 + t;
    o[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    o[16] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  };
#pragma unroll
  for (int j = 0; j < KEEP; j++)
    if (tid + j * NTH < nitem) emit(tid + j * NTH, kv[j][0], kv[j][1]);
  for (int it = tid + KEEP * NTH; it < nitem; it += NTH) {
    int b, kb, t;
    item_ptr(it, b, kb, t);
    const float *x = a.xr + (size_t)b * a.xrs + (size_t)ka0 * 64 + kb * 32 + 4 * t;
    float4 u0 = __ldg(reinterpret_cast<const float4 *>(x)), u1 = __ldg(reinterpret_cast<const float4 *>(x + 16));
    if (a.xw) {
      const float *w = a.xw + (size_t)ka0 * 64 + kb * 32 + 4 * t;
      const float4 w0 = __ldg(reinterpret_cast<const float4 *>(w)), w1 = __ldg(reinterpret_cast<const float4 *>(w + 16));
      u0 = make_float4(w0.x * u0.x, w0.y * u0.y, w0.z * u0.z, w0.w * u0.w);
      u1 = make_float4(w1.x * u1.x, w1.y * u1.y, w1.z * u1.z, w1.w * u1.w);
    }
    emit(it, u0, u1);
  }
  named_bar(1, NTH);
}

template <int TYPE, int NT, bool XL>
__global__ void __launch_bounds__(QGM_THREADS, 1) qgemv_kernel(GemvArgs a) {
  using Lay = QgLayout<TYPE, NT, XL>;
  constexpr int S = Lay::STAGES;
  constexpr int XL_AHEAD = Lay::XL_AHEAD;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Lay::BAR_OFF);
  uint64_t *empty = full + S;
  uint64_t *xready = empty + S;  // local X: the prologue's fragments are in shared memory
  volatile int *abort_p = reinterpret_cast<volatile int *>(xready + 1);
  int *last_p = const_cast<int *>(abort_p) + 1;  // [2]

  const int c = blockIdx.x;
  // unit arithmetic in 32 bits (the launcher checks units * (G + 1) < 2^31):
  // a 64-bit division is a long software sequence on the critical path
  const int units = (int)a.units;
  const int u_begin = c * units / a.G, u_end = (c + 1) * units / a.G;
  if (u_begin >= u_end) return;  // whole CTA, before any barrier
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&full[i], XL ? 1 : 2);  // the weight and the X producer
      mbar_init(&empty[i], QG_CONS_WARPS);
    }
    mbar_init(xready, 1);
    *abort_p = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp >= QG_CONS_WARPS) {
    // ---------------- producers ----------------
    // Two producer threads in two warps, one for the weights and one for X:
    // a bulk copy occupies its issuing thread for ~0.3 us whatever its size,
    // so one thread issuing both copies of a stage would cap the stream.
    // Consecutive units are consecutive (tile, k-pair) blocks of the repacked
    // weights, so the weight source just advances; no divisions in the loops.
    if (lane == 0 && (!XL || warp == QG_CONS_WARPS)) {  // local X: no X copies
      const bool wprod = warp == QG_CONS_WARPS;
      const int n = u_end - u_begin;
      const uint8_t *wsrc = a.w + (size_t)u_begin * Lay::WB;
      const uint8_t *xbase = reinterpret_cast<const uint8_t *>(a.xf);
      // Weights are not written by any kernel of the decode step: the weight
      // producer never waits for the previous kernel (PDL), so the ring fills
      // while that kernel finishes.  X is that kernel's output.
      if (!wprod) pdl_wait();
      int k = u_begin % a.kp;
      int st = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      for (; issued < n; issued++) {
        if (!mbar_wait(&empty[st], ph ^ 1, abort_p)) {
          ok = false;
          break;
        }
        if (*abort_p) break;  // consumers gave up: issue nothing more
        // Local X: XL_AHEAD weight stages go ahead, the rest after the
        // prologue has read X -- its loads would otherwise queue behind a
        // full ring of weights.
        if (XL && wprod && issued == XL_AHEAD && !mbar_wait(xready, 0, abort_p)) {
          ok = false;
          break;
        }
        uint8_t *dst = smem + st * Lay::STAGE;
        if (wprod) {
          mbar_expect_tx(&full[st], Lay::WB);
          bulk_g2s(dst, wsrc, Lay::WB, &full[st]);
          wsrc += Lay::WB;
        } else {
          mbar_expect_tx(&full[st], Lay::XB);
          bulk_g2s(dst + Lay::WB, xbase + (size_t)k * Lay::XB, Lay::XB, &full[st]);
          if (++k == a.kp) k = 0;
        }
        if (++st == S) {
          st = 0;
          ph ^= 1;
        }
      }
      if (!ok) {
        atomicExch(a.err, 1);
        *abort_p = 1;
      }
      // never leave bulk copies in flight: wait (bounded, one deadline) for
      // the last stages issued
      const long long t0 = cycles_now();
      for (int i = issued > S ? issued - S : 0; i < issued; i++) {
        while (!mbar_try_wait(&full[i % S], (uint32_t)((i / S) & 1)) && !spin_expired(t0)) {
        }
      }
    }
    if (a.cl > 1) {  // the two cluster barriers of the split-tile reduction
      cluster_sync_all();
      cluster_sync_all();
    }
    return;  // the producers take part in no later CTA barrier
  }

  // ---------------- consumers ----------------
  pdl_wait();  // before touching Y, the split-K partials or the tile counters
  const int g = lane >> 2, t = lane & 3;
  const int ka0 = u_begin % a.kp;  // local X: the CTA's one segment starts here
  float *xun = XL ? reinterpret_cast<float *>(smem + Lay::XE_OFF) : nullptr;
  float *wst = XL ? xun + 16 + warp * 16 : nullptr;  // this warp's output sums of squares per column
  if (XL && a.st_out && lane < 16) wst[lane] = 0.f;
  if (XL) {
    x_local_prologue<NT>(a, reinterpret_cast<uint4 *>(smem + Lay::XL_OFF), xun,
                         reinterpret_cast<int *>(xun + 16 + 16 * 16), xun + 16 + 16 * 16 + 16, ka0,
                         u_end - u_begin);
    if (threadIdx.x == 0) mbar_arrive(xready);
  }
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
  bool ok = true;
  int st = 0;        // ring position, advanced identically by every consumer warp and the producer
  uint32_t ph = 0;   // its phase parity
  int u = u_begin;
  bool first_seg = true;
  int ptile[2], pslot[2];  // split tiles of this CTA (its first and last segments) and their partial slots
  int np = 0;
  while (u < u_end) {
    const int tile = u / a.kp;
    const int ka = u - tile * a.kp;
    const int remain = u_end - u;
    const int kb_end = a.kp - ka < remain ? a.kp : ka + remain;
    const int nk = kb_end - ka;
    const int mt0 = tile * QG_TILE_MT + warp * 2;
    const bool has0 = mt0 < a.n_mt, has1 = mt0 + 1 < a.n_mt;

    float acc[2][NT][4];
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
      for (int n = 0; n < NT; n++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[mt][n][i] = 0.f;

    for (int i = 0; i < nk; i++) {
      if (ok && !mbar_wait(&full[st], ph, abort_p)) {
        ok = false;
        atomicExch(a.err, 2);
        *abort_p = 1;
      }
      if (ok && has0) {
        const uint8_t *stg = smem + st * Lay::STAGE;
        const uint4 *xs = XL ? reinterpret_cast<const uint4 *>(smem + Lay::XL_OFF) + (size_t)(ka + i - ka0) * (2 * NT * 32)
                             : reinterpret_cast<const uint4 *>(stg + Lay::WB);
        // up to two n-tiles: both m-tiles share the stage's X loads; more:
        // reload per m-tile (registers)
        constexpr bool XH = NT <= 2;
        constexpr int NH = XH ? NT : 1;
        uint4 xh[2][NH];
        if (XH) {
#pragma unroll
          for (int kbi = 0; kbi < 2; kbi++)
#pragma unroll
            for (int n = 0; n < NH; n++) xh[kbi][n] = xs[(kbi * NT + n) * 32 + lane];
        }
#pragma unroll
        for (int mt = 0; mt < 2; mt++) {
          if (mt == 1 && !has1) break;
          const uint8_t *ch = stg + (warp * 2 + mt) * Lay::CHUNK;
          const uint2 scw = *reinterpret_cast<const uint2 *>(ch + Lay::QB + g * 8);
#pragma unroll
          for (int kbi = 0; kbi < 2; kbi++) {
            uint32_t a0s0, a1s0, a2s0, a3s0, a0s1, a1s1, a2s1, a3s1;
            if (TYPE == 8) {
              const uint4 qw = *reinterpret_cast<const uint4 *>(ch + lane * 32 + kbi * 16);
              q8_to_f16(qw.x, a0s0, a2s0);  // row g, bytes 4t..4t+3
              q8_to_f16(qw.y, a0s1, a2s1);  // row g, bytes 16+4t..
              q8_to_f16(qw.z, a1s0, a3s0);  // row g+8
              q8_to_f16(qw.w, a1s1, a3s1);
            } else {
              const uint4 qw = *reinterpret_cast<const uint4 *>(ch + lane * 16);
              const uint32_t wg = kbi ? qw.z : qw.x, wg8 = kbi ? qw.w : qw.y;
              q4_to_f16(wg, a0s0, a2s0, a0s1, a2s1);
              q4_to_f16(wg8, a1s0, a3s0, a1s1, a3s1);
            }
            const uint32_t dw = kbi ? scw.y : scw.x;
            const float dg = __half2float(__ushort_as_half((unsigned short)(dw & 0xFFFFu)));
            const float dg8 = __half2float(__ushort_as_half((unsigned short)(dw >> 16)));
#pragma unroll
            for (int n = 0; n < NT; n++) {
              const uint4 xv = XH ? xh[kbi][XH ? n : 0] : xs[(kbi * NT + n) * 32 + lane];
              float cc[4];
              mma_16816(cc, a0s0, a1s0, a2s0, a3s0, xv.x, xv.y, zero4);
              mma_16816(cc, a0s1, a1s1, a2s1, a3s1, xv.z, xv.w, cc);
              acc[mt][n][0] = fmaf(dg, cc[0], acc[mt][n][0]);
              acc[mt][n][1] = fmaf(dg, cc[1], acc[mt][n][1]);
              acc[mt][n][2] = fmaf(dg8, cc[2], acc[mt][n][2]);
              acc[mt][n][3] = fmaf(dg8, cc[3], acc[mt][n][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (++st == S) {
        st = 0;
        ph ^= 1;
      }
    }

    fold_lo<NT>(acc);
    const bool full_tile = (ka == 0 && kb_end == a.kp);
    if (full_tile) {
      if (ok && has0) gemv_epilogue<NT>(a, mt0, has1, acc, g, t, xun);
    } else {
      // Partial tile: park this segment's sums; the arrival count and the
      // reduction wait until this CTA's last segment, so the stream never stalls.
      // In cluster mode the CTA holds its one segment in its own shared
      // memory (the drained ring), read by the other CTAs of the cluster.
      const int slot = first_seg ? 0 : 1;
      float *mine = a.cl > 1 ? reinterpret_cast<float *>(smem) : a.ws + ((size_t)c * 2 + slot) * WS_TILE_FLOATS;
      if (a.cl > 1) named_bar(1, QG_CONS_WARPS * 32);  // every warp is done with the ring
      if (has0 && t < 2) {
#pragma unroll
        for (int mt = 0; mt < 2; mt++)
#pragma unroll
          for (int n = 0; n < NT; n++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
              float *p = mine + ((warp * 2 + mt) * 16 + g + 8 * h) * 16 + n * 4 + 2 * t;
              float2 v = make_float2(acc[mt][n][2 * h], acc[mt][n][2 * h + 1]);
              if (XL) {  // local exponents differ between contributors: unscale before the sum (exact)
                v.x *= xun[n * 4 + 2 * t];
                v.y *= xun[n * 4 + 2 * t + 1];
              }
              *reinterpret_cast<float2 *>(p) = v;
            }
      }
      pslot[np] = slot;
      ptile[np++] = tile;
    }
    u += nk;
    first_seg = false;
  }

  if (np == 0) return;  // (sums of squares are only asked of fully split grids)
  // ---- split tiles: every contributor reduces a share of the rows ----
  // warp w's two m-tiles are reduced by contributor w % ncon: lane l sums row
  // l & 15 of m-tile l >> 4, four columns per n-tile (one float4 per
  // contributor and n-tile), over all contributors in CTA order.
  const int mt = lane >> 4, row = lane & 15;
  if (a.cl > 1) {
    // Cluster mode: the tile's contributors are the cluster's CTAs (ranks 0..cl-1
    // in CTA order); partials are read from their shared memory.  Both cluster
    // barriers are hardware barriers that every thread of the cluster reaches
    // (all earlier waits are bounded).
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster_sync_all();  // every CTA's partials are in its shared memory
    const int tile = ptile[0], r = (int)cluster.block_rank();
    const int mt0 = tile * QG_TILE_MT + warp * 2;
    if (__all_sync(0xffffffffu, ok) && warp % a.cl == r) {  // warp-uniform: split_epilogue shuffles
      const bool live = mt0 + mt < a.n_mt;
      float4 sum[NT];
#pragma unroll
      for (int n = 0; n < NT; n++) sum[n] = make_float4(0.f, 0.f, 0.f, 0.f);
      const int off = ((warp * 2 + mt) * 16 + row) * 16;
      if (live) {
        float4 v[4][NT];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          if (q >= a.cl) break;
          const float *src = cluster.map_shared_rank(reinterpret_cast<float *>(smem), q) + off;
#pragma unroll
          for (int n = 0; n < NT; n++) v[q][n] = *reinterpret_cast<const float4 *>(src + 4 * n);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
          if (q >= a.cl) break;
#pragma unroll
          for (int n = 0; n < NT; n++) {
            sum[n].x += v[q][n].x;
            sum[n].y += v[q][n].y;
            sum[n].z += v[q][n].z;
            sum[n].w += v[q][n].w;
          }
        }
      }
      split_epilogue<NT>(a, mt0, mt, row, live, sum, wst);
    }
    cluster_sync_all();  // no CTA leaves while another reads its shared memory
    if (XL && a.st_out && threadIdx.x < QG_STAT_COLS) {  // this CTA's slot: the warps' sums in warp order
      const float *w0 = xun + 16;
      float ss = 0.f;
      for (int w = 0; w < QG_CONS_WARPS; w++) ss += w0[w * 16 + threadIdx.x];
      a.st_out[(size_t)c * QG_STAT_COLS + threadIdx.x] = ss;
    }
    y_fence(a);  // row-sharded output: peer stores before the cross-GPU barrier
    return;
  }
  // Global mode.  All contributors of a split tile are resident (one CTA per
  // SM, G <= SMs, and PDL successors start only after every CTA of this grid
  // started), and each first publishes all its partials and only then waits,
  // so the waits below end; they are bounded all the same.  A contributor
  // publishes a partial by storing this launch's epoch into the flag of its
  // (CTA, slot) with release semantics; flags are never reset (a flag holding
  // an older epoch is simply not ready), so the CTA leaves right after its
  // share of the reduction.
  named_bar(1, QG_CONS_WARPS * 32);  // every partial of this CTA is stored
  if (threadIdx.x == 0)
    for (int j = 0; j < np; j++) st_release_gpu(a.cnt + c * 2 + pslot[j], a.epoch);
  for (int j = 0; j < np; j++) {
    const int tile = ptile[j];
    const int tu0 = tile * a.kp, tu1 = tu0 + a.kp - 1;
    const int c_first = ((tu0 + 1) * a.G - 1) / units;
    const int c_last = ((tu1 + 1) * a.G - 1) / units;
    const int ncon = c_last - c_first + 1, r = c - c_first;
    // partial slot of contributor cc: only the first contributor can have
    // begun before the tile (its slot 1); the tile opens every other's range
    const int slot_first = c_first * units / a.G >= tu0 ? 0 : 1;
    const int mt0 = tile * QG_TILE_MT + warp * 2;
    const bool mine = warp % ncon == r;
    const bool live = mt0 + mt < a.n_mt;
    // the rows this lane's share adds onto (EPI_ADD), loaded before the wait
    float yv[NT * 4];
    if (mine && a.epi == EPI_ADD)
#pragma unroll
      for (int i = 0; i < NT * 4; i++) {
        const int grow = (mt0 + mt) * 16 + row;
        yv[i] = live && i < a.B && grow < a.M ? __ldcg(a.y + y_off(a, i, grow)) : 0.f;
      }
    if (warp == 0) {  // lane q waits for contributors q, q + 32, ...
      const long long t0 = cycles_now();
      bool good = ok;
      for (int q = lane; q < ncon && good; q += 32) {
        const int cc = c_first + q;
        const int *f = a.cnt + cc * 2 + (q == 0 ? slot_first : 0);
        while (ld_acquire_gpu(f) != a.epoch) {
          if (spin_expired(t0)) {
            atomicExch(a.err, 3);
            good = false;
            break;
          }
        }
      }
      good = __all_sync(0xffffffffu, good);
      if (lane == 0) last_p[0] = good;
    }
    named_bar(1, QG_CONS_WARPS * 32);  // warp 0 saw every flag: the partials are visible to the CTA
    const bool go = last_p[0] != 0;
    if (go && mine) {
      float4 sum[NT];
#pragma unroll
      for (int n = 0; n < NT; n++) sum[n] = make_float4(0.f, 0.f, 0.f, 0.f);
      const size_t off = (size_t)((warp * 2 + mt) * 16 + row) * 16;
      constexpr int CH = NT == 1 ? 16 : (NT == 2 ? 4 : 2);  // independent loads in flight per lane
      if (live) {
        for (int c0 = c_first; c0 <= c_last; c0 += CH) {
          float4 v[CH][NT];
#pragma unroll
          for (int q = 0; q < CH; q++) {
            const int cc = c0 + q;
            if (cc > c_last) break;
            const float *src = a.ws + ((size_t)cc * 2 + (cc == c_first ? slot_first : 0)) * WS_TILE_FLOATS + off;
#pragma unroll
            for (int n = 0; n < NT; n++) v[q][n] = __ldcg(reinterpret_cast<const float4 *>(src + 4 * n));
          }
#pragma unroll
          for (int q = 0; q < CH; q++) {
            if (c0 + q > c_last) break;
#pragma unroll
            for (int n = 0; n < NT; n++) {
              sum[n].x += v[q][n].x;
              sum[n].y += v[q][n].y;
              sum[n].z += v[q][n].z;
              sum[n].w += v[q][n].w;
            }
          }
        }
      }
      split_epilogue<NT>(a, mt0, mt, row, live, sum, wst, a.epi == EPI_ADD ? yv : nullptr);
    }
    if (j + 1 < np) named_bar(1, QG_CONS_WARPS * 32);  // last_p is reused by the next tile
  }
  if (XL && a.st_out) named_bar(1, QG_CONS_WARPS * 32);  // every warp's sums of squares are in
  if (XL && a.st_out && threadIdx.x < QG_STAT_COLS) {  // this CTA's slot: the warps' sums in warp order
    const float *w0 = xun + 16;
    float ss = 0.f;
    for (int w = 0; w < QG_CONS_WARPS; w++) ss += w0[w * 16 + threadIdx.x];
    a.st_out[(size_t)c * QG_STAT_COLS + threadIdx.x] = ss;
  }
  y_fence(a);  // row-sharded output: peer stores before the cross-GPU barrier
}

// Thread-block clusters of cl CTAs of this kernel that can be resident at once
// (0: none / not queryable).
template <int TYPE, int NT, bool XL>
static int max_clusters(int cl) {
  using Lay = QgLayout<TYPE, NT, XL>;
  static int cache[5] = {-1, -1, -1, -1, -1};
  if (cl < 2 || cl > 4) return 0;
  if (cache[cl] < 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl * 64);
    cfg.blockDim = dim3(QGM_THREADS);
    cfg.dynamicSmemBytes = Lay::SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cl;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, qgemv_kernel<TYPE, NT, XL>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    cache[cl] = n;
  }
  return cache[cl];
}

template <int TYPE, int NT, bool XL>
static cudaError_t launch_t(GemvArgs a, cudaStream_t st) {
  using Lay = QgLayout<TYPE, NT, XL>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(qgemv_kernel<TYPE, NT, XL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Lay::SMEM);
    if (e != cudaSuccess) return e;
    e = carveout_max(qgemv_kernel<TYPE, NT, XL>);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  // Split tiles reduced inside thread-block clusters only when every tile's
  // cluster can be resident at once (the grid is one wave); the sums are the
  // same as the global path's (contributors in CTA order).
  if (a.cl > 1 && max_clusters<TYPE, NT, XL>(a.cl) < a.G / a.cl) a.cl = 1;
  if (a.cl > 1) return launch_pdl_cluster(qgemv_kernel<TYPE, NT, XL>, a.G, QGM_THREADS, Lay::SMEM, st, a.cl, a);
  return launch_pdl(qgemv_kernel<TYPE, NT, XL>, a.G, QGM_THREADS, Lay::SMEM, st, a);
}


cudaError_t launch(const GemvArgs &a, int type, bool xl, cudaStream_t st) {
  if (a.units * (a.G + 1) >= (1ll << 31)) return cudaErrorInvalidValue;  // the kernel's 32-bit unit arithmetic
  const int nt = (a.B + 3) / 4;  // n-tiles of 4 columns (hi | lo)
  if (xl) switch (nt) {
      case 1: return launch_t<2, 1, true>(a, st);
      case 2: return launch_t<2, 2, true>(a, st);
      case 3: return launch_t<2, 3, true>(a, st);
      default: return launch_t<2, 4, true>(a, st);
    }
  switch (nt * 16 + type) {
    case 16 + 8: return launch_t<8, 1, false>(a, st);
    case 32 + 8: return launch_t<8, 2, false>(a, st);
    case 48 + 8: return launch_t<8, 3, false>(a, st);
    case 64 + 8: return launch_t<8, 4, false>(a, st);
    case 16 + 2: return launch_t<2, 1, false>(a, st);
    case 32 + 2: return launch_t<2, 2, false>(a, st);
    case 48 + 2: return launch_t<2, 3, false>(a, st);
    default: return launch_t<2, 4, false>(a, st);
  }
}

cudaError_t configure() {
  cudaError_t e;
  if ((e = carveout_max(repack_kernel<2>)) != cudaSuccess) return e;
  if ((e = carveout_max(repack_kernel<8>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 1, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 2, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 3, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 4, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<8, 1, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<8, 2, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<8, 3, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<8, 4, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 1, true>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 2, true>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 3, true>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 4, true>)) != cudaSuccess) return e;
  return cudaSuccess;
}

}  // namespace mma
}  // namespace cw
