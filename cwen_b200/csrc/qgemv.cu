// Batched Q4_0 / Q8_0 GEMV for B <= 16 verify rows on sm_100a, on the
// 5th-generation tensor cores (tcgen05.mma with tensor memory).
//
// Replaces the reference's gemvb()/gemv() (run.c:1577-1680, 1419-1527) and
// the row dots under them (dot_q4_0 run.c:1009-1025, dot_nib16 run.c:432,
// dot_q8_0 run.c:1248-1274).
//
// Arithmetic.  The reference computes, per row and per 32-weight block,
//   y += d * sum_j (q_j - 8) * x_j          (fp32).
// Per block the dot runs on the tensor cores: (q - 8) (and the Q8_0 int8) is
// exact in f16, and X is split into f16 hi + lo parts (x = hi + lo to ~2^-22
// relative) after a per-column power-of-two scale that keeps it inside f16
// range.  For 128 rows x 32 weights x 16 columns four tcgen05.mma (M=128,
// N=16, K=16; A = the unpacked weights in tensor memory, B = X hi or lo in
// shared memory) accumulate
//   D = A*Xhi(k0..15) + A*Xlo(k0..15) + A*Xhi(k16..31) + A*Xlo(k16..31)
// in fp32 in tensor memory (products exact), and each row's thread applies
// the block's scale to its row of D on the CUDA cores: acc = fma(d, D, acc) --
// the reference's per-block scale on an fp32 block partial; y = acc * 2^-e.
// The legacy warp-level mma.sync path runs the same arithmetic at a fraction
// of this rate on sm_100a (its tensor pipe was the limit of the verify GEMV).
//
// Batch invariance.  Column b of any call depends only on column b of X: the
// MMAs are always 16 columns wide, each column of D is its own dot product,
// and the K partition (below) depends on the matrix shape and grid only,
// never on B.  So a B-row verify block produces the same bits as B single-row
// calls.
//
// Work split.  A fixed persistent grid of G <= #SM CTAs, one per SM, takes
// equal contiguous shares of the (512-row tile, k-pair) space ("stream-K").
// A tile cut between CTAs is reduced by its contributors, each summing a
// share of the rows over all contributors' partials in CTA (k) order, so the
// result does not depend on arrival order.
//
// Memory.  The weights of one (tile, k-pair) -- one contiguous 18 KB (Q4_0) /
// 34 KB (Q8_0) block of the repacked layout -- and the X operands of that
// k-pair stream HBM -> shared memory as two bulk (TMA) copies per stage into a
// ring, issued by two producer threads; 16 row warps unpack each stage into
// tensor memory and one thread issues the MMAs.  Every wait is bounded in
// time; a timeout raises an error flag and the CTA finishes without touching
// memory further.
#include <utility>

#include "common.cuh"
#include "qgemv.cuh"
#include "qgemv_dev.cuh"
#include "qmv.cuh"
#include "rowops.cuh"
#include "rowprep.cuh"
#include "sm100.cuh"

namespace cw {

// ---- weight repack: GGUF rows -> row-contiguous blocks per (tile, k-pair) ----
// One stage = one 512-row tile x one k-pair (two 32-blocks):
//   [block 0: 512 rows x QROW quant bytes][block 1: same][f16 scales: block 0 [512], block 1 [512]]
// QROW = 16 (Q4_0 nibbles) or 32 (Q8_0 int8).  Within every 4-byte group of a
// row's quant bytes the bytes are stored in the order [b0 b2 b1 b3], so that
// the exponent-trick unpack (q4_to_f16 / q8_to_f16) yields f16 pairs of
// consecutive K, the order of an A operand in tensor memory.  Rows at or past
// M stay zero.  Source row r lands in m-tile mt_off + (r/16)*mt_stride, row r%16.
template <int TYPE>
__global__ void repack_kernel(uint8_t *dst, int dst_kp, const uint8_t *src, int M, int K, int mt_off,
                              int mt_stride) {
  using S = QgStage<TYPE>;
  const int nb = K / 32, kp = K / 64;
  const long long total = (long long)M * kp;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(idx % kp);
    const int r = (int)(idx / kp);
    const int dmt = mt_off + (r / 16) * mt_stride;
    const int drow = (dmt % QG_TILE_MT) * 16 + r % 16;
    uint8_t *stg = dst + ((size_t)(dmt / QG_TILE_MT) * dst_kp + p) * S::WB;
    for (int kbi = 0; kbi < 2; kbi++) {
      const uint8_t *blk = src + ((size_t)r * nb + 2 * p + kbi) * (TYPE == 8 ? 34 : 18);
      uint8_t *q = stg + kbi * S::QB + drow * S::QROW;
#pragma unroll
      for (int g = 0; g < S::QROW; g += 4) {
        q[g + 0] = blk[2 + g + 0];
        q[g + 1] = blk[2 + g + 2];
        q[g + 2] = blk[2 + g + 1];
        q[g + 3] = blk[2 + g + 3];
      }
      uint8_t *sc = stg + 2 * S::QB + (kbi * QG_TILE_ROWS + drow) * 2;
      sc[0] = blk[0];
      sc[1] = blk[1];
    }
  }
}

cudaError_t qmat_repack(const QMat &dst, const uint8_t *src, int M, int mt_off, int mt_stride, cudaStream_t st) {
  const int src_mt = (M + 15) / 16;
  if (dst.kern == GK_QMV || dst.K % 64 || mt_off < 0 || mt_stride < 1 || mt_off + (src_mt - 1) * mt_stride >= dst.n_mt)
    return cudaErrorInvalidValue;
  if (!dst.tc) return mma::repack(dst, src, M, mt_off, mt_stride, st);
  const long long total = (long long)M * (dst.K / 64);
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  const int grid = (int)(blocks < 65535 ? blocks : 65535);
  if (dst.type == 8)
    repack_kernel<8><<<grid, threads, 0, st>>>(dst.w, dst.K / 64, src, M, dst.K, mt_off, mt_stride);
  else
    repack_kernel<2><<<grid, threads, 0, st>>>(dst.w, dst.K / 64, src, M, dst.K, mt_off, mt_stride);
  return cudaGetLastError();
}

// ---- X preparation (launch_row_prep: one thread-block cluster per column) ----
// Per column b: exponent e with max|x|*2^e in [2^14, 2^15), then the f16 hi
// and lo parts of the scaled column as B operands of the tensor cores: per
// 32-block 2 KB = two k16 steps x (hi tile 512 B, lo tile 512 B); a tile is
// 16 columns x 16 K, K-major without swizzle: column n, element k at byte
// (n % 8) * 16 + (n / 8) * 256 + (k / 8) * 128 + (k % 8) * 2.
cudaError_t gemv_prep_x(const float *X, int xs, int B, int K, GemvScratch &s, cudaStream_t st) {
  if (B < 1 || B > QG_MAXB || K % 64 || K > s.kmax) return cudaErrorInvalidValue;
  return launch_row_prep(X, xs, K, B, s, st);
}

// Tensor-memory plan of a CTA (512 columns): per row group rg (128 rows,
// tensor-memory lanes 0..127) 128 columns, two stage slots of 64 -- the
// stage's A operands (32 columns: two 32-blocks of K in f16 pairs) then its
// accumulators D (32 columns: two blocks x N = 16).
CW_DEV uint32_t tc_col_a(int rg, int ss) { return (uint32_t)(rg * 128 + ss * 64); }
CW_DEV uint32_t tc_col_d(int rg, int ss) { return tc_col_a(rg, ss) + 32; }
constexpr uint32_t TC_IDESC = tc_idesc_f16(128, 16);
constexpr int QG_MMA_WARP = QG_CONS_WARPS + 2;  // warps 18..21: one MMA issuer per row group

// Shared-memory layout of the GEMV.
template <int TYPE, bool XL>
struct QgLayout {
  using S = QgStage<TYPE>;
  static constexpr int WB = S::WB;                 // weights of one (tile, k-pair)
  static constexpr int XKP = 4096;                 // X operands of one k-pair (2 blocks x 2 KB)
  static constexpr int XB = XL ? 0 : XKP;          // ... streamed with each stage
  static constexpr int STAGE = WB + XB;
  static constexpr int STAGES = TYPE == 8 ? 5 : (XL ? 6 : 8);
  static constexpr int BAR_OFF = STAGES * STAGE;
  // full[S], empty[S], xready, a_ready[16], d_ready[16], fin, abort flag, tmem base
  static constexpr int BAR_BYTES = 1024;
  static constexpr int XL_OFF = BAR_OFF + BAR_BYTES;  // the CTA's k-range of X operands (<= QG_XL_KP k-pairs)
  static constexpr int XL_BYTES = XL ? QG_XL_KP * XKP : 0;
  // per column: 2^-e [16] floats, the warps' output sums of squares [16][16],
  // the prologue's per-warp column maxima [16]
  static constexpr int XE_OFF = XL_OFF + XL_BYTES;
  static constexpr int SMEM = XE_OFF + (XL ? 64 + 16 * 16 * 4 + 16 * 4 : 0);
  static_assert(WB % 16 == 0 && XB % 16 == 0 && STAGE % 128 == 0, "bulk copies need 16-byte multiples");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(2 * STAGES + 2 + 2 * 8 + 4 <= BAR_BYTES / 8, "barrier area");
};

// Byte offset of (column n, 8-K chunk c) of a 32-block's X operands:
// k16 step c / 2, hi (hl 0) or lo (hl 1) tile, K-chunk c % 2.
CW_DEV int xop_off(int n, int c, int hl) { return (c >> 1) * 1024 + hl * 512 + (n >> 3) * 256 + (c & 1) * 128 + (n & 7) * 16; }

// Local X (run by the 16 row warps once, after pdl_wait): the CTA's k-range
// [64*ka0, 64*(ka0+nkp)) of every column of the raw rows X becomes f16 hi/lo
// B operands in shared memory, scaled by the CTA's own power of two 2^e (max
// |x| over the range in [2^14, 2^15)); xun[col] = 2^-e unscales the CTA's
// results.  The operands hold the same values and layout gemv_prep_x emits,
// except for the exponent's range; columns B..15 hold stale values that only
// reach accumulator columns nobody reads.  A column gets
// 16 / B warps (at least one); each lane loads 8 values per item (item = one
// 8-K chunk), keeps them in registers while the column maxima are combined
// through shared memory (one barrier), then converts them.
// MAXI: items per lane, the most a column's warps need for the batch sizes
// of the caller (5 with one warp per column, 3 with two, 1 with sixteen).
template <int MAXI>
CW_DEV void x_local_prologue(const GemvArgs &a, uint8_t *xl, float *xun, float *cmax, int ka0, int nkp) {
  constexpr int NTH = QG_CONS_WARPS * 32;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nitems = nkp * 8;
  const int wpc = a.B >= QG_CONS_WARPS ? 1 : QG_CONS_WARPS / a.B;  // warps per column
  const int b = w / wpc, sub = w - b * wpc;
  const bool live = b < a.B;
  float4 v[MAXI][2];
  float m = 0.f, ss = 0.f;
  if (live) {
    const float *x = a.xr + (size_t)b * a.xrs + (size_t)ka0 * 64;
    const float *wn = a.xw ? a.xw + (size_t)ka0 * 64 : nullptr;
    // RMSNorm: the row's sum of squares from the per-CTA partials of the GEMV
    // that wrote it, in slot order then a fixed xor tree (every CTA, every B)
    if (a.xw)
#pragma unroll
      for (int i = 0; i < 5; i++)
        if (lane + 32 * i < a.st_g) ss += __ldcg(a.st_in + (size_t)(lane + 32 * i) * QG_STAT_COLS + b);
#pragma unroll
    for (int j = 0; j < MAXI; j++) {
      const int it = (sub + j * wpc) * 32 + lane;
      if (it < nitems) {
        float4 p = __ldg(reinterpret_cast<const float4 *>(x + it * 8));
        float4 q = __ldg(reinterpret_cast<const float4 *>(x + it * 8 + 4));
        if (wn) {
          const float4 wp = __ldg(reinterpret_cast<const float4 *>(wn + it * 8));
          const float4 wq = __ldg(reinterpret_cast<const float4 *>(wn + it * 8 + 4));
          p = make_float4(wp.x * p.x, wp.y * p.y, wp.z * p.z, wp.w * p.w);
          q = make_float4(wq.x * q.x, wq.y * q.y, wq.z * q.z, wq.w * q.w);
        }
        v[j][0] = p;
        v[j][1] = q;
        m = fmaxf(m, fmaxf(fmaxf(fabsf(p.x), fabsf(p.y)), fmaxf(fabsf(p.z), fabsf(p.w))));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w))));
      }
    }
    m = warp_max(m);
    if (lane == 0) cmax[w] = m;
  }
  // Columns B..15 of the B operands are left as they are: column n of D
  // depends only on column n of B, and those accumulator columns are never read.
  named_bar(1, NTH);
  if (live) {
    m = 0.f;
    for (int i = 0; i < wpc; i++) m = fmaxf(m, cmax[b * wpc + i]);
    float s = 1.f;
    if (a.xw) {
      s = 1.f / sqrtf(warp_sum(ss) / (float)(a.kp * 64) + 1e-6f);
      m *= s;  // max |(w x) s| = max |w x| * s: s > 0 and rounding is monotonic
    }
    const int e = xfrag_exponent(m);
    // ((w x) s) 2^e == (w x) (s 2^e) exactly: 2^e only shifts the exponent
    const float sc = s * __int_as_float((127 + e) << 23);
    if (sub == 0 && lane == 0) xun[b] = __int_as_float((127 - e) << 23);
#pragma unroll
    for (int j = 0; j < MAXI; j++) {
      const int it = (sub + j * wpc) * 32 + lane;
      if (it < nitems) {
        const float r[8] = {v[j][0].x, v[j][0].y, v[j][0].z, v[j][0].w, v[j][1].x, v[j][1].y, v[j][1].z, v[j][1].w};
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float v0 = r[2 * i] * sc, v1 = r[2 * i + 1] * sc;
          const half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
          const half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
          hw[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
          lw[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        uint8_t *o = xl + (it >> 2) * 2048 + xop_off(b, it & 3, 0);
        *reinterpret_cast<uint4 *>(o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(o + 512) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
    }
  }
  if (threadIdx.x >= a.B && threadIdx.x < 16) xun[threadIdx.x] = 1.f;  // padding column
  fence_proxy_async_smem();  // the operands are read by the tensor cores (async proxy)
  named_bar(1, NTH);
}

// One row's 32-block of quant bytes (QROW bytes at q) -> 16 f16 pairs of
// consecutive K (the A operand row in tensor memory), exact.
template <int TYPE>
CW_DEV void unpack_row_block(const uint8_t *q, uint32_t (&r)[16]) {
  if (TYPE == 8) {
    const uint4 u0 = *reinterpret_cast<const uint4 *>(q), u1 = *reinterpret_cast<const uint4 *>(q + 16);
    const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
    for (int i = 0; i < 8; i++) q8_to_f16(w[i], r[2 * i], r[2 * i + 1]);
  } else {
    const uint4 u = *reinterpret_cast<const uint4 *>(q);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    // word i holds K 4i..4i+3 (low nibbles) and 16+4i..16+4i+3 (high nibbles)
#pragma unroll
    for (int i = 0; i < 4; i++) q4_to_f16(w[i], r[2 * i], r[2 * i + 1], r[8 + 2 * i], r[8 + 2 * i + 1]);
  }
}

// Persistent stream-K GEMV on the 5th-generation tensor cores.
//
// Warps 0..15 ("row warps") own rows 32w..32w+31 of the current 512-row tile
// (row group w / 4 of 128 rows, tensor-memory lanes 32 (w % 4)..+31).  Lane 0
// of warp 16 streams the weights, lane 0 of warp 17 the X operands, and lane
// 0 of warp 18 + rg issues the MMAs of row group rg (one issuing thread
// sustains only ~one tcgen05.mma per 50 cycles; four in parallel ~one per 15).
// Per stage s (two 32-blocks) of the CTA's range:
//   row thread: unpack its row's quant bytes of both blocks to f16 and store
//     them as the A operands of stage slot s % 2 in tensor memory
//     (tcgen05.st), arrive on a_ready;
//   issuer of the row group: per block D[128 x 16] = A * Xhi(k 0..15)
//     + A * Xlo(k 0..15) + A * Xhi(k 16..31) + A * Xlo(k 16..31) (four
//     tcgen05.mma M=128 N=16 K=16, fp32 accumulate), commit -> d_ready;
//   row thread, one stage later: read its row of both blocks' D (tcgen05.ld)
//     and apply each block's f16 scale: acc[col] = fma(d, D[col], acc[col])
//     -- the reference's per-block scale on an fp32 block partial.
// NC: the accumulator columns read (1, 8 or 16 >= B).
template <int TYPE, int NC, bool XL>
__global__ void __launch_bounds__(QG_THREADS, 1) qgemv_kernel(GemvArgs a) {
  using Lay = QgLayout<TYPE, XL>;
  using Stg = QgStage<TYPE>;
  constexpr int S = Lay::STAGES;
  constexpr int NC4 = NC >= 16 ? 4 : (NC >= 8 ? 2 : 1);  // float4 column groups of a split-tile row
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Lay::BAR_OFF);
  uint64_t *empty = full + S;
  uint64_t *xready = empty + S;      // local X: the prologue's operands are in shared memory
  uint64_t *a_ready = xready + 1;  // [4 row groups][2 stage slots]
  uint64_t *d_ready = a_ready + 8;
  uint64_t *fin = d_ready + 8;      // [4]: every MMA of a row group's issuer has completed
  volatile int *abort_p = reinterpret_cast<volatile int *>(fin + 4);
  int *last_p = const_cast<int *>(abort_p) + 1;  // [2]
  uint32_t *tmem_base_p = reinterpret_cast<uint32_t *>(last_p + 2);
  static_assert(2 * Lay::STAGES + 1 + 8 + 8 + 4 + 2 <= Lay::BAR_BYTES / 8, "barrier area");

  const int c = blockIdx.x;
  const long long u_begin = (long long)c * a.units / a.G, u_end = (long long)(c + 1) * a.units / a.G;
  if (u_begin >= u_end) return;  // whole CTA, before any barrier
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nst = (int)(u_end - u_begin);  // stages (k-pairs) of this CTA
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&full[i], XL ? 1 : 2);  // the weight and the X producer
      mbar_init(&empty[i], QG_CONS_WARPS);
    }
    mbar_init(xready, 1);
    for (int i = 0; i < 8; i++) {
      mbar_init(&a_ready[i], 4);  // the 4 row warps of a row group
      mbar_init(&d_ready[i], 1);  // tcgen05.commit
    }
    for (int i = 0; i < 4; i++) mbar_init(&fin[i], 1);
    *abort_p = 0;
    mbar_fence_init();
  }
  if (warp == QG_MMA_WARP) tmem_alloc(tmem_base_p, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_base_p;

  if (warp >= QG_CONS_WARPS && warp < QG_MMA_WARP) {
    // ---------------- producers ----------------
    // Two producer threads in two warps, one for the weights and one for X:
    // a bulk copy occupies its issuing thread for ~0.3 us whatever its size,
    // so one thread issuing both copies of a stage would cap the stream.
    // Consecutive units are consecutive (tile, k-pair) blocks of the repacked
    // weights, so the weight source just advances; no divisions in the loops.
    if (lane == 0 && (!XL || warp == QG_CONS_WARPS)) {  // local X: no X copies
      const bool wprod = warp == QG_CONS_WARPS;
      const int n = (int)(u_end - u_begin);
      const uint8_t *wsrc = a.w + (size_t)u_begin * Lay::WB;
      const uint8_t *xbase = reinterpret_cast<const uint8_t *>(a.xf);
      // Weights are not written by any kernel of the decode step: the weight
      // producer never waits for the previous kernel (PDL), so the ring fills
      // while that kernel finishes.  X is that kernel's output.
      if (!wprod) pdl_wait();
      int k = (int)(u_begin % a.kp);
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
        // Local X: two weight stages go ahead, the rest after the prologue has
        // read X -- its loads would otherwise queue behind a full ring of weights.
        if (XL && wprod && issued == 2 && !mbar_wait(xready, 0, abort_p)) {
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

  if (warp >= QG_MMA_WARP) {
    // ---------------- MMA issuers (one per row group) ----------------
    const int rg = warp - QG_MMA_WARP;
    if (lane == 0) {
      bool ok = true;
      if (XL && !mbar_wait(xready, 0, abort_p)) ok = false;
      const uint32_t xl_s = smem_u32(smem + Lay::XL_OFF);
      for (int sg = 0; sg < nst && ok; sg++) {
        const int stage = sg % S, ss = sg & 1;
        uint32_t xs;
        if (XL) {
          xs = xl_s + (uint32_t)sg * 4096u;
        } else {
          // the X operands of the stage have landed (the row warps waited too)
          if (!mbar_wait(&full[stage], (uint32_t)((sg / S) & 1), abort_p)) {
            ok = false;
            break;
          }
          xs = smem_u32(smem + stage * Lay::STAGE + Lay::WB);
        }
        if (!mbar_wait(&a_ready[rg * 2 + ss], (uint32_t)((sg >> 1) & 1), abort_p)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kbi = 0; kbi < 2; kbi++) {
          const uint32_t xb = xs + (uint32_t)kbi * 2048u;
          const uint32_t ta = tbase + tc_col_a(rg, ss) + 16 * kbi, td = tbase + tc_col_d(rg, ss) + 16 * kbi;
          tc_mma_ts(td, ta, smem_desc_kmajor(xb, 128, 256), TC_IDESC, 0u);
          tc_mma_ts(td, ta, smem_desc_kmajor(xb + 512, 128, 256), TC_IDESC, 1u);
          tc_mma_ts(td, ta + 8, smem_desc_kmajor(xb + 1024, 128, 256), TC_IDESC, 1u);
          tc_mma_ts(td, ta + 8, smem_desc_kmajor(xb + 1536, 128, 256), TC_IDESC, 1u);
        }
        tc_commit(&d_ready[rg * 2 + ss]);
      }
      if (!ok) {
        atomicExch(a.err, 4);
        *abort_p = 1;
      }
      // every MMA issued has completed before the tensor memory is released
      tc_commit(&fin[rg]);
      const long long t0 = cycles_now();
      while (!mbar_try_wait(&fin[rg], 0) && !spin_expired(t0)) {
      }
    }
    __syncwarp();
    named_bar(2, (QG_CONS_WARPS + 4) * 32);  // the row warps are done with the tensor memory
    if (warp == QG_MMA_WARP) {
      tc_fence_after();
      tmem_dealloc(tbase, 512);
    }
    if (a.cl > 1) {
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }

  // ---------------- row warps ----------------
  pdl_wait();  // before touching Y, the split-K partials or the tile counters
  const int rg = warp >> 2;
  const uint32_t tl = tbase + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's lanes
  const int rrow = warp * 32 + lane;                                   // row within the tile
  const int ka0 = (int)(u_begin % a.kp);  // local X: the CTA's one segment starts here
  float *xun = XL ? reinterpret_cast<float *>(smem + Lay::XE_OFF) : nullptr;
  float *wst = XL ? xun + 16 + warp * 16 : nullptr;  // this warp's output sums of squares per column
  if (XL && a.st_out && lane < 16) wst[lane] = 0.f;
  if (XL) {
    // items per lane: ceil(QG_XL_KP * 8 / (32 * warps per column)), warps per column 16 / B
    constexpr int MAXI = NC == 1 ? 1 : (NC == 8 ? 3 : 5);
    static_assert(QG_XL_KP * 8 <= 32 * 5 && QG_XL_KP * 8 <= 64 * 3 && QG_XL_KP * 8 <= 512 * 1, "prologue items");
    x_local_prologue<MAXI>(a, smem + Lay::XL_OFF, xun, xun + 16 + 16 * 16, ka0, (int)(u_end - u_begin));
    if (threadIdx.x == 0) mbar_arrive(xready);
  }
  bool ok = true;
  long long u = u_begin;
  int sg = 0;  // the CTA's stage counter (ring stage sg % S, tensor-memory stage slot sg % 2)
  bool first_seg = true;
  int ptile[2];  // split tiles of this CTA (its first and last segments), uniform across the CTA
  int np = 0;
  float dp0 = 0.f, dp1 = 0.f;  // scales of the stage whose accumulators are pending

  // accumulate stage sp's two blocks of D into acc (block 0 first); for
  // streamed X the ring stage is released once its MMAs have completed
  auto drain = [&](int sp, float (&acc)[NC]) {
    const int ss = sp & 1;
    if (ok && !mbar_wait(&d_ready[rg * 2 + ss], (uint32_t)((sp >> 1) & 1), abort_p)) {
      ok = false;
      atomicExch(a.err, 2);
      *abort_p = 1;
    }
    tc_fence_after();
    const uint32_t td = tl + tc_col_d(rg, ss);
#pragma unroll
    for (int kbi = 0; kbi < 2; kbi++) {
      const float d = kbi ? dp1 : dp0;
      if (NC == 1) {
        uint32_t r[1];
        tmem_ld1(td + 16 * kbi, r);
        tmem_wait_ld();
        acc[0] = fmaf(d, __uint_as_float(r[0]), acc[0]);
      } else if (NC == 8) {
        uint32_t r[8];
        tmem_ld8(td + 16 * kbi, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < NC; i++) acc[i] = fmaf(d, __uint_as_float(r[i]), acc[i]);
      } else {
        uint32_t r[16];
        tmem_ld16(td + 16 * kbi, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < NC; i++) acc[i] = fmaf(d, __uint_as_float(r[i]), acc[i]);
      }
    }
    if (!XL) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[sp % S]);
    }
  };

  while (u < u_end) {
    const int tile = (int)(u / a.kp);
    const int ka = (int)(u % a.kp);
    const long long remain = u_end - u;
    const int kb_end = (int)((long long)(a.kp - ka) < remain ? a.kp : ka + remain);
    const int nk = kb_end - ka;
    const int s0 = sg;
    float acc[NC];
#pragma unroll
    for (int i = 0; i < NC; i++) acc[i] = 0.f;

    for (int i = 0; i < nk; i++, sg++) {
      const int stage = sg % S, ss = sg & 1;
      if (ok && !mbar_wait(&full[stage], (uint32_t)((sg / S) & 1), abort_p)) {
        ok = false;
        atomicExch(a.err, 2);
        *abort_p = 1;
      }
      const uint8_t *stg = smem + stage * Lay::STAGE;
      const float d0 = __half2float(*reinterpret_cast<const __half *>(stg + 2 * Stg::QB + rrow * 2));
      const float d1 = __half2float(*reinterpret_cast<const __half *>(stg + 2 * Stg::QB + (QG_TILE_ROWS + rrow) * 2));
#pragma unroll
      for (int kbi = 0; kbi < 2; kbi++) {  // one block at a time: 16 live registers
        uint32_t r[16];
        unpack_row_block<TYPE>(stg + kbi * Stg::QB + rrow * Stg::QROW, r);
        tmem_st16(tl + tc_col_a(rg, ss) + 16 * kbi, r);
      }
      if (XL) {  // the stage's quant bytes and scales have been read
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_ready[rg * 2 + ss]);  // this stage's MMAs may start ...
      if (sg > s0) drain(sg - 1, acc);  // ... while the previous stage's accumulators are read
      dp0 = d0;
      dp1 = d1;
    }
    if (sg > s0) drain(sg - 1, acc);

    const bool full_tile = (ka == 0 && kb_end == a.kp);
    const int mt0 = tile * QG_TILE_MT + warp * 2;  // this warp's rows: m-tiles mt0 (lanes 0-15), mt0 + 1
    if (full_tile) {
      if (ok) {
        if (a.epi == EPI_SWIGLU) {  // gate rows in lanes 0-15, their up rows in lanes 16-31
#pragma unroll
          for (int col = 0; col < NC; col++) {
            const float up = __shfl_down_sync(0xffffffffu, acc[col], 16);
            if (col < a.B && lane < 16) {
              const float sc = xun ? xun[col] : __int_as_float((127 - __ldg(a.xexp + col)) << 23);
              const int row = (mt0 >> 1) * 16 + lane;
              if (row * 2 < a.M) y_put(a, y_off(a, col, row), silu_f(acc[col] * sc) * (up * sc));
            }
          }
        } else {
          const int row = tile * QG_TILE_ROWS + rrow;
#pragma unroll
          for (int col = 0; col < NC; col++) {
            if (col >= a.B || row >= a.M) continue;
            const float sc = xun ? xun[col] : __int_as_float((127 - __ldg(a.xexp + col)) << 23);
            y_out(a, col, row, acc[col] * sc);
          }
        }
      }
    } else {
      // Partial tile: park this segment's sums; the arrival count and the
      // reduction wait until this CTA's last segment, so the stream never stalls.
      // In cluster mode the CTA holds its one segment in its own shared
      // memory (the drained ring), read by the other CTAs of the cluster.
      const int slot = first_seg ? 0 : 1;
      float *mine = a.cl > 1 ? reinterpret_cast<float *>(smem) : a.ws + ((size_t)c * 2 + slot) * WS_TILE_FLOATS;
      if (a.cl > 1) named_bar(1, QG_CONS_WARPS * 32);  // every warp is done with the ring
      float *p = mine + rrow * 16;
#pragma unroll
      for (int col = 0; col < NC; col += 4) {
        float4 v;
        if (NC == 1) {
          v = make_float4(acc[0], 0.f, 0.f, 0.f);
        } else {
          v = make_float4(acc[col], acc[col + 1], acc[col + 2], acc[col + 3]);
        }
        if (XL) {  // local exponents differ between contributors: unscale before the sum (exact)
          v.x *= xun[col];
          if (NC > 1) {
            v.y *= xun[col + 1];
            v.z *= xun[col + 2];
            v.w *= xun[col + 3];
          }
        }
        *reinterpret_cast<float4 *>(p + col) = v;
      }
      ptile[np++] = tile;
    }
    u += nk;
    first_seg = false;
  }
  // the tensor memory is no longer read by this warp
  tc_fence_before();
  named_bar(2, (QG_CONS_WARPS + 4) * 32);
  y_fence(a);  // full tiles' peer stores

  if (np == 0) {
    if (a.cl > 1) {
      cluster_sync_all();
      cluster_sync_all();
    }
    return;  // (sums of squares are only asked of fully split grids)
  }
  // ---- split tiles: every contributor reduces a share of the rows ----
  // warp w's two m-tiles are reduced by contributor w % ncon: lane l sums row
  // l & 15 of m-tile l >> 4, four columns per float4 (NC4 float4s per
  // contributor), over all contributors in CTA order.
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
      float4 sum[NC4];
#pragma unroll
      for (int n = 0; n < NC4; n++) sum[n] = make_float4(0.f, 0.f, 0.f, 0.f);
      const int off = ((warp * 2 + mt) * 16 + row) * 16;
      if (live) {
        float4 v[4][NC4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          if (q >= a.cl) break;
          const float *src = cluster.map_shared_rank(reinterpret_cast<float *>(smem), q) + off;
#pragma unroll
          for (int n = 0; n < NC4; n++) v[q][n] = *reinterpret_cast<const float4 *>(src + 4 * n);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
          if (q >= a.cl) break;
#pragma unroll
          for (int n = 0; n < NC4; n++) {
            sum[n].x += v[q][n].x;
            sum[n].y += v[q][n].y;
            sum[n].z += v[q][n].z;
            sum[n].w += v[q][n].w;
          }
        }
      }
      split_epilogue<NC4>(a, mt0, mt, row, live, sum, wst);
    }
    y_fence(a);
    cluster_sync_all();  // no CTA leaves while another reads its shared memory
    if (XL && a.st_out && threadIdx.x < QG_STAT_COLS) {  // this CTA's slot: the warps' sums in warp order
      const float *w0 = xun + 16;
      float ss = 0.f;
      for (int w = 0; w < QG_CONS_WARPS; w++) ss += w0[w * 16 + threadIdx.x];
      a.st_out[(size_t)c * QG_STAT_COLS + threadIdx.x] = ss;
    }
    return;
  }
  // Global mode.  All contributors of a split tile are resident (one CTA per
  // SM, G <= SMs, and PDL successors start only after every CTA of this grid
  // started), and each first counts itself in for all its split tiles and
  // only then waits, so the waits below end; they are bounded all the same.
  // The counter of a tile goes 0 -> n (partials parked) -> 2n (shares
  // reduced) -> 0.
  named_bar(1, QG_CONS_WARPS * 32);
  if (threadIdx.x == 0) {
    __threadfence();  // the CTA's partials (ordered before by the barrier), before the arrival
    for (int jt = 0; jt < np; jt++) atomicAdd(a.cnt + ptile[jt], 1);
  }
  for (int jt = 0; jt < np; jt++) {
    const int tile = ptile[jt];
    const long long tu0 = (long long)tile * a.kp, tu1 = tu0 + a.kp - 1;
    const int c_first = (int)(((tu0 + 1) * a.G - 1) / a.units);
    const int c_last = (int)(((tu1 + 1) * a.G - 1) / a.units);
    const int ncon = c_last - c_first + 1, r = c - c_first;
    if (threadIdx.x == 0) {
      const long long t0 = cycles_now();
      while (ok && *(volatile int *)(a.cnt + tile) < ncon) {
        if (spin_expired(t0)) {
          atomicExch(a.err, 3);
          ok = false;
        }
      }
      __threadfence();  // the other contributors' partials, after their arrivals
      last_p[0] = ok;
    }
    named_bar(1, QG_CONS_WARPS * 32);
    const bool go = last_p[0] != 0;
    const int mt0 = tile * QG_TILE_MT + warp * 2;
    if (go && warp % ncon == r) {
      const bool live = mt0 + mt < a.n_mt;
      float4 sum[NC4];
#pragma unroll
      for (int n = 0; n < NC4; n++) sum[n] = make_float4(0.f, 0.f, 0.f, 0.f);
      const size_t off = (size_t)((warp * 2 + mt) * 16 + row) * 16;
      constexpr int CH = NC4 <= 2 ? 4 : 2;  // independent loads in flight per lane
      if (live) {
        for (int c0 = c_first; c0 <= c_last; c0 += CH) {
          float4 v[CH][NC4];
#pragma unroll
          for (int q = 0; q < CH; q++) {
            const int cc = c0 + q;
            if (cc > c_last) break;
            const long long cu0 = (long long)cc * a.units / a.G;
            const float *src = a.ws + ((size_t)cc * 2 + (cu0 >= tu0 ? 0 : 1)) * WS_TILE_FLOATS + off;
#pragma unroll
            for (int n = 0; n < NC4; n++) v[q][n] = __ldcg(reinterpret_cast<const float4 *>(src + 4 * n));
          }
#pragma unroll
          for (int q = 0; q < CH; q++) {
            if (c0 + q > c_last) break;
#pragma unroll
            for (int n = 0; n < NC4; n++) {
              sum[n].x += v[q][n].x;
              sum[n].y += v[q][n].y;
              sum[n].z += v[q][n].z;
              sum[n].w += v[q][n].w;
            }
          }
        }
      }
      split_epilogue<NC4>(a, mt0, mt, row, live, sum, wst);
    }
    named_bar(1, QG_CONS_WARPS * 32);  // every read of the partials of this tile is done
    if (threadIdx.x == 0 && go) {
      if (atomicAdd(a.cnt + tile, 1) == 2 * ncon - 1) a.cnt[tile] = 0;
    }
  }
  y_fence(a);
  if (XL && a.st_out && threadIdx.x < QG_STAT_COLS) {  // this CTA's slot: the warps' sums in warp order
    const float *w0 = xun + 16;
    float ss = 0.f;
    for (int w = 0; w < QG_CONS_WARPS; w++) ss += w0[w * 16 + threadIdx.x];
    a.st_out[(size_t)c * QG_STAT_COLS + threadIdx.x] = ss;
  }
}

size_t gemv_scratch_ws_floats(int G) { return (size_t)G * 2 * WS_TILE_FLOATS; }

// Thread-block clusters of cl CTAs of this kernel that can be resident at once
// (0: none / not queryable).
template <int TYPE, int NC, bool XL>
static int max_clusters(int cl) {
  using Lay = QgLayout<TYPE, XL>;
  static int cache[5] = {-1, -1, -1, -1, -1};
  if (cl < 2 || cl > 4) return 0;
  if (cache[cl] < 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl * 64);
    cfg.blockDim = dim3(QG_THREADS);
    cfg.dynamicSmemBytes = Lay::SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cl;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, qgemv_kernel<TYPE, NC, XL>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    cache[cl] = n;
  }
  return cache[cl];
}

template <int TYPE, int NC, bool XL>
static cudaError_t launch_t(GemvArgs a, cudaStream_t st) {
  using Lay = QgLayout<TYPE, XL>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(qgemv_kernel<TYPE, NC, XL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Lay::SMEM);
    if (e != cudaSuccess) return e;
    e = carveout_max(qgemv_kernel<TYPE, NC, XL>);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  // Split tiles reduced inside thread-block clusters only when every tile's
  // cluster can be resident at once (the grid is one wave); the sums are the
  // same as the global path's (contributors in CTA order).
  if (a.cl > 1 && max_clusters<TYPE, NC, XL>(a.cl) < a.G / a.cl) a.cl = 1;
  if (a.cl > 1) return launch_pdl_cluster(qgemv_kernel<TYPE, NC, XL>, a.G, QG_THREADS, Lay::SMEM, st, a.cl, a);
  return launch_pdl(qgemv_kernel<TYPE, NC, XL>, a.G, QG_THREADS, Lay::SMEM, st, a);
}

// Grid of a GEMV: a function of the shape only (never of B), >= 4 k-pairs per
// CTA.  When the tiles are fewer than the CTAs, a multiple of the tile count:
// every tile is then split evenly between the same number of CTAs and every
// CTA holds exactly one segment (one split tile at most), instead of the
// arbitrary cuts of stream-K that give some CTAs two split tiles and two
// reductions.
static long long gemv_grid(const QMat &m, const GemvScratch &s, int &n_tiles, long long &units) {
  n_tiles = (m.n_mt + QG_TILE_MT - 1) / QG_TILE_MT;
  units = (long long)n_tiles * (m.K / 64);
  long long g = (units + 3) / 4;
  if (g > s.G) g = s.G;
  if (n_tiles <= g) g = g / n_tiles * n_tiles;
  return g;
}

// The local-X variant applies when the grid is tile-aligned and every CTA's
// k-range holds at most QG_XL_KP (tcgen05) / QG_XL_KP_MMA k-pairs -- decided on the shape alone, so
// that every B takes the same path (batch invariance).
static bool gemv_local_x(const QMat &m, const GemvScratch &s) {
  int n_tiles;
  long long units;
  const long long g = gemv_grid(m, s, n_tiles, units);
  if (m.type != 2 || n_tiles > g) return false;
  const long long ncon = g / n_tiles, kp = m.K / 64;
  return (kp + ncon - 1) / ncon <= (s.tc ? QG_XL_KP : QG_XL_KP_MMA);
}

// Every tile split between >= 2 CTAs (each CTA one segment): the epilogue's
// row statistics are then all taken in the split-tile reduction.
static bool gemv_all_split(const QMat &m, const GemvScratch &s) {
  int n_tiles;
  long long units;
  const long long g = gemv_grid(m, s, n_tiles, units);
  return n_tiles <= g && g / n_tiles >= 2;
}

static cudaError_t gemv_launch(const QMat &m, int B, float *Y, int ys, int epi, GemvScratch &s, cudaStream_t st,
                               const float *xr, int xrs, const float *norm_w = nullptr, bool want_stats = false) {
  if (B < 1 || B > QG_MAXB || m.K % 64 || m.K > s.kmax || !m.w || !s.err || m.tc != s.tc || m.kern != s.kern ||
      m.kern == GK_QMV)
    return cudaErrorInvalidValue;
  if (epi == EPI_SWIGLU && (m.n_mt % 2)) return cudaErrorInvalidValue;
  GemvArgs a;
  a.w = m.w;
  a.n_mt = m.n_mt;
  a.kp = m.K / 64;
  a.M = m.M;
  a.xf = s.xf;
  a.xexp = s.xexp;
  a.B = B;
  a.y = Y;
  a.ys = ys;
  a.epi = epi;
  a.ws = s.ws;
  a.cnt = s.cnt;
  if (++s.epoch == 0) s.epoch = 1;
  a.epoch = s.epoch;
  a.err = s.err;
  a.xr = xr;
  a.xrs = xrs;
  a.xw = nullptr;
  a.st_in = nullptr;
  a.st_g = 0;
  a.st_out = nullptr;
  if (xr && norm_w) {
    a.xw = norm_w;
    a.st_in = s.stat;
    a.st_g = s.stat_g;
  }
  if (xr && want_stats) a.st_out = s.stat_next;
  a.row0 = s.row0;
  a.np = s.np;
  for (int i = 0; i < QG_MAX_PEERS; i++) a.yp[i] = i < s.np ? s.yp[i] : nullptr;
  int n_tiles;
  const long long g = gemv_grid(m, s, n_tiles, a.units);
  if (n_tiles > s.max_tiles || 2 * g > s.max_tiles) return cudaErrorInvalidValue;  // counters / flags
  a.G = (int)g;
  // 2 to 4 contributors per tile: reduce inside a thread-block cluster
  // (distributed shared memory) instead of through global scratch
  a.cl = 1;
  if (n_tiles <= g && g / n_tiles >= 2 && g / n_tiles <= 4) a.cl = (int)(g / n_tiles);
  // accumulator columns read per block: 1, 8 or 16 (the MMAs are 16 wide either way)
  const int nc = B == 1 ? 1 : (B <= 8 ? 8 : 16);
  s.stat_ok = false;  // statistics describe the output of the GEMV right before
  if (xr) {
    cudaError_t e;
    if (!s.tc) e = mma::launch(a, m.type, true, st);
    else switch (nc) {
      case 1: e = launch_t<2, 1, true>(a, st); break;
      case 8: e = launch_t<2, 8, true>(a, st); break;
      default: e = launch_t<2, 16, true>(a, st); break;
    }
    if (e == cudaSuccess && a.st_out) {
      std::swap(s.stat, s.stat_next);
      s.stat_ok = true;
      s.stat_g = a.G;
      s.stat_y = Y;
      s.stat_ys = ys;
      s.stat_len = m.M;
      s.stat_cols = B;
    }
    return e;
  }
  if (!s.tc) return mma::launch(a, m.type, false, st);
  switch (nc * 16 + m.type) {
    case 16 + 8: return launch_t<8, 1, false>(a, st);
    case 128 + 8: return launch_t<8, 8, false>(a, st);
    case 256 + 8: return launch_t<8, 16, false>(a, st);
    case 16 + 2: return launch_t<2, 1, false>(a, st);
    case 128 + 2: return launch_t<2, 8, false>(a, st);
    default: return launch_t<2, 16, false>(a, st);
  }
}

cudaError_t gemv_run(const QMat &m, int B, float *Y, int ys, int epi, GemvScratch &s, cudaStream_t st) {
  return gemv_launch(m, B, Y, ys, epi, s, st, nullptr, 0);
}

bool gemv_uses_local_x(const QMat &m, const float *X, int xs, const GemvScratch &s) {
  if (m.kern == GK_QMV) return true;  // raw X, one launch
  return gemv_local_x(m, s) && (reinterpret_cast<uintptr_t>(X) & 15) == 0 && xs % 4 == 0;
}

cudaError_t gemv_run_x(const QMat &m, const float *X, int xs, int B, float *Y, int ys, int epi, GemvScratch &s,
                       cudaStream_t st, bool want_stats) {
  if (!X || xs < m.K) return cudaErrorInvalidValue;
  if (m.kern == GK_QMV) return qmv_run(m, X, xs, nullptr, B, Y, ys, epi, s, st);
  // the local-X prologue reads X as float4: rows must start on 16 bytes
  if (gemv_local_x(m, s) && (reinterpret_cast<uintptr_t>(X) & 15) == 0 && xs % 4 == 0)
    return gemv_launch(m, B, Y, ys, epi, s, st, X, xs, nullptr,
                       want_stats && epi == EPI_ADD && s.stat && s.stat_next && gemv_all_split(m, s));
  CW_TRY(gemv_prep_x(X, xs, B, m.K, s, st));
  return gemv_launch(m, B, Y, ys, epi, s, st, nullptr, 0);
}

bool gemv_norm_fused(const QMat &m, const float *X, int xs, int B, const GemvScratch &s) {
  if (m.kern == GK_QMV) return true;  // the norm is folded into the kernel
  return gemv_local_x(m, s) && (reinterpret_cast<uintptr_t>(X) & 15) == 0 && xs % 4 == 0 && s.stat_ok && s.stat_y == X && s.stat_ys == xs && s.stat_len == m.K &&
         s.stat_cols >= B && s.stat_g >= 1 && s.stat_g <= 160;
}

cudaError_t gemv_run_xn(const QMat &m, const float *X, int xs, const float *w, int B, float *Y, int ys, int epi,
                        GemvScratch &s, cudaStream_t st) {
  if (!X || !w || xs < m.K) return cudaErrorInvalidValue;
  if (m.kern == GK_QMV) return qmv_run(m, X, xs, w, B, Y, ys, epi, s, st);
  if (gemv_norm_fused(m, X, xs, B, s)) return gemv_launch(m, B, Y, ys, epi, s, st, X, xs, w, false);
  CW_TRY(launch_norm_prep(X, w, m.K, B, s, nullptr, st));
  return gemv_launch(m, B, Y, ys, epi, s, st, nullptr, 0);
}

// One-time kernel attributes (called at engine set-up).
cudaError_t qgemv_configure() {
  cudaError_t e;
  if ((e = qmv_configure()) != cudaSuccess) return e;
  if ((e = mma::configure()) != cudaSuccess) return e;
  if ((e = carveout_max(repack_kernel<2>)) != cudaSuccess) return e;
  if ((e = carveout_max(repack_kernel<8>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 1, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 8, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 16, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<8, 1, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<8, 8, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<8, 16, false>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 1, true>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 8, true>)) != cudaSuccess) return e;
  if ((e = carveout_max(qgemv_kernel<2, 16, true>)) != cudaSuccess) return e;
  return cudaSuccess;
}

}  // namespace cw
