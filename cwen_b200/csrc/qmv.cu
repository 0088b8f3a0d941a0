// Batched Q4_0 / Q8_0 GEMV for B <= 16 verify rows, the alternative to the
// mma kernel ("qmv", CWEN_GEMV=qmv).  Replaces the reference's gemvb()/gemv() (run.c:1577-1680,
// 1419-1527) and the row dots under them (dot_q4_0 run.c:1009-1025,
// dot_nib16 run.c:432, dot_q8_0 run.c:1248-1274); with a norm weight it also
// takes the rmsnorm that precedes the projection (run.c:346-368).
//
// Arithmetic.  The reference computes, per row and 32-weight block,
//   y += d * sum_j (q_j - 8) * x_j            (fp32).
// Here the block dot runs on the tensor cores (mma.sync m16n8k16, f16 in,
// fp32 accumulate): (q - 8) is exact in f16, and X is split into f16 hi + lo
// parts (x = hi + lo to ~2^-22 relative) after a power-of-two scale that
// brings the largest |x| of the column in the current K phase (512 values)
// into [2^14, 2^15).  An n-tile of the B operand holds the hi parts of 4
// columns (n 0..3) and their lo parts (n 4..7), so per 16 rows x 32 weights
// two chained MMAs (k 0..15, k 16..31) give fp32 block partials of the hi and
// the lo halves, and one FFMA per element applies the block's f16 scale:
// acc = fma(d, c, acc).  When the phase changes, the accumulators are moved
// to the new phase's scale by an exact power-of-two multiply -- the same
// bits as accumulating fma(d * 2^-e, c, acc) in the unscaled domain -- and y
// = (sum of hi partials + sum of lo partials) * 2^-e at the end.  With a norm
// weight w, X = w x and the row scale 1/sqrt(mean(x^2) + 1e-6) multiplies
// the outputs.
//
// Batch invariance.  Column b of the output depends only on column b of X:
// its exponents come from its own values, every MMA column is its own dot
// product, and the K split between warps (block-cyclic inside each phase,
// summed in warp order) is a function of the matrix shape only.  So a B-row
// verify block gives the bits of B single-row calls; the spec decode is
// lossless by construction.
//
// Work split.  Rows come in 8-row half-tiles.  A persistent grid of G = #SM
// CTAs takes equal contiguous ranges of half-tiles (of half-tile pairs for
// an interleaved gate/up matrix), each over the whole K: no row is split
// between CTAs, so there is no cross-CTA reduction of outputs.  Inside a
// CTA the 16 warps form a WM x WK grid: warp (i, j) owns a contiguous group
// of "v-tiles" (two half-tiles stacked into one 16-row MMA tile) and the
// blocks b of each phase with b % WK == j.  When the accumulators of a CTA's
// rows would not fit in registers (large M or B), the rows run in passes,
// each over the whole K.
//
// X.  Every CTA needs the whole X, converted the same way, so the conversion
// is done once per call: CTA f converts phase f (its columns' exponents, the
// f16 hi/lo operands in MMA-fragment order, the phase's sums of squares)
// into a global buffer and publishes it with an epoch flag; the operands of
// a phase then travel from L2 with each weight stage.
//
// Memory.  The weights are repacked at upload into exactly the order a CTA
// streams them: per CTA [32-block][half-tile], a 144-byte chunk (Q4_0: 8
// rows x 16 nibble bytes, 8 f16 scales) or 272 (Q8_0).  A stage = a few
// consecutive blocks of the pass's rows plus their X operands, bulk-copied
// (TMA) into a ring of 32 KB slots.  The weights of the first ring-full are
// requested before the previous kernel finishes (PDL: weights are constant);
// afterwards the warp that releases a stage last refills its slot -- no
// producer warp, so all 16 warps compute and each keeps 128 registers.  Every
// wait is bounded; a timeout raises the error flag (CWEN_ETIMEOUT on the host).
#include "common.cuh"
#include "qgemv.cuh"
#include "qgemv_dev.cuh"
#include "qmv.cuh"
#include "sm100.cuh"

namespace cw {
namespace qmv {

constexpr int CONS = 16;  // warps; every one computes
constexpr int THREADS = CONS * 32;
constexpr int PH = 16;           // 32-blocks per K phase
constexpr int SLOT = 45056;      // bytes of one ring stage: a whole phase of a ~15-half-tile CTA
constexpr int NSLOT = 4;
constexpr int RED_BYTES = 32768; // end-of-pass partial sums: >= one v-tile slot of every warp at 4 n-tiles
constexpr int MAXSTAGE = 512;    // stages of a CTA (the launcher checks)
constexpr int MAXPASS = 32;
constexpr int MISC_BYTES = 3072;
constexpr int SMEM = NSLOT * SLOT + RED_BYTES + MISC_BYTES;
static_assert(SMEM <= 227 * 1024, "shared memory plan");
static_assert(RED_BYTES >= CONS * 4 * 512, "reduction area holds one v-tile slot at NT = 4");
constexpr int HDR = 128;  // per phase: exponents e[16] (int), sums of squares ss[16] (float)

CW_HOST_DEV constexpr int chunk_bytes(int type) { return type == 8 ? 272 : 144; }
// v-tiles a warp accumulates per pass (registers: 4 * NT floats each)
CW_HOST_DEV constexpr int rw_max(int nt) { return nt == 1 ? 8 : (nt == 2 ? 6 : (nt == 3 ? 4 : 3)); }
// bytes of one phase of X operands in the global buffer
CW_HOST_DEV constexpr int phase_bytes(int nt) { return HDR + PH * nt * 512; }

// The half-tiles [h0, h0 + nh) of CTA c: equal contiguous shares of the
// units (half-tiles, or gate/up pairs of half-tiles).
struct Part {
  int h0, nh;
};
CW_HOST_DEV Part cta_part(int n_ht, bool pair, int G, int c) {
  const int unit = pair ? 2 : 1, nu = n_ht / unit;
  const int u0 = c * nu / G, u1 = (c + 1) * nu / G;  // nu * G < 2^31 (the launcher checks)
  return Part{(int)u0 * unit, (int)(u1 - u0) * unit};
}
// Row groups of the warp grid (WM; WK = 16 / WM): a function of the shape
// only, so the K split of every row is the same for every B.
CW_HOST_DEV int warp_rows(int n_ht, bool pair, int G) {
  const int unit = pair ? 2 : 1, nu = n_ht / unit;
  const int nh_max = (nu + G - 1) / G * unit;
  const int nv_max = (nh_max + 1) / 2;
  int wm = 1;
  while (wm < CONS && (nv_max + wm - 1) / wm > rw_max(1)) wm *= 2;
  return wm;
}
// v-tiles per warp and pass for NT n-tiles (one block of a pass fits a slot).
CW_HOST_DEV int rw_for(int nt, int type, int wm) {
  int rw = rw_max(nt);
  const int cap = (SLOT - HDR - nt * 512) / (2 * wm * chunk_bytes(type));
  if (cap < rw) rw = cap;
  return rw < 1 ? 1 : rw;
}
// Blocks per stage for a pass of hp half-tiles: the largest power of two
// <= PH whose weights and X operands fit a slot.
CW_HOST_DEV int stage_blocks(int hp, int ch, int nt) {
  int sb = PH;
  while (sb > 1 && sb * (hp * ch + nt * 512) + HDR > SLOT) sb >>= 1;
  return sb;
}

// max|x| * 2^e in [2^14, 2^15) (clamped to |e| <= 62, so that the exponent
// difference of two phases is one exact power-of-two factor)
CW_DEV int qexp(float mx) {
  int e = 0;
  if (mx > 0.f && mx <= 3.0e38f) {
    int p;
    frexpf(mx, &p);
    e = 15 - p;
    e = e < -62 ? -62 : (e > 62 ? 62 : e);
  }
  return e;
}
CW_DEV float pow2i(int d) { return __int_as_float((127 + d) << 23); }  // |d| <= 126
// v * 2^d, exact for |d| <= 128 (two power-of-two steps)
CW_DEV float scale2(float v, int d) {
  const int d1 = d / 2;
  return v * pow2i(d1) * pow2i(d - d1);
}

// One pass of a CTA: v-tiles [v0, v1), half-tiles [hp0, hp1), stages of sb blocks.
struct Pass {
  int v0, v1, hp0, hp1, hp, sb, nst;
};
CW_HOST_DEV Pass pass_of(int p, int npass, int nv, int nh, int nblk, int ch, int nt) {
  Pass q;
  q.v0 = p * nv / npass;
  q.v1 = (p + 1) * nv / npass;
  q.hp0 = 2 * q.v0;
  q.hp1 = 2 * q.v1 < nh ? 2 * q.v1 : nh;
  q.hp = q.hp1 - q.hp0;
  q.sb = stage_blocks(q.hp, ch, nt);
  const int nph = (nblk + PH - 1) / PH, nb_last = nblk - PH * (nph - 1);
  q.nst = (nph - 1) * (PH / q.sb) + (nb_last + q.sb - 1) / q.sb;
  return q;
}
// Stage n of a CTA: its pass, phase f and blocks [s0, s1) of the phase.
struct Stage {
  Pass q;
  int f, s0, s1;
};
CW_DEV Stage stage_of(int n, int npass, int nv, int nh, int nblk, int ch, int nt) {
  Stage s;
  int p = 0, k = n;
  s.q = pass_of(0, npass, nv, nh, nblk, ch, nt);
  while (k >= s.q.nst && p + 1 < npass) {
    k -= s.q.nst;
    s.q = pass_of(++p, npass, nv, nh, nblk, ch, nt);
  }
  const int nph = (nblk + PH - 1) / PH, spp = PH / s.q.sb;
  s.f = min(k / spp, nph - 1);
  s.s0 = (k - s.f * spp) * s.q.sb;
  s.s1 = min(s.s0 + s.q.sb, min(PH, nblk - PH * s.f));
  return s;
}

CW_DEV int ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
CW_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Shared state of a CTA besides the ring and the reduction area.
struct Misc {
  uint64_t full[NSLOT];
  int rel[NSLOT];         // warps done with the slot's stage
  int last_issued[NSLOT]; // the stage last issued into each slot
  int abort;
  int elast[16];          // exponents of the last phase seen
  float ssq[16];          // sums of squares of the columns (norm)
  float cmax[32], css[32];  // conversion: per warp and round
  int4 ptab[MAXPASS];       // per pass: first half-tile, half-tiles, blocks per stage
  uint32_t stab[MAXSTAGE];  // per stage: phase | first block << 8 | end block << 13 | pass << 18
};
static_assert(sizeof(Misc) <= MISC_BYTES, "misc area");

// Weights of stage n into its slot; arms the slot's mbarrier for the
// weights and the X operands together.  Called by one whole warp.
CW_DEV Stage stage_at(const Misc &ms, int n) {
  const uint32_t e = ms.stab[n];
  Stage s;
  s.f = (int)(e & 255u);
  s.s0 = (int)((e >> 8) & 31u);
  s.s1 = (int)((e >> 13) & 31u);
  const int4 pp = ms.ptab[e >> 18];
  s.q.hp0 = pp.x;
  s.q.hp = pp.y;
  s.q.sb = pp.z;
  return s;
}
template <int CH, int NT>
CW_DEV void issue_w(const Stage &s, int n, int nh, const uint8_t *wbase, uint8_t *ring, Misc &ms, int lane) {
  const int slot = n % NSLOT;
  uint8_t *dst = ring + slot * SLOT;
  const uint32_t wbytes = (uint32_t)((s.s1 - s.s0) * s.q.hp * CH);
  const uint32_t xbytes = (uint32_t)((s.s0 == 0 ? HDR : 0) + (s.s1 - s.s0) * NT * 512);
  if (lane == 0) {
    ms.last_issued[slot] = n;
    mbar_expect_tx(&ms.full[slot], wbytes + xbytes);
  }
  __syncwarp();
  if (s.q.hp == nh) {
    if (lane == 0) bulk_g2s(dst, wbase + (size_t)(PH * s.f + s.s0) * nh * CH, wbytes, &ms.full[slot]);
  } else if (lane < s.s1 - s.s0) {
    bulk_g2s(dst + lane * s.q.hp * CH, wbase + ((size_t)(PH * s.f + s.s0 + lane) * nh + s.q.hp0) * CH,
             (uint32_t)(s.q.hp * CH), &ms.full[slot]);
  }
  __syncwarp();
}
// X operands of stage n (every phase of the call is published by then):
// slot layout [weights: sb blocks][header (first stage of a phase) |
// operands of the blocks].  One lane.
template <int CH, int NT>
CW_DEV void issue_x(const Stage &s, int n, const QmvArgs &a, uint8_t *ring, Misc &ms) {
  const int slot = n % NSLOT;
  uint8_t *dst = ring + slot * SLOT + s.q.sb * s.q.hp * CH;
  const uint8_t *src = a.xg + (size_t)s.f * phase_bytes(NT);
  if (s.s0 == 0)
    bulk_g2s(dst, src, (uint32_t)(HDR + (s.s1 - s.s0) * NT * 512), &ms.full[slot]);
  else
    bulk_g2s(dst + HDR, src + HDR + s.s0 * NT * 512, (uint32_t)((s.s1 - s.s0) * NT * 512), &ms.full[slot]);
}
// Wait (bounded) until every phase of this call is published.  One warp,
// the lanes checking phases in parallel (a lane's acquire orders only its
// own later accesses: the caller synchronizes the warp and fences before
// another lane reads what a flag published).
CW_DEV bool wait_phases(const QmvArgs &a, int nph, int lane) {
  const long long t0 = cycles_now();
  bool ok = true;
  for (int f = lane; f < nph && ok; f += 32)
    for (uint32_t it = 0; ld_acquire(a.flags + f) != a.epoch; it++)
      if ((it & 63u) == 63u && spin_expired(t0)) {
        ok = false;
        break;
      }
  return __all_sync(0xffffffffu, ok);
}

CW_DEV void qput(const QmvArgs &a, size_t off, float v) {
  if (a.np == 0) {
    a.y[off] = v;
  } else {
    for (int p = 0; p < a.np; p++) a.yp[p][off] = v;
  }
}

// Phase f of X into the global buffer: exponents, f16 hi/lo operands in
// MMA-fragment order (lane (g, t) of n-tile u: (x[4t], x[4t+2]) (x[4t+1],
// x[4t+3]) (x[16+4t], x[18+4t]) (x[17+4t], x[19+4t]) of column 4u + g % 4,
// hi parts for g < 4, lo parts for g >= 4), the columns' sums of squares;
// then the phase's flag.  All 512 threads of the CTA.
template <int NT>
CW_DEV void convert_phase(const QmvArgs &a, int f, Misc &ms) {
  constexpr int NITEM = 64 * 4 * NT;  // (column, block of the phase, lane quad)
  constexpr int NR = (NITEM + THREADS - 1) / THREADS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float xv[NR][8];
  float m[NR], s2[NR];
  uint8_t *dst = a.xg + (size_t)f * phase_bytes(NT);
#pragma unroll
  for (int q = 0; q < NR; q++) {
    const int it = tid + THREADS * q;
    const int col = it >> 6, lb = (it & 63) >> 2, tt = it & 3;
    const int kb = PH * f + lb;
    m[q] = 0.f;
    s2[q] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) xv[q][i] = 0.f;
    if (it < NITEM && col < a.B && kb < a.nblk) {
      const float *p = a.x + (size_t)col * a.xs + (size_t)kb * 32 + 4 * tt;
      if (a.xal) {
        const float4 u = __ldg(reinterpret_cast<const float4 *>(p));
        const float4 w = __ldg(reinterpret_cast<const float4 *>(p + 16));
        xv[q][0] = u.x; xv[q][1] = u.y; xv[q][2] = u.z; xv[q][3] = u.w;
        xv[q][4] = w.x; xv[q][5] = w.y; xv[q][6] = w.z; xv[q][7] = w.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; i++) {
          xv[q][i] = __ldg(p + i);
          xv[q][4 + i] = __ldg(p + 16 + i);
        }
      }
      if (a.xw) {  // X = w x; the row scale is applied to the outputs
        const float *wp = a.xw + (size_t)kb * 32 + 4 * tt;
#pragma unroll
        for (int i = 0; i < 8; i++) s2[q] = fmaf(xv[q][i], xv[q][i], s2[q]);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          xv[q][i] *= __ldg(wp + i);
          xv[q][4 + i] *= __ldg(wp + 16 + i);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; i++) m[q] = fmaxf(m[q], fabsf(xv[q][i]));
    }
  }
#pragma unroll
  for (int q = 0; q < NR; q++) {
    const float wm = warp_max(m[q]), ws = warp_sum(s2[q]);  // the warp's lanes share one column
    if (lane == 0) {
      ms.cmax[warp * 2 + q] = wm;
      ms.css[warp * 2 + q] = ws;
    }
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < NR; q++) {
    const int it = tid + THREADS * q;
    const int col = it >> 6, lb = (it & 63) >> 2, tt = it & 3;
    const int kb = PH * f + lb;
    if (it >= NITEM) continue;
    const int w0 = warp & ~1;
    const int e = qexp(fmaxf(ms.cmax[w0 * 2 + q], ms.cmax[(w0 + 1) * 2 + q]));
    if (lane == 0 && warp == w0) {
      reinterpret_cast<int *>(dst)[col] = e;
      reinterpret_cast<float *>(dst)[16 + col] = ms.css[w0 * 2 + q] + ms.css[(w0 + 1) * 2 + q];
    }
    if (kb < a.nblk) {
      const float sc = pow2i(e);
      uint32_t hw[4], lw[4];
      const int ord[8] = {0, 2, 1, 3, 4, 6, 5, 7};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float v0 = xv[q][ord[2 * i]] * sc, v1 = xv[q][ord[2 * i + 1]] * sc;
        const half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
        const half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
        hw[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        lw[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
      }
      uint8_t *o = dst + HDR + (lb * NT + (col >> 2)) * 512;
      *reinterpret_cast<uint4 *>(o + ((col & 3) * 4 + tt) * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4 *>(o + ((4 + (col & 3)) * 4 + tt) * 16) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
  fence_proxy_async_global();  // the operands are read by bulk copies (async proxy)
  __threadfence();
  __syncthreads();
  if (tid == 0) asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(a.flags + f), "r"(a.epoch) : "memory");
}

template <int TYPE, int NT>
__global__ void __launch_bounds__(THREADS, 1) qmv_kernel(const QmvArgs a) {
  constexpr int RW = rw_max(NT);
  constexpr int CH = chunk_bytes(TYPE);
  constexpr int SPR = RED_BYTES / (CONS * NT * 512) >= 1 ? RED_BYTES / (CONS * NT * 512) : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  float *red = reinterpret_cast<float *>(smem + NSLOT * SLOT);
  Misc &ms = *reinterpret_cast<Misc *>(smem + NSLOT * SLOT + RED_BYTES);
  volatile int *abort_p = &ms.abort;

  const int c = blockIdx.x;
  const Part pt = cta_part(a.n_ht, a.pair, a.G, c);
  const int nph = (a.nblk + PH - 1) / PH;
  const bool conv = c < nph;  // converts phases c, c + G, ...
  if (pt.nh == 0 && !conv) return;  // whole CTA, before any barrier
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int WM = a.wm, WK = CONS / WM;
  const int rw = rw_for(NT, TYPE, WM);
  const int nv = (pt.nh + 1) / 2;
  const int npass = nv ? (nv + WM * rw - 1) / (WM * rw) : 0;
  const uint8_t *wbase = a.w + (size_t)pt.h0 * a.nblk * CH;
  // The pass table, then the stage table (which pass, phase and blocks each
  // stage holds); the launcher checks that the plan fits the tables.
  if (npass > MAXPASS) return;  // unreachable: the launcher checks the plan (uniform over the CTA)
  for (int p = threadIdx.x; p < npass; p += THREADS) {
    const Pass q = pass_of(p, npass, nv, pt.nh, a.nblk, CH, NT);
    ms.ptab[p] = make_int4(q.hp0, q.hp, q.sb, q.nst);
  }
  __syncthreads();
  int nstage = 0;  // stages of the CTA
  for (int p = 0; p < npass; p++) nstage += ms.ptab[p].w;
  if (nstage > MAXSTAGE) return;  // unreachable, as above
  for (int i = threadIdx.x; i < nstage; i += THREADS) {
    int p = 0, k = i;
    while (k >= ms.ptab[p].w) k -= ms.ptab[p++].w;
    const int sb = ms.ptab[p].z, spp = PH / sb;
    const int f = min(k / spp, nph - 1);
    const int s0 = (k - f * spp) * sb, s1 = min(s0 + sb, min(PH, a.nblk - PH * f));
    ms.stab[i] = (uint32_t)f | ((uint32_t)s0 << 8) | ((uint32_t)s1 << 13) | ((uint32_t)p << 18);
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSLOT; i++) {
      mbar_init(&ms.full[i], 1);
      ms.rel[i] = 0;
      ms.last_issued[i] = -1;
    }
    ms.abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  const int npre = nstage < NSLOT ? nstage : NSLOT;
  // The weights of the first ring-full, before waiting for the previous kernel.
  if (warp == 0)
    for (int i = 0; i < npre; i++)
      issue_w<CH, NT>(stage_at(ms, i), i, pt.nh, wbase, smem, ms, lane);
  pdl_wait();  // X is the previous kernel's output
  for (int f = c; f < nph; f += a.G) convert_phase<NT>(a, f, ms);
  // Every phase published (acquired once here, so that no refill waits on
  // a flag), then the X operands of the first ring-full.
  if (warp == 0 && npass > 0) {
    // lane 0 issues: the copies must follow the acquires in one thread's order
    const bool ready = wait_phases(a, nph, lane);
    __syncwarp();
    if (ready) {
      if (lane == 0) {
        __threadfence();
        fence_proxy_async_global();
        for (int i = 0; i < npre; i++) issue_x<CH, NT>(stage_at(ms, i), i, a, smem, ms);
      }
    } else if (lane == 0) {
      atomicExch(a.err, 3);
      ms.abort = 1;
    }
  }
  __syncthreads();
  // the X operands published by other CTAs (generic stores, then a release)
  // are read by this CTA's bulk copies (async proxy) from here on
  if (lane == 0) fence_proxy_async_global();

  const int gi = warp / WK, kj = warp % WK;
  const int g = lane >> 2, t = lane & 3;
  const int tid = threadIdx.x;
  bool ok = true;
  int n = 0;  // stage counter
  float ssum = 0.f;  // warp 0, lane < 16: sum of squares of column `lane` (norm)
  int ecur[NT][2];

  for (int p = 0; p < npass; p++) {
    const Pass pq = pass_of(p, npass, nv, pt.nh, a.nblk, CH, NT);
    const int v0 = pq.v0, hp0 = pq.hp0, hp1 = pq.hp1, hp = pq.hp, sb = pq.sb;
    const int vp = pq.v1 - pq.v0;
    const int gv0 = (int)((long long)gi * vp / WM), gv1 = (int)((long long)(gi + 1) * vp / WM);
    const int nvg = gv1 - gv0;  // v-tiles of this warp's group (<= rw <= RW)
    float acc[RW][NT][4];
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
      for (int u = 0; u < NT; u++)
#pragma unroll
        for (int k = 0; k < 4; k++) acc[r][u][k] = 0.f;

    for (int f = 0; f < nph; f++) {
      const int nb = min(PH, a.nblk - PH * f);
      for (int s0 = 0; s0 < nb; s0 += sb, n++) {
        const int s1 = min(s0 + sb, nb);
        const int slot = n % NSLOT;
        if (ok && !mbar_wait(&ms.full[slot], (uint32_t)((n / NSLOT) & 1), abort_p)) {
          ok = false;
          atomicExch(a.err, 2);
          *abort_p = 1;
        }
        const uint8_t *stg = smem + slot * SLOT;
        const uint8_t *xs = stg + sb * hp * CH;  // [header][operands of the stage's blocks]
        if (ok && s0 == 0) {
          // a new phase: its exponents; move the accumulators to its scale
          // (an exact power-of-two factor, skipped when no column changed)
          const int *eh = reinterpret_cast<const int *>(xs);
          int en[NT][2];
          bool chg = false;
#pragma unroll
          for (int u = 0; u < NT; u++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
              en[u][h] = eh[4 * u + 2 * (t & 1) + h];
              chg |= f > 0 && en[u][h] != ecur[u][h];
            }
          if (__any_sync(0xffffffffu, chg)) {
#pragma unroll
            for (int u = 0; u < NT; u++)
#pragma unroll
              for (int h = 0; h < 2; h++) {
                const float fac = pow2i(en[u][h] - ecur[u][h]);  // |difference| <= 124
#pragma unroll
                for (int r = 0; r < RW; r++) {
                  acc[r][u][h] *= fac;
                  acc[r][u][2 + h] *= fac;
                }
              }
          }
#pragma unroll
          for (int u = 0; u < NT; u++)
#pragma unroll
            for (int h = 0; h < 2; h++) ecur[u][h] = en[u][h];
          if (warp == 0 && lane < 16) {
            ms.elast[lane] = eh[lane];
            if (p == 0) ssum += reinterpret_cast<const float *>(xs)[16 + lane];
          }
        }
        if (ok && nvg > 0) {
          for (int lb = s0 + ((kj - s0) & (WK - 1)); lb < s1; lb += WK) {  // WK is a power of two
            uint4 xf[NT];
#pragma unroll
            for (int u = 0; u < NT; u++)
              xf[u] = *reinterpret_cast<const uint4 *>(xs + HDR + ((lb - s0) * NT + u) * 512 + lane * 16);
            const uint8_t *cb = stg + (size_t)(lb - s0) * hp * CH;
            // The warp's v-tiles in pairs, branch-free inside a pair so that two
            // load -> unpack -> MMA -> FFMA chains interleave; the second of a
            // pair past the warp's count reads a valid chunk with scale 0 (its
            // accumulators, never stored, stay unchanged); a missing bottom
            // half-tile likewise.
            constexpr int NW = TYPE == 8 ? 2 : 1;  // quant words per row and lane
#pragma unroll
            for (int r0 = 0; r0 < RW; r0 += 2) {
              if (r0 < nvg) {
                uint32_t wt[2][NW], wb[2][NW];
                float dt[2], db[2];
#pragma unroll
                for (int q = 0; q < 2; q++) {
                  const int r = r0 + q;
                  const int rr = r < nvg ? r : nvg - 1;
                  const int ht = 2 * (v0 + gv0 + rr);  // CTA-relative top half-tile
                  const bool hb = ht + 1 < hp1;
                  const uint8_t *ct = cb + (ht - hp0) * CH;
                  const uint8_t *cbt = hb ? ct + CH : ct;
#pragma unroll
                  for (int i = 0; i < NW; i++) {
                    wt[q][i] = *reinterpret_cast<const uint32_t *>(ct + i * 128 + lane * 4);
                    wb[q][i] = *reinterpret_cast<const uint32_t *>(cbt + i * 128 + lane * 4);
                  }
                  const float ht_d = __half2float(*reinterpret_cast<const half *>(ct + NW * 128 + 2 * g));
                  const float hb_d = __half2float(*reinterpret_cast<const half *>(cbt + NW * 128 + 2 * g));
                  dt[q] = r < nvg ? ht_d : 0.f;
                  db[q] = (r < nvg && hb) ? hb_d : 0.f;
                }
#pragma unroll
                for (int q = 0; q < 2; q++) {
                  const int r = r0 + q;
                  if (r >= RW) break;
                  uint32_t a0s0, a1s0, a2s0, a3s0, a0s1, a1s1, a2s1, a3s1;
                  if (TYPE == 8) {
                    q8_to_f16(wt[q][0], a0s0, a2s0);
                    q8_to_f16(wt[q][NW - 1], a0s1, a2s1);
                    q8_to_f16(wb[q][0], a1s0, a3s0);
                    q8_to_f16(wb[q][NW - 1], a1s1, a3s1);
                  } else {
                    q4_to_f16(wt[q][0], a0s0, a2s0, a0s1, a2s1);
                    q4_to_f16(wb[q][0], a1s0, a3s0, a1s1, a3s1);
                  }
#pragma unroll
                  for (int u = 0; u < NT; u++) {
                    float cc[4];
                    const float z4[4] = {0.f, 0.f, 0.f, 0.f};
                    mma_16816(cc, a0s0, a1s0, a2s0, a3s0, xf[u].x, xf[u].y, z4);
                    mma_16816(cc, a0s1, a1s1, a2s1, a3s1, xf[u].z, xf[u].w, cc);
                    acc[r][u][0] = fmaf(dt[q], cc[0], acc[r][u][0]);
                    acc[r][u][1] = fmaf(dt[q], cc[1], acc[r][u][1]);
                    acc[r][u][2] = fmaf(db[q], cc[2], acc[r][u][2]);
                    acc[r][u][3] = fmaf(db[q], cc[3], acc[r][u][3]);
                  }
                }
              }
            }
          }
        }
        // Release: the warp that finishes the stage last refills the slot
        // with stage n + NSLOT (its reads are ordered before the copies).
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          uint32_t old;
          asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;" : "=r"(old) : "r"(smem_u32(&ms.rel[slot])) : "memory");
          last = old == CONS - 1;
          if (last) ms.rel[slot] = 0;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last && n + NSLOT < nstage && !*abort_p) {
          const Stage sn = stage_at(ms, n + NSLOT);
          issue_w<CH, NT>(sn, n + NSLOT, pt.nh, wbase, smem, ms, lane);
          if (lane == 0) issue_x<CH, NT>(sn, n + NSLOT, a, smem, ms);
        }
      }
    }

    // ---- end of pass: reduction over the K warps, epilogue ----
    if (p == 0 && a.xw && warp == 0 && lane < 16) ms.ssq[lane] = ssum;
    for (int r0 = 0; r0 < RW; r0 += SPR) {
#pragma unroll
      for (int r = 0; r < RW; r++) {
        if (r >= r0 && r < r0 + SPR) {
#pragma unroll
          for (int u = 0; u < NT; u++)
            *reinterpret_cast<float4 *>(red + ((((r - r0) * CONS + warp) * NT + u) * 32 + lane) * 4) =
                make_float4(acc[r][u][0], acc[r][u][1], acc[r][u][2], acc[r][u][3]);
        }
      }
      __syncthreads();
      const int rows = a.epi == EPI_SWIGLU ? 8 : 16;
      const int nout = SPR * WM * rows * a.B;
      for (int o = tid; o < nout; o += THREADS) {
        const int col = o % a.B;
        int rest = o / a.B;
        const int rr = rest % rows;
        rest /= rows;
        const int ig = rest % WM, rin = rest / WM;
        const int r = r0 + rin;
        const int g0 = (int)((long long)ig * vp / WM), g1 = (int)((long long)(ig + 1) * vp / WM);
        if (r >= g1 - g0) continue;
        const int vt = v0 + g0 + r;  // CTA-relative v-tile
        const int u = col >> 2, th = (col & 3) >> 1;
        const float nsc = a.xw ? 1.f / sqrtf(ms.ssq[col] / (float)a.K + 1e-6f) : 1.f;
        const int e = ms.elast[col];
        // total of row `row` (0..15) of the v-tile, column col, over the K warps
        auto total = [&](int row) {
          const int gg = row & 7, k = (row >= 8 ? 2 : 0) + (col & 1);
          float sh = 0.f, sl = 0.f;
          for (int j = 0; j < WK; j++) {
            const float *b = red + (((rin * CONS + ig * WK + j) * NT + u) * 32) * 4;
            sh += b[(gg * 4 + th) * 4 + k];
            sl += b[(gg * 4 + th + 2) * 4 + k];
          }
          return scale2(sh + sl, -e) * nsc;
        };
        if (a.epi == EPI_SWIGLU) {
          const int orow = 4 * (pt.h0 + 2 * vt) + rr;  // gate/up unit (h0 + 2 vt) / 2, row rr
          if (2 * orow < a.M) {
            const float gt = total(rr), up = total(rr + 8);
            qput(a, (size_t)col * a.ys + a.row0 + orow, silu_f(gt) * up);
          }
        } else {
          const int h = 2 * vt + (rr >> 3);
          if (h < hp1) {
            const int row = 8 * (pt.h0 + h) + (rr & 7);
            if (row < a.M) {
              const size_t off = (size_t)col * a.ys + a.row0 + row;
              const float v = total(rr);
              qput(a, off, a.epi == EPI_ADD ? a.y[off] + v : v);
            }
          }
        }
      }
      __syncthreads();
    }
  }
  if (a.np) __threadfence_system();  // peer stores before the cross-GPU barrier kernel
  if (threadIdx.x == 0 && *abort_p) {
    // after a timeout: no bulk copy may still be in flight when the CTA exits
    const long long t0 = cycles_now();
    for (int i = 0; i < NSLOT; i++) {
      const int m = ms.last_issued[i];
      if (m >= 0)
        while (!mbar_try_wait(&ms.full[i], (uint32_t)((m / NSLOT) & 1)) && !spin_expired(t0)) {
        }
    }
  }
}

// ---- weight repack: GGUF rows -> [CTA][32-block][half-tile] chunks ----
// Source row r of this upload (absolute row a0 + r of the tensor) lands in
// half-tile ht_base + ((a0 + r) / 8) * ht_stride, row (a0 + r) % 8.
template <int TYPE>
__global__ void repack_kernel(uint8_t *dst, int n_ht, bool pair, int G, int nblk, const uint8_t *src, int nrows,
                              long long a0, int ht_base, int ht_stride) {
  constexpr int CH = chunk_bytes(TYPE);
  const int unit = pair ? 2 : 1, nu = n_ht / unit;
  const long long total = (long long)nrows * nblk;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(idx / nblk), kb = (int)(idx % nblk);
    const long long ar = a0 + r;
    const int h = ht_base + (int)(ar / 8) * ht_stride, i = (int)(ar % 8);
    const int x = h / unit;
    int c = (int)(((long long)x * G) / nu);
    while (c + 1 < G && (long long)(c + 1) * nu / G <= x) c++;
    while (c > 0 && (long long)c * nu / G > x) c--;
    const Part p = cta_part(n_ht, pair, G, c);
    uint8_t *ch = dst + ((size_t)p.h0 * nblk + (size_t)kb * p.nh + (h - p.h0)) * CH;
    const uint8_t *blk = src + ((size_t)r * nblk + kb) * (TYPE == 8 ? 34 : 18);
    if (TYPE == 8) {
      for (int j = 0; j < 16; j++) {
        ch[i * 16 + j] = blk[2 + j];
        ch[128 + i * 16 + j] = blk[18 + j];
      }
      ch[256 + 2 * i] = blk[0];
      ch[257 + 2 * i] = blk[1];
    } else {
      for (int j = 0; j < 16; j++) ch[i * 16 + j] = blk[2 + j];
      ch[128 + 2 * i] = blk[0];
      ch[129 + 2 * i] = blk[1];
    }
  }
}

}  // namespace qmv

size_t qmv_bytes(int type, int K, int n_ht) { return (size_t)n_ht * (K / 32) * qmv::chunk_bytes(type); }

cudaError_t qmv_repack(const QMat &m, const uint8_t *src, int nrows, long long a0, int ht_base, int ht_stride,
                       cudaStream_t st) {
  if (m.K % 64 || ht_base < 0 || ht_stride < 1 || nrows < 1) return cudaErrorInvalidValue;
  const long long last = ht_base + ((a0 + nrows - 1) / 8) * ht_stride;
  if (last >= m.n_ht) return cudaErrorInvalidValue;
  const long long total = (long long)nrows * (m.K / 32);
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  const int grid = (int)(blocks < 65535 ? blocks : 65535);
  if (m.type == 8)
    qmv::repack_kernel<8><<<grid, threads, 0, st>>>(m.w, m.n_ht, m.pair, m.G, m.K / 32, src, nrows, a0, ht_base,
                                                     ht_stride);
  else
    qmv::repack_kernel<2><<<grid, threads, 0, st>>>(m.w, m.n_ht, m.pair, m.G, m.K / 32, src, nrows, a0, ht_base,
                                                     ht_stride);
  return cudaGetLastError();
}

template <int TYPE, int NT>
static cudaError_t qmv_launch_t(const QmvArgs &a, cudaStream_t st) {
  return launch_pdl(qmv::qmv_kernel<TYPE, NT>, a.G, qmv::THREADS, (size_t)qmv::SMEM, st, a);
}

size_t qmv_xbuf_bytes(int kmax) { return (size_t)((kmax + qmv::PH * 32 - 1) / (qmv::PH * 32)) * qmv::phase_bytes(4); }
int qmv_nflags(int kmax) { return (kmax + qmv::PH * 32 - 1) / (qmv::PH * 32); }

cudaError_t qmv_run(const QMat &m, const float *X, int xs, const float *norm_w, int B, float *Y, int ys, int epi,
                    GemvScratch &s, cudaStream_t st) {
  if (B < 1 || B > QG_MAXB || m.K % 64 || !m.w || !X || xs < m.K || !s.err || m.kern != GK_QMV || !s.qx ||
      !s.qflag || m.K > s.kmax)
    return cudaErrorInvalidValue;
  if (epi == EPI_SWIGLU && (!m.pair || m.n_ht % 2)) return cudaErrorInvalidValue;
  QmvArgs a;
  a.w = m.w;
  a.K = m.K;
  a.nblk = m.K / 32;
  a.n_ht = m.n_ht;
  a.M = m.M;
  a.pair = m.pair;
  a.G = m.G;
  a.wm = qmv::warp_rows(m.n_ht, m.pair, m.G);
  a.x = X;
  a.xs = xs;
  a.xal = ((reinterpret_cast<uintptr_t>(X) & 15) == 0 && xs % 4 == 0) ? 1 : 0;
  a.xw = norm_w;
  a.B = B;
  a.y = Y;
  a.ys = ys;
  a.epi = epi;
  a.row0 = s.row0;
  a.np = s.np;
  for (int i = 0; i < QG_MAX_PEERS; i++) a.yp[i] = i < s.np ? s.yp[i] : nullptr;
  a.err = s.err;
  {  // the plan of the CTA with the most rows must fit the kernel's tables
    const int unit = m.pair ? 2 : 1, nu = m.n_ht / unit;
    if ((long long)nu * m.G >= (1ll << 31)) return cudaErrorInvalidValue;
    const int nh = (nu + m.G - 1) / m.G * unit, nv = (nh + 1) / 2, nt = (B + 3) / 4;
    const int rw = qmv::rw_for(nt, m.type, a.wm), npass = (nv + a.wm * rw - 1) / (a.wm * rw);
    long long nst = 0;
    for (int p = 0; p < npass; p++) nst += qmv::pass_of(p, npass, nv, nh, a.nblk, qmv::chunk_bytes(m.type), nt).nst;
    if (npass > qmv::MAXPASS || nst > qmv::MAXSTAGE) return cudaErrorInvalidValue;
  }
  a.xg = s.qx;
  a.flags = s.qflag;
  if (++s.qepoch == 0) s.qepoch = 1;  // flags start at 0: an epoch is never 0
  a.epoch = s.qepoch;
  const int nt = (B + 3) / 4;
  switch (nt * 16 + m.type) {
    case 16 + 2: return qmv_launch_t<2, 1>(a, st);
    case 32 + 2: return qmv_launch_t<2, 2>(a, st);
    case 48 + 2: return qmv_launch_t<2, 3>(a, st);
    case 64 + 2: return qmv_launch_t<2, 4>(a, st);
    case 16 + 8: return qmv_launch_t<8, 1>(a, st);
    case 32 + 8: return qmv_launch_t<8, 2>(a, st);
    case 48 + 8: return qmv_launch_t<8, 3>(a, st);
    default: return qmv_launch_t<8, 4>(a, st);
  }
}

template <int TYPE, int NT>
static cudaError_t qmv_attr() {
  cudaError_t e = cudaFuncSetAttribute(qmv::qmv_kernel<TYPE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       qmv::SMEM);
  if (e != cudaSuccess) return e;
  return carveout_max(qmv::qmv_kernel<TYPE, NT>);
}

cudaError_t qmv_configure() {
  CW_TRY((qmv_attr<2, 1>()));
  CW_TRY((qmv_attr<2, 2>()));
  CW_TRY((qmv_attr<2, 3>()));
  CW_TRY((qmv_attr<2, 4>()));
  CW_TRY((qmv_attr<8, 1>()));
  CW_TRY((qmv_attr<8, 2>()));
  CW_TRY((qmv_attr<8, 3>()));
  CW_TRY((qmv_attr<8, 4>()));
  CW_TRY(carveout_max(qmv::repack_kernel<2>));
  CW_TRY(carveout_max(qmv::repack_kernel<8>));
  return cudaSuccess;
}

}  // namespace cw
