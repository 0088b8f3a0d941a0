// Batched Q4_0 / Q8_0 GEMV for B <= 16 verify rows on sm_100a.
//
// Replaces the reference's gemvb()/gemv() (run.c:1577-1680, 1419-1527) and
// the row dots under them (dot_q4_0 run.c:1009-1025, dot_nib16 run.c:432,
// dot_q8_0 run.c:1248-1274).
//
// Arithmetic.  The reference computes, per row and per 32-weight block,
//   y += d * sum_j (q_j - 8) * x_j          (fp32).
// B = 8 columns at 28 FLOP/byte is beyond what the CUDA cores can do at HBM
// speed, so the block dot runs on the tensor cores: (q - 8) is exact in f16,
// and X is split into f16 hi + lo parts (x = hi + lo to ~2^-22 relative) after
// a per-column power-of-two scale that keeps it inside f16 range.  Per block:
//   c = A*Xhi(k0..15) + A*Xlo(k0..15) + A*Xhi(k16..31) + A*Xlo(k16..31)
// (fp32 accumulate inside the MMA), then acc = fma(d, c, acc) on the CUDA
// cores -- the reference's per-block scale, applied to an fp32 partial.
//
// Batch invariance.  Column b of any call depends only on column b of X: the
// n-tile of 8 columns a column falls in runs the same MMA/FMA chain whether
// or not another n-tile runs, and the K partition (below) depends on the
// matrix shape and grid only, never on B.  So a B-row verify block produces
// the same bits as B single-row calls.
//
// Work split.  A fixed persistent grid of G CTAs (8 warps, 2 m-tiles = 32
// rows per warp, so 256 rows per CTA tile) takes an equal contiguous share
// of the (tile, k-pair) space ("stream-K").  A tile cut between CTAs is
// reduced by the last CTA to arrive, summing the partials in k order, so
// the result does not depend on arrival order.
//
// Memory.  Weights stream HBM -> shared memory through a 6-stage per-warp
// cp.async ring (16-byte LDGSTS, no L1 allocation); X fragments (small,
// shared by every warp) come through L1.
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
    uint8_t *c = dst + ((size_t)dmt * dst_kp + p) * chunk;
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

cudaError_t qmat_repack(const QMat &dst, const uint8_t *src, int M, int mt_off, int mt_stride, cudaStream_t st) {
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

// ---- X preparation ----
// One CTA per column b < nt*8: exponent e with max|x|*2^e in [2^14, 2^15),
// then per (32-block, lane) the f16 hi/lo fragment words in the K order the
// A fragments use: lane (g,t) of n-tile b/8 (g = b%8) holds
//   (x[4t], x[4t+2]) (x[4t+1], x[4t+3]) (x[4t+16], x[4t+18]) (x[4t+17], x[4t+19]).
__global__ void prep_x_kernel(const float *__restrict__ X, int xs, int B, int K, int nt, uint4 *__restrict__ xf,
                              int *__restrict__ xexp) {
  const int b = blockIdx.x;
  __shared__ float red[32];
  __shared__ int s_e;
  float mx = 0.f;
  if (b < B)
    for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(X[(size_t)b * xs + k]));
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) {
      int e = 0;
      if (v > 0.f && v <= 3.0e38f) {
        int p;
        frexpf(v, &p);  // v = m * 2^p, m in [0.5, 1)
        e = 15 - p;
        e = e < -100 ? -100 : (e > 100 ? 100 : e);
      }
      s_e = e;
      xexp[b] = e;
    }
  }
  __syncthreads();
  const int e = s_e;
  const float scale = __int_as_float((127 + e) << 23);
  const int g = b & 7, n = b >> 3, nb = K / 32;
  for (int item = threadIdx.x; item < nb * 4; item += blockDim.x) {
    const int kb = item >> 2, t = item & 3;
    const int base = kb * 32;
    const int js[8] = {4 * t, 4 * t + 2, 4 * t + 1, 4 * t + 3, 4 * t + 16, 4 * t + 18, 4 * t + 17, 4 * t + 19};
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float v0 = 0.f, v1 = 0.f;
      if (b < B) {
        v0 = X[(size_t)b * xs + base + js[2 * i]] * scale;
        v1 = X[(size_t)b * xs + base + js[2 * i + 1]] * scale;
      }
      const half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
      const half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
      hi[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      lo[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    const int lane = g * 4 + t;
    const size_t o = ((size_t)(kb * nt + n) * 2) * 32 + lane;
    xf[o] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    xf[o + 32] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

cudaError_t gemv_prep_x(const float *X, int xs, int B, int K, GemvScratch &s, cudaStream_t st) {
  if (B < 1 || B > QG_MAXB || K % 64 || K > s.kmax) return cudaErrorInvalidValue;
  const int nt = (B + 7) / 8;
  prep_x_kernel<<<nt * 8, 256, 0, st>>>(X, xs, B, K, nt, s.xf, s.xexp);
  return cudaGetLastError();
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
  int G;
  long long units;
};

CW_DEV float silu_f(float x) { return x * (1.f / (1.f + expf(-x))); }

// Apply the epilogue for one warp's accumulators (rows of m-tiles mt0, mt0+1).
template <int NT>
CW_DEV void gemv_epilogue(const GemvArgs &a, int mt0, bool has1, const float (&acc)[2][NT][4], int g, int t) {
#pragma unroll
  for (int n = 0; n < NT; n++) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int col = n * 8 + 2 * t + (i & 1);
      if (col >= a.B) continue;
      const float sc = __int_as_float((127 - __ldg(a.xexp + col)) << 23);
      const int rr = g + ((i >> 1) << 3);
      if (a.epi == EPI_SWIGLU) {
        const int row = (mt0 >> 1) * 16 + rr;
        if (row * 2 < a.M) {
          const float gt = acc[0][n][i] * sc, up = acc[1][n][i] * sc;
          a.y[(size_t)col * a.ys + row] = silu_f(gt) * up;
        }
      } else {
#pragma unroll
        for (int mt = 0; mt < 2; mt++) {
          if (mt == 1 && !has1) continue;
          const int row = (mt0 + mt) * 16 + rr;
          if (row >= a.M) continue;
          const float v = acc[mt][n][i] * sc;
          float *p = a.y + (size_t)col * a.ys + row;
          if (a.epi == EPI_ADD) *p += v;
          else *p = v;
        }
      }
    }
  }
}

template <int TYPE, int NT>
__global__ void __launch_bounds__(QG_WARPS * 32, 2) qgemv_kernel(GemvArgs a) {
  constexpr int CHUNK = TYPE == 8 ? 1088 : 576;
  constexpr int QB = TYPE == 8 ? 1024 : 512;
  constexpr int STAGE = 2 * CHUNK;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int s_last;
  const int c = blockIdx.x;
  const long long u_begin = (long long)c * a.units / a.G, u_end = (long long)(c + 1) * a.units / a.G;
  if (u_begin >= u_end) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  uint8_t *ring = smem + warp * QG_STAGES * STAGE;
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};

  long long u = u_begin;
  bool first_seg = true;
  while (u < u_end) {
    const int tile = (int)(u / a.kp);
    const int ka = (int)(u % a.kp);
    const long long remain = u_end - u;
    const int kb_end = (int)((long long)(a.kp - ka) < remain ? a.kp : ka + remain);
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

    if (has0) {
      const uint8_t *w0 = a.w + (size_t)mt0 * a.kp * CHUNK;
      const uint8_t *w1 = w0 + (size_t)a.kp * CHUNK;
      auto issue = [&](int i) {
        if (i < nk) {
          const int k = ka + i;
          uint8_t *dst = ring + (i % QG_STAGES) * STAGE;
          const uint8_t *s0 = w0 + (size_t)k * CHUNK, *s1 = w1 + (size_t)k * CHUNK;
#pragma unroll
          for (int q = 0; q < QB / 512; q++) {
            cp_async16(dst + q * 512 + lane * 16, s0 + q * 512 + lane * 16);
            if (has1) cp_async16(dst + CHUNK + q * 512 + lane * 16, s1 + q * 512 + lane * 16);
          }
          if (lane < 4) cp_async16(dst + QB + lane * 16, s0 + QB + lane * 16);
          else if (lane < 8 && has1) cp_async16(dst + CHUNK + QB + (lane - 4) * 16, s1 + QB + (lane - 4) * 16);
        }
        cp_async_commit();
      };
#pragma unroll
      for (int i = 0; i < QG_STAGES - 1; i++) issue(i);

      // X fragments for k-pair k: [kb 2][n NT][hi/lo 2] uint4 at lane.
      auto load_x = [&](int k, uint4 (&xr)[2][NT][2]) {
#pragma unroll
        for (int kbi = 0; kbi < 2; kbi++)
#pragma unroll
          for (int n = 0; n < NT; n++) {
            const size_t o = ((size_t)((2 * k + kbi) * NT + n) * 2) * 32 + lane;
            xr[kbi][n][0] = ldg_u4(a.xf + o);
            xr[kbi][n][1] = ldg_u4(a.xf + o + 32);
          }
      };
      uint4 xcur[2][NT][2], xnext[2][NT][2];
      load_x(ka, xcur);

      for (int i = 0; i < nk; i++) {
        issue(i + QG_STAGES - 1);
        if (i + 1 < nk) load_x(ka + i + 1, xnext);
        cp_async_wait<QG_STAGES - 1>();
        __syncwarp();
        const uint8_t *stg = ring + (i % QG_STAGES) * STAGE;
#pragma unroll
        for (int mt = 0; mt < 2; mt++) {
          if (mt == 1 && !has1) break;
          const uint8_t *ch = stg + mt * CHUNK;
          const uint2 scw = *reinterpret_cast<const uint2 *>(ch + QB + g * 8);
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
              const uint4 xh = xcur[kbi][n][0], xl = xcur[kbi][n][1];
              float cc[4];
              mma_16816(cc, a0s0, a1s0, a2s0, a3s0, xh.x, xh.y, zero4);
              mma_16816(cc, a0s0, a1s0, a2s0, a3s0, xl.x, xl.y, cc);
              mma_16816(cc, a0s1, a1s1, a2s1, a3s1, xh.z, xh.w, cc);
              mma_16816(cc, a0s1, a1s1, a2s1, a3s1, xl.z, xl.w, cc);
              acc[mt][n][0] = fmaf(dg, cc[0], acc[mt][n][0]);
              acc[mt][n][1] = fmaf(dg, cc[1], acc[mt][n][1]);
              acc[mt][n][2] = fmaf(dg8, cc[2], acc[mt][n][2]);
              acc[mt][n][3] = fmaf(dg8, cc[3], acc[mt][n][3]);
            }
          }
        }
        __syncwarp();
#pragma unroll
        for (int kbi = 0; kbi < 2; kbi++)
#pragma unroll
          for (int n = 0; n < NT; n++) {
            xcur[kbi][n][0] = xnext[kbi][n][0];
            xcur[kbi][n][1] = xnext[kbi][n][1];
          }
      }
      cp_async_wait<0>();
    }

    const bool full = (ka == 0 && kb_end == a.kp);
    if (full) {
      if (has0) gemv_epilogue<NT>(a, mt0, has1, acc, g, t);
    } else {
      // Partial tile: park this segment's sums, last CTA to arrive reduces.
      const int slot = first_seg ? 0 : 1;
      float *mine = a.ws + ((size_t)c * 2 + slot) * (QG_TILE_MT * 16 * 16);
      if (has0) {
#pragma unroll
        for (int mt = 0; mt < 2; mt++)
#pragma unroll
          for (int n = 0; n < NT; n++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
              float *p = mine + ((warp * 2 + mt) * 16 + g + 8 * h) * 16 + n * 8 + 2 * t;
              *reinterpret_cast<float2 *>(p) = make_float2(acc[mt][n][2 * h], acc[mt][n][2 * h + 1]);
            }
      }
      __threadfence();
      __syncthreads();
      const long long tu0 = (long long)tile * a.kp, tu1 = tu0 + a.kp - 1;
      const int c_first = (int)(((tu0 + 1) * a.G - 1) / a.units);
      const int c_last = (int)(((tu1 + 1) * a.G - 1) / a.units);
      if (threadIdx.x == 0) {
        const int old = atomicAdd(a.cnt + tile, 1);
        s_last = (old == c_last - c_first);
      }
      __syncthreads();
      if (s_last) {
        __threadfence();
        if (has0) {
          float sum[2][NT][4];
#pragma unroll
          for (int mt = 0; mt < 2; mt++)
#pragma unroll
            for (int n = 0; n < NT; n++)
#pragma unroll
              for (int i = 0; i < 4; i++) sum[mt][n][i] = 0.f;
          for (int cc = c_first; cc <= c_last; cc++) {
            const long long cu0 = (long long)cc * a.units / a.G;
            const int sl = cu0 >= tu0 ? 0 : 1;
            const float *src = a.ws + ((size_t)cc * 2 + sl) * (QG_TILE_MT * 16 * 16);
#pragma unroll
            for (int mt = 0; mt < 2; mt++)
#pragma unroll
              for (int n = 0; n < NT; n++)
#pragma unroll
                for (int h = 0; h < 2; h++) {
                  const float *p = src + ((warp * 2 + mt) * 16 + g + 8 * h) * 16 + n * 8 + 2 * t;
                  const float2 v = __ldcg(reinterpret_cast<const float2 *>(p));
                  sum[mt][n][2 * h] += v.x;
                  sum[mt][n][2 * h + 1] += v.y;
                }
          }
          gemv_epilogue<NT>(a, mt0, has1, sum, g, t);
        }
        if (threadIdx.x == 0) a.cnt[tile] = 0;
      }
      __syncthreads();
    }
    u += nk;
    first_seg = false;
  }
}

size_t gemv_scratch_ws_floats(int G) { return (size_t)G * 2 * QG_TILE_MT * 16 * 16; }

template <int TYPE, int NT>
static cudaError_t launch_t(const GemvArgs &a, cudaStream_t st) {
  constexpr int CHUNK = TYPE == 8 ? 1088 : 576;
  const int smem = QG_WARPS * QG_STAGES * 2 * CHUNK;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(qgemv_kernel<TYPE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  qgemv_kernel<TYPE, NT><<<a.G, QG_WARPS * 32, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t gemv_run(const QMat &m, int B, float *Y, int ys, int epi, GemvScratch &s, cudaStream_t st) {
  if (B < 1 || B > QG_MAXB || m.K % 64 || m.K > s.kmax || !m.w) return cudaErrorInvalidValue;
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
  const int n_tiles = (m.n_mt + QG_TILE_MT - 1) / QG_TILE_MT;
  if (n_tiles > s.max_tiles) return cudaErrorInvalidValue;
  a.units = (long long)n_tiles * a.kp;
  // Grid: a function of the shape only (never of B), >= 4 k-pairs per CTA.
  long long g = (a.units + 3) / 4;
  a.G = (int)(g < s.G ? g : s.G);
  if (m.type == 8) return B > 8 ? launch_t<8, 2>(a, st) : launch_t<8, 1>(a, st);
  return B > 8 ? launch_t<2, 2>(a, st) : launch_t<2, 1>(a, st);
}

}  // namespace cw
