// GatedDeltaNet verify step (b): depthwise causal conv + the delta-rule
// recurrence over the B positions of a verify block, with rollback.
//
// Replaces conv1d_update (run.c:2183-2200), the decay/beta transform
// (run.c:2339-2344, 2693-2699), gdn_step with its gated norm
// (run.c:2014-2180) and the rollback snapshots snap_save/snap_load
// (run.c:2787-2809).
//
// Rollback.  A block reads the committed state (buffer `cur`) and writes the
// state after its last row to the other buffer.  Each row's rank-1 update
// (gate g_b, normalised key k_b, delta d_b) stays in per-layer HBM buffers,
// so the state after ANY row k is recoverable: a full accept flips `cur`
// (pointer swap); a short walk replays rows 0..k onto the committed state in
// place, with the same fp32 operations the block used, hence bit-identical to
// having stopped after row k.  No weight sweep is repeated.
#include "gdn.cuh"
#include "rowprep.cuh"

namespace cw {

// ---- conv + SiLU + q/k l2norm + decay/beta (one CTA per 128-channel group;
// the last CTA does the per-head gate/beta of all rows) ----
// proj row b: [qkv QKV | z | alpha at a_off | beta at b_off] (stride ps).
// gin row b:  [q NKH*128 | k NKH*128 | v NVH*128 | g NVH | beta NVH].
__global__ void __launch_bounds__(128) gdn_conv_kernel(const float *__restrict__ proj, int ps, int B, int nkh, int nvh,
                                                       int a_off, int b_off, const float *__restrict__ convw,
                                                       const float *__restrict__ cstate_in,
                                                       float *__restrict__ cstate_out, float *__restrict__ craw,
                                                       const float *__restrict__ A, const float *__restrict__ dt,
                                                       float *__restrict__ gin) {
  pdl_trigger();
  pdl_wait();
  const int QKV = (2 * nkh + nvh) * 128;
  const int GS = QKV + 2 * nvh;
  const int grp = blockIdx.x;
  __shared__ float red[32];
  if (grp == QKV / 128) {
    // decay / beta for every (row, head)
    for (int i = threadIdx.x; i < B * nvh; i += blockDim.x) {
      const int b = i / nvh, h = i % nvh;
      const float al = proj[(size_t)b * ps + a_off + h];
      const float be = proj[(size_t)b * ps + b_off + h];
      const float x = al + dt[h];
      const float sp = x > 20.f ? x : logf(1.f + expf(x));
      gin[(size_t)b * GS + QKV + h] = expf(A[h] * sp);
      gin[(size_t)b * GS + QKV + nvh + h] = 1.f / (1.f + expf(-be));
    }
    return;
  }
  const int c = grp * 128 + threadIdx.x;
  // every row's input at once: one memory round trip, not one per row
  float raw[GDN_MAXB];
#pragma unroll
  for (int b = 0; b < GDN_MAXB; b++) raw[b] = b < B ? proj[(size_t)b * ps + c] : 0.f;
  const float w0 = convw[c * 4 + 0], w1 = convw[c * 4 + 1], w2 = convw[c * 4 + 2], w3 = convw[c * 4 + 3];
  float s0 = cstate_in[c * 3 + 0], s1 = cstate_in[c * 3 + 1], s2 = cstate_in[c * 3 + 2];
  const bool is_qk = grp < 2 * nkh;
#pragma unroll
  for (int b = 0; b < GDN_MAXB; b++) {
    if (b >= B) break;
    const float cur = raw[b];
    craw[(size_t)b * QKV + c] = cur;
    float y = s0 * w0 + s1 * w1 + s2 * w2 + cur * w3;
    s0 = s1;
    s1 = s2;
    s2 = cur;
    y = silu_dev(y);
    if (is_qk) {
      // l2norm over the 128 channels of this head (l2norm_rows run.c:401);
      // the partial sums alternate between two slots, so one barrier per row
      // suffices (a slot is rewritten two rows later, after the next barrier)
      float ss = warp_sum(y * y);
      if ((threadIdx.x & 31) == 0) red[(b & 1) * 4 + (threadIdx.x >> 5)] = ss;
      __syncthreads();
      const float *r = red + (b & 1) * 4;
      ss = (r[0] + r[1]) + (r[2] + r[3]);
      y *= 1.f / sqrtf(ss + 1e-6f);
    }
    gin[(size_t)b * GS + c] = y;
  }
  cstate_out[c * 3 + 0] = s0;
  cstate_out[c * 3 + 1] = s1;
  cstate_out[c * 3 + 2] = s2;
}

// ---- the recurrence: CTA = (value head, half of the value columns),
// 256 threads; lane l of warp w owns value column w*8 + (l & 7) of the half
// and key rows 32*(l >> 3) .. +31 (a quarter), and keeps that 32x1 slice of
// S in registers for all B positions.  The quarters of a column sit in lanes
// l, l^8, l^16, l^24, so S^T k and S^T q are reduced with two xor shuffles
// ((q0 + q1) + (q2 + q3) in every lane) and the row loop has no barrier.  The
// rows' k, q, v, gate and beta are staged in shared memory before the loop.
// The two halves of a head form a thread-block cluster of 2 for the gated
// RMSNorm of the head's 128 outputs per row (run.c:2142-2178):
//   out[i] = wn[i] * o[i] * rsqrt(mean_i o^2 + eps) * silu(z[i]),
// one exchange of the halves' per-row sums of squares through distributed
// shared memory after the last row. ----
constexpr int GDN_T = 256;
// a quarter's 32 keys + 4: the 4 quarters' float4 reads start on banks 0, 4, 8
// and 12 (conflict-free) and stay 16-byte aligned
constexpr int KQ_PAD = 36;

// One row of the delta rule on this thread's quarter (32 keys) of value
// column j, the state slice s in registers:
//   s *= g;  sk = S^T k (this quarter, then the four quarters);
//   d = beta (v - sk);  s += k d;  o = S^T q (likewise).
// The quarter's dot products run as four interleaved partial sums (keys i,
// i+4, ... in each) added pairwise, so the dependent FMA chains are 8 long;
// the state update is the plain fma(k, d, s * g) the rollback replay
// repeats from the stored (g, k, d).
CW_DEV void gdn_row(float (&s)[32], const float *kk, const float *qq, float g, float beta, float v, float &d,
                    float &o) {
  const float4 *k4 = reinterpret_cast<const float4 *>(kk), *q4v = reinterpret_cast<const float4 *>(qq);
  float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
  for (int m = 0; m < 8; m++) {
    const float4 k = k4[m];
    s[4 * m + 0] *= g;
    s[4 * m + 1] *= g;
    s[4 * m + 2] *= g;
    s[4 * m + 3] *= g;
    p0 = fmaf(s[4 * m + 0], k.x, p0);
    p1 = fmaf(s[4 * m + 1], k.y, p1);
    p2 = fmaf(s[4 * m + 2], k.z, p2);
    p3 = fmaf(s[4 * m + 3], k.w, p3);
  }
  float sk = (p0 + p1) + (p2 + p3);
  sk += __shfl_xor_sync(0xffffffffu, sk, 8);
  sk += __shfl_xor_sync(0xffffffffu, sk, 16);
  d = beta * (v - sk);
  p0 = p1 = p2 = p3 = 0.f;
#pragma unroll
  for (int m = 0; m < 8; m++) {
    const float4 k = k4[m], q = q4v[m];
    s[4 * m + 0] = fmaf(k.x, d, s[4 * m + 0]);
    s[4 * m + 1] = fmaf(k.y, d, s[4 * m + 1]);
    s[4 * m + 2] = fmaf(k.z, d, s[4 * m + 2]);
    s[4 * m + 3] = fmaf(k.w, d, s[4 * m + 3]);
    p0 = fmaf(s[4 * m + 0], q.x, p0);
    p1 = fmaf(s[4 * m + 1], q.y, p1);
    p2 = fmaf(s[4 * m + 2], q.z, p2);
    p3 = fmaf(s[4 * m + 3], q.w, p3);
  }
  o = (p0 + p1) + (p2 + p3);
  o += __shfl_xor_sync(0xffffffffu, o, 8);
  o += __shfl_xor_sync(0xffffffffu, o, 16);
}

__global__ void __launch_bounds__(GDN_T) gdn_recur_kernel(const float *__restrict__ Sin, float *__restrict__ Sout,
                                                          const float *__restrict__ gin, int B, int nkh, int nvh,
                                                          float *__restrict__ out, float *__restrict__ delta,
                                                          const float *__restrict__ z, int zs,
                                                          const float *__restrict__ wn) {
  pdl_trigger();
  pdl_wait();
  const int hv = blockIdx.x >> 1, half = blockIdx.x & 1;
  const int hk = hv % nkh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q4 = lane >> 3, col = warp * 8 + (lane & 7);
  const int j = half * 64 + col;
  const int QKV = (2 * nkh + nvh) * 128;
  const int GS = QKV + 2 * nvh;
  __shared__ __align__(16) float kq[GDN_MAXB][2][4 * KQ_PAD];  // per row: k, q of key head hk
  __shared__ float vsh[GDN_MAXB][64];             // v of this half's columns
  __shared__ float gb[GDN_MAXB][2];               // gate, beta
  __shared__ float ob[GDN_MAXB][64];              // raw outputs of this half, per row
  __shared__ float oss[GDN_MAXB];                 // their sums of squares (read by the other half)
  const float *S0 = Sin + (size_t)hv * 128 * 128;
  float s[32];
#pragma unroll
  for (int i = 0; i < 32; i++) s[i] = S0[(size_t)(q4 * 32 + i) * 128 + j];
  for (int i = threadIdx.x; i < B * 256; i += GDN_T) {
    const int b = i >> 8, w = (i >> 7) & 1, e = i & 127;
    const float *row = gin + (size_t)b * GS;
    kq[b][w][(e >> 5) * KQ_PAD + (e & 31)] = w == 0 ? row[nkh * 128 + hk * 128 + e] : row[hk * 128 + e];
  }
  for (int i = threadIdx.x; i < B * 64; i += GDN_T) {
    const int b = i >> 6, c = i & 63;
    vsh[b][c] = gin[(size_t)b * GS + 2 * nkh * 128 + hv * 128 + half * 64 + c];
  }
  if (threadIdx.x < B) {
    gb[threadIdx.x][0] = gin[(size_t)threadIdx.x * GS + QKV + hv];
    gb[threadIdx.x][1] = gin[(size_t)threadIdx.x * GS + QKV + nvh + hv];
  }
  __syncthreads();
  const float scale = 1.f / sqrtf(128.f);
  for (int b = 0; b < B; b++) {
    const float *kk = &kq[b][0][q4 * KQ_PAD], *qq = &kq[b][1][q4 * KQ_PAD];
    float d, o;
    gdn_row(s, kk, qq, gb[b][0], gb[b][1], vsh[b][col], d, o);
    if (q4 == 0) delta[(size_t)b * nvh * 128 + hv * 128 + j] = d;
    if (q4 == 0) ob[b][col] = o * scale;
  }
  float *S1 = Sout + (size_t)hv * 128 * 128;
#pragma unroll
  for (int i = 0; i < 32; i++) S1[(size_t)(q4 * 32 + i) * 128 + j] = s[i];
  __syncthreads();  // every row's outputs are in ob
  // gated RMSNorm: warp b (< 8) sums row b's 64 squares of this half (and row
  // b + 8), then the halves' sums are added in rank order
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  for (int b = warp; b < B; b += GDN_T / 32) {
    const float a0 = ob[b][lane], a1 = ob[b][lane + 32];
    float ss = fmaf(a0, a0, a1 * a1);
    ss = warp_sum(ss);
    if (lane == 0) oss[b] = ss;
  }
  cl.sync();
  const float *oth = cl.map_shared_rank(oss, half ^ 1);
  for (int i = threadIdx.x; i < B * 64; i += GDN_T) {
    const int b = i >> 6, c = i & 63, jj = half * 64 + c;
    const float tot = half == 0 ? oss[b] + oth[b] : oth[b] + oss[b];
    const float sn = 1.f / sqrtf(tot / 128.f + 1e-6f);
    out[(size_t)b * nvh * 128 + hv * 128 + jj] =
        wn[jj] * ob[b][c] * sn * silu_dev(z[(size_t)b * zs + hv * 128 + jj]);
  }
  cl.sync();  // the other half has read oss before this CTA leaves
}

// ---- the whole layer step in one launch: conv + SiLU + q/k l2norm +
// decay/beta + the recurrence + the gated norm.  A thread-block cluster holds
// every value head of one key head (R = nvh / nkh heads x 2 halves, R <= 4):
// rank r = 2 * (value head index within the key head) + half, value head
// hv = hk + nkh * (r / 2).  Each CTA convolves the channels it reads (the key
// head's 128 q and 128 k channels, its half's 64 v channels) itself, so no
// intermediate rows go through global memory; the q/k channels' conv state
// and rollback records are written by rank 0 after a cluster barrier (every
// CTA of the cluster has read the old state by then), the v channels' by
// their own CTA.  The arithmetic is the two-kernel path's, operation for
// operation, so both give the same bits.
// keep < 0: the engine's verify block -- the state after the last row goes to
// S_out / cstate_out and the rank-1 records (normalised k, gate, delta, raw
// rows) stay for a later commit.  keep >= 0: rollback on the caller's
// buffers in place (S_out == S_in, cstate_out == cstate_in): the state after
// row keep - 1 is written (nothing when keep == 0), no records. ----
__global__ void __launch_bounds__(GDN_T) gdn_fused_kernel(const GdnLayerArgs a, int keep) {
  pdl_trigger();
  pdl_wait();
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int nkh = a.nkh, nvh = a.nvh, B = a.B;
  const int R2 = 2 * (nvh / nkh);
  const int hk = blockIdx.x / R2, rank = blockIdx.x % R2;
  const int half = rank & 1, hv = hk + nkh * (rank >> 1);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int q4 = lane >> 3, col = warp * 8 + (lane & 7);
  const int j = half * 64 + col;
  const int QKV = (2 * nkh + nvh) * 128;
  const int GS = QKV + 2 * nvh;
  __shared__ __align__(16) float kq[GDN_MAXB][2][4 * KQ_PAD];
  __shared__ float vsh[GDN_MAXB][64];
  __shared__ float gb[GDN_MAXB][2];
  __shared__ float ob[GDN_MAXB][64];
  __shared__ float oss[GDN_MAXB];
  __shared__ float red[GDN_MAXB][8];
  const int nsnap = keep < 0 ? B : keep;  // rows in the state written
  constexpr int NZ = GDN_MAXB * 64 / GDN_T;  // output items per thread at most

  // ---- every global read first: one memory round trip for the whole step ----
  const bool isk = t >= 128;
  const int ch = isk ? nkh * 128 + hk * 128 + (t - 128) : hk * 128 + t;  // this thread's q or k channel
  float raw[GDN_MAXB];
#pragma unroll
  for (int b = 0; b < GDN_MAXB; b++) raw[b] = b < B ? a.proj[(size_t)b * a.ps + ch] : 0.f;
  const float w0 = a.convw[ch * 4 + 0], w1 = a.convw[ch * 4 + 1], w2 = a.convw[ch * 4 + 2], w3 = a.convw[ch * 4 + 3];
  const float o0 = a.cstate_in[ch * 3 + 0], o1 = a.cstate_in[ch * 3 + 1], o2 = a.cstate_in[ch * 3 + 2];
  const int vc = 2 * nkh * 128 + hv * 128 + half * 64 + (t & 63);  // v channel (threads < 64)
  float vr[GDN_MAXB];
  float u0 = 0.f, u1 = 0.f, u2 = 0.f, u3 = 0.f, p0 = 0.f, p1 = 0.f, p2 = 0.f;
  if (t < 64) {
#pragma unroll
    for (int b = 0; b < GDN_MAXB; b++) vr[b] = b < B ? a.proj[(size_t)b * a.ps + vc] : 0.f;
    u0 = a.convw[vc * 4 + 0]; u1 = a.convw[vc * 4 + 1]; u2 = a.convw[vc * 4 + 2]; u3 = a.convw[vc * 4 + 3];
    p0 = a.cstate_in[vc * 3 + 0]; p1 = a.cstate_in[vc * 3 + 1]; p2 = a.cstate_in[vc * 3 + 2];
  }
  float al = 0.f, be = 0.f, dtv = 0.f, Av = 0.f;
  if (t < B) {
    al = a.proj[(size_t)t * a.ps + a.a_off + hv];
    be = a.proj[(size_t)t * a.ps + a.b_off + hv];
    dtv = a.dt[hv];
    Av = a.A[hv];
  }
  const float *S0 = a.S_in + (size_t)hv * 128 * 128;
  float s[32];
#pragma unroll
  for (int i = 0; i < 32; i++) s[i] = S0[(size_t)(q4 * 32 + i) * 128 + j];
  float zv[NZ], wnv[NZ];
#pragma unroll
  for (int m = 0; m < NZ; m++) {
    const int i = t + GDN_T * m, b = i >> 6, c = i & 63, jj = half * 64 + c;
    zv[m] = b < B ? a.z[(size_t)b * a.ps + hv * 128 + jj] : 0.f;
    wnv[m] = a.wn[jj];
  }

  // ---- conv + SiLU + l2norm of the q/k channels, all rows ----
  float y[GDN_MAXB];
  {
    float c0 = o0, c1 = o1, c2 = o2;
#pragma unroll
    for (int b = 0; b < GDN_MAXB; b++) {
      if (b >= B) break;
      const float cur = raw[b];
      const float v = c0 * w0 + c1 * w1 + c2 * w2 + cur * w3;
      c0 = c1;
      c1 = c2;
      c2 = cur;
      y[b] = silu_dev(v);
      const float ss = warp_sum(y[b] * y[b]);
      if (lane == 0) red[b][warp] = ss;
    }
  }
  // ---- v channels of this half (threads 0..63), their conv state owned here ----
  if (t < 64) {
    float c0 = p0, c1 = p1, c2 = p2;
#pragma unroll
    for (int b = 0; b < GDN_MAXB; b++) {
      if (b >= B) break;
      const float cur = vr[b];
      const float v = c0 * u0 + c1 * u1 + c2 * u2 + cur * u3;
      c0 = c1;
      c1 = c2;
      c2 = cur;
      const float yv = silu_dev(v);
      vsh[b][t] = yv;
      if (keep < 0) {
        a.gin[(size_t)b * GS + vc] = yv;
        a.craw[(size_t)b * QKV + vc] = cur;
      }
    }
    if (nsnap > 0 || keep < 0) {
#pragma unroll
      for (int m = 0; m < 3; m++) {
        const int pidx = nsnap + m;  // position in [old0 old1 old2 raw0 raw1 ...]
        float st = pidx == 0 ? p0 : (pidx == 1 ? p1 : p2);
#pragma unroll
        for (int b = 0; b < GDN_MAXB; b++)
          if (pidx == b + 3) st = vr[b];
        a.cstate_out[vc * 3 + m] = st;
      }
    }
  }
  // ---- decay / beta of this value head for every row ----
  if (t < B) {
    const float x = al + dtv;
    const float sp = x > 20.f ? x : logf(1.f + expf(x));
    gb[t][0] = expf(Av * sp);
    gb[t][1] = 1.f / (1.f + expf(-be));
    if (keep < 0 && half == 0) {
      a.gin[(size_t)t * GS + QKV + hv] = gb[t][0];
      a.gin[(size_t)t * GS + QKV + nvh + hv] = gb[t][1];
    }
  }
  __syncthreads();
  {
    const int w4 = isk ? 4 : 0;  // the 4 warps of this head's q or k channels
    const int e = t & 127;
#pragma unroll
    for (int b = 0; b < GDN_MAXB; b++) {
      if (b >= B) break;
      const float *r = red[b] + w4;
      const float ss = (r[0] + r[1]) + (r[2] + r[3]);
      const float yn = y[b] * (1.f / sqrtf(ss + 1e-6f));
      kq[b][isk ? 0 : 1][(e >> 5) * KQ_PAD + (e & 31)] = yn;
      if (keep < 0 && rank == 0) {
        a.gin[(size_t)b * GS + ch] = yn;
        a.craw[(size_t)b * QKV + ch] = raw[b];
      }
    }
  }
  __syncthreads();

  // ---- the recurrence (as gdn_recur_kernel) ----
  float sn[32];
#pragma unroll
  for (int i = 0; i < 32; i++) sn[i] = s[i];
  const float scale = 1.f / sqrtf(128.f);
  for (int b = 0; b < B; b++) {
    const float *kk = &kq[b][0][q4 * KQ_PAD], *qq = &kq[b][1][q4 * KQ_PAD];
    float d, o;
    gdn_row(s, kk, qq, gb[b][0], gb[b][1], vsh[b][col], d, o);
    if (keep < 0 && q4 == 0) a.delta[(size_t)b * nvh * 128 + hv * 128 + j] = d;
    if (q4 == 0) ob[b][col] = o * scale;
    if (b == nsnap - 1) {
#pragma unroll
      for (int i = 0; i < 32; i++) sn[i] = s[i];
    }
  }
  if (nsnap > 0) {
    float *S1 = a.S_out + (size_t)hv * 128 * 128;
#pragma unroll
    for (int i = 0; i < 32; i++) S1[(size_t)(q4 * 32 + i) * 128 + j] = sn[i];
  }
  __syncthreads();
  // ---- gated RMSNorm of the head's outputs (the halves exchange sums) ----
  for (int b = warp; b < B; b += GDN_T / 32) {
    const float a0 = ob[b][lane], a1 = ob[b][lane + 32];
    float ss = fmaf(a0, a0, a1 * a1);
    ss = warp_sum(ss);
    if (lane == 0) oss[b] = ss;
  }
  cl.sync();  // also: every CTA of the key head has read the old conv state
  const float *oth = cl.map_shared_rank(oss, rank ^ 1);
#pragma unroll
  for (int m = 0; m < NZ; m++) {
    const int i = t + GDN_T * m, b = i >> 6, c = i & 63, jj = half * 64 + c;
    if (b < B) {
      const float tot = half == 0 ? oss[b] + oth[b] : oth[b] + oss[b];
      const float sq = 1.f / sqrtf(tot / 128.f + 1e-6f);
      a.out[(size_t)b * nvh * 128 + hv * 128 + jj] = wnv[m] * ob[b][c] * sq * silu_dev(zv[m]);
    }
  }
  // the key head's q/k conv state (in place for the caller's rollback: every
  // CTA of the cluster has read it before the barrier above)
  if (rank == 0 && (nsnap > 0 || keep < 0)) {
#pragma unroll
    for (int m = 0; m < 3; m++) {
      const int pidx = nsnap + m;
      float st = pidx == 0 ? o0 : (pidx == 1 ? o1 : o2);
#pragma unroll
      for (int b = 0; b < GDN_MAXB; b++)
        if (pidx == b + 3) st = raw[b];
      a.cstate_out[ch * 3 + m] = st;
    }
  }
  cl.sync();  // the pair has read oss before this CTA leaves
}

bool gdn_fusable(int nkh, int nvh) { return nkh >= 1 && nvh % nkh == 0 && 2 * (nvh / nkh) <= 8; }

cudaError_t launch_gdn_fused(const GdnLayerArgs &a, int keep, cudaStream_t st) {
  if (a.B < 1 || a.B > GDN_MAXB || !gdn_fusable(a.nkh, a.nvh) || keep > a.B) return cudaErrorInvalidValue;
  const int r2 = 2 * (a.nvh / a.nkh);
  CW_TRY(launch_pdl_cluster(gdn_fused_kernel, a.nkh * r2, GDN_T, 0, st, r2, a, keep));
  return cudaGetLastError();
}

// ---- rollback: replay rows 0..k (inclusive) onto the committed state in
// place; conv state <- last three raw inputs. One CTA per (layer, head, half)
// for S, plus conv CTAs. ----
__device__ __forceinline__ void replay_layer(const GdnLayerPtrs &P, int k, int nkh, int nvh) {
  const int QKV = (2 * nkh + nvh) * 128;
  const int GS = QKV + 2 * nvh;
  const int nS = nvh * 2;
  if ((int)blockIdx.x >= nS) {
    // conv state after rows 0..k: the last three of [old state | raw rows]
    const int c = (blockIdx.x - nS) * GDN_T + threadIdx.x;
    if (c >= QKV) return;
    const float o1 = P.cstate[c * 3 + 1], o2 = P.cstate[c * 3 + 2];
    float st[3];
#pragma unroll
    for (int m = 0; m < 3; m++) {
      const int src = k - 2 + m;  // >= -2; -2 and -1 are old slots 1 and 2
      st[m] = src >= 0 ? P.craw[(size_t)src * QKV + c] : (src == -1 ? o2 : o1);
    }
    P.cstate[c * 3 + 0] = st[0];
    P.cstate[c * 3 + 1] = st[1];
    P.cstate[c * 3 + 2] = st[2];
    return;
  }
  const int hv = blockIdx.x >> 1, half = blockIdx.x & 1;
  const int hk = hv % nkh;
  const int col = threadIdx.x & 63, q4 = threadIdx.x >> 6;
  const int j = half * 64 + col;
  const int n = k + 1;  // rows replayed, <= GDN_MAXB (checked at launch)
  __shared__ float kr[GDN_MAXB][128];  // the rows' normalised keys of key head hk
  __shared__ float gr[GDN_MAXB];       // the rows' gates
  float *S = P.S + (size_t)hv * 128 * 128;
  float s[32];
#pragma unroll
  for (int i = 0; i < 32; i++) s[i] = S[(size_t)(q4 * 32 + i) * 128 + j];
  for (int i = threadIdx.x; i < n * 128; i += GDN_T)
    kr[i >> 7][i & 127] = P.gin[(size_t)(i >> 7) * GS + nkh * 128 + hk * 128 + (i & 127)];
  if ((int)threadIdx.x < n) gr[threadIdx.x] = P.gin[(size_t)threadIdx.x * GS + QKV + hv];
  float dr[GDN_MAXB];
#pragma unroll
  for (int b = 0; b < GDN_MAXB; b++) dr[b] = b < n ? P.delta[(size_t)b * nvh * 128 + hv * 128 + j] : 0.f;
  __syncthreads();
#pragma unroll
  for (int b = 0; b < GDN_MAXB; b++) {
    if (b >= n) break;
    const float g = gr[b];
    const float *kk = &kr[b][q4 * 32];
#pragma unroll
    for (int i = 0; i < 32; i++) s[i] = fmaf(kk[i], dr[b], s[i] * g);
  }
#pragma unroll
  for (int i = 0; i < 32; i++) S[(size_t)(q4 * 32 + i) * 128 + j] = s[i];
}

// Every linear layer of the model (layer = blockIdx.y) from a device table.
__global__ void __launch_bounds__(GDN_T) gdn_replay_kernel(GdnLayerPtrs *__restrict__ lp, int k, int nkh, int nvh) {
  pdl_trigger();
  pdl_wait();
  const GdnLayerPtrs P = lp[blockIdx.y];
  replay_layer(P, k, nkh, nvh);
}

// One layer whose pointers come as a kernel parameter (no table to upload).
__global__ void __launch_bounds__(GDN_T) gdn_replay1_kernel(const GdnLayerPtrs P, int k, int nkh, int nvh) {
  pdl_trigger();
  pdl_wait();
  replay_layer(P, k, nkh, nvh);
}

cudaError_t launch_gdn_layer(const GdnLayerArgs &a, cudaStream_t st) {
  const int QKV = (2 * a.nkh + a.nvh) * 128;
  if (a.B < 1 || a.B > GDN_MAXB) return cudaErrorInvalidValue;
  if (gdn_fusable(a.nkh, a.nvh)) return launch_gdn_fused(a, -1, st);
  CW_TRY(launch_pdl(gdn_conv_kernel, QKV / 128 + 1, 128, 0, st, a.proj, a.ps, a.B, a.nkh, a.nvh, a.a_off, a.b_off, a.convw,
                                                  a.cstate_in, a.cstate_out, a.craw, a.A, a.dt, a.gin));
  CW_TRY(launch_pdl_cluster(gdn_recur_kernel, a.nvh * 2, GDN_T, 0, st, 2, a.S_in, a.S_out, a.gin, a.B, a.nkh, a.nvh,
                            a.out, a.delta, a.z, a.ps, a.wn));
  return cudaGetLastError();
}

cudaError_t launch_gdn_replay(GdnLayerPtrs *dev_layers, int n_layers, int k, int nkh, int nvh, cudaStream_t st) {
  const int QKV = (2 * nkh + nvh) * 128;
  if (k < 0 || k >= GDN_MAXB) return cudaErrorInvalidValue;
  dim3 grid(nvh * 2 + (QKV + GDN_T - 1) / GDN_T, n_layers);
  CW_TRY(launch_pdl(gdn_replay_kernel, grid, GDN_T, 0, st, dev_layers, k, nkh, nvh));
  return cudaGetLastError();
}

cudaError_t launch_gdn_replay1(const GdnLayerPtrs &layer, int k, int nkh, int nvh, cudaStream_t st) {
  const int QKV = (2 * nkh + nvh) * 128;
  if (k < 0 || k >= GDN_MAXB) return cudaErrorInvalidValue;
  CW_TRY(launch_pdl(gdn_replay1_kernel, nvh * 2 + (QKV + GDN_T - 1) / GDN_T, GDN_T, 0, st, layer, k, nkh, nvh));
  return cudaGetLastError();
}

// One-time kernel attributes (called at engine set-up).
cudaError_t gdn_configure() {
  cudaError_t e;
  if ((e = carveout_max(gdn_conv_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(gdn_recur_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(gdn_fused_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(gdn_replay_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(gdn_replay1_kernel)) != cudaSuccess) return e;
  return cudaSuccess;
}

}  // namespace cw
