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
  const float w0 = convw[c * 4 + 0], w1 = convw[c * 4 + 1], w2 = convw[c * 4 + 2], w3 = convw[c * 4 + 3];
  float s0 = cstate_in[c * 3 + 0], s1 = cstate_in[c * 3 + 1], s2 = cstate_in[c * 3 + 2];
  const bool is_qk = grp < 2 * nkh;
  for (int b = 0; b < B; b++) {
    const float cur = proj[(size_t)b * ps + c];
    craw[(size_t)b * QKV + c] = cur;
    float y = s0 * w0 + s1 * w1 + s2 * w2 + cur * w3;
    s0 = s1;
    s1 = s2;
    s2 = cur;
    y = silu_dev(y);
    if (is_qk) {
      // l2norm over the 128 channels of this head (l2norm_rows run.c:401)
      float ss = warp_sum(y * y);
      __syncthreads();
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      ss = (red[0] + red[1]) + (red[2] + red[3]);
      y *= 1.f / sqrtf(ss + 1e-6f);
    }
    gin[(size_t)b * GS + c] = y;
  }
  cstate_out[c * 3 + 0] = s0;
  cstate_out[c * 3 + 1] = s1;
  cstate_out[c * 3 + 2] = s2;
}

// ---- the recurrence: CTA = (value head, half of the value columns),
// 256 threads = 64 columns x 4 quarters of the key rows; each thread keeps
// its 32x1 slice of S in registers for all B positions.  The two halves of a
// head form a thread-block cluster of 2 for the gated RMSNorm of the head's
// 128 outputs per row (run.c:2142-2178):
//   out[i] = wn[i] * o[i] * rsqrt(mean_i o^2 + eps) * silu(z[i]),
// one exchange of the halves' per-row sums of squares through distributed
// shared memory after the last row. ----
constexpr int GDN_T = 256;

__global__ void __launch_bounds__(GDN_T) gdn_recur_kernel(const float *__restrict__ Sin, float *__restrict__ Sout,
                                                          const float *__restrict__ gin, int B, int nkh, int nvh,
                                                          float *__restrict__ out, float *__restrict__ delta,
                                                          const float *__restrict__ z, int zs,
                                                          const float *__restrict__ wn) {
  pdl_trigger();
  pdl_wait();
  const int hv = blockIdx.x >> 1, half = blockIdx.x & 1;
  const int hk = hv % nkh;
  const int col = threadIdx.x & 63, q4 = threadIdx.x >> 6;
  const int j = half * 64 + col;
  const int QKV = (2 * nkh + nvh) * 128;
  const int GS = QKV + 2 * nvh;
  __shared__ float kq[2][128];
  __shared__ float part[4][64];
  __shared__ float dl[64];
  __shared__ float ob[GDN_MAXB][64];   // raw outputs of this half, per row
  __shared__ float oss[GDN_MAXB];      // their sums of squares (read by the other half)
  const float *S0 = Sin + (size_t)hv * 128 * 128;
  float s[32];
#pragma unroll
  for (int i = 0; i < 32; i++) s[i] = S0[(size_t)(q4 * 32 + i) * 128 + j];
  const float scale = 1.f / sqrtf(128.f);
  for (int b = 0; b < B; b++) {
    const float *row = gin + (size_t)b * GS;
    __syncthreads();
    if (threadIdx.x < 128) kq[0][threadIdx.x] = row[nkh * 128 + hk * 128 + threadIdx.x];
    else kq[1][threadIdx.x - 128] = row[hk * 128 + threadIdx.x - 128];
    const float g = row[QKV + hv], beta = row[QKV + nvh + hv];
    const float v = row[2 * nkh * 128 + hv * 128 + j];
    __syncthreads();
    // S *= g; partial S^T k over this quarter
    float sk = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) {
      s[i] = s[i] * g;
      sk = fmaf(s[i], kq[0][q4 * 32 + i], sk);
    }
    part[q4][col] = sk;
    __syncthreads();
    if (q4 == 0) {
      const float tot = (part[0][col] + part[1][col]) + (part[2][col] + part[3][col]);
      const float d = beta * (v - tot);
      dl[col] = d;
      delta[(size_t)b * nvh * 128 + hv * 128 + j] = d;
    }
    __syncthreads();
    const float d = dl[col];
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) {
      s[i] = fmaf(kq[0][q4 * 32 + i], d, s[i]);
      o = fmaf(s[i], kq[1][q4 * 32 + i], o);
    }
    __syncthreads();
    part[q4][col] = o;
    __syncthreads();
    if (q4 == 0) ob[b][col] = ((part[0][col] + part[1][col]) + (part[2][col] + part[3][col])) * scale;
  }
  float *S1 = Sout + (size_t)hv * 128 * 128;
#pragma unroll
  for (int i = 0; i < 32; i++) S1[(size_t)(q4 * 32 + i) * 128 + j] = s[i];
  // gated RMSNorm: warp b (< 8) sums row b's 64 squares of this half (and row
  // b + 8), then the halves' sums are added in rank order
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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

// ---- rollback: replay rows 0..k (inclusive) onto the committed state in
// place; conv state <- last three raw inputs. One CTA per (layer, head, half)
// for S, plus conv CTAs. ----
__device__ __forceinline__ void replay_layer(const GdnLayerPtrs &P, int k, int nkh, int nvh) {
  const int QKV = (2 * nkh + nvh) * 128;
  const int GS = QKV + 2 * nvh;
  const int nS = nvh * 2;
  if ((int)blockIdx.x >= nS) {
    // conv state: channels handled by the remaining CTAs
    const int c = (blockIdx.x - nS) * GDN_T + threadIdx.x;
    if (c >= QKV) return;
    float st[3] = {P.cstate[c * 3 + 0], P.cstate[c * 3 + 1], P.cstate[c * 3 + 2]};
    for (int b = 0; b <= k; b++) {
      st[0] = st[1];
      st[1] = st[2];
      st[2] = P.craw[(size_t)b * QKV + c];
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
  float *S = P.S + (size_t)hv * 128 * 128;
  float s[32];
#pragma unroll
  for (int i = 0; i < 32; i++) s[i] = S[(size_t)(q4 * 32 + i) * 128 + j];
  for (int b = 0; b <= k; b++) {
    const float *row = P.gin + (size_t)b * GS;
    const float g = row[QKV + hv];
    const float d = P.delta[(size_t)b * nvh * 128 + hv * 128 + j];
    const float *kk = row + nkh * 128 + hk * 128 + q4 * 32;
#pragma unroll
    for (int i = 0; i < 32; i++) s[i] = fmaf(kk[i], d, s[i] * g);
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
  CW_TRY(launch_pdl(gdn_conv_kernel, QKV / 128 + 1, 128, 0, st, a.proj, a.ps, a.B, a.nkh, a.nvh, a.a_off, a.b_off, a.convw,
                                                  a.cstate_in, a.cstate_out, a.craw, a.A, a.dt, a.gin));
  CW_TRY(launch_pdl_cluster(gdn_recur_kernel, a.nvh * 2, GDN_T, 0, st, 2, a.S_in, a.S_out, a.gin, a.B, a.nkh, a.nvh,
                            a.out, a.delta, a.z, a.ps, a.wn));
  return cudaGetLastError();
}

cudaError_t launch_gdn_replay(GdnLayerPtrs *dev_layers, int n_layers, int k, int nkh, int nvh, cudaStream_t st) {
  const int QKV = (2 * nkh + nvh) * 128;
  dim3 grid(nvh * 2 + (QKV + GDN_T - 1) / GDN_T, n_layers);
  CW_TRY(launch_pdl(gdn_replay_kernel, grid, GDN_T, 0, st, dev_layers, k, nkh, nvh));
  return cudaGetLastError();
}

cudaError_t launch_gdn_replay1(const GdnLayerPtrs &layer, int k, int nkh, int nvh, cudaStream_t st) {
  const int QKV = (2 * nkh + nvh) * 128;
  CW_TRY(launch_pdl(gdn_replay1_kernel, nvh * 2 + (QKV + GDN_T - 1) / GDN_T, GDN_T, 0, st, layer, k, nkh, nvh));
  return cudaGetLastError();
}

// One-time kernel attributes (called at engine set-up).
cudaError_t gdn_configure() {
  cudaError_t e;
  if ((e = carveout_max(gdn_conv_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(gdn_recur_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(gdn_replay_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(gdn_replay1_kernel)) != cudaSuccess) return e;
  return cudaSuccess;
}

}  // namespace cw
