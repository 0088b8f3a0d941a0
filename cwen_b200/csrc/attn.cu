// Gated GQA attention over the KV cache with partial RoPE (c).
//
// Replaces layer_full_blk's per-row head split, q/k RMSNorm, RoPE and KV
// write (run.c:2714-2737) and attention_heads_kv (run.c:2362-2409).
//
// Split-K decode: the KV range [t0, pos] of a query row is cut into fixed
// 64-slot chunks; one CTA per (kv head, chunk) scores every query row of the
// block that reaches the chunk against one shared K/V tile in shared memory,
// and keeps (max, sum, weighted V) per query; the combine pass merges the
// chunks of a row in chunk order.  The chunking depends on the row's position
// only, so a row's output does not depend on the other rows of the block.
#include "attn.cuh"
#include "rowprep.cuh"

namespace cw {

constexpr int HD = 256;
constexpr int ACH = 64;     // slots per chunk
constexpr int KPAD = 260;   // padded K row (floats) in shared memory
constexpr int PART = 4 + HD;

// q/k RMSNorm (per head, shared 256-vector weight), RoPE on dims 0..63, KV write.
__global__ void __launch_bounds__(HD) attn_prep_kernel(const float *__restrict__ proj, int ps, int nh, int nkv,
                                                       const float *__restrict__ qn, const float *__restrict__ kn,
                                                       const float2 *__restrict__ rope, int pos0,
                                                       float *__restrict__ qbuf, float *__restrict__ Kc,
                                                       float *__restrict__ Vc) {
  pdl_trigger();
  pdl_wait();
  const int y = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int pos = pos0 + b;
  const float *row = proj + (size_t)b * ps;
  const int kofs = nh * 2 * HD, vofs = kofs + nkv * HD;
  __shared__ float v[HD];
  __shared__ float red[8];
  if (y >= nh + nkv) {  // V head: plain copy into the cache
    const int h = y - nh - nkv;
    Vc[((size_t)pos * nkv + h) * HD + d] = row[vofs + h * HD + d];
    return;
  }
  const bool isq = y < nh;
  const int h = isq ? y : y - nh;
  const float x = isq ? row[h * 2 * HD + d] : row[kofs + h * HD + d];
  float ss = warp_sum(x * x);
  if ((d & 31) == 0) red[d >> 5] = ss;
  __syncthreads();
  ss = ((red[0] + red[1]) + (red[2] + red[3])) + ((red[4] + red[5]) + (red[6] + red[7]));
  const float s = 1.f / sqrtf(ss / (float)HD + 1e-6f);
  const float o = (isq ? qn[d] : kn[d]) * x * s;
  v[d] = o;
  __syncthreads();
  float r = o;
  if (d < 64) {
    const float2 cs = rope[(size_t)pos * 32 + (d >> 1)];
    const float a = v[d & ~1], bb = v[d | 1];
    r = (d & 1) ? (a * cs.y + bb * cs.x) : (a * cs.x - bb * cs.y);
  }
  if (isq) qbuf[((size_t)b * nh + h) * HD + d] = r;
  else Kc[((size_t)pos * nkv + h) * HD + d] = r;
}

// Partial attention of every (row, head of kv group) against one chunk.
// Grid (kv head, chunk, row group): rows [z*rb, z*rb + rb) of the block, so a
// verify block spreads over rb-times more CTAs than a single row.
__global__ void __launch_bounds__(256) attn_chunk_kernel(const float *__restrict__ qbuf, const float *__restrict__ Kc,
                                                         const float *__restrict__ Vc, int nh, int nkv, int pos0,
                                                         int B, int t0, int nch_max, int rb, float *__restrict__ part) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm[];
  float *Ks = sm;                       // [ACH][KPAD]
  float *Vs = Ks + ACH * KPAD;          // [ACH][HD]
  float *Qs = Vs + ACH * HD;            // [8 warps][HD]
  const int hkv = blockIdx.x, c = blockIdx.y;
  const int b0 = blockIdx.z * rb, b1 = min(B, b0 + rb);
  const int c0 = c * ACH;
  const int last = pos0 + b1 - 1;
  if (c0 > last) return;
  const int tmax = min(c0 + ACH - 1, last);
  // stage the chunk (slots beyond the last row are zero-filled and masked)
  for (int i = threadIdx.x; i < ACH * (HD / 4); i += blockDim.x) {
    const int t = i / (HD / 4), d4 = (i % (HD / 4)) * 4;
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
    if (c0 + t <= tmax) {
      kv = *reinterpret_cast<const float4 *>(Kc + ((size_t)(c0 + t) * nkv + hkv) * HD + d4);
      vv = *reinterpret_cast<const float4 *>(Vc + ((size_t)(c0 + t) * nkv + hkv) * HD + d4);
    }
    *reinterpret_cast<float4 *>(Ks + t * KPAD + d4) = kv;
    *reinterpret_cast<float4 *>(Vs + t * HD + d4) = vv;
  }
  __syncthreads();
  const int G = nh / nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float *q = Qs + warp * HD;
  const float scale = 1.f / sqrtf((float)HD);
  for (int qi = warp; qi < (b1 - b0) * G; qi += 8) {
    const int b = b0 + qi / G, h = hkv * G + qi % G;
    const int p = pos0 + b;
    if (c0 > p || c0 + ACH - 1 < t0) continue;  // warp-uniform
    __syncwarp();
    for (int d = lane; d < HD; d += 32) q[d] = qbuf[((size_t)b * nh + h) * HD + d];
    __syncwarp();
    float sc[2];
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int t = lane + 32 * u;
      const float *kr = Ks + t * KPAD;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 8
      for (int d = 0; d < HD; d += 4) {
        const float4 kk = *reinterpret_cast<const float4 *>(kr + d);
        const float4 qq = *reinterpret_cast<const float4 *>(q + d);
        a0 = fmaf(qq.x, kk.x, a0);
        a1 = fmaf(qq.y, kk.y, a1);
        a2 = fmaf(qq.z, kk.z, a2);
        a3 = fmaf(qq.w, kk.w, a3);
      }
      const int tt = c0 + t;
      sc[u] = (tt >= t0 && tt <= p) ? ((a0 + a1) + (a2 + a3)) * scale : -INFINITY;
    }
    float m = warp_max(fmaxf(sc[0], sc[1]));
    const float e0 = sc[0] == -INFINITY ? 0.f : expf(sc[0] - m);
    const float e1 = sc[1] == -INFINITY ? 0.f : expf(sc[1] - m);
    const float l = warp_sum(e0 + e1);
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.f;
    for (int t = 0; t < ACH; t++) {
      const float pt = __shfl_sync(0xffffffffu, t < 32 ? e0 : e1, t & 31);
      const float4 v0 = *reinterpret_cast<const float4 *>(Vs + t * HD + lane * 8);
      const float4 v1 = *reinterpret_cast<const float4 *>(Vs + t * HD + lane * 8 + 4);
      acc[0] = fmaf(pt, v0.x, acc[0]);
      acc[1] = fmaf(pt, v0.y, acc[1]);
      acc[2] = fmaf(pt, v0.z, acc[2]);
      acc[3] = fmaf(pt, v0.w, acc[3]);
      acc[4] = fmaf(pt, v1.x, acc[4]);
      acc[5] = fmaf(pt, v1.y, acc[5]);
      acc[6] = fmaf(pt, v1.z, acc[6]);
      acc[7] = fmaf(pt, v1.w, acc[7]);
    }
    float *o = part + (((size_t)b * nh + h) * nch_max + c) * PART;
    if (lane == 0) {
      o[0] = m;
      o[1] = l;
    }
    *reinterpret_cast<float4 *>(o + 4 + lane * 8) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4 *>(o + 4 + lane * 8 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// Merge the chunks of each (row, head), apply the sigmoid gate
// (run.c:2396-2406) and emit the wo GEMV input.  One thread-block cluster per
// row (blockIdx.y); each CTA owns whole heads: per head one warp turns the
// chunk maxima into chunk weights w_c = exp(m_c - M) and l = sum l_c w_c, then
// every element sums its chunks' weighted partials in chunk order.
constexpr int COMB_THREADS = 256;
__global__ void __launch_bounds__(COMB_THREADS) attn_combine_kernel(const float *__restrict__ part,
                                                                   const float *__restrict__ proj, int ps, int nh,
                                                                   int pos0, int t0, int nch_max, int nt,
                                                                   uint4 *__restrict__ xf, int *__restrict__ xexp,
                                                                   float *__restrict__ yout) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[32], slot, linv[32];
  const int b = blockIdx.y, r = blockIdx.x, hper = nh / gridDim.x, h0 = r * hper;
  float *v = sm;                    // [hper][HD]
  float *wts = sm + hper * HD;      // [hper][nch_max]
  const int p = pos0 + b, cf = t0 / ACH, cl = p / ACH, nc = cl - cf + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int hl = warp; hl < hper; hl += nw) {
    const float *ph = part + ((size_t)b * nh + h0 + hl) * nch_max * PART;
    float M = -INFINITY;
    for (int c = cf + lane; c <= cl; c += 32) M = fmaxf(M, ph[(size_t)c * PART]);
    M = warp_max(M);
    float l = 0.f;
    for (int c = cf + lane; c <= cl; c += 32) {
      const float w = expf(ph[(size_t)c * PART] - M);
      wts[hl * nch_max + (c - cf)] = w;
      l = fmaf(ph[(size_t)c * PART + 1], w, l);
    }
    l = warp_sum(l);
    if (lane == 0) linv[hl] = l;
  }
  __syncthreads();
  float mx = 0.f;
  for (int i = threadIdx.x; i < hper * HD; i += blockDim.x) {
    const int hl = i / HD, d = i % HD, h = h0 + hl;
    const float *ph = part + ((size_t)b * nh + h) * nch_max * PART + 4 + d;
    const float *wh = wts + hl * nch_max;
    float a = 0.f;
#pragma unroll 4
    for (int c = 0; c < nc; c++) a = fmaf(ph[(size_t)(cf + c) * PART], wh[c], a);
    const float o = (a / linv[hl]) * sigmoid_dev(proj[(size_t)b * ps + h * 2 * HD + HD + d]);
    v[i] = o;
    mx = fmaxf(mx, fabsf(o));
    if (yout) yout[(size_t)b * nh * HD + h * HD + d] = o;
  }
  mx = cluster_reduce<true>(block_max(mx, red), &slot);
  const int e = xfrag_exponent(mx);
  if (r == 0 && threadIdx.x == 0) xexp[b] = e;
  emit_xfrag_blocks(v, h0 * (HD / 32), hper * (HD / 32), b, nt, xf, __int_as_float((127 + e) << 23), true);
}

cudaError_t launch_attention(const AttnArgs &a, GemvScratch &s, cudaStream_t st) {
  CW_TRY(launch_pdl(attn_prep_kernel, dim3(a.nh + 2 * a.nkv, a.B), HD, 0, st, a.proj, a.ps, a.nh, a.nkv, a.qn, a.kn, a.rope, a.pos0,
                                                               a.qbuf, a.Kc, a.Vc));
  const int last = a.pos0 + a.B - 1;
  const int nch = last / ACH + 1;
  if (nch > a.nch_max) return cudaErrorInvalidValue;
  const size_t smem = (size_t)(ACH * KPAD + ACH * HD + 8 * HD) * sizeof(float);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  // Rows per CTA: split the block's rows over more CTAs only while the
  // (kv head, chunk) grid alone is short of two CTAs per SM -- each extra row
  // group stages the chunk's K/V again, which long contexts cannot afford.
  static int n_sm = 0;
  if (!n_sm) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (n_sm <= 0) n_sm = 148;
  }
  const int G = a.nh / a.nkv, base = a.nkv * nch;
  const int min_rb = G >= 8 ? 1 : 8 / G;                       // about one (row, head) item per warp
  int groups = (2 * n_sm + base - 1) / base;
  const int max_groups = (a.B + min_rb - 1) / min_rb;
  groups = groups < 1 ? 1 : (groups > max_groups ? max_groups : groups);
  const int rb = (a.B + groups - 1) / groups;
  CW_TRY(launch_pdl(attn_chunk_kernel, dim3(a.nkv, nch, (a.B + rb - 1) / rb), 256, smem, st, a.qbuf, a.Kc, a.Vc, a.nh,
                    a.nkv, a.pos0, a.B, a.t0, a.nch_max, rb, a.part));
  const int cl = cluster_split(a.nh);
  if (a.nh / cl > 32) return cudaErrorInvalidValue;  // per-CTA heads must fit linv[32]
  const size_t csmem = (size_t)(a.nh / cl) * (HD + a.nch_max) * sizeof(float);
  static size_t cdone = 48 * 1024;
  if (csmem > cdone) {
    cudaError_t e = cudaFuncSetAttribute(attn_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem);
    if (e != cudaSuccess) return e;
    cdone = csmem;
  }
  CW_TRY(launch_pdl_cluster(attn_combine_kernel, dim3(cl, a.B), COMB_THREADS, csmem, st, cl, a.part, a.proj, a.ps,
                            a.nh, a.pos0, a.t0, a.nch_max, gemv_ntiles(a.B), s.xf, s.xexp, a.yout));
  return cudaGetLastError();
}

int attn_chunk_slots() { return ACH; }
size_t attn_part_floats(int bmax, int nh, int nch_max) { return (size_t)bmax * nh * nch_max * PART; }

// One-time kernel attributes (called at engine set-up).
cudaError_t attn_configure() {
  cudaError_t e;
  if ((e = carveout_max(attn_prep_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(attn_chunk_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(attn_combine_kernel)) != cudaSuccess) return e;
  return cudaSuccess;
}

}  // namespace cw
