// Gated GQA attention over the KV cache with partial RoPE (c).
//
// Replaces layer_full_blk's per-row head split, q/k RMSNorm, RoPE and KV
// write (run.c:2714-2737) and attention_heads_kv (run.c:2362-2409).
//
// Split-K decode: the KV range [t0, pos] of a query row is cut into splits of
// S(pos) slots, the smallest power of two >= 32 with pos < 64 * S -- at most
// 64 splits per row, so short contexts spread over many CTAs and long ones
// leave few partials to merge.  One CTA per (kv head, slot range, row group)
// runs an online softmax over its range in 32-slot chunks staged in shared
// memory -- every query row of the group and every q head of the kv group
// against one staged tile, state in registers -- and leaves (max, sum,
// weighted V) per (row, head, split) at each of the row's split boundaries;
// the combine pass merges a row's splits in split order.  Split boundaries
// depend on the row's own position only (a CTA's range is S of the block's
// last row, the largest, and holds whole splits of every smaller S), so a
// row's output does not depend on the other rows of the block.
#include "attn.cuh"
#include "rowprep.cuh"

namespace cw {

constexpr int HD = 256;
constexpr int ACH = 32;     // slots per staged chunk
static_assert(ACH <= 32, "one slot per lane");
constexpr int SPS = 32;     // smallest split (>= ACH: a staged chunk never crosses a split)
constexpr int NSPLIT = 64;  // splits per row at most
CW_HOST_DEV int split_of(int p) {
  int S = SPS;
  while (p >= NSPLIT * S) S *= 2;
  return S;
}
constexpr int KPAD = 260;   // padded K row (floats) in shared memory
constexpr int PART = 4 + HD;
constexpr int IPW = 3;      // (row, head) items per warp
constexpr int MAXIT = 8 * IPW;
// dynamic shared memory of attn_split_kernel: K chunk (padded rows), V chunk, the CTA's queries
constexpr size_t SPLIT_SMEM = (size_t)(ACH * KPAD + ACH * HD + MAXIT * HD) * sizeof(float);

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

// Online-softmax attention of every (row, head of the kv group) over one
// split.  Grid (kv head, split, row group): rows [z*rb, z*rb + rb) of the
// block (rb * G <= MAXIT items; warp w owns items w, w + 8, w + 16).
__global__ void __launch_bounds__(256) attn_split_kernel(const float *__restrict__ qbuf, const float *__restrict__ Kc,
                                                         const float *__restrict__ Vc, int nh, int nkv, int pos0,
                                                         int B, int t0, int nsp_max, int rb, int range,
                                                         float *__restrict__ part) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm[];
  float *Ks = sm;                       // [ACH][KPAD]
  float *Vs = Ks + ACH * KPAD;          // [ACH][HD]
  float *Qs = Vs + ACH * HD;            // [MAXIT][HD]
  const int hkv = blockIdx.x, sp = blockIdx.y;
  const int b0 = blockIdx.z * rb, b1 = min(B, b0 + rb);
  const int G = nh / nkv, nit = (b1 - b0) * G;
  const int last = pos0 + b1 - 1, s0 = sp * range;
  if (s0 > last || s0 + range - 1 < t0) return;  // no row of the group reaches the range (whole CTA)
  const int send = min(s0 + range - 1, last);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < nit * HD; i += blockDim.x) {
    const int it = i / HD, d = i % HD;
    Qs[i] = qbuf[((size_t)(b0 + it / G) * nh + hkv * G + it % G) * HD + d];
  }
  float m[IPW], l[IPW], acc[IPW][8];
#pragma unroll
  for (int j = 0; j < IPW; j++) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) acc[j][i] = 0.f;
  }
  const float scale = 1.f / sqrtf((float)HD);
  for (int c0 = s0; c0 <= send; c0 += ACH) {
    __syncthreads();  // the previous chunk's reads (and the q stores) are done
    for (int i = threadIdx.x; i < ACH * (HD / 4); i += blockDim.x) {
      const int t = i / (HD / 4), d4 = (i % (HD / 4)) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (c0 + t <= send) {
        kv = *reinterpret_cast<const float4 *>(Kc + ((size_t)(c0 + t) * nkv + hkv) * HD + d4);
        vv = *reinterpret_cast<const float4 *>(Vc + ((size_t)(c0 + t) * nkv + hkv) * HD + d4);
      }
      *reinterpret_cast<float4 *>(Ks + t * KPAD + d4) = kv;
      *reinterpret_cast<float4 *>(Vs + t * HD + d4) = vv;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < IPW; j++) {
      const int it = warp + 8 * j;
      if (it >= nit) break;
      const int p = pos0 + b0 + it / G;
      if (c0 > p || c0 + ACH - 1 < t0) continue;  // warp-uniform: no slot of the chunk for this row
      const float *q = Qs + it * HD;
      const float *kr = Ks + lane * KPAD;
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
      const int tt = c0 + lane;
      const float sc = (tt >= t0 && tt <= p) ? ((a0 + a1) + (a2 + a3)) * scale : -INFINITY;
      const float mn = fmaxf(m[j], warp_max(sc));  // finite: the chunk holds a slot of the row
      const float corr = m[j] == -INFINITY ? 0.f : expf(m[j] - mn);
      const float e = sc == -INFINITY ? 0.f : expf(sc - mn);
      l[j] = fmaf(l[j], corr, warp_sum(e));
      m[j] = mn;
#pragma unroll
      for (int i = 0; i < 8; i++) acc[j][i] *= corr;
      for (int t = 0; t < ACH; t++) {
        const float pt = __shfl_sync(0xffffffffu, e, t);
        const float4 v0 = *reinterpret_cast<const float4 *>(Vs + t * HD + lane * 8);
        const float4 v1 = *reinterpret_cast<const float4 *>(Vs + t * HD + lane * 8 + 4);
        acc[j][0] = fmaf(pt, v0.x, acc[j][0]);
        acc[j][1] = fmaf(pt, v0.y, acc[j][1]);
        acc[j][2] = fmaf(pt, v0.z, acc[j][2]);
        acc[j][3] = fmaf(pt, v0.w, acc[j][3]);
        acc[j][4] = fmaf(pt, v1.x, acc[j][4]);
        acc[j][5] = fmaf(pt, v1.y, acc[j][5]);
        acc[j][6] = fmaf(pt, v1.z, acc[j][6]);
        acc[j][7] = fmaf(pt, v1.w, acc[j][7]);
      }
    }
    // the end of a row's split (or of this CTA's range): leave its partial
#pragma unroll
    for (int j = 0; j < IPW; j++) {
      const int it = warp + 8 * j;
      if (it >= nit) break;
      const int b = b0 + it / G, S = split_of(pos0 + b);
      if ((c0 + ACH) % S != 0 && c0 + ACH <= send) continue;
      if (m[j] != -INFINITY) {  // the split held a slot of the row
        float *o = part + (((size_t)b * nh + hkv * G + it % G) * nsp_max + c0 / S) * PART;
        if (lane == 0) {
          o[0] = m[j];
          o[1] = l[j];
        }
        *reinterpret_cast<float4 *>(o + 4 + lane * 8) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
        *reinterpret_cast<float4 *>(o + 4 + lane * 8 + 4) = make_float4(acc[j][4], acc[j][5], acc[j][6], acc[j][7]);
      }
      m[j] = -INFINITY;
      l[j] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i++) acc[j][i] = 0.f;
    }
  }
}

// Merge the splits of each (row, head) and apply the sigmoid gate
// (run.c:2396-2406): o = (sum_s w_s a_s) / (sum_s w_s l_s) * sigmoid(gate),
// w_s = exp(m_s - M), splits in order.  One CTA per (head, row), one thread
// per dimension; the rows go to the wo GEMV as raw fp32 (local X).
constexpr int COMB_THREADS = HD;
__global__ void __launch_bounds__(COMB_THREADS) attn_combine_kernel(const float *__restrict__ part,
                                                                   const float *__restrict__ proj, int ps, int nh,
                                                                   int pos0, int t0, int nsp_max,
                                                                   float *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float wts[];  // [nsp_max]
  __shared__ float lsum;
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int p = pos0 + b, S = split_of(p), sf = t0 / S, sl = p / S, ns = sl - sf + 1;
  const float *ph = part + ((size_t)b * nh + h) * nsp_max * PART;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float M = -INFINITY;
    for (int s = sf + lane; s <= sl; s += 32) M = fmaxf(M, ph[(size_t)s * PART]);
    M = warp_max(M);
    float l = 0.f;
    for (int s = sf + lane; s <= sl; s += 32) {
      const float w = expf(ph[(size_t)s * PART] - M);
      wts[s - sf] = w;
      l = fmaf(ph[(size_t)s * PART + 1], w, l);
    }
    l = warp_sum(l);
    if (lane == 0) lsum = l;
  }
  __syncthreads();
  const float *pd = ph + (size_t)sf * PART + 4 + d;
  float a = 0.f;
#pragma unroll 8
  for (int s = 0; s < ns; s++) a = fmaf(pd[(size_t)s * PART], wts[s], a);
  out[(size_t)b * nh * HD + h * HD + d] = (a / lsum) * sigmoid_dev(proj[(size_t)b * ps + h * 2 * HD + HD + d]);
}

cudaError_t launch_attention(const AttnArgs &a, GemvScratch &s, cudaStream_t st) {
  CW_TRY(launch_pdl(attn_prep_kernel, dim3(a.nh + 2 * a.nkv, a.B), HD, 0, st, a.proj, a.ps, a.nh, a.nkv, a.qn, a.kn, a.rope, a.pos0,
                                                               a.qbuf, a.Kc, a.Vc));
  const int last = a.pos0 + a.B - 1;
  const int range = split_of(last);  // a CTA's slot range: the block's largest split
  const int nsp = last / range + 1;
  const int G = a.nh / a.nkv;
  if (a.nch_max < NSPLIT || G > MAXIT || !a.out) return cudaErrorInvalidValue;
  const size_t smem = SPLIT_SMEM;
  // Rows per CTA: split the block's rows over more CTAs only while the
  // (kv head, split) grid alone is short of two CTAs per SM -- each extra row
  // group stages the split's K/V again, which long contexts cannot afford --
  // and at most MAXIT (row, head) items per CTA.
  const int n_sm = s.G > 0 ? s.G : 148;  // the GEMV grid: one CTA per SM
  const int base = a.nkv * nsp;
  const int min_rb = G >= 8 ? 1 : 8 / G;  // about one (row, head) item per warp
  const int max_rb = MAXIT / G;
  int groups = (2 * n_sm + base - 1) / base;
  const int max_groups = (a.B + min_rb - 1) / min_rb;
  groups = groups < 1 ? 1 : (groups > max_groups ? max_groups : groups);
  int rb = (a.B + groups - 1) / groups;
  if (rb > max_rb) rb = max_rb;
  CW_TRY(launch_pdl(attn_split_kernel, dim3(a.nkv, nsp, (a.B + rb - 1) / rb), 256, smem, st, a.qbuf, a.Kc, a.Vc,
                    a.nh, a.nkv, a.pos0, a.B, a.t0, a.nch_max, rb, range, a.part));
  CW_TRY(launch_pdl(attn_combine_kernel, dim3(a.nh, a.B), COMB_THREADS, (size_t)a.nch_max * sizeof(float), st, a.part,
                    a.proj, a.ps, a.nh, a.pos0, a.t0, a.nch_max, a.out));
  return cudaGetLastError();
}

// Partial slots per (row, head): at most NSPLIT splits per row.
int attn_splits_max(int ctx) {
  (void)ctx;
  return NSPLIT;
}
size_t attn_part_floats(int bmax, int nh, int nch_max) { return (size_t)bmax * nh * nch_max * PART; }

// One-time kernel attributes (called at engine set-up).
cudaError_t attn_configure() {
  cudaError_t e;
  if ((e = carveout_max(attn_prep_kernel)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SPLIT_SMEM)) !=
      cudaSuccess)
    return e;
  if ((e = carveout_max(attn_split_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(attn_combine_kernel)) != cudaSuccess) return e;
  return cudaSuccess;
}

}  // namespace cw
