// Row-wise kernels of the forward pass: embedding, RMSNorm -> GEMV input,
// gated GDN norm -> GEMV input, generic row -> GEMV input, argmax.
#include "rowops.cuh"
#include "rowprep.cuh"

namespace cw {

// Layout selector of the X operands for the engine's GEMV kernel: 0 for the
// tcgen05 kernel, else the n-tile count of the mma.sync kernel.
static int xops_nt(const GemvScratch &s, int B) { return s.kern == GK_TC ? 0 : (B + 3) / 4; }

// Dynamic shared memory above the 48 KB default needs an explicit opt-in.
template <typename F>
static cudaError_t smem_optin(F *fn, size_t bytes, size_t &done) {
  if (bytes <= 48 * 1024 || bytes <= done) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) done = bytes;
  return e;
}

// ---- embedding (embed_token_to, Q4_0 branch run.c:1873-1881) ----
// x[b][k] = d * (q - 8) of row toks[b] of token_embd (GGUF Q4_0 layout).
// The token ids come from `toks` or, when dtok is set, from device memory
// (a drafted token produced by an earlier kernel).
__global__ void embed_kernel(const uint8_t *__restrict__ emb, int H, int V, const Toks16 toks, const int *dtok,
                             int B, float *__restrict__ x, int *__restrict__ err) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.y;
  const int tok = dtok ? dtok[b] : toks.t[b];
  if (tok < 0 || tok >= V) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(err, 1);
    return;
  }
  const int nb = H / 32;
  const uint8_t *row = emb + (size_t)tok * nb * 18;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nb * 16; i += gridDim.x * blockDim.x) {
    const int blk = i >> 4, j = i & 15;
    const uint8_t *p = row + blk * 18;
    const float d = __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
    const uint8_t q = p[2 + j];
    x[(size_t)b * H + blk * 32 + j] = (float)((q & 0xF) - 8) * d;
    x[(size_t)b * H + blk * 32 + j + 16] = (float)((q >> 4) - 8) * d;
  }
}

cudaError_t launch_embed(const uint8_t *emb, int H, int V, const Toks16 &toks, int B, float *x, int *err,
                         cudaStream_t st, const int *dtok) {
  CW_TRY(launch_pdl(embed_kernel, dim3(4, B), 256, 0, st, emb, H, V, toks, dtok, B, x, err));
  return cudaGetLastError();
}

// ---- MTP input: [rmsnorm(e, enorm) | rmsnorm(h, hnorm)] -> GEMV input (run.c:3100-3102) ----
// One CTA per row b < B (column b; padding columns are not read into any
// live result: a GEMV column depends only on its own X column).
__global__ void __launch_bounds__(PREP_THREADS) cat_norm_prep_kernel(const float *__restrict__ e,
                                                                     const float *__restrict__ h,
                                                                     const float *__restrict__ we,
                                                                     const float *__restrict__ wh, int H, int mma_nt,
                                                                     uint4 *__restrict__ xf, int *__restrict__ xexp,
                                                                     float *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float v[];
  __shared__ float red[32];
  const int b = blockIdx.x;
  e += (size_t)b * H;
  h += (size_t)b * H;
  float se = 0.f, sh = 0.f;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float a = e[k], c = h[k];
    v[k] = a;
    v[H + k] = c;
    se = fmaf(a, a, se);
    sh = fmaf(c, c, sh);
  }
  se = block_sum(se, red);
  sh = block_sum(sh, red);
  const float re = 1.f / sqrtf(se / (float)H + 1e-6f), rh = 1.f / sqrtf(sh / (float)H + 1e-6f);
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    v[k] = we[k] * v[k] * re;
    v[H + k] = wh[k] * v[H + k] * rh;
  }
  __syncthreads();
  if (out) {  // the concatenated rows for a GEMV kernel that takes raw X
    for (int k = threadIdx.x; k < 2 * H; k += blockDim.x) out[(size_t)b * 2 * H + k] = v[k];
    return;
  }
  emit_xfrag(v, 2 * H, b, mma_nt, xf, xexp, red, true);
}

cudaError_t launch_cat_norm_prep(const float *e, const float *h, const float *we, const float *wh, int H, int B,
                                 GemvScratch &s, cudaStream_t st, float *out) {
  const size_t smem = (size_t)2 * H * sizeof(float);
  static size_t done = 0;
  cudaError_t err = smem_optin(cat_norm_prep_kernel, smem, done);
  if (err != cudaSuccess) return err;
  CW_TRY(launch_pdl(cat_norm_prep_kernel, B, PREP_THREADS, smem, st, e, h, we, wh, H, xops_nt(s, B), s.xf, s.xexp, out));
  return cudaGetLastError();
}

// Row kernels below run one thread-block cluster of CL CTAs per row (blockIdx.y
// = row b < B, cluster rank = blockIdx.x): each CTA owns a contiguous slice of
// the row; row-wide sums and maxima go through distributed shared memory in
// cluster-rank order (deterministic, independent of B), and each CTA emits the
// GEMV fragments of its own slice.  Only live rows run: a GEMV column depends
// only on its own X column, so stale padding columns are never read into a
// live result.
constexpr int ROW_THREADS = 256;

// ---- RMSNorm (run.c:346) fused with GEMV input preparation ----
// Optional copy of the normed row to `out`.
__global__ void __launch_bounds__(ROW_THREADS) norm_prep_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                                int H, int mma_nt, uint4 *__restrict__ xf,
                                                                int *__restrict__ xexp, float *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float v[];
  __shared__ float red[64];
  __shared__ float2 slot;
  const int b = blockIdx.y, r = blockIdx.x, n = H / gridDim.x, k0 = r * n;
  // one pass: sum x^2 and max |w x|; one cluster exchange for both.
  // max |(w x) s| = max |w x| * s exactly: s > 0 and rounding is monotonic.
  float ss = 0.f, m = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float t = x[(size_t)b * H + k0 + i];
    const float wt = w[k0 + i] * t;
    v[i] = wt;
    ss = fmaf(t, t, ss);
    m = fmaxf(m, fabsf(wt));
  }
  const float2 sm = cluster_reduce_sum_max(block_sum_max(ss, m, red), &slot);
  const float s = 1.f / sqrtf(sm.x / (float)H + 1e-6f);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float o = v[i] * s;  // (w x) s, the reference's order
    v[i] = o;
    if (out) out[(size_t)b * H + k0 + i] = o;
  }
  __syncthreads();
  const int e = xfrag_exponent(sm.y * s);
  if (r == 0 && threadIdx.x == 0) xexp[b] = e;
  emit_xops(v, k0 / 32, n / 32, b, mma_nt, xf, __int_as_float((127 + e) << 23), true);
}

cudaError_t launch_norm_prep(const float *x, const float *w, int H, int B, GemvScratch &s, float *out,
                             cudaStream_t st) {
  const int cl = cluster_split(H / 32);
  CW_TRY(launch_pdl_cluster(norm_prep_kernel, dim3(cl, B), ROW_THREADS, (size_t)(H / cl) * sizeof(float), st, cl, x, w,
                            H, xops_nt(s, B), s.xf, s.xexp, out));
  return cudaGetLastError();
}

// ---- plain row -> GEMV input (e.g. the SwiGLU output feeding ffn_down) ----
__global__ void __launch_bounds__(ROW_THREADS) row_prep_kernel(const float *__restrict__ x, int xs, int K, int mma_nt,
                                                               uint4 *__restrict__ xf, int *__restrict__ xexp) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float v[];
  __shared__ float red[32], slot;
  const int b = blockIdx.y, r = blockIdx.x, n = K / gridDim.x, k0 = r * n;
  float mx = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float t = x[(size_t)b * xs + k0 + i];
    v[i] = t;
    mx = fmaxf(mx, fabsf(t));
  }
  mx = cluster_reduce<true>(block_max(mx, red), &slot);
  const int e = xfrag_exponent(mx);
  if (r == 0 && threadIdx.x == 0) xexp[b] = e;
  emit_xops(v, k0 / 32, n / 32, b, mma_nt, xf, __int_as_float((127 + e) << 23), true);
}

cudaError_t launch_row_prep(const float *x, int xs, int K, int B, GemvScratch &s, cudaStream_t st) {
  const int cl = cluster_split(K / 32);
  CW_TRY(launch_pdl_cluster(row_prep_kernel, dim3(cl, B), ROW_THREADS, (size_t)(K / cl) * sizeof(float), st, cl, x, xs,
                            K, xops_nt(s, B), s.xf, s.xexp));
  return cudaGetLastError();
}

// ---- argmax (argmax_of run.c:2647) + greedy walk (run.c:4954-4959), one launch ----
// Packed key: order-preserving float bits in the high word, ~index in the low
// word, so a 64-bit max picks the largest value and, among equal values, the
// lowest index -- independent of the order CTAs finish.  The reference scans
// with a strict `>` from bv = lg[0]: -0.0 and +0.0 compare equal (canonicalised
// to +0.0 here, so the lower index wins), a NaN never replaces the running
// maximum (a NaN at index i > 0 is skipped: key of -inf), and a NaN at index 0
// is never replaced, so the answer is 0 (top key).
CW_DEV unsigned long long argmax_key(float v, int i) {
  if (v != v) return i == 0 ? ~0ull : 0ull;
  if (v == 0.f) v = 0.f;  // -0.0 -> +0.0
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (uint32_t)(~(uint32_t)i);
}

constexpr int AW_THREADS = 256;
constexpr int AW_CTAS = 64;  // CTAs per logits row

// Grid (AW_CTAS, B): each CTA reduces a strided slice of row b to one key and
// parks it in part[b][cta]; the last CTA to arrive (arrival counter, reset by
// that CTA) reduces every row's parked keys and walks the block:
//   k = longest prefix with argmax(row j) == blk[j+1] (j < E), ustar = argmax(row k)
//   res = [k, ustar, argmax(row 0..B-1)].
__global__ void __launch_bounds__(AW_THREADS) argmax_walk_kernel(const float *__restrict__ lg, int n, int ldl, int E,
                                                                 const Toks16 blk, unsigned long long *__restrict__ part,
                                                                 unsigned int *__restrict__ count, int *__restrict__ res) {
  pdl_trigger();
  pdl_wait();
  __shared__ unsigned long long red[AW_THREADS / 32];
  __shared__ int am[16];
  __shared__ bool last;
  const int b = blockIdx.y, B = gridDim.y, nb = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned long long k = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long kk = argmax_key(lg[(size_t)b * ldl + i], i);
    k = kk > k ? kk : k;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, k, o);
    k = t > k ? t : k;
  }
  if (lane == 0) red[warp] = k;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < AW_THREADS / 32; w++) k = red[w] > k ? red[w] : k;
    part[b * nb + blockIdx.x] = k;
    __threadfence();  // the parked key before the arrival
    last = atomicAdd(count, 1u) == (unsigned)(nb * B - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();  // every other CTA's parked key, after its arrival
  for (int r = warp; r < B; r += AW_THREADS / 32) {
    unsigned long long m = 0;
    for (int c = lane; c < nb; c += 32) {
      const unsigned long long t = __ldcg(part + r * nb + c);
      m = t > m ? t : m;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, m, o);
      m = t > m ? t : m;
    }
    if (lane == 0) am[r] = (int)(~(uint32_t)(m & 0xffffffffu));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int kk = 0;
    while (kk < E && am[kk] == blk.t[kk + 1]) kk++;
    res[0] = kk;
    res[1] = am[kk];
    for (int r = 0; r < B; r++) res[2 + r] = am[r];
    *count = 0u;  // ready for the next launch (launches on a stream are ordered)
  }
}

size_t argmax_part_bytes(int bmax) { return (size_t)bmax * AW_CTAS * sizeof(unsigned long long) + 256; }

cudaError_t launch_argmax_walk(const float *lg, int n, int ldl, int B, int E, const Toks16 &blk, void *scratch,
                               int *res, cudaStream_t st) {
  if (B < 1 || B > 16 || E < 0 || E >= B) return cudaErrorInvalidValue;
  auto *count = reinterpret_cast<unsigned int *>(scratch);  // first 256 bytes: the arrival counter
  auto *part = reinterpret_cast<unsigned long long *>(static_cast<char *>(scratch) + 256);
  CW_TRY(launch_pdl(argmax_walk_kernel, dim3(AW_CTAS, B), AW_THREADS, 0, st, lg, n, ldl, E, blk, part, count, res));
  return cudaGetLastError();
}

// One-time kernel attributes (called at engine set-up).
cudaError_t rowops_configure() {
  cudaError_t e;
  if ((e = carveout_max(embed_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(norm_prep_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(row_prep_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(argmax_walk_kernel)) != cudaSuccess) return e;
  if ((e = carveout_max(cat_norm_prep_kernel)) != cudaSuccess) return e;
  return cudaSuccess;
}

}  // namespace cw
