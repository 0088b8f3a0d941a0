// Row sharding of the decode step across the GPUs of one node (one engine,
// one process per GPU).
//
// The FFN matrices (ffn_gate/ffn_up, ffn_down) and the lm_head are split by
// output rows -- the reference's gemvb rows are independent (run.c:1577-1680,
// OpenMP over output rows at run.c:1588, 1656) -- and K is never split, so
// every output element is computed whole on one GPU.  Everything else (the
// GDN and attention projections, the recurrent state, the KV cache, the MTP
// block) is replicated and computes the same bits on every GPU.  A sharded
// GEMV stores its rows straight into every GPU's copy of the output buffer
// (NVLink stores into buffers opened through CUDA IPC), then a barrier kernel
// signals the other GPUs and waits until they have all signalled the same
// epoch: after it, every copy holds the full output.  Three buffers are
// exchanged this way: the SwiGLU rows h (gate_up), the residual stream x
// (ffn_down adds its rows onto it) and the logits (lm_head).
#include <stdio.h>
#include <string.h>

#include "common.cuh"
#include "engine.cuh"
#include "model.cuh"
#include "shard.cuh"

namespace cw {

static Shard g_shard;
Shard &shard() { return g_shard; }

// One thread: release this GPU's writes system-wide, store the epoch into
// slot `rank` of every GPU's flag array, then wait (bounded) until every
// other GPU has stored the epoch into this GPU's array.  On a timeout the
// error flag is set and the kernel returns; the host reports CWEN_ETIMEOUT.
struct FlagPtrs {
  int *f[QG_MAX_PEERS];
};
__global__ void xrank_barrier_kernel(FlagPtrs peers, int *local, int rank, int world, int epoch, int *err) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x != 0) return;
  __threadfence_system();
  for (int p = 0; p < world; p++) {
    if (p == rank) continue;
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(peers.f[p] + rank), "r"(epoch) : "memory");
  }
  const long long t0 = clock64();
  for (int q = 0; q < world; q++) {
    if (q == rank) continue;
    for (;;) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(local + q) : "memory");
      if (v - epoch >= 0) break;  // epochs only grow (wrap-safe difference)
      if (clock64() - t0 > SHARD_SPIN_CYCLES) {
        atomicExch(err, 1);
        return;
      }
    }
  }
}

cudaError_t shard_barrier(cudaStream_t st) {
  Shard &S = g_shard;
  if (!S.on()) return cudaSuccess;
  FlagPtrs fp;
  for (int p = 0; p < QG_MAX_PEERS; p++) fp.f[p] = p < S.world ? S.flags[p] : nullptr;
  S.epoch++;
  engine().prof.launches++;
  return launch_pdl(xrank_barrier_kernel, 1, 32, 0, st, fp, S.flags[S.rank], S.rank, S.world, S.epoch, S.err);
}

// The shard of rows [r0, r1) of a matrix of M rows held by this GPU: equal
// contiguous shares, multiples of `align` rows.
static void rows_of(int M, int align, int rank, int world, int &r0, int &r1) {
  const int units = (M + align - 1) / align;
  const int u0 = (int)((long long)units * rank / world), u1 = (int)((long long)units * (rank + 1) / world);
  r0 = u0 * align < M ? u0 * align : M;
  r1 = u1 * align < M ? u1 * align : M;
}
void shard_rows(int M, int align, int &r0, int &r1) {
  Shard &S = g_shard;
  if (!S.configured) {
    r0 = 0;
    r1 = M;
    return;
  }
  rows_of(M, align, S.rank, S.world, r0, r1);
}

// Point the GEMV launch that follows at every GPU's copy of `local` (one of
// the exchanged buffers) as rows row0.. of the full output.
void shard_target(GemvScratch &s, const float *local, int row0) {
  Shard &S = g_shard;
  Model &M = model();
  float *const *peers = local == M.h ? S.h : (local == M.x ? S.x : S.lg);
  s.np = S.world;
  s.row0 = row0;
  for (int p = 0; p < S.world; p++) s.yp[p] = peers[p];
}
void shard_untarget(GemvScratch &s) {
  s.np = 0;
  s.row0 = 0;
}

void shard_free() {
  Shard &S = g_shard;
  for (int p = 0; p < S.world; p++) {
    if (p == S.rank || !S.opened) continue;
    if (S.h[p]) cudaIpcCloseMemHandle(S.h[p]);
    if (S.x[p]) cudaIpcCloseMemHandle(S.x[p]);
    if (S.lg[p]) cudaIpcCloseMemHandle(S.lg[p]);
    if (S.flags[p]) cudaIpcCloseMemHandle(S.flags[p]);
  }
  if (S.flags[S.rank]) cudaFree(S.flags[S.rank]);
  if (S.err) cudaFree(S.err);
  S = Shard();
}

// Buffers of this GPU (after cwen_cuda_model_finalize): the local copies.
int shard_alloc_local() {
  Shard &S = g_shard;
  Model &M = model();
  if (!S.configured) return CWEN_OK;
  S.h[S.rank] = M.h;
  S.x[S.rank] = M.x;
  S.lg[S.rank] = M.logits;
  CW_CHECK(cudaMalloc(&S.flags[S.rank], 64 * sizeof(int)));
  CW_CHECK(cudaMemset(S.flags[S.rank], 0, 64 * sizeof(int)));
  CW_CHECK(cudaMalloc(&S.err, sizeof(int)));
  CW_CHECK(cudaMemset(S.err, 0, sizeof(int)));
  return CWEN_OK;
}

int shard_status() {
  Shard &S = g_shard;
  if (!S.on()) return CWEN_OK;
  int e = 0;
  CW_CHECK(cudaMemcpy(&e, S.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (!e) return CWEN_OK;
  set_error("row-sharded decode: a cross-GPU barrier gave up waiting for another GPU");
  return CWEN_ETIMEOUT;
}

}  // namespace cw

using namespace cw;

extern "C" {

int cwen_cuda_shard_config(int rank, int world) {
  Shard &S = shard();
  if (!engine().live || model().configured) {
    set_error("cwen_cuda_shard_config: call after cwen_cuda_init and before cwen_cuda_model_config");
    return CWEN_ESTATE;
  }
  if (world < 1 || world > QG_MAX_PEERS || rank < 0 || rank >= world) {
    set_error("cwen_cuda_shard_config: need 1 <= world <= %d and 0 <= rank < world", QG_MAX_PEERS);
    return CWEN_EINVAL;
  }
  S = Shard();
  S.rank = rank;
  S.world = world;
  S.configured = world > 1;
  return CWEN_OK;
}

int cwen_cuda_shard_handle(void *out, int cap) {
  Shard &S = shard();
  if (!S.configured || !model().finalized || !S.flags[S.rank]) {
    set_error("cwen_cuda_shard_handle: no shard group configured, or the model is not finalised");
    return CWEN_ESTATE;
  }
  if (!out || cap < CWEN_SHARD_HANDLE_BYTES) {
    set_error("cwen_cuda_shard_handle: need %d bytes", CWEN_SHARD_HANDLE_BYTES);
    return CWEN_EINVAL;
  }
  cudaIpcMemHandle_t h[4];
  CW_CHECK(cudaIpcGetMemHandle(&h[0], S.h[S.rank]));
  CW_CHECK(cudaIpcGetMemHandle(&h[1], S.x[S.rank]));
  CW_CHECK(cudaIpcGetMemHandle(&h[2], S.lg[S.rank]));
  CW_CHECK(cudaIpcGetMemHandle(&h[3], S.flags[S.rank]));
  memcpy(out, h, sizeof h);
  return CWEN_OK;
}

int cwen_cuda_shard_open(const void *handles, int world) {
  Shard &S = shard();
  if (!S.configured || !model().finalized || S.opened || world != S.world || !handles) {
    set_error("cwen_cuda_shard_open: need the %d handles of the configured group, once, after finalize", S.world);
    return CWEN_ESTATE;
  }
  const uint8_t *all = (const uint8_t *)handles;
  for (int p = 0; p < S.world; p++) {
    if (p == S.rank) continue;
    cudaIpcMemHandle_t h[4];
    memcpy(h, all + (size_t)p * CWEN_SHARD_HANDLE_BYTES, sizeof h);
    void *ptr[4] = {};
    for (int i = 0; i < 4; i++) CW_CHECK(cudaIpcOpenMemHandle(&ptr[i], h[i], cudaIpcMemLazyEnablePeerAccess));
    S.h[p] = (float *)ptr[0];
    S.x[p] = (float *)ptr[1];
    S.lg[p] = (float *)ptr[2];
    S.flags[p] = (int *)ptr[3];
  }
  S.opened = true;
  return CWEN_OK;
}

int cwen_cuda_shard_rows_for(const char *name, int ne1, int *r0, int *r1) {
  if (!name || !r0 || !r1 || ne1 < 0) {
    set_error("cwen_cuda_shard_rows_for: need a name, ne1 >= 0 and two outputs");
    return CWEN_EINVAL;
  }
  *r0 = 0;
  *r1 = ne1;
  if (!shard().configured || !model().configured) return CWEN_OK;
  int l = -1, n = 0;
  const bool ffn = sscanf(name, "blk.%d.%n", &l, &n) == 1 && n > 0 && l >= 0 && l < model().d.n_layer &&
                   (!strcmp(name + n, "ffn_gate.weight") || !strcmp(name + n, "ffn_up.weight") ||
                    !strcmp(name + n, "ffn_down.weight"));
  if (ffn || !strcmp(name, "output.weight")) shard_rows(ne1, 16, *r0, *r1);
  return CWEN_OK;
}

int cwen_shard_rows(int M, int align, int rank, int world, int *r0, int *r1) {
  if (M < 0 || align < 1 || world < 1 || rank < 0 || rank >= world || !r0 || !r1) {
    set_error("cwen_shard_rows: need M >= 0, align >= 1, 0 <= rank < world");
    return CWEN_EINVAL;
  }
  rows_of(M, align, rank, world, *r0, *r1);
  return CWEN_OK;
}

}  // extern "C"
