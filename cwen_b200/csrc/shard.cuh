// Row sharding of the decode step across the GPUs of one node (shard.cu).
#pragma once
#include <cuda_runtime.h>

#include "qgemv.cuh"

namespace cw {

// A cross-GPU barrier waits at most this many SM cycles (~2 s at the maximum
// clock) for another GPU before it reports a timeout.
constexpr long long SHARD_SPIN_CYCLES = 4000000000ll;

struct Shard {
  int rank = 0, world = 1;
  bool configured = false;  // world > 1 (cwen_cuda_shard_config)
  bool opened = false;      // the other GPUs' buffers are mapped (cwen_cuda_shard_open)
  // every GPU's copy (index = rank) of the exchanged buffers and flag arrays
  float *h[QG_MAX_PEERS] = {}, *x[QG_MAX_PEERS] = {}, *lg[QG_MAX_PEERS] = {};
  int *flags[QG_MAX_PEERS] = {};
  int *err = nullptr;
  int epoch = 0;
  bool on() const { return configured && opened; }
};

Shard &shard();
// This GPU's rows [r0, r1) of a matrix of M rows (equal shares in units of align rows).
void shard_rows(int M, int align, int &r0, int &r1);
// Route the next GEMV's output (local buffer `local`, rows row0..) to every GPU's copy.
void shard_target(GemvScratch &s, const float *local, int row0);
void shard_untarget(GemvScratch &s);
// The cross-GPU barrier after a sharded GEMV (no-op without a shard group).
cudaError_t shard_barrier(cudaStream_t st);
int shard_alloc_local();
int shard_status();
void shard_free();

}  // namespace cw
