// GatedDeltaNet verify step -- host interface (gdn.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace cw {

// Rows of one verify block the recurrence kernel holds in shared memory.
constexpr int GDN_MAXB = 16;

struct GdnLayerArgs {
  const float *proj;  // in_proj output rows [B][ps]: qkv | z | alpha | beta
  int ps, B, nkh, nvh;
  int a_off, b_off;        // columns of alpha / beta in a proj row
  const float *convw;      // [QKV][4]
  const float *cstate_in;  // committed conv state [QKV][3]
  float *cstate_out;       // conv state after the block's last row
  float *craw;             // raw (pre-conv) qkv rows [B][QKV], kept for rollback
  const float *A, *dt;     // ssm_a, ssm_dt.bias [nvh]
  float *gin;              // recurrence inputs [B][QKV + 2*nvh]
  const float *S_in;       // committed state [nvh][128][128]
  float *S_out;            // state after the last row
  float *out;              // gated-norm head outputs [B][nvh*128] (the ssm_out GEMV's rows)
  float *delta;            // per-row delta [B][nvh*128], kept for rollback
  const float *z;          // gate rows (z of proj), stride ps
  const float *wn;         // ssm_norm weight [128]
};

// Committed-state view of one GDN layer for the rollback replay.
struct GdnLayerPtrs {
  float *S;             // committed state (updated in place)
  float *cstate;        // committed conv state
  const float *gin;     // block rows
  const float *craw;
  const float *delta;
};

cudaError_t launch_gdn_layer(const GdnLayerArgs &a, cudaStream_t st);
// The same step in one launch (a cluster per key head; gdn_fusable: at most 4
// value heads per key head).  keep < 0: as launch_gdn_layer.  keep >= 0: roll
// the caller's state forward by rows 0..keep-1 in place (S_out == S_in,
// cstate_out == cstate_in), no rollback records.
bool gdn_fusable(int nkh, int nvh);
cudaError_t launch_gdn_fused(const GdnLayerArgs &a, int keep, cudaStream_t st);
// Advance every layer's committed state by block rows 0..k.
cudaError_t launch_gdn_replay(GdnLayerPtrs *dev_layers, int n_layers, int k, int nkh, int nvh, cudaStream_t st);
// The same for one layer given by value.
cudaError_t launch_gdn_replay1(const GdnLayerPtrs &layer, int k, int nkh, int nvh, cudaStream_t st);

// Kernel attributes set once per process (shared-memory carveout).
cudaError_t gdn_configure();
// Frees the scratch of the stand-alone entry point (cwen_cuda_gdn_verify).
void gdn_verify_free();

}  // namespace cw
