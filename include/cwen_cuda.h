/* cwen_cuda.h -- C ABI of the B200 speculative block-verify decode engine.
 *
 * The reference (maci0/cwen, single file run.c) has no FFI: its hot path is a
 * set of static C functions over process globals.  Each entry point below
 * replaces one of them for a C host that keeps the reference's loaders,
 * knobs and drafters; the reference function it stands in for is cited.
 *
 * Conventions (differences from the reference are deliberate):
 *  - every function returns 0 or a negative CWEN_E* code and never exits the
 *    process (the reference calls exit(1) on bad input);
 *    cwen_cuda_last_error() describes the most recent failure;
 *  - the library owns all device memory; one engine per process, driven
 *    from one host thread (the reference is likewise single-threaded and
 *    not re-entrant), bound to one GPU;
 *  - weights arrive in GGUF layout (Q4_0 / Q8_0 / F32) from host memory and
 *    are repacked on the device.
 */
#ifndef CWEN_CUDA_H
#define CWEN_CUDA_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

enum {
  CWEN_OK = 0,
  CWEN_EINVAL = -1,   /* bad argument (the reference: exit(1)/assert) */
  CWEN_ECUDA = -2,    /* CUDA runtime error */
  CWEN_ENOMEM = -3,   /* device allocation failed */
  CWEN_ESTATE = -4,   /* call out of order (no init / model incomplete) */
  CWEN_ERANGE = -5,   /* token id or position out of range */
  CWEN_ETIMEOUT = -6  /* a bounded device wait gave up */
};

/* ggml tensor types accepted by the upload calls (GGUF numbering). */
enum { CWEN_T_F32 = 0, CWEN_T_Q4_0 = 2, CWEN_T_Q8_0 = 8 };

/* Model geometry; the reference fixes it at compile time (run.c:83-91). */
typedef struct {
  int n_embd, n_ff, n_vocab, n_layer;
  int n_head, n_head_kv, head_dim, n_rot;
  int ssm_n_kh, ssm_n_vh, ssm_d, conv_k;
  int full_interval;
  int has_mtp;
} cwen_dims;

/* Description of the last failure (static storage, never NULL). */
const char *cwen_cuda_last_error(void);

/* Select `device`, create the engine's stream and GEMV scratch.  `ctx` is the
 * context window (CWEN_CTX, run.c:4098-4104) and `bmax` the largest verify
 * block (SPEC_BMAX = 16, run.c:192).  Replaces alloc_state (run.c:3928) for
 * the kernel-level scratch.  The verify GEMV of the engine is chosen here,
 * for its lifetime: the warp-level mma.sync kernel (default), or with
 * CWEN_GEMV=tcgen05 in the environment the 5th-generation tensor-core kernel
 * (faster for verify blocks of 9-16 rows, slower for serial decode); weights
 * are repacked for the chosen kernel. */
int cwen_cuda_init(int device, int ctx, int bmax);
/* Free everything (process exit in the reference). */
void cwen_cuda_shutdown(void);
/* Context window the engine was initialised with (0 before init). */
int cwen_cuda_ctx(void);
/* The engine's CUDA stream (a cudaStream_t), for callers that time or order
 * their own work against it. */
void *cwen_cuda_stream(void);

/* ---- stand-alone verify GEMV (gemvb, run.c:1577) ---- */
/* Upload one GGUF Q4_0/Q8_0 matrix (ne0 = K row length, ne1 = M rows) from
 * host memory; returns a handle in *wid. */
int cwen_cuda_weight_upload(int type, const void *host, int ne0, int ne1, int *wid);
/* Y[b*ys + i] = row i of W . X[b*xs ...], b < B <= 16, device pointers,
 * ordered on `stream` (NULL: the engine's stream).  Batch-invariant: column b
 * is bit-identical for every B.  Replaces gemvb (run.c:1577). */
int cwen_cuda_gemvb(int wid, const float *dX, int xs, float *dY, int ys, int B, void *stream);
/* The same with host buffers: copies X in, runs, copies Y out, synchronizes. */
int cwen_cuda_gemvb_host(int wid, const float *hX, int xs, float *hY, int ys, int B);

/* The same GEMV with no allocation at all: its scratch (prepared X, split-K
 * partials, tile counters) is a fixed array of device memory inside the
 * library (about 24 MiB on every GPU that loads it, held until exit) instead
 * of the engine's.  No counterpart in the reference, which has no device
 * memory.  For callers that must not call cudaMalloc while they run -- a
 * framework whose caching allocator already holds the device memory, or a
 * latency-critical loop where cudaMalloc/cudaFree would synchronize the device.
 * Weights come from cwen_cuda_weight_upload at set-up; X and Y are the
 * caller's device buffers.  Limits: K <= 32768, M <= 1,048,576, B <= 16;
 * larger shapes return CWEN_EINVAL.  The first call on a device looks up the
 * array's device address (no allocation); make that first call before any
 * stream capture.  All calls share the one array: calls that overlap on the
 * GPU (different streams, no ordering between them) race and corrupt each
 * other's results.  Runs the kernels cwen_cuda_gemvb runs for the shape, so
 * the output is bit-identical to it.  The call itself does not synchronize:
 * cwen_cuda_gemvb_static_status tells whether a call gave up on a wait. */
int cwen_cuda_gemvb_static(int wid, const float *dX, int xs, float *dY, int ys, int B, void *stream);
/* Synchronize `stream` (NULL: the engine's stream) and report whether any
 * cwen_cuda_gemvb_static call since the last status check gave up on a
 * bounded device wait: CWEN_OK, or CWEN_ETIMEOUT (those calls' outputs are not
 * valid; the flag and the static tile counters are cleared).  No counterpart
 * in the reference; the status half of cwen_cuda_gemvb_host's synchronous
 * check. */
int cwen_cuda_gemvb_static_status(void *stream);

/* ---- stand-alone GatedDeltaNet verify step with rollback ---- */
/* One linear-attention layer over the B <= 16 rows of a verify block, on
 * caller device buffers, ordered on `stream` (NULL: the engine's stream):
 * conv1d_update + SiLU + q/k l2norm (run.c:2183-2200, 2019-2020), the
 * decay/beta transform (run.c:2339-2344), gdn_step with its gated RMSNorm
 * (run.c:2014-2180) for every row; then the committed state is advanced by
 * rows 0..keep-1 only, 0 <= keep <= B (the snap_save / snap_load rollback of
 * a short walk, run.c:2787-2809, 4975-4988).
 *   proj  [B][ps] rows [q nkh*128 | k nkh*128 | v nvh*128 | z nvh*128 |
 *         alpha nvh | beta nvh] (the layer's input projections, pre-conv)
 *   convw [QKV][4] (ssm_conv1d), A / dt [nvh] (ssm_a, ssm_dt.bias),
 *   wn [128] (ssm_norm), QKV = (2 nkh + nvh) * 128
 *   S [nvh][128][128], conv [QKV][3]: the committed state, updated in place
 *   out [B][nvh*128]: the gated-norm head outputs of all B rows
 * Value head h reads key head h % nkh.  The engine keeps one scratch for this
 * call (the state after the block and the rows' rank-1 records, ~3.5 MB at
 * nvh = 48): calls that overlap on the GPU race on it. */
int cwen_cuda_gdn_verify(int nkh, int nvh, int B, const float *proj, int ps, const float *convw, const float *A,
                         const float *dt, const float *wn, float *S, float *conv, int keep, float *out,
                         void *stream);

/* ---- the model ---- */
/* Declare the geometry (run.c:83-91 constants) before any upload. */
int cwen_cuda_model_config(const cwen_dims *dims);
/* The configured geometry (CWEN_ESTATE before cwen_cuda_model_config). */
int cwen_cuda_model_dims(cwen_dims *out);
/* Upload one GGUF tensor by its GGUF name ("token_embd.weight",
 * "blk.<l>.ffn_gate.weight", "blk.<n_layer>.nextn.eh_proj.weight", ...),
 * validating type and shape like rebind_layers_from_tens (run.c:3366-3465).
 * Matrices are repacked on the device (fused where they share an input);
 * names the path does not use are accepted and ignored. */
int cwen_cuda_upload(const char *name, int type, const void *host, int ne0, int ne1);
/* Check every required tensor is bound and allocate the decode state:
 * alloc_state (run.c:3928); KV cache only for the attention layers. */
int cwen_cuda_model_finalize(void);
/* Fresh sequence: zero the GDN/conv state, rewind (reset_state, run.c:4011). */
int cwen_cuda_reset(void);
/* Tokens in the committed state (the reference's pos_n + 1). */
int cwen_cuda_n_past(void);
/* Score toks[0..B) at slots n_past..n_past+B-1 (forward_block, run.c:2752).
 * nlogits in [0,B]: logits + argmax for rows 0..nlogits-1; -1: last row only
 * (the prefill convention of run.c:4850-4854).  The block stays pending until
 * cwen_cuda_commit.  Row j's argmax is compared with toks[j+1] on the device
 * (the greedy walk of run.c:4954-4956). */
int cwen_cuda_forward_block(const int *toks, int B, int nlogits);
/* Result of the fused argmax + greedy walk of the pending block:
 * k = accepted drafts, ustar = bonus token, argmax_out[0..nlogits) (optional).
 * Synchronizes. */
int cwen_cuda_accept(int *k_out, int *ustar_out, int *argmax_out);
/* Keep rows 0..k of the pending block: pointer swap when k is the last row,
 * otherwise a replay of the stored per-row GDN updates (snap_load + replay of
 * run.c:4975-4988 without a second weight sweep). */
int cwen_cuda_commit(int k);
/* One token at slot n_past, committed (forward_ex, run.c:2594); with
 * need_logits the argmax of its logits goes to *argmax_out. */
int cwen_cuda_forward_serial(int token, int need_logits, int *argmax_out);
/* ---- MTP (nextn) drafter, blk.<n_layer> of the GGUF ---- */
/* 1 when the model carries the MTP block (all 15 nextn tensors bound). */
int cwen_cuda_mtp_ready(void);
/* Fold the token committed at slot pos into the nextn stream and park the
 * normed hidden of row `row` of the last forward (its residual stream before
 * output_norm) for slot pos+1.  Call once per committed slot, in order
 * (mtp_commit, run.c:3147-3159). */
int cwen_cuda_mtp_commit(int pos, int token, int row);
/* The same for rows 0..n-1 of the last forward at slots pos0..pos0+n-1
 * (tokens toks[0..n)) in one pass over the nextn weights instead of n: the
 * rows' steps attend causally over the nextn cache, so the result is the bits
 * of n cwen_cuda_mtp_commit calls in order (the prefill and verify-cycle folds
 * of run.c:4830-4849, 4987-4994). */
int cwen_cuda_mtp_commit_block(int pos0, const int *toks, int n);
/* Draft up to max_d tokens after the last committed slot from the pending
 * token `pend`: a chain of nextn steps, each scored by the shared lm_head and
 * argmax'ed on the device; one synchronization at the end.  Returns the
 * number drafted (0 when the stream is not at the last committed slot), or a
 * negative CWEN_E* code (mtp_draft, run.c:3166-3187). */
int cwen_cuda_mtp_draft(int pend, int *out, int max_d);

/* Hidden-state slots of the nextn stream: the predecessor hidden parked by
 * cwen_cuda_mtp_commit (rmsnorm(x_pre, output_norm) of the last committed
 * slot, the reference's NHprev) and two output slots. */
enum { CWEN_MTP_PARKED = 0, CWEN_MTP_OUT0 = 1, CWEN_MTP_OUT1 = 2 };
/* One nextn step (mtp_step, run.c:3099-3131) at stream slot pos (1 <= pos <
 * ctx): input token tok, predecessor hidden from slot src, the
 * shared-head-normed output hidden into slot dst (CWEN_MTP_OUT0/OUT1); writes
 * K/V at pos of the nextn cache, which later steps attend over (slots 1..pos).
 * The parked slot and the stream position of cwen_cuda_mtp_commit are left as
 * they are.  Synchronizes. */
int cwen_cuda_mtp_step(int tok, int pos, int src, int dst);
/* Copy slot `slot`'s hidden (n_embd floats) to host memory. */
int cwen_cuda_mtp_read(int slot, float *host);

/* Copies of device rows for parity checks: logits row (n_vocab floats), the
 * residual stream after the last layer (n_embd), per-layer residual streams
 * (the CWEN_DUMP layerNN files, run.c:2601-2629) while dumps are on, and a
 * GDN layer's committed state [n_vh][128][128] + conv state [qkv][3]. */
int cwen_cuda_logits(int row, float *host);
int cwen_cuda_hidden(int row, float *host);
int cwen_cuda_dump_layers(int on);
int cwen_cuda_dump_read(int layer, int row, float *host);
int cwen_cuda_gdn_state(int layer, float *S_host, float *conv_host);

/* The fused argmax + greedy walk of cwen_cuda_accept on caller device logits:
 * rows b < B (1 <= B <= 16) of n logits at stride ldl; row j's argmax is
 * compared with blk[j+1] for j < E_drafts (0 <= E_drafts < B; blk may be
 * NULL when E_drafts is 0).  res[0] = k (drafts accepted), res[1] = ustar
 * (argmax of row k), res[2..2+B) = the rows' argmaxes.  First maximum, ties to
 * the lowest index, -0.0 equal to +0.0, NaN never replacing the maximum, a NaN
 * at index 0 kept (argmax_of, run.c:2647-2669; the walk, run.c:4954-4959).
 * One kernel launch on `stream` (NULL: the engine's); synchronizes. */
int cwen_cuda_accept_logits(const float *dlogits, int n, int ldl, int B, const int *blk, int E_drafts, int *res,
                            void *stream);

/* ---- row sharding across the GPUs of one node (one engine per GPU) ----
 * The FFN matrices (ffn_gate, ffn_up, ffn_down) and the lm_head (output.weight)
 * are split by output rows, K never split (gemvb rows are independent,
 * run.c:1577-1680; OpenMP over rows at run.c:1588, 1656); the GDN and
 * attention layers, the recurrent state, the KV cache and the MTP block are
 * replicated.  A sharded GEMV writes its rows into every GPU's copy of its
 * output (NVLink stores into buffers opened through CUDA IPC) and a bounded
 * cross-GPU barrier follows it.  Sequence: cwen_cuda_init, cwen_cuda_shard_config,
 * cwen_cuda_model_config, uploads (each GPU keeps its rows), finalize,
 * cwen_cuda_shard_handle on every GPU, exchange the blobs (rank order),
 * cwen_cuda_shard_open; then every GPU runs the same calls.  Output bits do
 * not depend on the batch size for a given group size; they may differ from
 * a single GPU's in fp32 summation order only.  No counterpart in the
 * reference (a CPU program). */
enum { CWEN_SHARD_HANDLE_BYTES = 256 };
int cwen_cuda_shard_config(int rank, int world);
/* This GPU's exchange buffers as a CWEN_SHARD_HANDLE_BYTES blob. */
int cwen_cuda_shard_handle(void *out, int cap);
/* Map the other GPUs' buffers: `handles` holds world blobs in rank order. */
int cwen_cuda_shard_open(const void *handles, int world);
/* The rows [r0, r1) of a matrix of M rows that GPU `rank` of `world` holds
 * (equal shares in units of `align` rows); needs no GPU. */
int cwen_shard_rows(int M, int align, int rank, int world, int *r0, int *r1);
/* The rows [r0, r1) of GGUF tensor `name` (ne1 rows) this GPU keeps: a
 * shard for the FFN matrices and output.weight under a shard group, all rows
 * otherwise (so a loader need only read or generate those). */
int cwen_cuda_shard_rows_for(const char *name, int ne1, int *r0, int *r1);

/* ---- instrumentation (the reference's CWEN_SPEC_DEBUG timers, run.c:3133) ---- */
/* Reset counters and turn per-launch CUDA-event timing of the verify-GEMV
 * kernel on or off (timing adds two event records per GEMV launch). */
int cwen_cuda_profile(int on);
/* Sum of GEMV kernel durations (ms) and of their algorithmic bytes, number of
 * timed GEMV launches, and the number of kernels the engine launched since
 * cwen_cuda_profile(); synchronizes on the recorded events. */
int cwen_cuda_profile_read(double *gemv_ms, double *gemv_bytes, long long *gemv_calls, long long *launches);

#ifdef __cplusplus
}
#endif
#endif
