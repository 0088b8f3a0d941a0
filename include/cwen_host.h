/* cwen_host.h -- the C host side kept from the reference (maci0/cwen run.c):
 * model loading (GGUF, or the seeded synthetic model), the n-gram drafter,
 * and the serial / speculative decode drivers.  They run on the CPU and call
 * the GPU engine only through include/cwen_cuda.h.
 */
#ifndef CWEN_HOST_H
#define CWEN_HOST_H
#include <stdint.h>

#include "cwen_cuda.h"
#ifdef __cplusplus
extern "C" {
#endif

/* ---- loading ---- */
/* Parse a GGUF v2/v3 file (bounds-checked like load_gguf, run.c:3230-3303),
 * derive the geometry from the tensor shapes, upload every tensor and
 * finalize.  The engine must be initialised (cwen_cuda_init).  Q4_0 tensors
 * that the file's CWENR sidecar binds (load_cwenr, run.c:3305-3643: v2
 * packed, v3 split, v4 split + interleaved pairs; path from CWEN_REPACK, else
 * MODEL.gguf -> MODEL.cwenr) are uploaded from the sidecar's bytes; a
 * missing, stale or malformed sidecar is ignored with a note on stderr, as
 * the reference does. */
int cwen_load_gguf(const char *path);
/* The bytes cwen_load_gguf uploads for tensor `name` of the GGUF at `path`
 * (GGUF block layout: f32 rows, or 18-byte Q4_0 / 34-byte Q8_0 blocks): from
 * its CWENR sidecar when one binds the tensor, else from the GGUF.  Writes
 * them to out (when out is non-NULL and cap is large enough), sets
 * *from_sidecar (when non-NULL), and returns the byte count, or a negative
 * CWEN_E* code.  No GPU needed. */
int cwen_gguf_tensor_bytes(const char *path, const char *name, void *out, size_t cap, int *from_sidecar);
/* The geometry cwen_load_gguf would derive from the file's tensor shapes,
 * with the same parse and bounds checks, without touching the engine (no
 * GPU needed).  CWEN_EINVAL with the reason in cwen_cuda_last_error() for a
 * malformed file. */
int cwen_gguf_dims(const char *path, cwen_dims *out);
/* The seeded random-init model of the benchmark configurations: every tensor
 * generated on the host (`threads` threads, <= 0: all cores) and uploaded. */
int cwen_load_synth(uint64_t seed, const cwen_dims *dims, int threads);
/* Write that seeded model as a GGUF v3 file (the reference's tensor names,
 * shapes and types; 32-byte aligned data) that cwen_load_gguf and the
 * reference's own loader (load_gguf, run.c:3230) read back to the same bytes
 * cwen_load_synth uploads.  No GPU needed. */
int cwen_write_synth_gguf(const char *path, const cwen_dims *dims, uint64_t seed, int threads);
/* Geometry of the reference (run.c:83-91) and the small test geometry. */
void cwen_dims_reference(cwen_dims *d);
void cwen_dims_small(cwen_dims *d);

/* ---- speculation knobs (spec_config_init, run.c:4021-4053) ---- */
typedef struct {
  int spec;       /* CWEN_SPEC: block speculation on */
  int use_mtp;    /* CWEN_MTP: draft with the blk.<L> nextn head when present */
  int max_draft;  /* CWEN_SPEC_MAX_DRAFT / -d: drafts per block, 1..15 */
  int min_draft;  /* CWEN_SPEC_MIN_DRAFT: smaller proposals run a plain step */
  int n_key;      /* CWEN_SPEC_NGRAM_N: n-gram key length, 2..256 */
  int cooldown;   /* CWEN_SPEC_COOLDOWN: plain steps after 3 short walks */
  int debug;      /* CWEN_SPEC_DEBUG: per-cycle trace on stderr */
} cwen_spec_cfg;
/* (CWEN_NGRAM_CACHE=FILE, read by cwen_generate itself: the n-gram map of a
 * speculative run is loaded from FILE before the prompt and saved after.) */
void cwen_spec_defaults(cwen_spec_cfg *c);
/* Apply the CWEN_SPEC* / CWEN_MTP environment with the reference's strict
 * parsing; returns CWEN_EINVAL (message in cwen_cuda_last_error) on a bad
 * value instead of exiting. */
int cwen_spec_from_env(cwen_spec_cfg *c);

typedef struct {
  long long cycles, drafted, full, shortw, kept;  /* the "spec:" stats line */
  long long plain_steps;
} cwen_spec_stats;

/* Prefill tokens[0..n_tok) and greedily generate up to n_gen ids into out
 * (generate_tokens run.c:5027 / generate_tokens_spec run.c:4882).  Returns the
 * number emitted (< n_gen only when the context window fills), or a negative
 * CWEN_E* code.  Speculative output is identical to serial output. */
int cwen_generate(const int32_t *tokens, int n_tok, int n_gen, int32_t *out, const cwen_spec_cfg *cfg,
                  cwen_spec_stats *stats);

/* ---- binary-frame server (CWEN_SERVER=1: server_loop, run.c:5063-5078) ---- */
/* Generate for one request: prefill tokens[0..n_tok) and write up to n_gen
 * ids to out; the number written, or a negative CWEN_E* code (which ends the
 * server with that code). */
typedef int (*cwen_generate_fn)(void *user, const int32_t *tokens, int n_tok, int n_gen, int32_t *out);
/* Serve request frames from in_fd until end of input: {u32 n_prompt, u32
 * n_gen, n_prompt x int32 ids} -> {u32 n_out, n_out x int32 ids}.  Frames with
 * a count outside [1, ctx] or an id outside [0, n_vocab) get the reply 0
 * (server_read_frame, run.c:4216-4235).  Returns 0 at end of input, or the
 * error that ended it (a failed reply write, a generation error). */
int cwen_serve(int in_fd, int out_fd, int ctx, int n_vocab, cwen_generate_fn gen, void *user);

/* ---- drafters (the contract of run.c:4527-4532) ---- */
/* Prompt-lookup scan (ngram_draft, run.c:4533): propose up to max_d ids that
 * followed the most useful earlier match of the last n_key ids. */
int cwen_ngram_draft(const int32_t *hist, int hn, int32_t *out, int n_key, int max_d);
/* The counted n-gram map (run.c:205-221, 4552-4654): key of n_key ids ->
 * latest continuation and hit count, 2^18 entries, least-hit eviction when
 * full.  The speculative driver keeps one per generation when n-gram
 * drafting is on.  NULL (message in cwen_cuda_last_error) for n_key outside
 * [2,256] or no memory. */
typedef struct cwen_ngram_map cwen_ngram_map;
cwen_ngram_map *cwen_ngram_map_new(int n_key);
void cwen_ngram_map_free(cwen_ngram_map *m);
/* Fold hist[a..b): every position p >= n_key adds hist[p-n_key..p) -> hist[p]
 * (ng_update_range, run.c:4631). */
void cwen_ngram_map_update(cwen_ngram_map *m, const int32_t *hist, int a, int b);
/* The proposal of one speculative cycle (run.c:4925-4930): chained map
 * lookups from the last n_key ids, replaced by cwen_ngram_draft's history
 * scan when that proposes more; at most min(max_d, 256) ids. */
int cwen_ngram_map_draft(const cwen_ngram_map *m, const int32_t *hist, int hn, int32_t *out, int max_d);
/* NGC2 persistence (ng_save / ng_load, run.c:4656-4716; the CWEN_NGRAM_CACHE
 * knob, which the speculative driver honours the same way): save writes
 * {"NGC2", n_key, n_vocab, entries} and the occupied slots in slot order,
 * through a temporary file and a rename.  load merges a file's entries into
 * the map (hit counts add) and returns how many it merged: a missing file,
 * another n_key or vocabulary, or a damaged tail merges nothing or only the
 * valid records -- never an error, like the reference's cold start. */
int cwen_ngram_map_save(const cwen_ngram_map *m, const char *path, int n_vocab);
int cwen_ngram_map_load(cwen_ngram_map *m, const char *path, int n_vocab);

#ifdef __cplusplus
}
#endif
#endif
