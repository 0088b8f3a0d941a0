// Batched quantized GEMV (verify GEMV) -- host-side interface.
//
// Y[b*ys + i] = sum_k W[i,k] * X[b*xs + k] for b < B <= 16, W in GGUF Q4_0 or
// Q8_0 (f16 scale per 32 weights).  Replaces gemvb()/gemv() of the reference
// (run.c:1577, run.c:1419).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cw {

// Device layout of one (possibly fused) weight matrix: rows grouped in
// 16-row m-tiles, m-tiles in 512-row tiles of 32, one contiguous stage per
// (tile, pair of 32-blocks), stages stored [tile][k-pair].  Inside a stage:
// tcgen05 kernel [block 0: 512 rows x quant bytes | block 1 | f16 scales
// [2][512]] (QgStage); mma.sync kernel [m-tile][576-byte chunk in A-fragment
// order] (qgemv_mma.cu).  Same stage size either way.  The m-tile count is
// padded to whole tiles (zero padding).
// The verify-GEMV kernels an engine can run (chosen once at cwen_cuda_init;
// a matrix is stored in the layout of that kernel): the warp-level mma.sync
// kernel of qgemv_mma.cu (default), the tcgen05 kernel of qgemv.cu, and
// qmv.cu (whole rows per CTA, no split-K reduction).
enum { GK_MMA = 0, GK_QMV = 1, GK_TC = 2 };

struct QMat {
  uint8_t *w = nullptr;  // device
  int kern = GK_MMA;     // layout of this kernel
  bool tc = false;       // kern == GK_TC
  int n_ht = 0;          // qmv layout: 8-row half-tiles
  bool pair = false;     // qmv layout: gate/up rows interleaved by half-tile (SwiGLU)
  int G = 0;             // qmv layout: CTAs the rows are partitioned over
  int type = 0;          // 2 = Q4_0, 8 = Q8_0
  int K = 0;             // row length
  int n_mt = 0;          // m-tiles (16 rows) holding rows; storage is padded to QG_TILE_MT
  int M = 0;             // valid rows (n_mt*16 >= M)
  size_t bytes = 0;
};

enum { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };

constexpr int QG_MAXB = 16;
constexpr int QG_CONS_WARPS = 16;                    // row warps, 32 rows (two m-tiles) each
constexpr int QG_THREADS = (QG_CONS_WARPS + 6) * 32;  // + two producer warps + four MMA-issuing warps
constexpr int QG_TILE_MT = 2 * QG_CONS_WARPS;         // m-tiles per CTA tile (512 rows)
constexpr int QG_TILE_ROWS = 16 * QG_TILE_MT;
// One stage of the repacked weights: one 512-row tile x one k-pair.
template <int TYPE>
struct QgStage {
  static constexpr int QROW = TYPE == 8 ? 32 : 16;             // quant bytes per row and 32-block
  static constexpr int QB = QG_TILE_ROWS * QROW;               // one 32-block of the tile
  static constexpr int WB = 2 * QB + 2 * QG_TILE_ROWS * 2;     // both blocks + their f16 scales
};
constexpr int WS_TILE_FLOATS = QG_TILE_MT * 16 * 16;   // split-K partials of one tile (16 columns)
constexpr int QG_XL_KP = 20;  // local-X variant: at most this many k-pairs per CTA (tcgen05 kernel)
constexpr int QG_XL_KP_MMA = 40;  // the same for the mma.sync kernel (its ring shrinks to make room)
constexpr int QG_STAT_COLS = 16;  // per-CTA statistics slot: one float per column
constexpr int QG_MAX_PEERS = 8;   // GPUs of a row-shard group

inline size_t qmat_stage_bytes(int type) { return type == 8 ? QgStage<8>::WB : QgStage<2>::WB; }
inline size_t qmat_bytes(int type, int K, int n_mt) {
  const size_t tiles = (size_t)(n_mt + QG_TILE_MT - 1) / QG_TILE_MT;
  return qmat_stage_bytes(type) * (size_t)(K / 64) * tiles;
}

// Scratch the GEMV needs (owned by the caller, reused across calls on one stream).
struct GemvScratch {
  // Which kernel the engine runs (chosen once, before any weight upload, so
  // every batch size of an engine takes the same arithmetic): the tcgen05
  // kernel of qgemv.cu, or the mma.sync kernel of qgemv_mma.cu (default).
  int kern = GK_MMA;
  bool tc = false;  // kern == GK_TC
  // qmv: X operands converted once per call, published per K phase
  uint8_t *qx = nullptr;
  int *qflag = nullptr;  // zero-initialised
  int qepoch = 0;
  uint4 *xf = nullptr;   // X operands, >= (Kmax/32) * 128 uint4 (2 KB per 32-block)
  int *xexp = nullptr;   // [16] per-column exponents
  float *ws = nullptr;   // split-K partials [G][2][WS_TILE_FLOATS]
  int *cnt = nullptr;    // split-K sync words (zeroed at allocation): per-tile arrival counters
                         // of the tcgen05 kernel, per (CTA, slot) partial flags of the mma kernel
  int epoch = 0;         // the mma kernel's last flag value (never 0)
  int *err = nullptr;    // set when a bounded wait gave up (0 = fine)
  int G = 0;             // persistent grid size (CTAs), at most one per SM
  int kmax = 0;
  int max_tiles = 0;
  // Sums of squares of the output rows of the last GEMV, per CTA [G][16]
  // (two buffers: a GEMV never writes the one it reads), for an RMSNorm of
  // those rows inside the next GEMV.  Optional (nullptr: never fused).
  float *stat = nullptr, *stat_next = nullptr;
  bool stat_ok = false;  // stat describes the output (stat_y, stat_ys) of the GEMV right before
  int stat_g = 0, stat_len = 0, stat_cols = 0, stat_ys = 0;
  const float *stat_y = nullptr;
  // Row sharding of the next GEMV launch (set by the caller around it): the
  // output is rows row0.. of the full matrix, stored into np copies of Y
  // (yp[i] is GPU i's copy of the buffer passed as Y); np = 0: not sharded.
  int np = 0, row0 = 0;
  float *yp[QG_MAX_PEERS] = {};
};
size_t gemv_scratch_ws_floats(int G);
// The engine's kernel takes raw fp32 X (and an RMSNorm weight) in one launch:
// callers pass rows instead of preparing GEMV fragments first.
inline bool gemv_raw_x(const GemvScratch &s) { return s.kern == GK_QMV; }

// Repack `M` GGUF rows (Q4_0 18 B/block or Q8_0 34 B/block) already on the
// device at `src` into `dst`: source row r lands in m-tile
// mt_off + (r/16)*mt_stride, row r%16 of that tile.
cudaError_t qmat_repack(const QMat &dst, const uint8_t *src, int M, int mt_off, int mt_stride, cudaStream_t st);

// X fp32 [B][xs] -> fragments + exponents (scratch).
cudaError_t gemv_prep_x(const float *X, int xs, int B, int K, GemvScratch &s, cudaStream_t st);
// GEMV over prepared X.  epi selects the output: store, add into Y
// (residual), or SiLU(gate)*up of an interleaved gate/up matrix.
cudaError_t gemv_run(const QMat &m, int B, float *Y, int ys, int epi, GemvScratch &s, cudaStream_t st);

// GEMV over raw fp32 X [B][xs].  When the grid is tile-aligned and every
// CTA's k-range is short (the shape decides, never B), each CTA turns its own
// k-range of X into fragments with its own power-of-two column scale and
// unscales its partials before the reduction -- no separate X preparation;
// otherwise gemv_prep_x + gemv_run.
// want_stats (EPI_ADD): also leave the output rows' sums of squares for
// gemv_run_xn of the next GEMV.
cudaError_t gemv_run_x(const QMat &m, const float *X, int xs, int B, float *Y, int ys, int epi, GemvScratch &s,
                       cudaStream_t st, bool want_stats = false);
// GEMV over RMSNorm(X) * w (run.c:346) of rows X [B][xs].  When the GEMV right
// before wrote X with want_stats and this matrix takes the local-X variant,
// each CTA normalises its own k-range inside the GEMV; otherwise
// launch_norm_prep + gemv_run.  (Either way the choice is the shape's, not B's.)
cudaError_t gemv_run_xn(const QMat &m, const float *X, int xs, const float *w, int B, float *Y, int ys, int epi,
                        GemvScratch &s, cudaStream_t st);
bool gemv_norm_fused(const QMat &m, const float *X, int xs, int B, const GemvScratch &s);
// Whether gemv_run_x takes the local-X variant for this matrix (one launch) or
// prepares X first (two).
bool gemv_uses_local_x(const QMat &m, const float *X, int xs, const GemvScratch &s);

// Kernel attributes set once per process (shared-memory carveout).
cudaError_t qgemv_configure();

}  // namespace cw
