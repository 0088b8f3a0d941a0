/* Seeded synthetic weights and inputs for the cwen hybrid model.
 *
 * Every value is a pure function of (seed, tensor name, element index):
 * a counter-based splitmix64 stream keyed by an FNV-1a hash of the tensor
 * name.  Any tensor can therefore be generated alone, in any order, on any
 * number of threads, and the CPU reference, the oracle and the GPU engine
 * all see identical bytes without a 15 GB file changing hands.
 *
 * Distributions follow the benchmark configurations of the reference
 * (Q4_0 scales |N(0,0.01)| with uniform nibbles; Q8_0 scales |N(0,0.01)|
 * with uniform int8 in [-127,127]; F32 norm vectors = 1; ssm_a = -1,
 * ssm_dt.bias = 0; conv kernel ~N(0,0.1)).
 */
#ifndef CWEN_SYNTH_H
#define CWEN_SYNTH_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids used here (same numbering as GGUF files). */
enum { CW_T_F32 = 0, CW_T_Q4_0 = 2, CW_T_Q8_0 = 8 };

/* Model geometry.  The reference fixes these at compile time
 * (run.c:83-91); here they are runtime so tests can run a small model with
 * the same code.  head_dim, n_rot, ssm_d and conv_k are fixed by the
 * kernels (256, 64, 128, 4). */
typedef struct {
  int n_embd, n_ff, n_vocab, n_layer;
  int n_head, n_head_kv, head_dim, n_rot;
  int ssm_n_kh, ssm_n_vh, ssm_d, conv_k;
  int full_interval;
  int has_mtp;
} cw_dims;

/* The 27B geometry of the reference (run.c:83-91). */
void cw_dims_full(cw_dims *d);
/* A small geometry with the same structure (3 GDN layers + 1 attention
 * layer, 2 key heads / 4 value heads, 4 q heads / 2 kv heads). */
void cw_dims_tiny(cw_dims *d);
static inline int cw_qkv_dim(const cw_dims *d) { return 2 * d->ssm_n_kh * d->ssm_d + d->ssm_n_vh * d->ssm_d; }
static inline int cw_is_linear(const cw_dims *d, int layer) { return ((layer + 1) % d->full_interval) != 0; }

/* Tensor descriptor of one model tensor in GGUF terms. */
typedef struct {
  char name[96];
  int type;          /* CW_T_* */
  int ne0, ne1;      /* ne0 = row length (K), ne1 = rows (M) */
  int kind;          /* generator kind, CW_GEN_* */
} cw_tensor_desc;

enum { CW_GEN_QMAT = 0, CW_GEN_ONES = 1, CW_GEN_ZERO = 2, CW_GEN_NEG1 = 3, CW_GEN_CONV = 4 };

/* Number of tensors of the model (including blk.<L>.* when has_mtp). */
int cw_model_tensor_count(const cw_dims *d);
/* i-th tensor descriptor; returns 0 on success. */
int cw_model_tensor_desc(const cw_dims *d, int i, cw_tensor_desc *out);
/* Bytes of a tensor in GGUF layout. */
size_t cw_tensor_nbytes(int type, int ne0, int ne1);
/* Fill `dst` (cw_tensor_nbytes bytes) with the tensor's seeded contents,
 * using up to `threads` host threads (<=0: all cores). */
void cw_synth_tensor(uint64_t seed, const cw_tensor_desc *t, void *dst, int threads);
/* Only rows [r0, r1) of a quantized matrix, at their own offsets of the
 * full-size dst (other kinds: the whole tensor). */
void cw_synth_tensor_rows(uint64_t seed, const cw_tensor_desc *t, void *dst, int threads, int r0, int r1);

/* Generic seeded fills used by benches and tests. */
void cw_synth_q4_0(uint64_t seed, const char *stream, int ne0, int ne1, void *dst, int threads);
void cw_synth_q8_0(uint64_t seed, const char *stream, int ne0, int ne1, void *dst, int threads);
/* n floats ~ N(mean, std). */
void cw_synth_normal(uint64_t seed, const char *stream, float mean, float std, float *dst, size_t n);
/* n ints uniform in [0, hi). */
void cw_synth_ids(uint64_t seed, const char *stream, int hi, int32_t *dst, size_t n);

/* Write the whole seeded model as a GGUF v3 file.  Returns 0 on success. */
int cw_write_gguf(const char *path, const cw_dims *d, uint64_t seed, int threads);

/* IEEE half <-> float (round to nearest even). */
float cw_f16_to_f32(uint16_t h);
uint16_t cw_f32_to_f16(float x);

#ifdef __cplusplus
}
#endif
#endif
