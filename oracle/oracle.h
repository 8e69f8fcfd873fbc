/*
 * CPU oracle for the Llama decode step -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load this library, and only as the checker or the timed CPU
 * baseline. The product (llama-cuda-runtime_b200) never links it and never
 * falls back to it.
 *
 * What it restates, each function citing the file:line of the reference
 * (mohamadmsalman82/llama-cuda-runtime) it follows:
 *   - the decode step of Model::run_layers (src/model.cu:370-484), with the
 *     kernels it calls: RMSNorm (src/kernels/rmsnorm.cu:21-119), RoPE
 *     (src/kernels/rope.cu:33-87), GQA decode attention
 *     (src/kernels/attention.cu:110-299; nested-loop form of
 *     tests/test_kernels.cu:341-381), SwiGLU (src/kernels/elementwise.cu:64-121)
 *     and the tied lm_head (src/model.cu:212, 478-483);
 *   - the RoPE inverse-frequency table with llama3 scaling
 *     (src/config.cpp:223-259);
 *   - greedy argmax with the lowest-index tie rule (src/kernels/sampling.cu:42-67);
 *   - top-k / top-p sampling semantics (src/kernels/sampling.cu:97-224), in the
 *     deterministic form the CUDA sampler implements (see orc_sample);
 *   - the paged KV page allocator (src/kv_cache.cu:73-102).
 *
 * Two evaluation modes:
 *   ORC_MODE_FP32     every activation stays fp32 (the "fp32 host evaluation":
 *                     weights are the bf16 checkpoint values, nothing else is
 *                     rounded). Cross-checked against transformers'
 *                     LlamaForCausalLM in fp32 (tests/golden).
 *   ORC_MODE_BF16     rounds to bf16 exactly where the reference stores a bf16
 *                     tensor (normed, qkv, roped q/k, attention output,
 *                     projections, residual stream, SwiGLU output); math in
 *                     between is fp32/fp64. This is the reference algorithm.
 *   ORC_MODE_BF16_REORDERED  the same with every dot product summed in the
 *                     opposite order: the spread between the two bf16 modes
 *                     is the reproducibility floor of the algorithm itself.
 *   ORC_MODE_FP32_KV_BF16  fp32 activations with the K/V cache stored as bf16
 *                     (the reference's cache format, src/kv_cache.cuh:33-57):
 *                     the closest any implementation on that cache can get to
 *                     ORC_MODE_FP32.
 *
 * Parity pins: the RoPE table against tests/test_config.cpp:120-182, sampling
 * against tests/test_kernels.cu:468-508, page accounting against
 * tests/test_kernels.cu:442-464, the whole step against transformers fp32 and,
 * where the reference sources compile here, against the reference's own
 * compute_rope_inv_freq (oracle/_ref). The full-model logits are pinned only
 * through transformers (the reference ships no golden logits).
 */
#ifndef LCR_ORACLE_H
#define LCR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_MODE_FP32 = 0, ORC_MODE_BF16 = 1, ORC_MODE_BF16_REORDERED = 2, ORC_MODE_FP32_KV_BF16 = 3 };

typedef struct {
  int hidden, ffn, layers, heads, kv_heads, head_dim, vocab;
  float eps, theta;
  int rope_scaling; /* 1 = llama3 band scaling */
  float rope_factor, rope_low, rope_high;
  int rope_orig_ctx;
} orc_config;

/* bf16 bit patterns, reference layouts (src/model.h:29-43): qkv is [q;k;v]
 * rows, gate_up is [gate;up] rows, all row-major [out][in]. */
typedef struct {
  const uint16_t* embed;      /* [vocab][hidden] */
  const uint16_t* final_norm; /* [hidden] */
  const uint16_t* lm_head;    /* [vocab][hidden]; == embed when tied */
  const uint16_t* const* input_norm;
  const uint16_t* const* qkv;
  const uint16_t* const* o;
  const uint16_t* const* post_norm;
  const uint16_t* const* gate_up;
  const uint16_t* const* down;
} orc_weights;

typedef struct orc_state orc_state;

/* ---- numerics helpers ---- */
float orc_bf16_to_float(uint16_t b);
uint16_t orc_float_to_bf16(float f); /* round to nearest even */
void orc_round_bf16_inplace(float* x, size_t n);

/* ---- config-level ---- */
void orc_rope_inv_freq(const orc_config* c, float* out /* [head_dim/2] */);
size_t orc_weight_bytes_per_token(const orc_config* c); /* src/model.cu:91-102 */

/* ---- the decode step ---- */
orc_state* orc_state_new(const orc_config* c, int max_seq);
void orc_state_free(orc_state* s);
void orc_state_reset(orc_state* s);
/* One token at `position`; writes [vocab] fp32 logits. taps (optional) gets
 * [layers + 2][hidden]: embed, each layer's residual stream, final norm
 * (the tap names of src/model.cu:486-503). Returns 0 on success. */
int orc_decode(const orc_config* c, const orc_weights* w, orc_state* s,
               int token, int position, int mode, float* logits, float* taps);
void orc_set_threads(int n);
/* n consecutive tokens at positions start..start+n-1 as one chunk (the
 * reference's chunked prefill, src/model.cu:308-345 and 509-556): the
 * projections as GEMMs over the chunk, causal attention of each row over the
 * cache up to its own position; the K/V rows are appended to the state's
 * cache. Writes the last row's [vocab] logits when last_logits is not NULL.
 * ORC_MODE_FP32, ORC_MODE_BF16 (the rounding points of orc_decode, plus, for
 * n > 1, the bf16 probabilities of the reference's prefill softmax) and
 * ORC_MODE_FP32_KV_BF16. The summation order of the chunk GEMM differs from
 * the decode GEMV. Returns 0 on success. */
int orc_prefill(const orc_config* c, const orc_weights* w, orc_state* s,
                const int32_t* tokens, int n, int start, int mode,
                float* last_logits);

/* ---- individual kernels' maths, for the per-kernel parity tests ---- */
void orc_rmsnorm(float* out, const uint16_t* x, const uint16_t* weight,
                 int tokens, int dim, float eps, int round_out);
void orc_add_residual_rmsnorm(float* out, uint16_t* x, const uint16_t* delta,
                              const uint16_t* weight, int tokens, int dim,
                              float eps);
void orc_swiglu(float* out, const uint16_t* gate, const uint16_t* up,
                long count);
void orc_rope_rows(float* out, const uint16_t* in, const float* inv_freq,
                   int tokens, int start_position, int heads, int head_dim,
                   int src_row_stride, int head_major);
void orc_attention(float* out, const uint16_t* q, const uint16_t* keys,
                   const uint16_t* values, int num_heads, int num_kv_heads,
                   int head_dim, int positions, float scale);
void orc_gemv(float* y, const uint16_t* w, const uint16_t* x, int rows,
              int cols);

/* ---- sampling ---- */
int orc_argmax(const float* logits, int vocab);
float orc_det_expf(float x);
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2],
                       uint32_t out[4]);
float orc_philox_uniform(uint64_t seed, uint64_t counter, uint32_t stream);
float orc_tree_sum_1024(const float* e, int n);
int orc_sample(const float* logits, int vocab, float inv_temperature,
               int top_k, float top_p, float uniform);

/* ---- paged KV page allocator ---- */
/* Single-sequence KvCache::reserve_length (src/kv_cache.cu:73-102): pages are
 * handed out from a counter, layer by layer. `order` (nullable) maps the
 * counter to a physical page id (the shuffled physical order); `tables` is
 * [layers][max_pages], initialised to -1 by the caller. Returns the new
 * pages_mapped, or -1 if the pool is exhausted. */
int orc_paged_reserve(int32_t* tables, int layers, int max_pages,
                      int page_size, int old_length, int new_length,
                      int pages_mapped, int pool_pages, const int32_t* order);
/* Seeded permutation of [0, n) (Fisher-Yates over splitmix64). */
void orc_page_permutation(int32_t* out, int n, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
