/*
 * lcr_b200 -- C ABI of the B200 (sm_100a) Llama decode step.
 *
 * Drop-in boundary for the forward path of mohamadmsalman82/llama-cuda-runtime:
 *   - one entry point per host launcher of src/kernels.cuh (the `launch_*`
 *     free functions), same argument meaning, raw device pointers, async on
 *     the given stream, no allocation inside;
 *   - lcr_gemm_nt replacing the cuBLAS `gemm_nt` of src/model.cu:38-45;
 *   - a decode context replacing Model::decode / Model::sample / prefill
 *     (src/model.h:60-127, src/model.cu:308-597), whose whole step is a
 *     CUDA graph of hand-written sm_100a kernels with the token, position and
 *     sampling state resident on the device.
 *
 * Conventions: bf16 tensors are `void*` to 16-bit bf16 storage; every function
 * returns an lcr_status (0 = LCR_OK); no C++ exception crosses this boundary;
 * lcr_last_error_string() describes the last failure on the calling thread.
 * The caller owns every buffer passed in; buffers a context allocates are
 * freed by lcr_ctx_destroy. Where the reference threw lcr::Error (LCR_CHECK),
 * these functions return LCR_ERR_INVALID / LCR_ERR_SHAPE with the same text.
 */
#ifndef LCR_B200_H
#define LCR_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LCR_API __attribute__((visibility("default")))
#else
#define LCR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* lcr_stream_t; /* == cudaStream_t; NULL = legacy default stream */

enum lcr_status {
  LCR_OK = 0,
  LCR_ERR_INVALID = 1,     /* bad argument: null pointer, non-positive size */
  LCR_ERR_SHAPE = 2,       /* shape this build has no kernel for */
  LCR_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  LCR_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up */
  LCR_ERR_POOL = 5,        /* paged KV pool exhausted */
  LCR_ERR_STATE = 6,       /* call out of order (e.g. sequence full) */
  LCR_ERR_NO_DEVICE = 7    /* no sm_100 device */
};

LCR_API const char* lcr_last_error_string(void);
LCR_API const char* lcr_status_string(int status);
LCR_API int lcr_version(void); /* major * 10000 + minor * 100 + patch */

/* ------------------------------------------------------------------------- */
/* KV cache view -- KvCacheView, src/kv_cache.cuh:33-57.                      */
/* Element offset of (head, position): page * page_stride +                  */
/* head * head_stride + slot * head_dim, page = page_table[pos / page_size], */
/* slot = pos % page_size (contiguous: page 0, slot = pos).                  */
/* ------------------------------------------------------------------------- */
typedef struct lcr_kv_view {
  void* keys;
  void* values;
  const int32_t* page_table; /* NULL for the contiguous layout */
  int page_size;
  int page_stride;
  int head_stride;
  int num_kv_heads;
  int head_dim;
} lcr_kv_view;

/* ------------------------------------------------------------------------- */
/* Per-kernel entry points (src/kernels.cuh:17-132)                           */
/* ------------------------------------------------------------------------- */

/* launch_embedding_lookup, src/kernels.cuh:16-19: out[t,:] = table[ids[t],:] */
LCR_API int lcr_embedding_lookup(void* out, const void* table, const int32_t* ids,
                         int tokens, int dim, lcr_stream_t stream);

/* launch_rmsnorm, src/kernels.cuh:21-25 */
LCR_API int lcr_rmsnorm(void* out, const void* x, const void* weight, int tokens,
                int dim, float eps, lcr_stream_t stream);

/* launch_add_residual, src/kernels.cuh:27-29 */
LCR_API int lcr_add_residual(void* x, const void* delta, int64_t count,
                     lcr_stream_t stream);

/* launch_add_residual_rmsnorm, src/kernels.cuh:31-41 */
LCR_API int lcr_add_residual_rmsnorm(void* out, void* x, const void* delta,
                             const void* weight, int tokens, int dim,
                             float eps, lcr_stream_t stream);

/* launch_swiglu, src/kernels.cuh:43-45 */
LCR_API int lcr_swiglu(void* out, const void* gate, const void* up, int64_t count,
               lcr_stream_t stream);

/* launch_swiglu_strided, src/kernels.cuh:47-51 */
LCR_API int lcr_swiglu_strided(void* out, const void* gate, const void* up, int tokens,
                       int width, int src_row_stride, lcr_stream_t stream);

/* launch_rope_q, src/kernels.cuh:53-64: [tokens][heads*d] -> [heads][tokens][d] */
LCR_API int lcr_rope_q(void* q_heads, const void* q_proj, const float* inv_freq,
               int tokens, int start_position, int num_heads, int head_dim,
               int src_row_stride, lcr_stream_t stream);

/* launch_rope_write_kv, src/kernels.cuh:66-72 */
LCR_API int lcr_rope_write_kv(const lcr_kv_view* view, const void* k_proj,
                      const void* v_proj, const float* inv_freq, int tokens,
                      int start_position, int paged, int src_row_stride,
                      lcr_stream_t stream);

/* launch_causal_softmax, src/kernels.cuh:74-81: scores [heads][rows][keys]
 * fp32, row r is query position start_position + r and sees keys up to it;
 * probs (same layout, bf16) = softmax over those keys, 0 beyond them. */
LCR_API int lcr_causal_softmax(void* probs, const float* scores, int num_heads,
                       int rows, int keys, int start_position,
                       lcr_stream_t stream);

/* launch_merge_heads, src/kernels.cuh:83-86: heads [heads][tokens][d] ->
 * out [tokens][heads * d]. */
LCR_API int lcr_merge_heads(void* out, const void* heads, int tokens, int num_heads,
                    int head_dim, lcr_stream_t stream);

/* launch_gather_kv, src/kernels.cuh:88-94: the cached positions [0, positions)
 * of a (paged or contiguous) view as contiguous [kv_head][position][d] keys
 * and values. */
LCR_API int lcr_gather_kv(void* out_keys, void* out_values, const lcr_kv_view* view,
                  int positions, lcr_stream_t stream);

/* launch_decode_attention, src/kernels.cuh:106-110: single-token GQA attention
 * over seq_len cached positions, split-K over `splits` blocks per KV head. */
LCR_API int lcr_decode_attention(void* out, const void* q, const lcr_kv_view* view,
                         int num_heads, int heads_per_kv, int seq_len,
                         float scale, int paged, int splits, float* scratch,
                         lcr_stream_t stream);

/* No counterpart in the reference. lcr_decode_attention without caller
 * scratch, for callers that must not allocate device memory (an allocator
 * that forbids it, or a fixed memory budget set up before serving): the
 * split partials live in one static device array of
 * LCR_NOALLOC_ATTENTION_SCRATCH_FLOATS floats (2 MiB). A call that needs more
 * (num_heads x splits x (head_dim + 2), splits after the 16-position clamp)
 * returns LCR_ERR_SHAPE. The first call on each device looks the array up
 * (cudaGetSymbolAddress, with that device current): make it before any stream
 * capture, and do not use the entry point across a cudaDeviceReset (the
 * array may move; the looked-up address is kept). Every call on a device
 * shares the array, so calls whose kernels may overlap race; order them on
 * one stream. */
#define LCR_NOALLOC_ATTENTION_SCRATCH_FLOATS (1 << 19)
LCR_API int lcr_decode_attention_noalloc(void* out, const void* q,
                                 const lcr_kv_view* view, int num_heads,
                                 int heads_per_kv, int seq_len, float scale,
                                 int paged, int splits, lcr_stream_t stream);

/* decode_attention_scratch_floats, src/kernels.cuh:114 */
LCR_API size_t lcr_decode_attention_scratch_floats(int num_heads, int head_dim,
                                           int splits);

/* choose_attention_splits, src/kernels.cuh:118 */
LCR_API int lcr_choose_attention_splits(int num_kv_heads, int seq_len,
                                int multiprocessors);

/* launch_sample, src/kernels.cuh:128-130: temperature 0 = argmax (ties to the
 * lowest id); otherwise top-k/top-p over the full-vocab softmax with the
 * host's uniform in [0,1). Deterministic: equal inputs give equal ids. */
LCR_API int lcr_sample(int32_t* out_id, const float* logits, int vocab,
               float temperature, int top_k, float top_p, float uniform,
               float* scratch, lcr_stream_t stream);

/* sample_scratch_floats, src/kernels.cuh:132 */
LCR_API size_t lcr_sample_scratch_floats(int vocab, int top_k);

/* gemm_nt, src/model.cu:38-45: y[rows][out] = x[rows][in] * w[out][in]^T,
 * bf16 inputs, fp32 accumulation, bf16 output (y_fp32 = 0) or fp32 output
 * (y_fp32 = 1, the lm_head case of src/model.cu:481). */
LCR_API int lcr_gemm_nt(void* y, int y_fp32, const void* x, const void* w, int rows,
                int in_features, int out_features, lcr_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Decode context -- Model (src/model.h:60-127)                               */
/* ------------------------------------------------------------------------- */

typedef struct lcr_model_desc { /* ModelConfig, src/config.h:22-60 */
  int hidden_size;
  int intermediate_size;
  int num_layers;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int vocab_size;
  float rms_norm_eps;
  float rope_theta;
  int rope_scaling; /* 1 = llama3 */
  float rope_factor;
  float rope_low_freq_factor;
  float rope_high_freq_factor;
  int rope_original_max_position_embeddings;
} lcr_model_desc;

typedef struct lcr_layer_weights { /* LayerWeights, src/model.h:29-43 */
  const void* input_norm;          /* [hidden] */
  const void* qkv_proj;            /* [q_dim + 2 kv_dim][hidden], rows q;k;v */
  const void* o_proj;              /* [hidden][q_dim] */
  const void* post_attention_norm; /* [hidden] */
  const void* gate_up_proj;        /* [2 ffn][hidden], rows gate;up */
  const void* down_proj;           /* [hidden][ffn] */
} lcr_layer_weights;

typedef struct lcr_weights { /* device pointers, caller-owned */
  const void* embedding;  /* [vocab][hidden] */
  const void* final_norm; /* [hidden] */
  const void* lm_head;    /* [vocab][hidden]; the embedding when tied */
  const lcr_layer_weights* layers; /* host array of num_layers entries */
} lcr_weights;

typedef struct lcr_options { /* Model::Options, src/model.h:62-77 */
  int device;
  int max_seq;          /* KV positions per sequence */
  int paged;            /* 0 = contiguous, 1 = paged */
  int page_size;        /* positions per page (paged); 16 in the reference */
  int attention_splits; /* split-K blocks per KV head (at most; fewer only when
                           the context has fewer than 32 positions per split);
                           0 = choose: one split per ~384 cached positions */
  uint64_t page_order_seed; /* 0 = pages handed out in counter order;
                               otherwise a seeded permutation of the pool */
  int gemv_ctas;        /* CTAs per streaming GEMV; 0 = one per SM */
  int flags;            /* bit 0: no programmatic dependent launch,
                           bit 1: no CUDA graph, bit 2: multi-kernel step
                           instead of the persistent single-kernel step,
                           bit 3: record per-phase timestamps (trace),
                           bit 4: persistent step with fp32 activations,
                           bit 5: tests only (grid-barrier timeout path),
                           bit 6: lcr_prefill one decode step per token,
                           bit 7: persistent step's attention on CUDA cores
                           instead of the tensor pipe,
                           bit 8: persistent step's phases meet at grid
                           barriers instead of exchanging tagged words */
} lcr_options;

typedef struct lcr_ctx lcr_ctx;

LCR_API int lcr_ctx_create(const lcr_model_desc* desc, const lcr_weights* weights,
                   const lcr_options* options, lcr_ctx** out);
LCR_API void lcr_ctx_destroy(lcr_ctx* ctx);

/* compute_rope_inv_freq, src/config.cpp:223-259: the head_dim / 2 inverse
 * frequencies the context rotates with (theta^(-2i/d) in double, rounded to
 * float, then the llama3 band rescaling when rope_scaling is set), written to
 * out[0 .. head_dim / 2). Host only; needs no device. */
LCR_API int lcr_rope_inv_freq(const lcr_model_desc* desc, float* out, int capacity);

/* Model::reset, src/model.h:91: position back to 0 (the cache is reused). */
LCR_API int lcr_reset(lcr_ctx* ctx);
/* Model::position */
LCR_API int lcr_position(const lcr_ctx* ctx);

/* Model::decode, src/model.cu:347-368: one token at the current position;
 * *logits receives the device fp32 logits [vocab], valid until the next
 * call. Synchronous, like the reference. */
LCR_API int lcr_decode(lcr_ctx* ctx, int token, const float** logits);

/* Model::prefill, src/model.cu:308-345: the prompt at the current position;
 * *logits for the last token, and the device state ready for the next step
 * (next token = the argmax of those logits, position advanced). Like the
 * reference, which runs the prompt in chunks of prefill_chunk positions
 * (cuBLAS projections, a bf16 softmax and the P.V GEMM), prompts of two or
 * more tokens run in chunks -- of up to 2048 rows, on the tcgen05 path of
 * lcr_batch_prefill (projections as GEMMs over the chunk, causal flash
 * attention over the cache), writing this context's own cache. One decode
 * step per token instead with options bit 6, with fp32 activations (bit 4),
 * with a paged cache whose page size is not a multiple of 16, or for a model
 * the batch kernels are not built for. Synchronous. */
LCR_API int lcr_prefill(lcr_ctx* ctx, const int32_t* tokens, int count,
                const float** logits);

/* Model::logits_to_host, src/model.cu:599-604: copies the [vocab] fp32 logits
 * of the last step to host memory (synchronous). */
LCR_API int lcr_logits_to_host(lcr_ctx* ctx, float* host);

/* Model::sample, src/model.cu:584-597: a token id from device logits. */
LCR_API int lcr_sample_logits(lcr_ctx* ctx, const float* logits, float temperature,
                      int top_k, float top_p, float uniform, int* token);

/* Device-resident greedy generation: the step graph replayed `steps` times,
 * each step's argmax feeding the next with no host round trip. Starts from
 * `first_token` at the current position; tokens_out (host, nullable) receives
 * the `steps` generated ids. Synchronous. */
LCR_API int lcr_generate_greedy(lcr_ctx* ctx, int first_token, int steps,
                        int32_t* tokens_out);

/* Asynchronous pieces of the same loop, for timing and for host pipelines:
 * lcr_set_token reads the token from host memory during the call and stages
 * (token, position) into device state on the context's stream, as one
 * 8-byte copy; lcr_enqueue_steps launches `steps` step graphs
 * (mapping first, when paged, the pages of the positions they write);
 * lcr_read_token copies the latest device token to host memory (pinned for
 * true async) and lcr_sync waits for the stream. */
LCR_API int lcr_set_token(lcr_ctx* ctx, const int32_t* host_token, int position);
/* One step of the reference's host decode loop in one call: Model::decode
 * (src/model.cu:347-368) of `token` at `position`, then the greedy pick of
 * the logits that llama-run's loop reads back (src/main.cu:455-463,
 * temperature 0). The next token arrives in *next_token with the step's
 * status in the same read-back; synchronous. */
LCR_API int lcr_step_host(lcr_ctx* ctx, int32_t token, int position, int32_t* next_token);
LCR_API int lcr_enqueue_steps(lcr_ctx* ctx, int steps);
LCR_API int lcr_read_token(lcr_ctx* ctx, int32_t* host_token);
LCR_API int lcr_sync(lcr_ctx* ctx);
LCR_API lcr_stream_t lcr_ctx_stream(lcr_ctx* ctx);

/* The device KV view of one layer (KvCache::view, src/kv_cache.cu:121-144). */
LCR_API int lcr_kv_view_of(const lcr_ctx* ctx, int layer, lcr_kv_view* view);
/* Copies the host mirror of the page tables ([layers][max_pages] int32) to
 * `tables`; returns the number of pages handed out in *pages_mapped. */
LCR_API int lcr_page_tables(const lcr_ctx* ctx, int32_t* tables, int* pages_mapped);
/* KvCache::reserve_length, src/kv_cache.cu:73-102 */
LCR_API int lcr_reserve_length(lcr_ctx* ctx, int length);

/* Bytes one decode step streams from HBM (src/model.cu:91-102) and the KV
 * bytes per cached position (src/config.h:47-49). */
LCR_API size_t lcr_weight_bytes_per_token(const lcr_ctx* ctx);
LCR_API size_t lcr_kv_bytes_per_position(const lcr_ctx* ctx);
/* Kernel launches in one decode step. */
LCR_API int lcr_step_launches(const lcr_ctx* ctx);
/* Reads and clears the device status word the context's kernels report
 * bounded-wait failures and out-of-range tokens / positions / pages through:
 * LCR_OK, LCR_ERR_TIMEOUT, LCR_ERR_INVALID, LCR_ERR_POOL or LCR_ERR_STATE. */
LCR_API int lcr_device_status(lcr_ctx* ctx);

/* Measurement: `steps` step graphs timed with CUDA events on the context's
 * stream (device state advances as in lcr_enqueue_steps), and `reps`
 * back-to-back launches of one streaming GEMV of the step (matrix 0 qkv,
 * 1 o_proj, 2 gate_up, 3 down, 4 lm_head; reps <= 128), in ms per launch. */
LCR_API int lcr_time_steps(lcr_ctx* ctx, int steps, float* ms);
/* With flags bit 3 (trace) on a persistent-step context: copies the last
 * step's per-CTA phase timestamps (globaltimer ns unless noted; per CTA 1024
 * slots: [0] consumers start, [2k+1]/[2k+2] arrival at / departure from grid
 * barrier k, [163 + p] prologue of phase p done, [255] consumers end,
 * [256 + p] producer starting phase p, [340 + p] / [424 + p] SM cycles the
 * consumers / the producer waited on the ring in matrix phase p, and for
 * layer 8's gate/up phase per stage s: [512 + s] issued, [576 + s] ready,
 * [640 + s] released); *count gets the number of values copied. */
LCR_API int lcr_copy_trace(lcr_ctx* ctx, unsigned long long* host, int capacity, int* count);
LCR_API int lcr_time_gemv(lcr_ctx* ctx, int matrix, int layer, int reps, float* ms);

/* ------------------------------------------------------------------------- */
/* Batched decode -- no counterpart in the reference, whose Model decodes one  */
/* sequence at a time (src/model.h:60-127). Continuous batching keeps up to    */
/* max_batch sequences in slots; one step decodes one token of each of the     */
/* first n slots with tensor-core (tcgen05) projections, the paged decode      */
/* attention of every sequence, and per-slot sampling.                         */
/* ------------------------------------------------------------------------- */

typedef struct lcr_batch_options {
  int device;
  int max_batch;   /* slots (1..256) */
  int max_seq;     /* positions per sequence */
  int page_size;   /* positions per KV page, a multiple of 16 */
  int pool_pages;  /* pages in the shared KV pool; a page holds every layer */
  int flags;       /* bit 1: no CUDA graph; bit 2: projections of 128-row
                      batch tiles (prefill chunks) one CTA per tile instead of
                      the persistent kernel (same results) */
} lcr_batch_options;

typedef struct lcr_batch lcr_batch;

LCR_API int lcr_batch_create(const lcr_model_desc* desc, const lcr_weights* weights,
                             const lcr_batch_options* options, lcr_batch** out);
LCR_API void lcr_batch_destroy(lcr_batch* batch);
/* Physical pool pages of slot `slot` for positions [0, count * page_size):
 * page i holds positions [i * page_size, (i + 1) * page_size) in every layer.
 * Entries in [0, pool_pages); staged to the device with the next step. */
LCR_API int lcr_batch_set_pages(lcr_batch* batch, int slot, const int32_t* pages, int count);
/* Sampling of slot `slot`: temperature 0 = greedy (lowest id on ties);
 * otherwise top-k / top-p as lcr_sample with the uniform drawn by
 * Philox4x32-10 from (seed, position). */
LCR_API int lcr_batch_set_sampling(lcr_batch* batch, int slot, float temperature, int top_k,
                                   float top_p, uint64_t seed);
/* One step for slots [0, n): slot b decodes host tokens[b] at host
 * positions[b] (its K/V are written at that position; it attends to
 * positions 0..positions[b]), then samples its next token. tokens = NULL
 * continues every slot with the id it sampled in the previous step (no host
 * round trip). Asynchronous. */
LCR_API int lcr_batch_step(lcr_batch* batch, int n, const int32_t* tokens,
                           const int32_t* positions);
/* Writes a seeded synthetic context (approximately standard normal K and V,
 * bf16) for positions [0, length) of slot `slot` in every layer, through its
 * current page table: a stand-in for the prompt's prefill when a benchmark
 * admits a sequence. Asynchronous. */
LCR_API int lcr_batch_fill_kv(lcr_batch* batch, int slot, int length, uint64_t seed);
/* Chunked prefill, Model::prefill (src/model.cu:308-345 with the attention of
 * model.cu:509-560): `count` prompt tokens of slot `slot` at positions
 * start .. start + count - 1, through the projections as tcgen05 GEMMs over
 * the chunk's rows and causal flash attention over the slot's pages (which
 * must cover start + count positions; earlier positions come from earlier
 * chunks or steps). Writes the chunk's K/V into the cache, the last row's
 * logits into the slot's logits (lcr_batch_logits) and its sample, with the
 * slot's sampling parameters and Philox counter start + count - 1, into the
 * slot's next id (lcr_batch_read). The slot then decodes from position
 * start + count. Asynchronous; the first call (or a longer chunk) allocates
 * the chunk's activations. */
LCR_API int lcr_batch_prefill(lcr_batch* batch, int slot, const int32_t* tokens, int count, int start);
/* (lcr_batch_step, lcr_batch_fill_kv and lcr_batch_prefill reject positions
 * beyond the pages set for the slot with LCR_ERR_STATE.) */
/* The last step's sampled ids of slots [0, n) into host memory (synchronous). */
LCR_API int lcr_batch_read(lcr_batch* batch, int32_t* next_ids, int n);
/* The last step's fp32 logits [vocab] of one slot into host memory (synchronous). */
LCR_API int lcr_batch_logits(lcr_batch* batch, int slot, float* host);
LCR_API int lcr_batch_sync(lcr_batch* batch);
LCR_API lcr_stream_t lcr_batch_stream(lcr_batch* batch);
/* Kernel launches in one step of n slots (split projections add a reduction
 * launch each); 0 until a step of n slots has been issued. */
LCR_API int lcr_batch_step_launches(const lcr_batch* batch, int n);
/* Replays the step of the last lcr_batch_step `steps` times (same tokens and
 * positions) between CUDA events on the batch stream: ms in total. */
LCR_API int lcr_batch_time_steps(lcr_batch* batch, int steps, float* ms);

#ifdef __cplusplus
}
#endif
#endif
