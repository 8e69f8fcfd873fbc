// The drop-in of INTEGRATION.md section 1: the bodies of the reference's
// kernel launchers (src/kernels.cuh:16-132 of mohamadmsalman82/
// llama-cuda-runtime) forwarding to liblcr_b200's C ABI. Built in place of
// the reference's src/kernels/*.cu, the reference's own Model, loader, KV
// cache and cuBLAS projections run every hand-written kernel from this
// library. A non-OK status becomes the reference's lcr::Error through its
// LCR_CHECK (src/common.h:25-35).
#include "common.h"
#include "kernels.cuh"
#include "lcr_b200.h"

namespace lcr {
namespace {

inline void ok(int status, const char* what) {
  LCR_CHECK(status == LCR_OK, what << ": " << lcr_status_string(status) << ": " << lcr_last_error_string());
}
inline lcr_stream_t st(cudaStream_t s) { return reinterpret_cast<lcr_stream_t>(s); }
inline lcr_kv_view kv(const KvCacheView& k) {  // src/kv_cache.cuh:33-57, the same fields
  return {k.keys, k.values, k.page_table, k.page_size, k.page_stride, k.head_stride, k.num_kv_heads, k.head_dim};
}

}  // namespace

void launch_embedding_lookup(elem_t* out, const elem_t* table, const int32_t* ids, int tokens, int dim,
                             cudaStream_t s) {
  ok(lcr_embedding_lookup(out, table, ids, tokens, dim, st(s)), "embedding_lookup");
}
void launch_rmsnorm(elem_t* out, const elem_t* x, const elem_t* weight, int tokens, int dim, float eps,
                    cudaStream_t s) {
  ok(lcr_rmsnorm(out, x, weight, tokens, dim, eps, st(s)), "rmsnorm");
}
void launch_add_residual(elem_t* x, const elem_t* delta, int64_t count, cudaStream_t s) {
  ok(lcr_add_residual(x, delta, count, st(s)), "add_residual");
}
void launch_add_residual_rmsnorm(elem_t* out, elem_t* x, const elem_t* delta, const elem_t* weight, int tokens,
                                 int dim, float eps, cudaStream_t s) {
  ok(lcr_add_residual_rmsnorm(out, x, delta, weight, tokens, dim, eps, st(s)), "add_residual_rmsnorm");
}
void launch_swiglu(elem_t* out, const elem_t* gate, const elem_t* up, int64_t count, cudaStream_t s) {
  ok(lcr_swiglu(out, gate, up, count, st(s)), "swiglu");
}
void launch_swiglu_strided(elem_t* out, const elem_t* gate, const elem_t* up, int tokens, int width,
                           int src_row_stride, cudaStream_t s) {
  ok(lcr_swiglu_strided(out, gate, up, tokens, width, src_row_stride, st(s)), "swiglu_strided");
}
void launch_rope_q(elem_t* q_heads, const elem_t* q_proj, const float* inv_freq, int tokens, int start_position,
                   int num_heads, int head_dim, int src_row_stride, cudaStream_t s) {
  ok(lcr_rope_q(q_heads, q_proj, inv_freq, tokens, start_position, num_heads, head_dim, src_row_stride, st(s)),
     "rope_q");
}
void launch_rope_write_kv(const KvCacheView& view, const elem_t* k_proj, const elem_t* v_proj,
                          const float* inv_freq, int tokens, int start_position, bool paged, int src_row_stride,
                          cudaStream_t s) {
  const lcr_kv_view v = kv(view);
  ok(lcr_rope_write_kv(&v, k_proj, v_proj, inv_freq, tokens, start_position, paged ? 1 : 0, src_row_stride, st(s)),
     "rope_write_kv");
}
void launch_causal_softmax(elem_t* probs, const float* scores, int num_heads, int rows, int keys,
                           int start_position, cudaStream_t s) {
  ok(lcr_causal_softmax(probs, scores, num_heads, rows, keys, start_position, st(s)), "causal_softmax");
}
void launch_merge_heads(elem_t* out, const elem_t* heads, int tokens, int num_heads, int head_dim,
                        cudaStream_t s) {
  ok(lcr_merge_heads(out, heads, tokens, num_heads, head_dim, st(s)), "merge_heads");
}
void launch_gather_kv(elem_t* out_keys, elem_t* out_values, const KvCacheView& view, int positions,
                      cudaStream_t s) {
  const lcr_kv_view v = kv(view);
  ok(lcr_gather_kv(out_keys, out_values, &v, positions, st(s)), "gather_kv");
}
void launch_decode_attention(elem_t* out, const elem_t* q, const KvCacheView& view, int num_heads,
                             int heads_per_kv, int seq_len, float scale, bool paged, int splits, float* scratch,
                             cudaStream_t s) {
  const lcr_kv_view v = kv(view);
  ok(lcr_decode_attention(out, q, &v, num_heads, heads_per_kv, seq_len, scale, paged ? 1 : 0, splits, scratch,
                          st(s)),
     "decode_attention");
}
size_t decode_attention_scratch_floats(int num_heads, int head_dim, int splits) {
  return lcr_decode_attention_scratch_floats(num_heads, head_dim, splits);
}
int choose_attention_splits(int num_kv_heads, int seq_len, int multiprocessors) {
  return lcr_choose_attention_splits(num_kv_heads, seq_len, multiprocessors);
}
void launch_sample(int32_t* out_id, const float* logits, int vocab, float temperature, int top_k, float top_p,
                   float uniform, float* scratch, cudaStream_t s) {
  ok(lcr_sample(out_id, logits, vocab, temperature, top_k, top_p, uniform, scratch, st(s)), "sample");
}
size_t sample_scratch_floats(int vocab, int top_k) { return lcr_sample_scratch_floats(vocab, top_k); }

}  // namespace lcr
