// C ABI of the B200 decode step (include/lcr_b200.h): status plumbing, the
// per-kernel entry points that mirror src/kernels.cuh of the reference, and
// the decode context whose step is one CUDA graph of sm_100a kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "dispatch.h"
#include "gemv_dispatch.h"
#include "lcr_b200.h"
#include "sampling.cuh"
#include "small_kernels.cuh"
#include "gemm_tc.h"
#include "tmap.h"

namespace lcrb {

namespace {
thread_local char g_error[1024] = "";
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_error, sizeof g_error, fmt, ap);
  va_end(ap);
  return status;
}

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(LCR_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return LCR_OK;
}

namespace {

inline cudaStream_t cs(lcr_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

template <typename T>
inline const bf16* cb(T p) { return reinterpret_cast<const bf16*>(p); }
template <typename T>
inline bf16* mb(T p) { return reinterpret_cast<bf16*>(p); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace lcrb

using namespace lcrb;

// ===========================================================================
// Status
// ===========================================================================

extern "C" const char* lcr_last_error_string(void) { return g_error; }

extern "C" const char* lcr_status_string(int status) {
  switch (status) {
    case LCR_OK: return "ok";
    case LCR_ERR_INVALID: return "invalid argument";
    case LCR_ERR_SHAPE: return "unsupported shape";
    case LCR_ERR_CUDA: return "CUDA error";
    case LCR_ERR_TIMEOUT: return "device wait timed out";
    case LCR_ERR_POOL: return "paged KV pool exhausted";
    case LCR_ERR_STATE: return "invalid state";
    case LCR_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown status";
  }
}

extern "C" int lcr_version(void) { return 100; }

// ===========================================================================
// Per-kernel entry points (src/kernels.cuh)
// ===========================================================================

extern "C" int lcr_embedding_lookup(void* out, const void* table, const int32_t* ids, int tokens,
                                    int dim, lcr_stream_t stream) {
  if (tokens == 0) return LCR_OK;
  LCRB_REQUIRE(out && table && ids && tokens > 0 && dim > 0, LCR_ERR_INVALID,
               "embedding lookup: null pointer or non-positive size");
  LCRB_REQUIRE(dim % 8 == 0 && aligned16(out) && aligned16(table), LCR_ERR_SHAPE,
               "embedding lookup needs 16-byte aligned rows (dim %d)", dim);
  embedding_kernel<<<tokens, kSmallThreads, 0, cs(stream)>>>(mb(out), cb(table), ids, dim, INT32_MAX,
                                                             nullptr);
  return launch_status("embedding_lookup");
}

extern "C" int lcr_rmsnorm(void* out, const void* x, const void* weight, int tokens, int dim,
                           float eps, lcr_stream_t stream) {
  if (tokens == 0) return LCR_OK;
  LCRB_REQUIRE(out && x && weight && tokens > 0 && dim > 0, LCR_ERR_INVALID,
               "rmsnorm: null pointer or non-positive size");
  rmsnorm_kernel<<<tokens, kSmallThreads, 0, cs(stream)>>>(mb(out), const_cast<bf16*>(cb(x)), nullptr,
                                                          cb(weight), dim, eps);
  return launch_status("rmsnorm");
}

extern "C" int lcr_add_residual(void* x, const void* delta, int64_t count, lcr_stream_t stream) {
  if (count == 0) return LCR_OK;
  LCRB_REQUIRE(x && delta && count > 0, LCR_ERR_INVALID, "add_residual: bad arguments");
  const int blocks = static_cast<int>(std::min<int64_t>(8192, (count + kSmallThreads - 1) / kSmallThreads));
  add_residual_kernel<<<blocks, kSmallThreads, 0, cs(stream)>>>(mb(x), cb(delta), count);
  return launch_status("add_residual");
}

extern "C" int lcr_add_residual_rmsnorm(void* out, void* x, const void* delta, const void* weight,
                                        int tokens, int dim, float eps, lcr_stream_t stream) {
  if (tokens == 0) return LCR_OK;
  LCRB_REQUIRE(out && x && delta && weight && tokens > 0 && dim > 0, LCR_ERR_INVALID,
               "add_residual_rmsnorm: null pointer or non-positive size");
  rmsnorm_kernel<<<tokens, kSmallThreads, 0, cs(stream)>>>(mb(out), mb(x), cb(delta), cb(weight), dim,
                                                          eps);
  return launch_status("add_residual_rmsnorm");
}

extern "C" int lcr_swiglu(void* out, const void* gate, const void* up, int64_t count,
                          lcr_stream_t stream) {
  if (count == 0) return LCR_OK;
  LCRB_REQUIRE(out && gate && up && count > 0, LCR_ERR_INVALID, "swiglu: bad arguments");
  const int blocks = static_cast<int>(std::min<int64_t>(8192, (count + kSmallThreads - 1) / kSmallThreads));
  swiglu_kernel<<<blocks, kSmallThreads, 0, cs(stream)>>>(mb(out), cb(gate), cb(up), count, count, 1);
  return launch_status("swiglu");
}

extern "C" int lcr_swiglu_strided(void* out, const void* gate, const void* up, int tokens, int width,
                                  int src_row_stride, lcr_stream_t stream) {
  if (tokens == 0) return LCR_OK;
  LCRB_REQUIRE(out && gate && up && tokens > 0 && width > 0 && src_row_stride >= width,
               LCR_ERR_INVALID, "swiglu_strided: bad arguments");
  const int64_t total = static_cast<int64_t>(tokens) * width;
  const int blocks = static_cast<int>(std::min<int64_t>(8192, (total + kSmallThreads - 1) / kSmallThreads));
  swiglu_kernel<<<blocks, kSmallThreads, 0, cs(stream)>>>(mb(out), cb(gate), cb(up), width,
                                                         src_row_stride, tokens);
  return launch_status("swiglu_strided");
}

extern "C" int lcr_rope_q(void* q_heads, const void* q_proj, const float* inv_freq, int tokens,
                          int start_position, int num_heads, int head_dim, int src_row_stride,
                          lcr_stream_t stream) {
  if (tokens == 0) return LCR_OK;
  LCRB_REQUIRE(q_heads && q_proj && inv_freq && tokens > 0 && num_heads > 0 && head_dim > 0 &&
                   head_dim % 2 == 0,
               LCR_ERR_INVALID, "rope_q: bad arguments");
  const dim3 grid(static_cast<unsigned>(tokens), static_cast<unsigned>(num_heads));
  const int block = std::min(64, ((head_dim / 2 + 31) / 32) * 32);
  rope_q_kernel<<<grid, block, 0, cs(stream)>>>(mb(q_heads), cb(q_proj), inv_freq, tokens,
                                                start_position, head_dim, src_row_stride);
  return launch_status("rope_q");
}

extern "C" int lcr_rope_write_kv(const lcr_kv_view* view, const void* k_proj, const void* v_proj,
                                 const float* inv_freq, int tokens, int start_position, int paged,
                                 int src_row_stride, lcr_stream_t stream) {
  if (tokens == 0) return LCR_OK;
  LCRB_REQUIRE(view && view->keys && view->values && k_proj && v_proj && inv_freq && tokens > 0,
               LCR_ERR_INVALID, "rope_write_kv: bad arguments");
  LCRB_REQUIRE(!paged || view->page_table != nullptr, LCR_ERR_INVALID,
               "rope_write_kv: paged layout without a page table");
  const dim3 grid(static_cast<unsigned>(tokens), static_cast<unsigned>(view->num_kv_heads));
  const int block = std::min(64, ((view->head_dim + 31) / 32) * 32);
  rope_write_kv_kernel<<<grid, block, 0, cs(stream)>>>(
      mb(view->keys), mb(view->values), paged ? view->page_table : nullptr, view->page_size,
      view->page_stride, view->head_stride, view->head_dim, cb(k_proj), cb(v_proj), inv_freq,
      start_position, src_row_stride);
  return launch_status("rope_write_kv");
}

extern "C" size_t lcr_decode_attention_scratch_floats(int num_heads, int head_dim, int splits) {
  if (splits <= 1) return 0;
  return static_cast<size_t>(num_heads) * splits * (2 + head_dim);
}

extern "C" int lcr_choose_attention_splits(int num_kv_heads, int seq_len, int multiprocessors) {
  // The reference's rule (src/kernels/attention.cu:419-431): about two blocks
  // per SM, at least 256 positions per split, at most 64 splits.
  const int wanted = std::max(1, 2 * multiprocessors);
  int splits = (wanted + num_kv_heads - 1) / std::max(1, num_kv_heads);
  splits = std::min(splits, std::max(1, seq_len / 256));
  return std::max(1, std::min(splits, 64));
}

extern "C" int lcr_causal_softmax(void* probs, const float* scores, int num_heads, int rows, int keys,
                                  int start_position, lcr_stream_t stream) {
  if (rows == 0 || num_heads == 0) return LCR_OK;
  LCRB_REQUIRE(probs && scores && num_heads > 0 && rows > 0 && keys > 0 && start_position >= 0, LCR_ERR_INVALID,
               "causal_softmax: null pointer or bad size");
  LCRB_REQUIRE(rows <= 65535 * 64 && num_heads <= 65535, LCR_ERR_SHAPE, "causal_softmax: %d rows x %d heads",
               rows, num_heads);
  causal_softmax_kernel<<<dim3(rows, num_heads), kSmallThreads, 0, cs(stream)>>>(mb(probs), scores, rows, keys,
                                                                                start_position);
  return launch_status("causal_softmax");
}

extern "C" int lcr_merge_heads(void* out, const void* heads, int tokens, int num_heads, int head_dim,
                               lcr_stream_t stream) {
  if (tokens == 0) return LCR_OK;
  LCRB_REQUIRE(out && heads && tokens > 0 && num_heads > 0 && head_dim > 0, LCR_ERR_INVALID,
               "merge_heads: null pointer or non-positive size");
  LCRB_REQUIRE(head_dim % 8 != 0 || (aligned16(out) && aligned16(heads)), LCR_ERR_SHAPE,
               "merge_heads: buffers must be 16-byte aligned");
  const long long units = static_cast<long long>(tokens) * num_heads * head_dim / (head_dim % 8 == 0 ? 8 : 1);
  const int blocks = static_cast<int>(std::min<long long>(4096, (units + kSmallThreads - 1) / kSmallThreads));
  merge_heads_kernel<<<blocks, kSmallThreads, 0, cs(stream)>>>(mb(out), cb(heads), tokens, num_heads, head_dim);
  return launch_status("merge_heads");
}

extern "C" int lcr_gather_kv(void* out_keys, void* out_values, const lcr_kv_view* view, int positions,
                             lcr_stream_t stream) {
  if (positions == 0) return LCR_OK;
  LCRB_REQUIRE(out_keys && out_values && view && view->keys && view->values && positions > 0, LCR_ERR_INVALID,
               "gather_kv: null pointer or non-positive size");
  LCRB_REQUIRE(positions <= 65535 * 64 && view->num_kv_heads > 0 && view->num_kv_heads <= 65535 &&
                   view->head_dim > 0 && (view->page_table == nullptr || view->page_size > 0),
               LCR_ERR_SHAPE, "gather_kv: bad view or %d positions", positions);
  gather_kv_kernel<<<dim3(positions, view->num_kv_heads), 64, 0, cs(stream)>>>(
      mb(out_keys), mb(out_values), cb(view->keys), cb(view->values), view->page_table, view->page_size,
      view->page_stride, view->head_stride, view->head_dim, positions);
  return launch_status("gather_kv");
}

extern "C" int lcr_decode_attention(void* out, const void* q, const lcr_kv_view* view, int num_heads,
                                    int heads_per_kv, int seq_len, float scale, int paged, int splits,
                                    float* scratch, lcr_stream_t stream) {
  LCRB_REQUIRE(seq_len > 0, LCR_ERR_INVALID, "decode attention needs at least one cached position");
  LCRB_REQUIRE(splits >= 1, LCR_ERR_INVALID, "split count must be positive, got %d", splits);
  LCRB_REQUIRE(view && out && q && view->keys && view->values, LCR_ERR_INVALID,
               "decode attention: null pointer");
  LCRB_REQUIRE(view->head_dim % 32 == 0, LCR_ERR_SHAPE,
               "decode attention needs head_dim to be a multiple of the warp width, got %d",
               view->head_dim);
  LCRB_REQUIRE(heads_per_kv > 0 && num_heads == heads_per_kv * view->num_kv_heads, LCR_ERR_INVALID,
               "decode attention: %d heads is not %d x %d", num_heads, heads_per_kv,
               view->num_kv_heads);
  LCRB_REQUIRE(!paged || (view->page_table && view->page_size % kAttnBlock == 0), LCR_ERR_SHAPE,
               "paged decode attention needs a page table and a page size that is a multiple of %d",
               kAttnBlock);
  LCRB_REQUIRE(aligned16(view->keys) && aligned16(view->values) && aligned16(q), LCR_ERR_SHAPE,
               "decode attention needs 16-byte aligned cache and query");
  // A split that would leave blocks with no positions at all is pointless
  // (src/kernels/attention.cu:450-451); so is one shorter than a stage.
  splits = std::min(splits, std::max(1, (seq_len + kAttnBlock - 1) / kAttnBlock));
  LCRB_REQUIRE(splits == 1 || scratch != nullptr, LCR_ERR_INVALID,
               "a split decode attention needs scratch space for the partials");
  AttnArgs a = {};
  a.q = cb(q);
  a.kpool = mb(view->keys);
  a.vpool = mb(view->values);
  a.tables = view->page_table;
  a.table_seq_stride = 0;
  a.max_pages = INT32_MAX / 2;
  a.pool_pages = INT32_MAX;
  a.page_size = paged ? view->page_size : 1;
  a.page_stride = view->page_stride;
  a.head_stride = view->head_stride;
  a.seq_stride = 0;
  a.max_seq = paged ? INT32_MAX : std::max(1, view->head_stride / std::max(1, view->head_dim));
  a.seq_len = seq_len;
  a.splits = splits;
  a.scale_log2 = scale * kLog2e;
  a.out = mb(out);
  a.partials = scratch;
  a.status = nullptr;
  LCRB_TRY(attn_launch(a, false, view->head_dim, heads_per_kv, paged != 0, view->num_kv_heads, 1,
                       cs(stream), false));
  if (splits > 1) return attn_merge_launch(mb(out), scratch, num_heads, view->head_dim, splits, cs(stream));
  return LCR_OK;
}

extern "C" size_t lcr_sample_scratch_floats(int vocab, int top_k) {
  (void)vocab;
  (void)top_k;
  return 8;  // per-row parameters staged on the device
}

extern "C" int lcr_sample(int32_t* out_id, const float* logits, int vocab, float temperature,
                          int top_k, float top_p, float uniform, float* scratch,
                          lcr_stream_t stream) {
  LCRB_REQUIRE(vocab > 0, LCR_ERR_INVALID, "cannot sample from an empty vocabulary");
  LCRB_REQUIRE(out_id && logits && scratch, LCR_ERR_INVALID, "sample: null pointer");
  if (temperature > 0.0f) {
    LCRB_REQUIRE(top_p > 0.0f && top_p <= 1.0f, LCR_ERR_INVALID, "top_p must be in (0, 1], got %g",
                 static_cast<double>(top_p));
  }
  // The parameters travel by value in the launch: no host buffer is read at
  // run time, so the call may be captured in a graph. (The scratch the
  // reference's signature carries stays unused.)
  SampleArgs a = {};
  a.logits = logits;
  a.row_stride = vocab;
  a.vocab = vocab;
  a.inline_params = 1;
  a.inv_temperature_v = temperature > 0.0f ? 1.0f / temperature : 0.0f;
  a.top_k_v = top_k;
  a.top_p_v = top_p;
  a.uniform_v = uniform;
  a.out = out_id;
  return sample_launch(a, 1, cs(stream), false);
}

extern "C" int lcr_gemm_nt(void* y, int y_fp32, const void* x, const void* w, int rows,
                           int in_features, int out_features, lcr_stream_t stream) {
  if (rows == 0 || out_features == 0) return LCR_OK;
  LCRB_REQUIRE(y && x && w && rows > 0 && in_features > 0 && out_features > 0, LCR_ERR_INVALID,
               "gemm_nt: null pointer or non-positive size");
  const int epi = y_fp32 ? EPI_STORE_F32 : EPI_STORE;
  if (rows >= 16 && in_features % kTcSlabK == 0 && aligned16(x) && aligned16(w)) {
    // Batched: tcgen05 tiles of 128 weight rows x up to 128 batch rows.
    const int nb = gemm_tc_batch_tile(rows);
    CUtensorMap wmap, xmap;
    LCRB_TRY(make_kmajor_map(&wmap, w, out_features, in_features, 1, kTcTileM, 1));
    LCRB_TRY(make_kmajor_map(&xmap, x, rows, in_features, 1, nb, 1));
    TcArgs a = {};
    a.n_out = out_features;
    a.K = in_features;
    a.rows = rows;
    a.splits = 1;
    a.ldy = out_features;
    a.ctas = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&a.ctas, cudaDevAttrMultiProcessorCount, dev);
    if (y_fp32) a.yf = reinterpret_cast<float*>(y);
    else a.y = mb(y);
    return gemm_tc_launch(a, wmap, xmap, nb, epi, 1, cs(stream), false);
  }
  if (gemv_supported(in_features, PRO_PLAIN, epi) && aligned16(x) && aligned16(w)) {
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    const int per = gemv_outputs_per_chunk(in_features, epi);
    const int chunks = (out_features + per - 1) / per;
    CUtensorMap map;
    LCRB_TRY(make_weight_map(&map, w, out_features, in_features, false));
    for (int r = 0; r < rows; ++r) {
      GemvArgs a = {};
      a.w = cb(w);
      a.n_out = out_features;
      a.x_in = cb(x) + static_cast<size_t>(r) * in_features;
      if (y_fp32) a.yf = reinterpret_cast<float*>(y) + static_cast<size_t>(r) * out_features;
      else a.y = mb(y) + static_cast<size_t>(r) * out_features;
      LCRB_TRY(gemv_launch(a, map, in_features, PRO_PLAIN, epi, std::min(chunks, sms), cs(stream), false));
    }
    return LCR_OK;
  }
  const long long warps = static_cast<long long>(rows) * out_features;
  const int blocks = static_cast<int>((warps * 32 + 255) / 256);
  gemm_nt_simple_kernel<<<blocks, 256, 0, cs(stream)>>>(y, y_fp32, cb(x), cb(w), rows, in_features,
                                                        out_features);
  return launch_status("gemm_nt");
}
