// The decode context: Model (src/model.h:60-127) for the B200.
//
// A step is one token of one sequence through every layer. It is launched as
// a chain of 5 kernels per layer plus the output head, with programmatic
// dependent launch so each kernel's weight stream starts while the previous
// kernel drains, and captured once as a CUDA graph. Everything a step needs
// from the host -- the token and its position -- lives in device memory, and
// the output head's last CTA writes the argmax back there, so a greedy
// generation is a sequence of graph launches with no host round trip.
//
//   per layer  qkv GEMV   (RMSNorm prologue; embedding row for layer 0)
//              attention  (RoPE of q and the new k, KV write, split-K, merge)
//              o GEMV     (residual epilogue)
//              gate/up GEMV (RMSNorm prologue, SwiGLU epilogue)
//              down GEMV  (residual epilogue)
//   then       lm_head GEMV (final-norm prologue, fp32 logits + argmax)
//
// The KV cache is the reference's (src/kv_cache.cu): contiguous
// [layer][kv_head][max_seq][d], or a paged pool of [kv_head][page][d] pages
// with one table per layer, pages handed out layer by layer from a counter --
// optionally through a seeded permutation of the pool (shuffled physical
// order).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "batch_internal.h"
#include "common.cuh"
#include "dispatch.h"
#include "gemv_dispatch.h"
#include "rope_table.h"
#include "tmap.h"
#include "lcr_b200.h"
#include "mega_dispatch.h"

namespace lcrb {

// The RoPE table of src/config.cpp:223-259 (double math, float table).
std::vector<float> rope_inv_freq(const lcr_model_desc& d) {
  const int pairs = d.head_dim / 2;
  std::vector<float> f(static_cast<size_t>(pairs));
  for (int i = 0; i < pairs; ++i) {
    f[static_cast<size_t>(i)] = static_cast<float>(
        1.0 / std::pow(static_cast<double>(d.rope_theta), static_cast<double>(2 * i) / d.head_dim));
  }
  if (!d.rope_scaling) return f;
  const double old_context = d.rope_original_max_position_embeddings;
  const double low_wavelen = old_context / d.rope_low_freq_factor;
  const double high_wavelen = old_context / d.rope_high_freq_factor;
  for (int i = 0; i < pairs; ++i) {
    const double freq = f[static_cast<size_t>(i)];
    const double wavelen = 2.0 * M_PI / freq;
    double scaled;
    if (wavelen < high_wavelen) {
      scaled = freq;
    } else if (wavelen > low_wavelen) {
      scaled = freq / d.rope_factor;
    } else {
      const double smooth = (old_context / wavelen - d.rope_low_freq_factor) /
                            (d.rope_high_freq_factor - d.rope_low_freq_factor);
      scaled = (1.0 - smooth) * (freq / d.rope_factor) + smooth * freq;
    }
    f[static_cast<size_t>(i)] = static_cast<float>(scaled);
  }
  return f;
}

}  // namespace lcrb

using namespace lcrb;

namespace {

// Bit 4: the persistent step with fp32 activations instead of the
// reference's bf16 storage rounding (closer to the fp32 evaluation, slower).
// Bit 6: lcr_prefill runs the prompt one decode step per token instead of
// in tcgen05 chunks. Bit 7: the persistent step's attention phase on CUDA
// cores instead of the tensor pipe. Bit 8: the persistent step's phases meet
// at grid barriers instead of exchanging tagged words (ll.cuh).
// Bit 5 (tests only): the persistent step's waits give up after 50 ms and CTA
// 0 skips its first arrival at a grid barrier (with the exchange: its first
// q/k/v words), so the first wait times out -- the timeout path, exercised
// without faulting or hanging the GPU.
enum : int { kFlagNoPdl = 1, kFlagNoGraph = 2, kFlagNoPersistent = 4, kFlagTrace = 8, kFlagFp32Act = 16,
             kFlagTestTimeout = 32, kFlagPerTokenPrefill = 64, kFlagCudaCoreAttention = 128,
             kFlagGridBarriers = 256 };
// Prompt rows per tcgen05 prefill chunk, and the shortest prompt chunked.
constexpr int kPrefillChunk = 2048;
constexpr int kPrefillChunkMin = 2;
constexpr int kPinnedRing = 256;
constexpr int kTimingSlots = 128;

uint64_t splitmix64(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}


}  // namespace

struct lcr_ctx {
  int device = 0;
  lcr_model_desc d{};
  lcr_options o{};
  int sms = 148;
  cudaStream_t stream = nullptr;
  bool pdl = true;
  bool use_graph = true;
  bool persistent = false;  // the whole step as one cooperative kernel
  bool f32 = false;         // persistent step: fp32 activations

  const bf16* embed = nullptr;
  const bf16* final_norm = nullptr;
  const bf16* lm_head = nullptr;
  std::vector<lcr_layer_weights> layers;

  char* buf = nullptr;
  bf16* x = nullptr;
  float* xsum = nullptr;
  bf16* qkv = nullptr;
  bf16* attn = nullptr;
  bf16* act = nullptr;
  float* qkv_f = nullptr;   // fp32 activations of the persistent step
  float* attn_f = nullptr;
  float* act_f = nullptr;
  float* logits = nullptr;
  float* partials = nullptr;
  unsigned* attn_ctr = nullptr;
  unsigned* sched = nullptr;
  int sched_slots = 0;
  unsigned long long* argmax_acc = nullptr;
  int32_t* state = nullptr;  // [0] token, [1] position
  int32_t* history = nullptr;
  uint32_t* status = nullptr;
  float* inv_freq = nullptr;
  float* sample_params = nullptr;
  int32_t* sampled = nullptr;
  // Low-latency exchange words of the persistent step (ll.cuh), and the
  // per-step epoch base of their tags.
  bool ll = false;
  uint32_t* epoch = nullptr;
  uint32_t* qkv_ll = nullptr;
  unsigned long long* part_ll = nullptr;
  uint32_t* attn_ll = nullptr;
  unsigned long long* x_ll = nullptr;
  uint32_t* act_ll = nullptr;

  bf16* kpool = nullptr;
  bf16* vpool = nullptr;
  int32_t* tables_dev = nullptr;
  std::vector<int32_t> tables_host;
  std::vector<int32_t> order;
  int max_pages = 0, pool_pages = 0, pages_mapped = 0, length = 0;
  int splits = 1;

  MegaLayer* mega_layers = nullptr;  // device copy of the per-layer pointers
  // Tensor maps of every streamed matrix (make_weight_map): [layer * 4 + m],
  // m = 0 qkv, 1 o, 2 gate/up, 3 down; then the lm_head. Host copy for the
  // multi-kernel launches, device copy for the persistent kernel.
  std::vector<CUtensorMap> wmaps;
  CUtensorMap* wmaps_dev = nullptr;
  unsigned* mega_bar = nullptr;
  unsigned long long* trace = nullptr;  // kFlagTrace: per-CTA phase timestamps
  unsigned long long prefetch_bytes = 0;  // persistent step: L2 prefetch lead per CTA
  int split_positions = 0;                // persistent step: cached positions per attention split
  size_t ll_copy_bytes = 0;               // stride of the exchange buffers' replicas

  cudaGraphExec_t exec = nullptr;
  int launches = 0;
  int position = 0;

  int32_t* pinned = nullptr;  // ring of [token, position] pairs
  int ring_next = 0;
  int32_t* pinned_prompt = nullptr;
  size_t pinned_prompt_cap = 0;
  float* pinned_params = nullptr;

  // Tensor maps of the cache rows (16-row boxes, 128-byte swizzle): paged,
  // {K, V} over the whole pool; contiguous, {K, V} per layer. Empty when the
  // cache does not allow them (head_dim not a multiple of 64, pages of other
  // than a multiple of 16 positions). Host copy for the chunked prefill,
  // device copy for the persistent step's tensor-pipe attention.
  std::vector<CUtensorMap> kvmaps;
  CUtensorMap* kvmaps_dev = nullptr;
  // Chunked prefill: a one-slot batch context over the same weights, whose
  // tcgen05 prefill writes this context's cache (created on first use).
  lcr_batch* prefill_engine = nullptr;
  bool prefill_unavailable = false;
  int32_t* prefill_table = nullptr;  // contiguous cache: the one page, {0}
};

namespace {

int q_dim(const lcr_ctx* c) { return c->d.num_heads * c->d.head_dim; }
int kv_dim(const lcr_ctx* c) { return c->d.num_kv_heads * c->d.head_dim; }

int gemv_node(lcr_ctx* c, GemvArgs a, int K, int pro, int epi, int n_out, int* slot, int map) {
  const int per = gemv_outputs_per_chunk(K, epi);
  a.n_out = n_out;
  LCRB_REQUIRE(*slot < c->sched_slots, LCR_ERR_STATE, "GEMV scheduler slots exhausted");
  a.sched = c->sched + 2 * (*slot)++;
  a.status = c->status;
  a.eps = c->d.rms_norm_eps;
  const int want = c->o.gemv_ctas > 0 ? c->o.gemv_ctas : c->sms;
  const int ctas = std::max(1, std::min((n_out + per - 1) / per, want));
  ++c->launches;
  return gemv_launch(a, c->wmaps[static_cast<size_t>(map)], K, pro, epi, ctas, c->stream, c->pdl);
}

int attention_node(lcr_ctx* c, int layer) {
  const lcr_model_desc& d = c->d;
  AttnArgs a = {};
  a.qkv = c->qkv;
  a.qkv_stride = q_dim(c) + 2 * kv_dim(c);
  a.q_dim = q_dim(c);
  a.kv_dim = kv_dim(c);
  a.inv_freq = c->inv_freq;
  a.max_seq = c->o.max_seq;
  if (c->o.paged) {
    a.kpool = c->kpool;
    a.vpool = c->vpool;
    a.tables = c->tables_dev + static_cast<size_t>(layer) * c->max_pages;
    a.table_seq_stride = 0;
    a.max_pages = c->max_pages;
    a.pool_pages = c->pool_pages;
    a.page_size = c->o.page_size;
    a.page_stride = static_cast<long long>(d.num_kv_heads) * c->o.page_size * d.head_dim;
    a.head_stride = static_cast<long long>(c->o.page_size) * d.head_dim;
  } else {
    const size_t layer_elems = static_cast<size_t>(d.num_kv_heads) * c->o.max_seq * d.head_dim;
    a.kpool = c->kpool + layer * layer_elems;
    a.vpool = c->vpool + layer * layer_elems;
    a.page_size = 1;
    a.head_stride = static_cast<long long>(c->o.max_seq) * d.head_dim;
    a.seq_stride = static_cast<long long>(layer_elems);
  }
  a.positions = c->state + 1;
  a.splits = c->splits;
  a.scale_log2 = (1.0f / std::sqrt(static_cast<float>(d.head_dim))) * kLog2e;
  a.out = c->attn;
  a.partials = c->partials;
  a.counters = c->attn_ctr + static_cast<size_t>(layer) * d.num_kv_heads;
  a.status = c->status;
  ++c->launches;
  return attn_launch(a, true, d.head_dim, d.num_heads / d.num_kv_heads, c->o.paged != 0,
                     d.num_kv_heads, 1, c->stream, c->pdl);
}

int enqueue_persistent_step(lcr_ctx* c) {
  const lcr_model_desc& d = c->d;
  MegaArgs a = {};
  a.layers = d.num_layers;
  a.vocab = d.vocab_size;
  a.num_kv = d.num_kv_heads;
  a.max_seq = c->o.max_seq;
  a.splits = c->splits;
  a.eps = d.rms_norm_eps;
  a.scale_log2 = (1.0f / std::sqrt(static_cast<float>(d.head_dim))) * kLog2e;
  a.embed = c->embed;
  a.final_norm = c->final_norm;
  a.lm_head = c->lm_head;
  a.L = c->mega_layers;
  a.wmaps = c->wmaps_dev;
  a.inv_freq = c->inv_freq;
  a.state = c->state;
  a.x = c->x;
  a.xsum = c->xsum;
  a.qkv = c->qkv;
  a.attn = c->attn;
  a.act = c->act;
  a.qkv_f = c->qkv_f;
  a.attn_f = c->attn_f;
  a.act_f = c->act_f;
  a.logits = c->logits;
  a.partials = c->partials;
  a.attn_ctr = c->attn_ctr;
  a.bar = c->mega_bar;
  a.argmax_acc = c->argmax_acc;
  a.argmax_done = c->sched;  // slot 0 of the scheduler words
  a.history = c->history;
  a.history_len = c->o.max_seq;
  a.status = c->status;
  a.kpool = c->kpool;
  a.vpool = c->vpool;
  a.trace = c->trace;
  a.prefetch_bytes = c->prefetch_bytes;
  a.split_positions = c->split_positions;
  if (d.head_dim == 64 && !(c->o.flags & kFlagCudaCoreAttention)) {
    a.kvmaps = c->kvmaps_dev;  // nullptr when the cache has no tensor maps
    a.kvmap_layer_stride = c->o.paged ? 0 : 2;
  }
  if (c->ll) {
    a.ll = 1;
    a.epoch = c->epoch;
    a.qkv_ll = c->qkv_ll;
    a.part_ll = c->part_ll;
    a.attn_ll = c->attn_ll;
    a.x_ll = c->x_ll;
    a.act_ll = c->act_ll;
    a.ll_copy_bytes = c->ll_copy_bytes;
  }
  a.wait_ns = (c->o.flags & kFlagTestTimeout) ? 50000000ull : kWaitLimitNs;
  a.test_skip_arrival = (c->o.flags & kFlagTestTimeout) ? 1 : 0;
  if (c->o.paged) {
    a.tables = c->tables_dev;
    a.max_pages = c->max_pages;
    a.pool_pages = c->pool_pages;
    a.page_size = c->o.page_size;
    a.page_stride = static_cast<long long>(d.num_kv_heads) * c->o.page_size * d.head_dim;
    a.head_stride = static_cast<long long>(c->o.page_size) * d.head_dim;
  } else {
    a.head_stride = static_cast<long long>(c->o.max_seq) * d.head_dim;
    a.layer_stride = static_cast<long long>(d.num_kv_heads) * c->o.max_seq * d.head_dim;
  }
  c->launches = 1;
  return mega_launch(a, d.hidden_size, d.num_heads * d.head_dim, d.intermediate_size, d.head_dim,
                     d.num_heads / d.num_kv_heads, c->o.paged != 0, c->f32, c->sms, c->stream);
}

// Launches one decode step on the context's stream.
int enqueue_step(lcr_ctx* c) {
  if (c->persistent) return enqueue_persistent_step(c);
  const lcr_model_desc& d = c->d;
  const int H = d.hidden_size, F = d.intermediate_size;
  int slot = 1;  // slot 0 belongs to the persistent kernel's argmax hand-off
  c->launches = 0;
  for (int l = 0; l < d.num_layers; ++l) {
    const lcr_layer_weights& w = c->layers[static_cast<size_t>(l)];
    {
      GemvArgs a = {};
      a.w = static_cast<const bf16*>(w.qkv_proj);
      a.norm_w = static_cast<const bf16*>(w.input_norm);
      a.y = c->qkv;
      int pro = PRO_NORM;
      if (l == 0) {
        pro = PRO_EMBED_NORM;
        a.embed = c->embed;
        a.token = c->state;
        a.vocab = d.vocab_size;
        a.x_out = c->x;
        a.xsum_out = c->xsum;
      } else {
        a.x_in = c->x;
        a.xsum = c->xsum;
      }
      LCRB_TRY(gemv_node(c, a, H, pro, EPI_STORE, q_dim(c) + 2 * kv_dim(c), &slot, 4 * l));
    }
    LCRB_TRY(attention_node(c, l));
    {
      GemvArgs a = {};
      a.w = static_cast<const bf16*>(w.o_proj);
      a.x_in = c->attn;
      a.resid = c->x;
      a.resid_sum = c->xsum;
      LCRB_TRY(gemv_node(c, a, q_dim(c), PRO_PLAIN, EPI_RESID, H, &slot, 4 * l + 1));
    }
    {
      GemvArgs a = {};
      a.w = static_cast<const bf16*>(w.gate_up_proj);
      a.x_in = c->x;
      a.xsum = c->xsum;
      a.norm_w = static_cast<const bf16*>(w.post_attention_norm);
      a.y = c->act;
      LCRB_TRY(gemv_node(c, a, H, PRO_NORM, EPI_SWIGLU, F, &slot, 4 * l + 2));
    }
    {
      GemvArgs a = {};
      a.w = static_cast<const bf16*>(w.down_proj);
      a.x_in = c->act;
      a.resid = c->x;
      a.resid_sum = c->xsum;
      LCRB_TRY(gemv_node(c, a, F, PRO_PLAIN, EPI_RESID, H, &slot, 4 * l + 3));
    }
  }
  GemvArgs a = {};
  a.w = c->lm_head;
  a.x_in = c->x;
  a.xsum = c->xsum;
  a.norm_w = c->final_norm;
  a.yf = c->logits;
  a.argmax_acc = c->argmax_acc;
  a.state_token = c->state;
  a.state_pos = c->state + 1;
  a.history = c->history;
  a.history_len = c->o.max_seq;
  a.advance = 1;
  return gemv_node(c, a, H, PRO_NORM, EPI_LOGITS_ARGMAX, d.vocab_size, &slot, 4 * d.num_layers);
}

int build_graph(lcr_ctx* c) {
  if (!c->use_graph || c->exec != nullptr) return LCR_OK;
  cudaGraph_t graph = nullptr;
  LCRB_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  const int st = enqueue_step(c);
  const cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
  if (st != LCR_OK) {
    if (graph) cudaGraphDestroy(graph);
    return st;
  }
  if (e != cudaSuccess) return fail(LCR_ERR_CUDA, "step capture failed: %s", cudaGetErrorString(e));
  const cudaError_t ie = cudaGraphInstantiate(&c->exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) {
    c->exec = nullptr;
    return fail(LCR_ERR_CUDA, "step graph instantiation failed: %s", cudaGetErrorString(ie));
  }
  return LCR_OK;
}

int launch_steps(lcr_ctx* c, int steps) {
  LCRB_CUDA(cudaSetDevice(c->device));
  if (c->use_graph) {
    LCRB_TRY(build_graph(c));
    for (int i = 0; i < steps; ++i) LCRB_CUDA(cudaGraphLaunch(c->exec, c->stream));
    return LCR_OK;
  }
  for (int i = 0; i < steps; ++i) LCRB_TRY(enqueue_step(c));
  return LCR_OK;
}

int check_status(lcr_ctx* c) {
  // The status word comes back through a pinned word (an asynchronous copy;
  // a pageable destination would be a staged, slower one).
  uint32_t* pst = reinterpret_cast<uint32_t*>(c->pinned + 2 * kPinnedRing);
  *pst = 0;
  LCRB_CUDA(cudaMemcpyAsync(pst, c->status, sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream));
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  const uint32_t st = *pst;
  if (st == 0) return LCR_OK;
  LCRB_CUDA(cudaMemsetAsync(c->status, 0, sizeof st, c->stream));
  if (st & kStatusAbort) {
    // A stopped step may leave the many-split merge counters and the argmax
    // hand-off part way: start the next step from zero. Its exchange words
    // may carry tags the next step would expect (it did not advance the
    // epoch): move the epoch well past them.
    LCRB_CUDA(cudaMemsetAsync(c->attn_ctr, 0, sizeof(unsigned) * c->d.num_layers * c->d.num_kv_heads, c->stream));
    LCRB_CUDA(cudaMemsetAsync(c->sched, 0, 2 * sizeof(unsigned), c->stream));
    LCRB_CUDA(cudaMemsetAsync(c->argmax_acc, 0, sizeof(unsigned long long), c->stream));
    uint32_t ep = 0;
    LCRB_CUDA(cudaMemcpyAsync(&ep, c->epoch, sizeof ep, cudaMemcpyDeviceToHost, c->stream));
    LCRB_CUDA(cudaStreamSynchronize(c->stream));
    ep += 4096u;
    LCRB_CUDA(cudaMemcpyAsync(c->epoch, &ep, sizeof ep, cudaMemcpyHostToDevice, c->stream));
  }
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  if (st & (kStatusTimeoutFull | kStatusTimeoutEmpty | kStatusTimeoutBarrier | kStatusAbort)) {
    return fail(LCR_ERR_TIMEOUT, "a device-side wait gave up (status 0x%x)", st);
  }
  if (st & kStatusBadToken) return fail(LCR_ERR_INVALID, "token id outside the vocabulary (status 0x%x)", st);
  if (st & kStatusBadPage) return fail(LCR_ERR_POOL, "page table entry outside the pool (status 0x%x)", st);
  return fail(LCR_ERR_STATE, "position outside the KV cache (status 0x%x)", st);
}

int stage_state(lcr_ctx* c, const int32_t* token_src, int position) {
  int32_t* slot = c->pinned + 2 * c->ring_next;
  c->ring_next = (c->ring_next + 1) % kPinnedRing;
  if (token_src == nullptr) {
    slot[1] = position;
    LCRB_CUDA(cudaMemcpyAsync(c->state + 1, slot + 1, sizeof(int32_t), cudaMemcpyHostToDevice, c->stream));
    return LCR_OK;
  }
  // The token is read here, on the host, and travels with the position in
  // one 8-byte copy (one copy fewer per step than copying each from where
  // it lies).
  slot[0] = *token_src;
  slot[1] = position;
  LCRB_CUDA(cudaMemcpyAsync(c->state, slot, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, c->stream));
  return LCR_OK;
}

// The chunked-prefill engine and the tensor maps of this context's cache
// rows (created on first use). Returns false where the chunked path does not
// apply: the fp32-activation step, a paged cache with pages of other than a
// multiple of 16 positions, or a model the batch kernels are not built for
// (the prompt then runs one decode step per token).
bool prefill_engine_ready(lcr_ctx* c) {
  if (c->prefill_engine) return true;
  if (c->prefill_unavailable) return false;
  c->prefill_unavailable = true;
  const lcr_model_desc& d = c->d;
  if (c->f32 || (c->o.flags & kFlagPerTokenPrefill)) return false;
  lcr_weights w = {};
  w.embedding = c->embed;
  w.final_norm = c->final_norm;
  w.lm_head = c->lm_head;
  w.layers = c->layers.data();
  lcr_batch_options bo = {};
  bo.device = c->device;
  bo.max_batch = 1;
  bo.max_seq = 16;
  bo.page_size = 16;
  bo.pool_pages = 1;
  bo.flags = 0;
  if (c->kvmaps.empty()) return false;
  lcr_batch* engine = nullptr;
  if (lcr_batch_create(&d, &w, &bo, &engine) != LCR_OK) return false;
  int st = LCR_OK;
  if (!c->o.paged) {
    if (cudaMalloc(&c->prefill_table, sizeof(int32_t)) != cudaSuccess) st = LCR_ERR_CUDA;
    if (st == LCR_OK && cudaMemset(c->prefill_table, 0, sizeof(int32_t)) != cudaSuccess) st = LCR_ERR_CUDA;
  }
  if (st != LCR_OK) {
    lcr_batch_destroy(engine);
    cudaFree(c->prefill_table);
    c->prefill_table = nullptr;
    return false;
  }
  c->prefill_engine = engine;
  c->prefill_unavailable = false;
  return true;
}

// Prompt positions [c->position, c->position + count) in tcgen05 chunks of up
// to kPrefillChunk rows: projections as GEMMs over the chunk's rows, causal
// attention over the cache, K/V written into this context's cache. Leaves the
// last row's logits in c->logits and the device state as the per-token path
// does (next token = their argmax, position advanced, history entry set).
int prefill_chunked(lcr_ctx* c, const int32_t* tokens, int count) {
  const lcr_model_desc& d = c->d;
  PrefillKv kv = {};
  kv.kpool = c->kpool;
  kv.vpool = c->vpool;
  kv.kvmaps = c->kvmaps.data();
  if (c->o.paged) {
    kv.layer_elems = 0;
    kv.table = c->tables_dev;
    kv.table_layer_stride = static_cast<size_t>(c->max_pages);
    kv.page_size = c->o.page_size;
    kv.pool_pages = c->pool_pages;
    kv.kvmap_layer_stride = 0;
    kv.limit = c->max_pages * c->o.page_size;
  } else {
    kv.layer_elems = static_cast<size_t>(d.num_kv_heads) * c->o.max_seq * d.head_dim;
    kv.table = c->prefill_table;
    kv.table_layer_stride = 0;
    kv.page_size = c->o.max_seq;
    kv.pool_pages = 1;
    kv.kvmap_layer_stride = 2;
    kv.limit = c->o.max_seq;
  }
  // The engine's stream follows everything queued on this context's stream.
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  for (int done = 0; done < count;) {
    const int n = std::min(kPrefillChunk, count - done);
    LCRB_TRY(batch_prefill_into(c->prefill_engine, kv, tokens + done, n, c->position + done, c->logits));
    done += n;
  }
  LCRB_TRY(batch_check_status(c->prefill_engine));
  // Device state after the last prompt token: greedy pick of its logits.
  int32_t* slot = c->pinned + 2 * c->ring_next;
  c->ring_next = (c->ring_next + 1) % kPinnedRing;
  slot[0] = tokens[count - 1];
  slot[1] = c->position + count - 1;
  LCRB_CUDA(cudaMemcpyAsync(c->state, slot, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, c->stream));
  SampleArgs s = {};
  s.logits = c->logits;
  s.row_stride = d.vocab_size;
  s.vocab = d.vocab_size;
  s.inline_params = 1;
  s.inv_temperature_v = 0.f;
  s.top_p_v = 1.f;
  s.top_k_v = 0;
  s.out = c->sampled;
  s.state_token = c->state;
  s.state_pos = c->state + 1;
  s.history = c->history;
  s.history_len = c->o.max_seq;
  s.advance = 1;
  return sample_launch(s, 1, c->stream, false);
}

void release(lcr_ctx* c) {
  if (c == nullptr) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->exec) cudaGraphExecDestroy(c->exec);
  lcr_batch_destroy(c->prefill_engine);
  cudaFree(c->prefill_table);
  cudaFree(c->kvmaps_dev);
  cudaFree(c->buf);
  cudaFree(c->kpool);
  cudaFree(c->vpool);
  cudaFree(c->tables_dev);
  cudaFree(c->mega_layers);
  cudaFree(c->wmaps_dev);
  cudaFree(c->mega_bar);
  cudaFree(c->trace);
  cudaFreeHost(c->pinned);
  cudaFreeHost(c->pinned_prompt);
  cudaFreeHost(c->pinned_params);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

}  // namespace

// ===========================================================================

extern "C" int lcr_ctx_create(const lcr_model_desc* desc, const lcr_weights* weights,
                              const lcr_options* options, lcr_ctx** out) {
  LCRB_REQUIRE(desc && weights && options && out, LCR_ERR_INVALID, "lcr_ctx_create: null argument");
  *out = nullptr;
  const lcr_model_desc& d = *desc;
  LCRB_REQUIRE(d.hidden_size > 0 && d.intermediate_size > 0 && d.num_layers > 0, LCR_ERR_INVALID,
               "model has a non-positive hidden_size, intermediate_size, or num_hidden_layers");
  LCRB_REQUIRE(d.num_heads > 0 && d.num_kv_heads > 0 && d.num_heads % d.num_kv_heads == 0,
               LCR_ERR_INVALID, "num_attention_heads (%d) must be a multiple of num_key_value_heads (%d)",
               d.num_heads, d.num_kv_heads);
  LCRB_REQUIRE(d.head_dim == 64 || d.head_dim == 128, LCR_ERR_SHAPE,
               "decode attention is compiled for head_dim 64 or 128, this model has %d", d.head_dim);
  LCRB_REQUIRE(d.vocab_size > 0 && d.rms_norm_eps > 0.f && d.rope_theta > 1.f, LCR_ERR_INVALID,
               "bad vocab_size / rms_norm_eps / rope_theta");
  const int qd = d.num_heads * d.head_dim, kvd = d.num_kv_heads * d.head_dim;
  LCRB_REQUIRE(gemv_supported(d.hidden_size, PRO_NORM, EPI_SWIGLU) &&
                   gemv_supported(qd, PRO_PLAIN, EPI_RESID) &&
                   gemv_supported(d.intermediate_size, PRO_PLAIN, EPI_RESID),
               LCR_ERR_SHAPE, "no streaming GEMV for hidden %d / q_dim %d / ffn %d", d.hidden_size, qd,
               d.intermediate_size);
  LCRB_REQUIRE(weights->embedding && weights->final_norm && weights->layers, LCR_ERR_INVALID,
               "lcr_weights: null embedding, final_norm or layers");
  const lcr_options& o = *options;
  LCRB_REQUIRE(o.max_seq > 0, LCR_ERR_INVALID, "max_seq must be positive");
  LCRB_REQUIRE(!o.paged || (o.page_size > 0 && o.page_size % 16 == 0), LCR_ERR_SHAPE,
               "paged KV cache needs a page size that is a positive multiple of 16, got %d",
               o.page_size);

  int devices = 0;
  if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) {
    cudaGetLastError();
    return fail(LCR_ERR_NO_DEVICE, "no CUDA device");
  }
  LCRB_REQUIRE(o.device >= 0 && o.device < devices, LCR_ERR_INVALID, "device %d of %d", o.device, devices);
  LCRB_CUDA(cudaSetDevice(o.device));
  LCRB_REQUIRE(on_device(weights->embedding, o.device) && on_device(weights->final_norm, o.device), LCR_ERR_INVALID,
               "lcr_weights: the weights are not in device %d's memory", o.device);
  int major = 0;
  LCRB_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, o.device));
  LCRB_REQUIRE(major == 10, LCR_ERR_NO_DEVICE, "this library is built for sm_100a; device %d is sm_%d",
               o.device, major * 10);

  lcr_ctx* c = new (std::nothrow) lcr_ctx();
  LCRB_REQUIRE(c != nullptr, LCR_ERR_INVALID, "out of host memory");
  c->device = o.device;
  c->d = d;
  c->o = o;
  c->pdl = (o.flags & kFlagNoPdl) == 0;
  c->use_graph = (o.flags & kFlagNoGraph) == 0;
  cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, o.device);
  c->embed = static_cast<const bf16*>(weights->embedding);
  c->final_norm = static_cast<const bf16*>(weights->final_norm);
  c->lm_head = static_cast<const bf16*>(weights->lm_head ? weights->lm_head : weights->embedding);
  c->layers.assign(weights->layers, weights->layers + d.num_layers);
  for (const lcr_layer_weights& w : c->layers) {
    if (!(w.input_norm && w.qkv_proj && w.o_proj && w.post_attention_norm && w.gate_up_proj &&
          w.down_proj)) {
      release(c);
      return fail(LCR_ERR_INVALID, "lcr_layer_weights: null tensor pointer");
    }
    for (const void* p : {w.input_norm, w.qkv_proj, w.o_proj, w.post_attention_norm, w.gate_up_proj,
                          w.down_proj}) {
      if (reinterpret_cast<uintptr_t>(p) & 15u) {
        release(c);
        return fail(LCR_ERR_INVALID, "weights must be 16-byte aligned");
      }
    }
  }

  int st = LCR_OK;
  auto cuda = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && st == LCR_OK) st = fail(LCR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  };
  cuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate");

  const int group = d.num_heads / d.num_kv_heads;
  // LCR_PREFETCH_KIB: the persistent step's L2 prefetch lead per CTA, a tuning
  // knob for measurements. 384 KiB per CTA (57 MB over 148 CTAs) measured
  // best on the 1B model; from 768 KiB on, prefetched lines are evicted from
  // L2 before the ring reads them.
  if (const char* env = std::getenv("LCR_PREFETCH_KIB")) {
    c->prefetch_bytes = static_cast<unsigned long long>(std::max(0, std::atoi(env))) << 10;
  } else {
    c->prefetch_bytes = 384ull << 10;
  }
  // LCR_SPLIT_POSITIONS: the cached positions per attention split the
  // persistent step aims at, a tuning knob like the prefetch lead. Each merge
  // hop costs about as much as a few 128-position stages, so a split takes
  // about three stages: one split up to 384 positions (config 2), 18 at 8192
  // (config 3, the one-CTA-per-SM cap).
  // An explicit Options::attention_splits asks for that many splits: the
  // step then splits down to 32-position chunks.
  c->split_positions = o.attention_splits > 0 ? 32 : 384;
  if (const char* env = std::getenv("LCR_SPLIT_POSITIONS")) c->split_positions = std::max(32, std::atoi(env));
  c->persistent = (o.flags & kFlagNoPersistent) == 0 &&
                  mega_supported(d.hidden_size, qd, d.intermediate_size, d.head_dim, group);
  c->f32 = (o.flags & kFlagFp32Act) != 0;
  // Split-K width: about 128 cached positions per split at max_seq (short
  // caches merge fewer partials; measured at config 2: 4 splits 1615 tok/s
  // against 1590 for 8..18), at most one (kv_head, split) CTA per SM.
  c->splits = o.attention_splits > 0
                  ? o.attention_splits
                  : std::max(1, std::min(c->sms / d.num_kv_heads, (o.max_seq + 127) / 128));
  {
    // Keep the last CTA's merge in shared memory (attn_max_staged_splits).
    const int group = d.num_heads / d.num_kv_heads;
    const int cap = d.head_dim == 64 ? attn_max_staged_splits<64, kAttnStages>(group)
                                     : attn_max_staged_splits<128, kAttnStages>(group);
    if (o.attention_splits <= 0) c->splits = std::max(1, std::min(c->splits, cap));
    if (c->persistent) {
      c->splits = std::max(1, std::min({c->splits, mega_max_splits(c->sms, d.num_kv_heads),
                                        kMegaMaxMergeSplits}));
    }
  }
  // One scheduler slot per GEMV node of the step, plus kTimingSlots for
  // lcr_time_gemv (back-to-back launches may overlap, so none share a slot).
  c->sched_slots = 5 * d.num_layers + 8 + kTimingSlots;

  // One allocation for the activations and device state, 256-byte aligned.
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    const size_t at = off;
    off = (off + bytes + 255) / 256 * 256;
    return at;
  };
  const size_t o_x = carve(sizeof(bf16) * d.hidden_size);
  const size_t o_xsum = carve(sizeof(float) * d.hidden_size);
  const size_t o_qkv = carve(sizeof(bf16) * (qd + 2 * kvd));
  const size_t o_attn = carve(sizeof(bf16) * qd);
  const size_t o_act = carve(sizeof(bf16) * d.intermediate_size);
  const size_t o_qkvf = carve(sizeof(float) * (qd + 2 * kvd));
  const size_t o_attnf = carve(sizeof(float) * qd);
  const size_t o_actf = carve(sizeof(float) * d.intermediate_size);
  const size_t o_logits = carve(sizeof(float) * d.vocab_size);
  // Split partial records: (2 + D) floats in the multi-kernel step, (D + 4) in
  // the persistent one.
  const size_t o_part = carve(sizeof(float) * d.num_heads * c->splits * (4 + d.head_dim));
  const size_t o_actr = carve(sizeof(unsigned) * d.num_layers * d.num_kv_heads);
  const size_t o_sched = carve(sizeof(unsigned) * 2 * c->sched_slots);
  const size_t o_amax = carve(sizeof(unsigned long long));
  const size_t o_state = carve(sizeof(int32_t) * 4);
  const size_t o_hist = carve(sizeof(int32_t) * o.max_seq);
  const size_t o_freq = carve(sizeof(float) * d.head_dim / 2);
  const size_t o_sparams = carve(sizeof(float) * 8);
  const size_t o_sampled = carve(sizeof(int32_t) * 4);
  const size_t o_epoch = carve(sizeof(uint32_t));
  // The exchange buffers: qkv, attn, x and act are held in kLLCopies
  // replicas ll_copy_bytes apart (4 KB past a 64 KB multiple, so the
  // replicas start at different offsets within 64 KB).
  {
    const size_t biggest = std::max({sizeof(uint32_t) * (qd + 2 * kvd), sizeof(uint32_t) * qd,
                                     sizeof(unsigned long long) * d.hidden_size,
                                     sizeof(uint32_t) * d.intermediate_size});
    c->ll_copy_bytes = (biggest + 65535) / 65536 * 65536 + 4096;
  }
  const size_t rep = c->ll_copy_bytes * static_cast<size_t>(kLLCopies);
  const size_t o_qkvll = carve(rep);
  const size_t o_partll = carve(sizeof(unsigned long long) * d.num_heads * c->splits * (4 + d.head_dim));
  const size_t o_attnll = carve(rep);
  const size_t o_xll = carve(rep);
  const size_t o_actll = carve(rep);
  if (st == LCR_OK) cuda(cudaMalloc(&c->buf, off), "cudaMalloc(activations)");
  if (st == LCR_OK) cuda(cudaMemset(c->buf, 0, off), "cudaMemset(activations)");
  if (st == LCR_OK) {
    char* b = c->buf;
    c->x = reinterpret_cast<bf16*>(b + o_x);
    c->xsum = reinterpret_cast<float*>(b + o_xsum);
    c->qkv = reinterpret_cast<bf16*>(b + o_qkv);
    c->attn = reinterpret_cast<bf16*>(b + o_attn);
    c->act = reinterpret_cast<bf16*>(b + o_act);
    c->qkv_f = reinterpret_cast<float*>(b + o_qkvf);
    c->attn_f = reinterpret_cast<float*>(b + o_attnf);
    c->act_f = reinterpret_cast<float*>(b + o_actf);
    c->logits = reinterpret_cast<float*>(b + o_logits);
    c->partials = reinterpret_cast<float*>(b + o_part);
    c->attn_ctr = reinterpret_cast<unsigned*>(b + o_actr);
    c->sched = reinterpret_cast<unsigned*>(b + o_sched);
    c->argmax_acc = reinterpret_cast<unsigned long long*>(b + o_amax);
    c->state = reinterpret_cast<int32_t*>(b + o_state);
    c->history = reinterpret_cast<int32_t*>(b + o_hist);
    // The status word shares the state's 16 bytes (token, position, -,
    // status), so one read-back carries the next token and the status.
    c->status = reinterpret_cast<uint32_t*>(c->state + 3);
    c->inv_freq = reinterpret_cast<float*>(b + o_freq);
    c->sample_params = reinterpret_cast<float*>(b + o_sparams);
    c->sampled = reinterpret_cast<int32_t*>(b + o_sampled);
    c->epoch = reinterpret_cast<uint32_t*>(b + o_epoch);
    c->qkv_ll = reinterpret_cast<uint32_t*>(b + o_qkvll);
    c->part_ll = reinterpret_cast<unsigned long long*>(b + o_partll);
    c->attn_ll = reinterpret_cast<uint32_t*>(b + o_attnll);
    c->x_ll = reinterpret_cast<unsigned long long*>(b + o_xll);
    c->act_ll = reinterpret_cast<uint32_t*>(b + o_actll);
    const uint32_t epoch0 = 16;  // no tag of the first step is the zero of an unwritten word
    cuda(cudaMemcpy(c->epoch, &epoch0, sizeof epoch0, cudaMemcpyHostToDevice), "upload epoch");
    const std::vector<float> freq = rope_inv_freq(d);
    cuda(cudaMemcpy(c->inv_freq, freq.data(), freq.size() * sizeof(float), cudaMemcpyHostToDevice),
         "upload inv_freq");
  }

  // KV cache (src/kv_cache.cu:24-63).
  if (st == LCR_OK) {
    size_t elems;
    if (o.paged) {
      c->max_pages = (o.max_seq + o.page_size - 1) / o.page_size;
      c->pool_pages = c->max_pages * d.num_layers;
      elems = static_cast<size_t>(c->pool_pages) * d.num_kv_heads * o.page_size * d.head_dim;
      c->tables_host.assign(static_cast<size_t>(d.num_layers) * c->max_pages, -1);
      c->order.resize(static_cast<size_t>(c->pool_pages));
      for (int i = 0; i < c->pool_pages; ++i) c->order[static_cast<size_t>(i)] = i;
      if (o.page_order_seed != 0) {
        uint64_t s = o.page_order_seed;
        for (int i = c->pool_pages - 1; i > 0; --i) {
          const int j = static_cast<int>(splitmix64(&s) % static_cast<uint64_t>(i + 1));
          std::swap(c->order[static_cast<size_t>(i)], c->order[static_cast<size_t>(j)]);
        }
      }
      cuda(cudaMalloc(&c->tables_dev, c->tables_host.size() * sizeof(int32_t)), "cudaMalloc(page tables)");
      if (st == LCR_OK) {
        cuda(cudaMemcpy(c->tables_dev, c->tables_host.data(), c->tables_host.size() * sizeof(int32_t),
                        cudaMemcpyHostToDevice),
             "upload page tables");
      }
    } else {
      elems = static_cast<size_t>(d.num_layers) * d.num_kv_heads * o.max_seq * d.head_dim;
    }
    if (st == LCR_OK) cuda(cudaMalloc(&c->kpool, elems * sizeof(bf16)), "cudaMalloc(K pool)");
    if (st == LCR_OK) cuda(cudaMalloc(&c->vpool, elems * sizeof(bf16)), "cudaMalloc(V pool)");
    if (st == LCR_OK) cuda(cudaMemset(c->kpool, 0, elems * sizeof(bf16)), "cudaMemset(K pool)");
    if (st == LCR_OK) cuda(cudaMemset(c->vpool, 0, elems * sizeof(bf16)), "cudaMemset(V pool)");
  }
  // Tensor maps of the cache rows.
  if (st == LCR_OK && d.head_dim % 64 == 0 && (!o.paged || o.page_size % 16 == 0)) {
    const long long rows = o.paged ? static_cast<long long>(c->pool_pages) * d.num_kv_heads * o.page_size
                                   : static_cast<long long>(d.num_kv_heads) * o.max_seq;
    if (rows <= INT32_MAX) {
      const int maps = o.paged ? 1 : d.num_layers;
      const size_t layer_elems = o.paged ? 0 : static_cast<size_t>(d.num_kv_heads) * o.max_seq * d.head_dim;
      c->kvmaps.resize(static_cast<size_t>(2 * maps));
      for (int l = 0; l < maps && st == LCR_OK; ++l) {
        st = make_prefill_kv_map(&c->kvmaps[static_cast<size_t>(2 * l)], c->kpool + l * layer_elems,
                                 static_cast<int>(rows), d.head_dim);
        if (st == LCR_OK) {
          st = make_prefill_kv_map(&c->kvmaps[static_cast<size_t>(2 * l + 1)], c->vpool + l * layer_elems,
                                   static_cast<int>(rows), d.head_dim);
        }
      }
      if (st == LCR_OK) cuda(cudaMalloc(&c->kvmaps_dev, c->kvmaps.size() * sizeof(CUtensorMap)), "cudaMalloc(KV maps)");
      if (st == LCR_OK) {
        cuda(cudaMemcpy(c->kvmaps_dev, c->kvmaps.data(), c->kvmaps.size() * sizeof(CUtensorMap),
                        cudaMemcpyHostToDevice),
             "upload KV maps");
      }
    }
  }
  // Tensor maps of the streamed matrices (one TMA copy per GEMV stage).
  if (st == LCR_OK) {
    c->wmaps.resize(static_cast<size_t>(4 * d.num_layers + 1));
    for (int l = 0; l < d.num_layers && st == LCR_OK; ++l) {
      const lcr_layer_weights& w = c->layers[static_cast<size_t>(l)];
      CUtensorMap* m = &c->wmaps[static_cast<size_t>(4 * l)];
      st = make_weight_map(m, w.qkv_proj, qd + 2 * kvd, d.hidden_size, false);
      if (st == LCR_OK) st = make_weight_map(m + 1, w.o_proj, d.hidden_size, qd, false);
      if (st == LCR_OK) st = make_weight_map(m + 2, w.gate_up_proj, d.intermediate_size, d.hidden_size, true);
      if (st == LCR_OK) st = make_weight_map(m + 3, w.down_proj, d.hidden_size, d.intermediate_size, false);
    }
    if (st == LCR_OK) st = make_weight_map(&c->wmaps.back(), c->lm_head, d.vocab_size, d.hidden_size, false);
    if (st == LCR_OK) cuda(cudaMalloc(&c->wmaps_dev, c->wmaps.size() * sizeof(CUtensorMap)), "cudaMalloc(tensor maps)");
    if (st == LCR_OK) {
      cuda(cudaMemcpy(c->wmaps_dev, c->wmaps.data(), c->wmaps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice),
           "upload tensor maps");
    }
  }
  if (st == LCR_OK && c->persistent) {
    std::vector<MegaLayer> ml(static_cast<size_t>(d.num_layers));
    for (int l = 0; l < d.num_layers; ++l) {
      const lcr_layer_weights& w = c->layers[static_cast<size_t>(l)];
      ml[static_cast<size_t>(l)] = {static_cast<const bf16*>(w.input_norm), static_cast<const bf16*>(w.qkv_proj),
                                    static_cast<const bf16*>(w.o_proj), static_cast<const bf16*>(w.post_attention_norm),
                                    static_cast<const bf16*>(w.gate_up_proj), static_cast<const bf16*>(w.down_proj)};
    }
    cuda(cudaMalloc(&c->mega_layers, ml.size() * sizeof(MegaLayer)), "cudaMalloc(layer table)");
    if (st == LCR_OK) {
      cuda(cudaMemcpy(c->mega_layers, ml.data(), ml.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice),
           "upload layer table");
    }
    if (st == LCR_OK) cuda(cudaMalloc(&c->mega_bar, sizeof(unsigned)), "cudaMalloc(barrier)");
    if (st == LCR_OK) cuda(cudaMemset(c->mega_bar, 0, sizeof(unsigned)), "cudaMemset(barrier)");
    if (st == LCR_OK && (o.flags & kFlagTrace)) {
      const size_t n = static_cast<size_t>(c->sms) * kMegaTraceEvents;
      cuda(cudaMalloc(&c->trace, n * sizeof(unsigned long long)), "cudaMalloc(trace)");
      if (st == LCR_OK) cuda(cudaMemset(c->trace, 0, n * sizeof(unsigned long long)), "cudaMemset(trace)");
    }
  }
  // The exchange needs the tensor-pipe attention phase and bf16 activations.
  c->ll = c->persistent && !c->f32 && c->kvmaps_dev != nullptr && d.head_dim == 64 && group <= 8 &&
          !(o.flags & (kFlagGridBarriers | kFlagCudaCoreAttention));
  // The (token, position) ring, then four words for the state read-back.
  if (st == LCR_OK) cuda(cudaMallocHost(&c->pinned, sizeof(int32_t) * (2 * kPinnedRing + 4)), "cudaMallocHost");
  if (st == LCR_OK) cuda(cudaMallocHost(&c->pinned_params, sizeof(float) * 8), "cudaMallocHost");
  if (st != LCR_OK) {
    release(c);
    return st;
  }
  *out = c;
  return LCR_OK;
}

extern "C" void lcr_ctx_destroy(lcr_ctx* ctx) { release(ctx); }

extern "C" int lcr_rope_inv_freq(const lcr_model_desc* desc, float* out, int capacity) {
  LCRB_REQUIRE(desc && out, LCR_ERR_INVALID, "lcr_rope_inv_freq: null argument");
  LCRB_REQUIRE(desc->head_dim > 0 && desc->head_dim % 2 == 0 && desc->rope_theta > 1.f, LCR_ERR_INVALID,
               "lcr_rope_inv_freq: head_dim %d / rope_theta %g", desc->head_dim,
               static_cast<double>(desc->rope_theta));
  LCRB_REQUIRE(capacity >= desc->head_dim / 2, LCR_ERR_INVALID, "lcr_rope_inv_freq: %d floats needed, %d given",
               desc->head_dim / 2, capacity);
  const std::vector<float> f = rope_inv_freq(*desc);
  std::memcpy(out, f.data(), f.size() * sizeof(float));
  return LCR_OK;
}

extern "C" int lcr_reset(lcr_ctx* ctx) {
  LCRB_REQUIRE(ctx, LCR_ERR_INVALID, "null context");
  ctx->position = 0;
  return LCR_OK;
}

extern "C" int lcr_position(const lcr_ctx* ctx) { return ctx ? ctx->position : -1; }

extern "C" int lcr_reserve_length(lcr_ctx* c, int length) {
  LCRB_REQUIRE(c, LCR_ERR_INVALID, "null context");
  LCRB_REQUIRE(length <= c->o.max_seq, LCR_ERR_STATE,
               "sequence reached %d positions but the KV cache was built for %d", length, c->o.max_seq);
  if (length <= c->length) return LCR_OK;
  if (c->o.paged) {
    const int P = c->o.page_size;
    const int have = (c->length + P - 1) / P;
    const int need = (length + P - 1) / P;
    if (need > have) {
      LCRB_CUDA(cudaSetDevice(c->device));
      LCRB_CUDA(cudaStreamSynchronize(c->stream));
      for (int l = 0; l < c->d.num_layers; ++l) {
        int32_t* table = c->tables_host.data() + static_cast<size_t>(l) * c->max_pages;
        for (int p = have; p < need; ++p) {
          LCRB_REQUIRE(c->pages_mapped < c->pool_pages, LCR_ERR_POOL,
                       "paged KV cache pool is exhausted after %d pages", c->pages_mapped);
          table[p] = c->order[static_cast<size_t>(c->pages_mapped++)];
        }
        LCRB_CUDA(cudaMemcpy(c->tables_dev + static_cast<size_t>(l) * c->max_pages + have, table + have,
                             static_cast<size_t>(need - have) * sizeof(int32_t), cudaMemcpyHostToDevice));
      }
    }
  }
  c->length = length;
  return LCR_OK;
}

extern "C" int lcr_decode(lcr_ctx* c, int token, const float** logits) {
  LCRB_REQUIRE(c, LCR_ERR_INVALID, "null context");
  LCRB_REQUIRE(c->position < c->o.max_seq, LCR_ERR_STATE,
               "sequence reached %d positions, the cache limit", c->position);
  LCRB_REQUIRE(token >= 0 && token < c->d.vocab_size, LCR_ERR_INVALID, "token %d outside the vocabulary",
               token);
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_TRY(lcr_reserve_length(c, c->position + 1));
  int32_t* slot = c->pinned + 2 * c->ring_next;
  c->ring_next = (c->ring_next + 1) % kPinnedRing;
  slot[0] = token;
  slot[1] = c->position;
  LCRB_CUDA(cudaMemcpyAsync(c->state, slot, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, c->stream));
  LCRB_TRY(launch_steps(c, 1));
  LCRB_TRY(check_status(c));
  c->position += 1;
  if (logits) *logits = c->logits;
  return LCR_OK;
}

extern "C" int lcr_prefill(lcr_ctx* c, const int32_t* tokens, int count, const float** logits) {
  LCRB_REQUIRE(c && tokens, LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(count > 0, LCR_ERR_INVALID, "prefill needs at least one token");
  LCRB_REQUIRE(c->position + count <= c->o.max_seq, LCR_ERR_STATE,
               "prompt of %d tokens at position %d exceeds the cache built for %d", count, c->position,
               c->o.max_seq);
  for (int i = 0; i < count; ++i) {
    LCRB_REQUIRE(tokens[i] >= 0 && tokens[i] < c->d.vocab_size, LCR_ERR_INVALID,
                 "token %d outside the vocabulary", tokens[i]);
  }
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_TRY(lcr_reserve_length(c, c->position + count));
  if (count >= kPrefillChunkMin && prefill_engine_ready(c)) {
    LCRB_TRY(prefill_chunked(c, tokens, count));
    LCRB_TRY(check_status(c));
    c->position += count;
    if (logits) *logits = c->logits;
    return LCR_OK;
  }
  const size_t need = static_cast<size_t>(count) * 2;
  if (c->pinned_prompt_cap < need) {
    LCRB_CUDA(cudaStreamSynchronize(c->stream));
    cudaFreeHost(c->pinned_prompt);
    c->pinned_prompt = nullptr;
    c->pinned_prompt_cap = 0;
    LCRB_CUDA(cudaMallocHost(&c->pinned_prompt, need * sizeof(int32_t)));
    c->pinned_prompt_cap = need;
  } else {
    LCRB_CUDA(cudaStreamSynchronize(c->stream));
  }
  for (int i = 0; i < count; ++i) {
    c->pinned_prompt[2 * i] = tokens[i];
    c->pinned_prompt[2 * i + 1] = c->position + i;
  }
  for (int i = 0; i < count; ++i) {
    LCRB_CUDA(cudaMemcpyAsync(c->state, c->pinned_prompt + 2 * i, 2 * sizeof(int32_t),
                              cudaMemcpyHostToDevice, c->stream));
    LCRB_TRY(launch_steps(c, 1));
  }
  LCRB_TRY(check_status(c));
  c->position += count;
  if (logits) *logits = c->logits;
  return LCR_OK;
}

extern "C" int lcr_logits_to_host(lcr_ctx* c, float* host) {
  LCRB_REQUIRE(c && host, LCR_ERR_INVALID, "null argument");
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_CUDA(cudaMemcpyAsync(host, c->logits, sizeof(float) * c->d.vocab_size, cudaMemcpyDeviceToHost,
                            c->stream));
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  return LCR_OK;
}

extern "C" int lcr_sample_logits(lcr_ctx* c, const float* logits, float temperature, int top_k,
                                 float top_p, float uniform, int* token) {
  LCRB_REQUIRE(c && logits && token, LCR_ERR_INVALID, "null argument");
  if (temperature > 0.0f) {
    LCRB_REQUIRE(top_p > 0.0f && top_p <= 1.0f, LCR_ERR_INVALID, "top_p must be in (0, 1], got %g",
                 static_cast<double>(top_p));
  }
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  float* p = c->pinned_params;
  p[0] = temperature > 0.0f ? 1.0f / temperature : 0.0f;
  std::memcpy(&p[1], &top_k, sizeof(int));
  p[2] = top_p;
  p[3] = uniform;
  LCRB_CUDA(cudaMemcpyAsync(c->sample_params, p, 4 * sizeof(float), cudaMemcpyHostToDevice, c->stream));
  SampleArgs a = {};
  a.logits = logits;
  a.row_stride = c->d.vocab_size;
  a.vocab = c->d.vocab_size;
  a.inv_temperature = c->sample_params;
  a.top_k = reinterpret_cast<const int*>(c->sample_params + 1);
  a.top_p = c->sample_params + 2;
  a.uniform = c->sample_params + 3;
  a.out = c->sampled;
  LCRB_TRY(sample_launch(a, 1, c->stream, false));
  int32_t id = -1;
  LCRB_CUDA(cudaMemcpyAsync(&id, c->sampled, sizeof id, cudaMemcpyDeviceToHost, c->stream));
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  LCRB_REQUIRE(id >= 0 && id < c->d.vocab_size, LCR_ERR_STATE,
               "sampling produced token id %d, outside the vocabulary", id);
  *token = id;
  return LCR_OK;
}

extern "C" int lcr_generate_greedy(lcr_ctx* c, int first_token, int steps, int32_t* tokens_out) {
  LCRB_REQUIRE(c, LCR_ERR_INVALID, "null context");
  LCRB_REQUIRE(steps >= 0, LCR_ERR_INVALID, "negative step count");
  if (steps == 0) return LCR_OK;
  LCRB_REQUIRE(c->position + steps <= c->o.max_seq, LCR_ERR_STATE,
               "%d steps at position %d exceed the cache built for %d", steps, c->position, c->o.max_seq);
  LCRB_REQUIRE(first_token >= 0 && first_token < c->d.vocab_size, LCR_ERR_INVALID,
               "token %d outside the vocabulary", first_token);
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_TRY(lcr_reserve_length(c, c->position + steps));
  int32_t* slot = c->pinned + 2 * c->ring_next;
  c->ring_next = (c->ring_next + 1) % kPinnedRing;
  slot[0] = first_token;
  slot[1] = c->position;
  LCRB_CUDA(cudaMemcpyAsync(c->state, slot, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, c->stream));
  LCRB_TRY(launch_steps(c, steps));
  if (tokens_out) {
    LCRB_CUDA(cudaMemcpyAsync(tokens_out, c->history + c->position, sizeof(int32_t) * steps,
                              cudaMemcpyDeviceToHost, c->stream));
  }
  LCRB_TRY(check_status(c));
  c->position += steps;
  return LCR_OK;
}

extern "C" int lcr_set_token(lcr_ctx* c, const int32_t* host_token, int position) {
  LCRB_REQUIRE(c && host_token, LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(position >= 0 && position < c->o.max_seq, LCR_ERR_STATE,
               "position %d outside the cache built for %d", position, c->o.max_seq);
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_TRY(stage_state(c, host_token, position));
  c->position = position;
  return LCR_OK;
}

extern "C" int lcr_enqueue_steps(lcr_ctx* c, int steps) {
  LCRB_REQUIRE(c && steps >= 0, LCR_ERR_INVALID, "bad arguments");
  // Pages for the positions the steps write (a synchronisation only when
  // new pages are mapped).
  LCRB_TRY(lcr_reserve_length(c, c->position + steps));
  LCRB_TRY(launch_steps(c, steps));
  c->position += steps;
  return LCR_OK;
}

extern "C" int lcr_read_token(lcr_ctx* c, int32_t* host_token) {
  LCRB_REQUIRE(c && host_token, LCR_ERR_INVALID, "null argument");
  LCRB_CUDA(cudaMemcpyAsync(host_token, c->state, sizeof(int32_t), cudaMemcpyDeviceToHost, c->stream));
  return LCR_OK;
}

extern "C" int lcr_step_host(lcr_ctx* c, int32_t token, int position, int32_t* next_token) {
  LCRB_REQUIRE(c && next_token, LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(position >= 0 && position < c->o.max_seq, LCR_ERR_STATE,
               "position %d outside the cache built for %d", position, c->o.max_seq);
  LCRB_REQUIRE(token >= 0 && token < c->d.vocab_size, LCR_ERR_INVALID, "token %d outside the vocabulary", token);
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_TRY(stage_state(c, &token, position));
  c->position = position;
  LCRB_TRY(lcr_reserve_length(c, c->position + 1));
  LCRB_TRY(launch_steps(c, 1));
  c->position += 1;
  // One read-back: the next token and, in the same 16 bytes, the status.
  int32_t* back = c->pinned + 2 * kPinnedRing;
  LCRB_CUDA(cudaMemcpyAsync(back, c->state, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, c->stream));
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  if (back[3] != 0) return check_status(c);
  *next_token = back[0];
  return LCR_OK;
}

extern "C" int lcr_sync(lcr_ctx* c) {
  LCRB_REQUIRE(c, LCR_ERR_INVALID, "null context");
  LCRB_CUDA(cudaSetDevice(c->device));
  return check_status(c);
}

extern "C" lcr_stream_t lcr_ctx_stream(lcr_ctx* c) {
  return c ? reinterpret_cast<lcr_stream_t>(c->stream) : nullptr;
}

extern "C" int lcr_kv_view_of(const lcr_ctx* c, int layer, lcr_kv_view* v) {
  LCRB_REQUIRE(c && v, LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(layer >= 0 && layer < c->d.num_layers, LCR_ERR_INVALID, "layer %d is out of range", layer);
  const lcr_model_desc& d = c->d;
  v->num_kv_heads = d.num_kv_heads;
  v->head_dim = d.head_dim;
  if (c->o.paged) {
    v->keys = c->kpool;
    v->values = c->vpool;
    v->page_table = c->tables_dev + static_cast<size_t>(layer) * c->max_pages;
    v->page_size = c->o.page_size;
    v->page_stride = d.num_kv_heads * c->o.page_size * d.head_dim;
    v->head_stride = c->o.page_size * d.head_dim;
  } else {
    const size_t base = static_cast<size_t>(layer) * d.num_kv_heads * c->o.max_seq * d.head_dim;
    v->keys = c->kpool + base;
    v->values = c->vpool + base;
    v->page_table = nullptr;
    v->page_size = c->o.max_seq;
    v->page_stride = 0;
    v->head_stride = c->o.max_seq * d.head_dim;
  }
  return LCR_OK;
}

extern "C" int lcr_page_tables(const lcr_ctx* c, int32_t* tables, int* pages_mapped) {
  LCRB_REQUIRE(c, LCR_ERR_INVALID, "null context");
  if (tables && !c->tables_host.empty()) {
    std::memcpy(tables, c->tables_host.data(), c->tables_host.size() * sizeof(int32_t));
  }
  if (pages_mapped) *pages_mapped = c->pages_mapped;
  return LCR_OK;
}

extern "C" size_t lcr_weight_bytes_per_token(const lcr_ctx* c) {
  if (!c) return 0;
  const lcr_model_desc& d = c->d;
  const size_t h = d.hidden_size, q = static_cast<size_t>(d.num_heads) * d.head_dim;
  const size_t kv = static_cast<size_t>(d.num_kv_heads) * d.head_dim, f = d.intermediate_size;
  size_t per = static_cast<size_t>(d.num_layers) * (h * 2 + q * h + kv * h * 2 + h * q + f * h * 3);
  per += h + static_cast<size_t>(d.vocab_size) * h;
  return per * 2;
}

extern "C" size_t lcr_kv_bytes_per_position(const lcr_ctx* c) {
  if (!c) return 0;
  return static_cast<size_t>(c->d.num_layers) * 2 * c->d.num_kv_heads * c->d.head_dim * 2;
}

extern "C" int lcr_step_launches(const lcr_ctx* c) {
  if (!c) return 0;
  return c->persistent ? 1 : 5 * c->d.num_layers + 1;
}

extern "C" int lcr_device_status(lcr_ctx* c) {
  LCRB_REQUIRE(c, LCR_ERR_INVALID, "null context");
  LCRB_CUDA(cudaSetDevice(c->device));
  return check_status(c);
}

extern "C" int lcr_time_steps(lcr_ctx* c, int steps, float* ms) {
  LCRB_REQUIRE(c && ms && steps > 0, LCR_ERR_INVALID, "bad arguments");
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_TRY(build_graph(c));
  cudaEvent_t e0, e1;
  LCRB_CUDA(cudaEventCreate(&e0));
  LCRB_CUDA(cudaEventCreate(&e1));
  cudaEventRecord(e0, c->stream);
  int st = launch_steps(c, steps);
  cudaEventRecord(e1, c->stream);
  cudaEventSynchronize(e1);
  float t = 0.f;
  cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (st != LCR_OK) return st;
  c->position += steps;
  *ms = t;
  return check_status(c);
}

extern "C" int lcr_time_gemv(lcr_ctx* c, int matrix, int layer, int reps, float* ms) {
  LCRB_REQUIRE(c && ms && reps > 0, LCR_ERR_INVALID, "bad arguments");
  LCRB_REQUIRE(layer >= 0 && layer < c->d.num_layers, LCR_ERR_INVALID, "layer %d out of range", layer);
  LCRB_CUDA(cudaSetDevice(c->device));
  const lcr_model_desc& d = c->d;
  const lcr_layer_weights& w = c->layers[static_cast<size_t>(layer)];
  GemvArgs a = {};
  int K = d.hidden_size, pro = PRO_NORM, epi = EPI_STORE, n = 0;
  switch (matrix) {
    case 0:
      a.w = static_cast<const bf16*>(w.qkv_proj); a.x_in = c->x; a.xsum = c->xsum;
      a.norm_w = static_cast<const bf16*>(w.input_norm); a.y = c->qkv; n = q_dim(c) + 2 * kv_dim(c);
      break;
    case 1:
      a.w = static_cast<const bf16*>(w.o_proj); a.x_in = c->attn; a.y = c->qkv;
      K = q_dim(c); pro = PRO_PLAIN; n = d.hidden_size;
      break;
    case 2:
      a.w = static_cast<const bf16*>(w.gate_up_proj); a.x_in = c->x; a.xsum = c->xsum;
      a.norm_w = static_cast<const bf16*>(w.post_attention_norm); a.y = c->act; epi = EPI_SWIGLU;
      n = d.intermediate_size;
      break;
    case 3:
      a.w = static_cast<const bf16*>(w.down_proj); a.x_in = c->act; a.y = c->qkv;
      K = d.intermediate_size; pro = PRO_PLAIN; n = d.hidden_size;
      break;
    default:
      a.w = c->lm_head; a.x_in = c->x; a.xsum = c->xsum; a.norm_w = c->final_norm; a.yf = c->logits;
      epi = EPI_STORE_F32; n = d.vocab_size;
      break;
  }
  LCRB_REQUIRE(reps <= kTimingSlots, LCR_ERR_INVALID, "at most %d repetitions", kTimingSlots);
  cudaEvent_t e0, e1;
  LCRB_CUDA(cudaEventCreate(&e0));
  LCRB_CUDA(cudaEventCreate(&e1));
  cudaEventRecord(e0, c->stream);
  int st = LCR_OK;
  for (int i = 0; i < reps && st == LCR_OK; ++i) {
    int slot = c->sched_slots - kTimingSlots + i;
    st = gemv_node(c, a, K, pro, epi, n, &slot, matrix < 4 ? 4 * layer + matrix : 4 * d.num_layers);
  }
  cudaEventRecord(e1, c->stream);
  cudaEventSynchronize(e1);
  float t = 0.f;
  cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (st != LCR_OK) return st;
  *ms = t / reps;
  return check_status(c);
}

extern "C" int lcr_copy_trace(lcr_ctx* c, unsigned long long* host, int capacity, int* count) {
  LCRB_REQUIRE(c && host && count, LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(c->trace != nullptr, LCR_ERR_STATE,
               "tracing is off (create the context with flags bit 3 on the persistent step)");
  const int n = std::min(capacity, c->sms * kMegaTraceEvents);
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  LCRB_CUDA(cudaMemcpy(host, c->trace, sizeof(unsigned long long) * n, cudaMemcpyDeviceToHost));
  *count = n;
  return LCR_OK;
}
