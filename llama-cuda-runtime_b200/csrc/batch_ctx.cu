// Batched decode context (include/lcr_b200.h, lcr_batch_*): continuous
// batching of up to max_batch sequences, one token each per step.
//
// Every kernel after the first launches programmatically (PDL): it starts
// while its predecessor drains and waits (griddepcontrol.wait) before
// reading that predecessor's outputs; the projections stream their first
// weight stages before the wait. A step of n slots is, per layer:
//   norm_rows_kernel        x -> xn (layer 0: the token embeddings)
//   gemm_tc_kernel          qkv  = xn W_qkv^T, RoPE on q and k (the step's
//                           cos/sin table, written by the layer-0 norm)
//                           (split-K, + reduction)
//   attn_batch_kernel       K/V write at each slot's position, paged
//                           attention over 0..position on the tensor pipe,
//                           split merge -> attn
//   gemm_tc_kernel          x   += attn W_o^T (residual epilogue, split-K)
//   norm_rows_kernel        x -> xn
//   gemm_tc_kernel          act  = silu(xn W_gate^T) * (xn W_up^T)
//   gemm_tc_kernel          x   += act W_down^T (residual epilogue, split-K)
// then the final norm, the lm_head into fp32 logits [n][vocab] and one
// sampling row per slot (greedy or top-k/top-p with a Philox uniform of
// (seed, position)). The sequence of launches for a given n is captured once
// as a CUDA graph and replayed.
//
// KV cache: one pool per layer of pool_pages pages [kv_head][page_size][D];
// a slot's page table (shared by all layers) maps its positions to pages.
// The caller (the scheduler) owns page allocation through lcr_batch_set_pages.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <new>
#include <vector>

#include "attention.cuh"
#include "attn_batch.h"
#include "attn_prefill.h"
#include "batch.cuh"
#include "batch_internal.h"
#include "common.cuh"
#include "dispatch.h"
#include "gemm_tc.h"
#include "lcr_b200.h"
#include "rope_table.h"
#include "sampling.cuh"
#include "tmap.h"

using namespace lcrb;

namespace {

constexpr int kStaging = 16;  // pinned (tokens, positions) staging areas

struct StepMaps {  // activation tensor maps for one batch tile size
  CUtensorMap xn, attn, act;
};

// One set of activation rows: the step's (max_batch rows) or a prefill
// chunk's.
struct Acts {
  int32_t* tokens;
  int32_t* positions;
  bf16* x;       // residual stream (bf16)
  float* xsum;   // its unrounded sums
  bf16* xn;      // normalised rows
  bf16* qkv;
  bf16* attn;
  bf16* act;
  float2* rope;  // [rows][head_dim / 2] (cos, sin)
};

}  // namespace

struct lcr_batch {
  int device = 0;
  lcr_model_desc d{};
  lcr_batch_options o{};
  int sms = 148;
  bool use_graph = true;
  bool persist_gemm = true;  // 128-row projection tiles on gemm_tc_persist_kernel
  cudaStream_t stream = nullptr;

  const bf16* embed = nullptr;
  const bf16* final_norm = nullptr;
  const bf16* lm_head = nullptr;
  std::vector<lcr_layer_weights> layers;
  std::vector<CUtensorMap> wmaps;  // [layer * 4 + m]: qkv, o, gate/up, down; then lm_head
  std::vector<CUtensorMap> wmaps1; // the same with one 64-column chunk per copy (prefill chunks)
  std::map<int, StepMaps> xmaps;   // by batch tile
  std::vector<CUtensorMap> kvmaps; // [layer * 2 + {0: K, 1: V}] pool rows of head_dim

  char* buf = nullptr;
  bf16* x = nullptr;
  float* xsum = nullptr;
  bf16* xn = nullptr;
  bf16* qkv = nullptr;
  bf16* attn = nullptr;
  bf16* act = nullptr;
  float* logits = nullptr;
  float* partials = nullptr;
  unsigned* attn_work = nullptr;
  float* work = nullptr;
  float* inv_freq = nullptr;
  float2* rope = nullptr;  // [max_batch][head_dim / 2] (cos, sin) of this step
  int32_t* tokens = nullptr;
  int32_t* positions = nullptr;
  int32_t* tables = nullptr;  // [max_batch][max_pages]
  float* inv_temp = nullptr;
  int32_t* top_k = nullptr;
  float* top_p = nullptr;
  unsigned long long* seed = nullptr;
  int32_t* next = nullptr;
  uint32_t* status = nullptr;
  bf16* kpool = nullptr;
  bf16* vpool = nullptr;
  size_t layer_elems = 0;  // elements of one layer's pool
  int max_pages = 0;
  int tc_chunks = 2;        // 64-column K chunks per projection stage (fits batch tiles to 128)
  int attn_item_pos = 512;  // positions per attention work item
  int attn_slots = 1;       // partial slots per head: ceil(max_seq / attn_item_pos)
  int attn_ctas = 1;        // persistent attention CTAs
  size_t work_floats = 0;

  std::vector<int32_t> tables_host;
  std::vector<int> pages_set;  // pages each slot's table holds (lcr_batch_set_pages)
  std::vector<float> inv_temp_host, top_p_host;
  std::vector<int32_t> top_k_host;
  std::vector<unsigned long long> seed_host;
  bool tables_dirty = true, sampling_dirty = true;
  int32_t* pinned = nullptr;  // [kStaging][2 * max_batch]
  cudaEvent_t staged[kStaging] = {};
  int staging_next = 0;

  char* pre_buf = nullptr;  // prefill activations, grown to the largest chunk
  int pre_rows = 0;
  Acts pre{};

  std::map<int, cudaGraphExec_t> graphs;
  std::map<int, int> launches_by_n;  // kernels one step of n slots launches
  int last_n = 0;
  int launches = 0;
};

namespace {

void release(lcr_batch* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  for (auto& g : c->graphs) cudaGraphExecDestroy(g.second);
  for (cudaEvent_t e : c->staged) {
    if (e) cudaEventDestroy(e);
  }
  cudaFree(c->buf);
  cudaFree(c->logits);
  cudaFree(c->kpool);
  cudaFree(c->vpool);
  cudaFree(c->work);
  cudaFree(c->pre_buf);
  cudaFreeHost(c->pinned);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

int check_status(lcr_batch* c) {
  uint32_t st = 0;
  LCRB_CUDA(cudaMemcpyAsync(&st, c->status, sizeof st, cudaMemcpyDeviceToHost, c->stream));
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  if (st == 0) return LCR_OK;
  LCRB_CUDA(cudaMemsetAsync(c->status, 0, sizeof st, c->stream));
  LCRB_CUDA(cudaStreamSynchronize(c->stream));
  if (st & (kStatusTimeoutFull | kStatusTimeoutEmpty | kStatusTimeoutBarrier | kStatusAbort)) {
    return fail(LCR_ERR_TIMEOUT, "a device-side wait gave up (status 0x%x)", st);
  }
  if (st & kStatusBadToken) return fail(LCR_ERR_INVALID, "token id outside the vocabulary (status 0x%x)", st);
  if (st & kStatusBadPage) return fail(LCR_ERR_POOL, "page table entry outside the pool (status 0x%x)", st);
  return fail(LCR_ERR_STATE, "position outside the KV cache (status 0x%x)", st);
}

Acts step_acts(const lcr_batch* c) {
  return Acts{c->tokens, c->positions, c->x, c->xsum, c->xn, c->qkv, c->attn, c->act, c->rope};
}

int norm_launch(lcr_batch* c, const Acts& v, int n, bool embed, const void* gain) {
  NormRowsArgs a = {};
  a.tokens = v.tokens;
  a.embed = c->embed;
  a.vocab = c->d.vocab_size;
  a.x = v.x;
  a.xsum = v.xsum;
  a.gain = static_cast<const bf16*>(gain);
  a.eps = c->d.rms_norm_eps;
  a.out = v.xn;
  a.status = c->status;
  if (embed) {
    a.positions = v.positions;
    a.inv_freq = c->inv_freq;
    a.rope = v.rope;
    a.half = c->d.head_dim / 2;
  }
  ++c->launches;
  const dim3 grid(static_cast<unsigned>(n));
  void (*kernel)(NormRowsArgs) = nullptr;
  switch (c->d.hidden_size) {
    case 256: kernel = embed ? norm_rows_kernel<256, true> : norm_rows_kernel<256, false>; break;
    case 2048: kernel = embed ? norm_rows_kernel<2048, true> : norm_rows_kernel<2048, false>; break;
    case 4096: kernel = embed ? norm_rows_kernel<4096, true> : norm_rows_kernel<4096, false>; break;
    default:
      return fail(LCR_ERR_SHAPE, "batched RMSNorm has no kernel for hidden size %d", c->d.hidden_size);
  }
  // The step's first kernel follows the host copies of its inputs; the
  // others launch programmatically after their predecessor.
  return launch_kernel(kernel, grid, dim3(kNormThreads), 0, c->stream, !embed, a);
}

// One projection: n rows of `x` (tensor map `xm`, batch tile nb) against
// weight map `wm` ([n_out][K], or gate/up halves for SWIGLU).
// With `norm_gain` (a RESID projection), the RMSNorm of the updated rows into
// v.xn is fused into the split-K reduction when the projection splits;
// *normed says whether it was, so the caller launches the norm otherwise.
int gemm_node(lcr_batch* c, const Acts& v, const CUtensorMap& wm, const CUtensorMap& xm, int nb, int n, int n_out,
              int K, int epi, bf16* y, float* yf, int ldy, int ch, const void* norm_gain = nullptr,
              bool* normed = nullptr) {
  TcArgs a = {};
  a.n_out = n_out;
  a.K = K;
  a.rows = n;
  a.ldy = ldy;
  a.y = y;
  a.yf = yf;
  a.resid = v.x;
  a.resid_sum = v.xsum;
  a.status = c->status;
  a.rope = v.rope;
  a.head_dim = c->d.head_dim;
  a.rope_cols = (c->d.num_heads + c->d.num_kv_heads) * c->d.head_dim;
  const int tiles_n = epi == EPI_SWIGLU ? (n_out + 63) / 64 : (n_out + kTcTileM - 1) / kTcTileM;
  const int tiles = tiles_n * ((n + nb - 1) / nb);
  const int steps = K / (kTcSlabK * ch);
  // As many splits as fit the SMs in one wave (one CTA per SM), within the
  // K stages and the workspace.
  int splits = std::max(1, c->sms / tiles);
  splits = std::min(splits, steps);
  while (splits > 1 && gemm_tc_work_floats(n, n_out, epi, splits) > c->work_floats) --splits;
  a.splits = splits;
  a.work = c->work;
  a.ctas = c->persist_gemm ? c->sms : 0;
  const bool fuse = norm_gain != nullptr && epi == EPI_RESID && splits > 1;
  if (fuse) {
    a.norm_gain = static_cast<const bf16*>(norm_gain);
    a.norm_eps = c->d.rms_norm_eps;
    a.norm_out = v.xn;
  }
  if (normed) *normed = fuse;
  c->launches += splits > 1 ? 2 : 1;
  return gemm_tc_launch(a, wm, xm, nb, epi, ch, c->stream, true);
}

int attention_launch_layer(lcr_batch* c, int layer, int n) {
  const lcr_model_desc& d = c->d;
  const int qd = d.num_heads * d.head_dim, kvd = d.num_kv_heads * d.head_dim;
  AttnArgs a = {};
  a.qkv = c->qkv;
  a.qkv_stride = qd + 2 * kvd;
  a.q_dim = qd;
  a.kv_dim = kvd;
  a.inv_freq = c->inv_freq;
  a.kpool = c->kpool + static_cast<size_t>(layer) * c->layer_elems;
  a.vpool = c->vpool + static_cast<size_t>(layer) * c->layer_elems;
  a.tables = c->tables;
  a.table_seq_stride = c->max_pages;
  a.max_pages = c->max_pages;
  a.pool_pages = c->o.pool_pages;
  a.page_size = c->o.page_size;
  a.page_stride = static_cast<long long>(d.num_kv_heads) * c->o.page_size * d.head_dim;
  a.head_stride = static_cast<long long>(c->o.page_size) * d.head_dim;
  a.max_seq = c->o.max_seq;
  a.positions = c->positions;
  // Work items of attn_item_pos positions per (sequence, KV head), spread
  // over the persistent CTAs.
  a.item_pos = c->attn_item_pos;
  a.splits = c->attn_slots;
  a.seqs = n;
  a.work = c->attn_work;
  a.scale_log2 = (1.0f / std::sqrt(static_cast<float>(d.head_dim))) * kLog2e;
  a.out = c->attn;
  a.partials = c->partials;
  a.status = c->status;
  c->launches += 2;
  return attn_batch_launch(a, c->kvmaps[static_cast<size_t>(2 * layer)], c->kvmaps[static_cast<size_t>(2 * layer + 1)],
                           d.head_dim, d.num_heads / d.num_kv_heads, c->attn_ctas, c->stream);
}

int maps_for(lcr_batch* c, int nb, const StepMaps** out) {
  auto it = c->xmaps.find(nb);
  if (it == c->xmaps.end()) {
    const lcr_model_desc& d = c->d;
    StepMaps m;
    const int qd = d.num_heads * d.head_dim;
    const int ch = c->tc_chunks;
    LCRB_TRY(make_kmajor_map(&m.xn, c->xn, c->o.max_batch, d.hidden_size, 1, nb, ch));
    LCRB_TRY(make_kmajor_map(&m.attn, c->attn, c->o.max_batch, qd, 1, nb, ch));
    LCRB_TRY(make_kmajor_map(&m.act, c->act, c->o.max_batch, d.intermediate_size, 1, nb, ch));
    it = c->xmaps.emplace(nb, m).first;
  }
  *out = &it->second;
  return LCR_OK;
}

int enqueue_step(lcr_batch* c, int n) {
  const lcr_model_desc& d = c->d;
  const int H = d.hidden_size, F = d.intermediate_size;
  const int qd = d.num_heads * d.head_dim, kvd = d.num_kv_heads * d.head_dim;
  const int nb = gemm_tc_batch_tile(n);
  const StepMaps* m = nullptr;
  LCRB_TRY(maps_for(c, nb, &m));
  c->launches = 0;
  const Acts v = step_acts(c);
  bool normed = false;  // the previous down projection already wrote xn
  for (int l = 0; l < d.num_layers; ++l) {
    const lcr_layer_weights& w = c->layers[static_cast<size_t>(l)];
    const CUtensorMap* wm = &c->wmaps[static_cast<size_t>(4 * l)];
    if (!normed) LCRB_TRY(norm_launch(c, v, n, l == 0, w.input_norm));
    const int ch = c->tc_chunks;
    LCRB_TRY(gemm_node(c, v, wm[0], m->xn, nb, n, qd + 2 * kvd, H, EPI_ROPE, v.qkv, nullptr, qd + 2 * kvd, ch));
    LCRB_TRY(attention_launch_layer(c, l, n));
    LCRB_TRY(gemm_node(c, v, wm[1], m->attn, nb, n, H, qd, EPI_RESID, nullptr, nullptr, H, ch,
                       w.post_attention_norm, &normed));
    if (!normed) LCRB_TRY(norm_launch(c, v, n, false, w.post_attention_norm));
    LCRB_TRY(gemm_node(c, v, wm[2], m->xn, nb, n, F, H, EPI_SWIGLU, v.act, nullptr, F, ch));
    const void* next_gain = l + 1 < d.num_layers ? c->layers[static_cast<size_t>(l + 1)].input_norm : c->final_norm;
    LCRB_TRY(gemm_node(c, v, wm[3], m->act, nb, n, H, F, EPI_RESID, nullptr, nullptr, H, ch, next_gain, &normed));
  }
  if (!normed) LCRB_TRY(norm_launch(c, v, n, false, c->final_norm));
  LCRB_TRY(gemm_node(c, v, c->wmaps.back(), m->xn, nb, n, d.vocab_size, H, EPI_STORE_F32, nullptr, c->logits,
                     d.vocab_size, c->tc_chunks));
  SampleArgs s = {};
  s.logits = c->logits;
  s.row_stride = d.vocab_size;
  s.vocab = d.vocab_size;
  s.inv_temperature = c->inv_temp;
  s.top_k = c->top_k;
  s.top_p = c->top_p;
  s.uniform = nullptr;
  s.seed = c->seed;
  s.counter = c->positions;
  s.out = c->next;
  ++c->launches;
  return sample_launch(s, n, c->stream, true);
}

// Uploads changed page tables and sampling parameters (on the stream).
int upload_slot_state(lcr_batch* c) {
  const size_t B = static_cast<size_t>(c->o.max_batch);
  if (c->tables_dirty) {
    LCRB_CUDA(cudaMemcpyAsync(c->tables, c->tables_host.data(), sizeof(int32_t) * B * c->max_pages,
                              cudaMemcpyHostToDevice, c->stream));
    c->tables_dirty = false;
  }
  if (c->sampling_dirty) {
    LCRB_CUDA(cudaMemcpyAsync(c->inv_temp, c->inv_temp_host.data(), sizeof(float) * B, cudaMemcpyHostToDevice,
                              c->stream));
    LCRB_CUDA(cudaMemcpyAsync(c->top_k, c->top_k_host.data(), sizeof(int32_t) * B, cudaMemcpyHostToDevice,
                              c->stream));
    LCRB_CUDA(cudaMemcpyAsync(c->top_p, c->top_p_host.data(), sizeof(float) * B, cudaMemcpyHostToDevice,
                              c->stream));
    LCRB_CUDA(cudaMemcpyAsync(c->seed, c->seed_host.data(), sizeof(unsigned long long) * B,
                              cudaMemcpyHostToDevice, c->stream));
    c->sampling_dirty = false;
  }
  return LCR_OK;
}

int launch_step(lcr_batch* c, int n) {
  if (!c->use_graph) {
    LCRB_TRY(enqueue_step(c, n));
    c->launches_by_n[n] = c->launches;
    return LCR_OK;
  }
  auto it = c->graphs.find(n);
  if (it == c->graphs.end()) {
    cudaGraph_t g = nullptr;
    LCRB_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    const int st = enqueue_step(c, n);
    if (st == LCR_OK) c->launches_by_n[n] = c->launches;
    const cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (st != LCR_OK) {
      if (g) cudaGraphDestroy(g);
      return st;
    }
    LCRB_CUDA(e);
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    LCRB_CUDA(ie);
    it = c->graphs.emplace(n, exec).first;
  }
  LCRB_CUDA(cudaGraphLaunch(it->second, c->stream));
  return LCR_OK;
}

}  // namespace

extern "C" int lcr_batch_create(const lcr_model_desc* desc, const lcr_weights* weights,
                                const lcr_batch_options* options, lcr_batch** out) {
  LCRB_REQUIRE(desc && weights && options && out, LCR_ERR_INVALID, "lcr_batch_create: null argument");
  *out = nullptr;
  const lcr_model_desc& d = *desc;
  const lcr_batch_options& o = *options;
  LCRB_REQUIRE(d.hidden_size > 0 && d.intermediate_size > 0 && d.num_layers > 0 && d.num_heads > 0 &&
                   d.num_kv_heads > 0 && d.num_heads % d.num_kv_heads == 0 && d.vocab_size > 0,
               LCR_ERR_INVALID, "bad model description");
  LCRB_REQUIRE(d.head_dim == 64 || d.head_dim == 128, LCR_ERR_SHAPE,
               "decode attention is compiled for head_dim 64 or 128, this model has %d", d.head_dim);
  const int qd = d.num_heads * d.head_dim, kvd = d.num_kv_heads * d.head_dim;
  LCRB_REQUIRE(d.hidden_size % kTcSlabK == 0 && qd % kTcSlabK == 0 && d.intermediate_size % kTcSlabK == 0,
               LCR_ERR_SHAPE, "tensor-core projections need hidden, q_dim and ffn multiples of %d", kTcSlabK);
  LCRB_REQUIRE(d.hidden_size == 256 || d.hidden_size == 2048 || d.hidden_size == 4096, LCR_ERR_SHAPE,
               "batched RMSNorm has no kernel for hidden size %d", d.hidden_size);
  LCRB_REQUIRE(o.max_batch >= 1 && o.max_batch <= 256, LCR_ERR_INVALID, "max_batch %d outside 1..256",
               o.max_batch);
  LCRB_REQUIRE(o.max_seq > 0 && o.page_size > 0 && o.page_size % 16 == 0 && o.pool_pages > 0, LCR_ERR_SHAPE,
               "batched KV cache: max_seq, page_size (multiple of 16) and pool_pages must be positive");
  LCRB_REQUIRE(weights->embedding && weights->final_norm && weights->layers, LCR_ERR_INVALID,
               "lcr_weights: null embedding, final_norm or layers");
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
  LCRB_REQUIRE(major == 10, LCR_ERR_NO_DEVICE, "this library is built for sm_100a; device %d is sm_%d", o.device,
               major * 10);

  lcr_batch* c = new (std::nothrow) lcr_batch();
  LCRB_REQUIRE(c != nullptr, LCR_ERR_INVALID, "out of host memory");
  c->device = o.device;
  c->d = d;
  c->o = o;
  c->use_graph = (o.flags & 2) == 0;
  c->persist_gemm = (o.flags & 4) == 0;
  cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, o.device);
  c->embed = static_cast<const bf16*>(weights->embedding);
  c->final_norm = static_cast<const bf16*>(weights->final_norm);
  c->lm_head = static_cast<const bf16*>(weights->lm_head ? weights->lm_head : weights->embedding);
  c->layers.assign(weights->layers, weights->layers + d.num_layers);
  c->max_pages = (o.max_seq + o.page_size - 1) / o.page_size;

  int st = LCR_OK;
  auto cuda = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && st == LCR_OK) st = fail(LCR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  };
  cuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate");

  // Tensor maps of the weights (128 rows per tile; gate/up as two halves of 64).
  c->wmaps.resize(static_cast<size_t>(4 * d.num_layers + 1));
  for (int l = 0; l < d.num_layers && st == LCR_OK; ++l) {
    const lcr_layer_weights& w = c->layers[static_cast<size_t>(l)];
    if (!(w.input_norm && w.qkv_proj && w.o_proj && w.post_attention_norm && w.gate_up_proj && w.down_proj)) {
      st = fail(LCR_ERR_INVALID, "lcr_layer_weights: null tensor pointer");
      break;
    }
    CUtensorMap* m = &c->wmaps[static_cast<size_t>(4 * l)];
    const int ch = c->tc_chunks;
    st = make_kmajor_map(m, w.qkv_proj, qd + 2 * kvd, d.hidden_size, 1, kTcTileM, ch);
    if (st == LCR_OK) st = make_kmajor_map(m + 1, w.o_proj, d.hidden_size, qd, 1, kTcTileM, ch);
    if (st == LCR_OK) st = make_kmajor_map(m + 2, w.gate_up_proj, d.intermediate_size, d.hidden_size, 2, 64, ch);
    if (st == LCR_OK) st = make_kmajor_map(m + 3, w.down_proj, d.hidden_size, d.intermediate_size, 1, kTcTileM, ch);
  }
  if (st == LCR_OK) {
    st = make_kmajor_map(&c->wmaps.back(), c->lm_head, d.vocab_size, d.hidden_size, 1, kTcTileM, c->tc_chunks);
  }
  c->wmaps1.resize(static_cast<size_t>(4 * d.num_layers));
  for (int l = 0; l < d.num_layers && st == LCR_OK; ++l) {
    const lcr_layer_weights& w = c->layers[static_cast<size_t>(l)];
    CUtensorMap* m = &c->wmaps1[static_cast<size_t>(4 * l)];
    st = make_kmajor_map(m, w.qkv_proj, qd + 2 * kvd, d.hidden_size, 1, kTcTileM, 1);
    if (st == LCR_OK) st = make_kmajor_map(m + 1, w.o_proj, d.hidden_size, qd, 1, kTcTileM, 1);
    if (st == LCR_OK) st = make_kmajor_map(m + 2, w.gate_up_proj, d.intermediate_size, d.hidden_size, 2, 64, 1);
    if (st == LCR_OK) st = make_kmajor_map(m + 3, w.down_proj, d.hidden_size, d.intermediate_size, 1, kTcTileM, 1);
  }

  // Attention work items: 512 positions, or more for very long caches so
  // that a sequence has at most 64 partial slots per head.
  const int group = d.num_heads / d.num_kv_heads;
  c->attn_item_pos = std::max(512, ((o.max_seq + 63) / 64 + 15) / 16 * 16);
  c->attn_slots = (o.max_seq + c->attn_item_pos - 1) / c->attn_item_pos;
  if (st == LCR_OK) st = attn_batch_ctas(d.head_dim, group, o.max_batch, c->sms, &c->attn_ctas);

  // Activations and per-slot state, one allocation.
  const size_t B = static_cast<size_t>(o.max_batch);
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    const size_t at = off;
    off = (off + bytes + 255) / 256 * 256;
    return at;
  };
  const size_t o_x = carve(sizeof(bf16) * B * d.hidden_size);
  const size_t o_xsum = carve(sizeof(float) * B * d.hidden_size);
  const size_t o_xn = carve(sizeof(bf16) * B * d.hidden_size);
  const size_t o_qkv = carve(sizeof(bf16) * B * (qd + 2 * kvd));
  const size_t o_attn = carve(sizeof(bf16) * B * qd);
  const size_t o_act = carve(sizeof(bf16) * B * d.intermediate_size);
  const size_t o_part = carve(sizeof(float) * B * d.num_heads * c->attn_slots * (2 + d.head_dim));
  const size_t o_awork = carve(sizeof(unsigned) * 2);
  const size_t o_freq = carve(sizeof(float) * d.head_dim / 2);
  const size_t o_rope = carve(sizeof(float2) * B * (d.head_dim / 2));
  const size_t o_tok = carve(sizeof(int32_t) * B);
  const size_t o_pos = carve(sizeof(int32_t) * B);
  const size_t o_tab = carve(sizeof(int32_t) * B * c->max_pages);
  const size_t o_temp = carve(sizeof(float) * B);
  const size_t o_topk = carve(sizeof(int32_t) * B);
  const size_t o_topp = carve(sizeof(float) * B);
  const size_t o_seed = carve(sizeof(unsigned long long) * B);
  const size_t o_next = carve(sizeof(int32_t) * B);
  const size_t o_status = carve(sizeof(uint32_t));
  if (st == LCR_OK) cuda(cudaMalloc(&c->buf, off), "cudaMalloc(batch activations)");
  if (st == LCR_OK) cuda(cudaMemset(c->buf, 0, off), "cudaMemset(batch activations)");
  if (st == LCR_OK) {
    char* b = c->buf;
    c->x = reinterpret_cast<bf16*>(b + o_x);
    c->xsum = reinterpret_cast<float*>(b + o_xsum);
    c->xn = reinterpret_cast<bf16*>(b + o_xn);
    c->qkv = reinterpret_cast<bf16*>(b + o_qkv);
    c->attn = reinterpret_cast<bf16*>(b + o_attn);
    c->act = reinterpret_cast<bf16*>(b + o_act);
    c->partials = reinterpret_cast<float*>(b + o_part);
    c->attn_work = reinterpret_cast<unsigned*>(b + o_awork);
    c->inv_freq = reinterpret_cast<float*>(b + o_freq);
    c->rope = reinterpret_cast<float2*>(b + o_rope);
    c->tokens = reinterpret_cast<int32_t*>(b + o_tok);
    c->positions = reinterpret_cast<int32_t*>(b + o_pos);
    c->tables = reinterpret_cast<int32_t*>(b + o_tab);
    c->inv_temp = reinterpret_cast<float*>(b + o_temp);
    c->top_k = reinterpret_cast<int32_t*>(b + o_topk);
    c->top_p = reinterpret_cast<float*>(b + o_topp);
    c->seed = reinterpret_cast<unsigned long long*>(b + o_seed);
    c->next = reinterpret_cast<int32_t*>(b + o_next);
    c->status = reinterpret_cast<uint32_t*>(b + o_status);
    const std::vector<float> freq = rope_inv_freq(d);
    cuda(cudaMemcpy(c->inv_freq, freq.data(), freq.size() * sizeof(float), cudaMemcpyHostToDevice),
         "upload inv_freq");
  }
  if (st == LCR_OK) {
    cuda(cudaMalloc(&c->logits, sizeof(float) * B * d.vocab_size), "cudaMalloc(logits)");
  }
  // Split-K workspace, per batch row: two splits of the gate/up projection
  // (2 x 2F columns), or 32768 columns of the others (e.g. 10 splits of the
  // 1B model's QKV); a projection that would need more takes fewer splits.
  c->work_floats = B * std::max<size_t>(32768, 4 * static_cast<size_t>(d.intermediate_size));
  if (st == LCR_OK) cuda(cudaMalloc(&c->work, c->work_floats * sizeof(float)), "cudaMalloc(split-K workspace)");
  // KV pools: [layer][page][kv_head][page_size][D].
  c->layer_elems = static_cast<size_t>(o.pool_pages) * d.num_kv_heads * o.page_size * d.head_dim;
  const size_t kv_elems = c->layer_elems * d.num_layers;
  if (st == LCR_OK) cuda(cudaMalloc(&c->kpool, kv_elems * sizeof(bf16)), "cudaMalloc(K pool)");
  if (st == LCR_OK) cuda(cudaMalloc(&c->vpool, kv_elems * sizeof(bf16)), "cudaMalloc(V pool)");
  if (st == LCR_OK) cuda(cudaMemset(c->kpool, 0, kv_elems * sizeof(bf16)), "cudaMemset(K pool)");
  if (st == LCR_OK) cuda(cudaMemset(c->vpool, 0, kv_elems * sizeof(bf16)), "cudaMemset(V pool)");
  // Tensor maps of each layer's pools as rows of head_dim, 16-row boxes.
  const long long pool_rows = static_cast<long long>(o.pool_pages) * d.num_kv_heads * o.page_size;
  if (st == LCR_OK && pool_rows > 0x7fffffffLL) {
    st = fail(LCR_ERR_SHAPE, "KV pool of %lld rows per layer is too large", pool_rows);
  }
  c->kvmaps.resize(static_cast<size_t>(2 * d.num_layers));
  for (int l = 0; l < d.num_layers && st == LCR_OK; ++l) {
    const size_t at = static_cast<size_t>(l) * c->layer_elems;
    st = make_kmajor_map(&c->kvmaps[static_cast<size_t>(2 * l)], c->kpool + at, static_cast<int>(pool_rows),
                         d.head_dim, 1, kAbUnit, d.head_dim / 64);
    if (st == LCR_OK) {
      st = make_kmajor_map(&c->kvmaps[static_cast<size_t>(2 * l + 1)], c->vpool + at, static_cast<int>(pool_rows),
                           d.head_dim, 1, kAbUnit, d.head_dim / 64);
    }
  }
  if (st == LCR_OK) {
    cuda(cudaMallocHost(&c->pinned, sizeof(int32_t) * 2 * B * kStaging), "cudaMallocHost");
  }
  for (int i = 0; i < kStaging && st == LCR_OK; ++i) {
    cuda(cudaEventCreateWithFlags(&c->staged[i], cudaEventDisableTiming), "cudaEventCreate");
  }
  c->tables_host.assign(B * c->max_pages, 0);
  c->pages_set.assign(B, 0);
  c->inv_temp_host.assign(B, 0.f);
  c->top_k_host.assign(B, 0);
  c->top_p_host.assign(B, 1.f);
  c->seed_host.assign(B, 0ull);
  if (st != LCR_OK) {
    release(c);
    return st;
  }
  *out = c;
  return LCR_OK;
}

extern "C" void lcr_batch_destroy(lcr_batch* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  release(c);
}

extern "C" int lcr_batch_set_pages(lcr_batch* c, int slot, const int32_t* pages, int count) {
  LCRB_REQUIRE(c && (pages || count == 0), LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(slot >= 0 && slot < c->o.max_batch, LCR_ERR_INVALID, "slot %d outside 0..%d", slot,
               c->o.max_batch - 1);
  LCRB_REQUIRE(count >= 0 && count <= c->max_pages, LCR_ERR_INVALID, "%d pages; a slot holds at most %d", count,
               c->max_pages);
  for (int i = 0; i < count; ++i) {
    LCRB_REQUIRE(pages[i] >= 0 && pages[i] < c->o.pool_pages, LCR_ERR_POOL, "page %d outside the pool of %d",
                 pages[i], c->o.pool_pages);
  }
  int32_t* row = c->tables_host.data() + static_cast<size_t>(slot) * c->max_pages;
  std::memcpy(row, pages, sizeof(int32_t) * count);
  std::fill(row + count, row + c->max_pages, 0);
  c->pages_set[static_cast<size_t>(slot)] = count;
  c->tables_dirty = true;
  return LCR_OK;
}

extern "C" int lcr_batch_set_sampling(lcr_batch* c, int slot, float temperature, int top_k, float top_p,
                                      uint64_t seed) {
  LCRB_REQUIRE(c, LCR_ERR_INVALID, "null batch");
  LCRB_REQUIRE(slot >= 0 && slot < c->o.max_batch, LCR_ERR_INVALID, "slot %d outside 0..%d", slot,
               c->o.max_batch - 1);
  LCRB_REQUIRE(temperature >= 0.f && top_p > 0.f && top_p <= 1.f, LCR_ERR_INVALID,
               "bad sampling parameters (temperature %g, top_p %g)", temperature, top_p);
  c->inv_temp_host[static_cast<size_t>(slot)] = temperature > 0.f ? 1.0f / temperature : 0.f;
  c->top_k_host[static_cast<size_t>(slot)] = top_k;
  c->top_p_host[static_cast<size_t>(slot)] = top_p;
  c->seed_host[static_cast<size_t>(slot)] = seed;
  c->sampling_dirty = true;
  return LCR_OK;
}

extern "C" int lcr_batch_step(lcr_batch* c, int n, const int32_t* tokens, const int32_t* positions) {
  LCRB_REQUIRE(c && positions, LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(n >= 1 && n <= c->o.max_batch, LCR_ERR_INVALID, "batch of %d slots; this context holds %d", n,
               c->o.max_batch);
  for (int b = 0; b < n; ++b) {
    LCRB_REQUIRE(positions[b] >= 0 && positions[b] < c->o.max_seq, LCR_ERR_STATE,
                 "slot %d: position %d outside the cache built for %d", b, positions[b], c->o.max_seq);
    LCRB_REQUIRE(positions[b] / c->o.page_size < c->pages_set[static_cast<size_t>(b)], LCR_ERR_STATE,
                 "slot %d: no page for position %d (its table holds %d pages)", b, positions[b],
                 c->pages_set[static_cast<size_t>(b)]);
  }
  LCRB_CUDA(cudaSetDevice(c->device));
  const size_t B = static_cast<size_t>(c->o.max_batch);
  LCRB_TRY(upload_slot_state(c));
  // (token, position) staging: a pinned area is reused only after the copy
  // that last read it has completed.
  const int slot = c->staging_next;
  c->staging_next = (slot + 1) % kStaging;
  LCRB_CUDA(cudaEventSynchronize(c->staged[slot]));
  int32_t* area = c->pinned + static_cast<size_t>(slot) * 2 * B;
  std::memcpy(area + B, positions, sizeof(int32_t) * n);
  if (tokens) {
    std::memcpy(area, tokens, sizeof(int32_t) * n);
    LCRB_CUDA(cudaMemcpyAsync(c->tokens, area, sizeof(int32_t) * n, cudaMemcpyHostToDevice, c->stream));
  } else {  // each slot continues with the id it sampled last step
    LCRB_CUDA(cudaMemcpyAsync(c->tokens, c->next, sizeof(int32_t) * n, cudaMemcpyDeviceToDevice, c->stream));
  }
  LCRB_CUDA(cudaMemcpyAsync(c->positions, area + B, sizeof(int32_t) * n, cudaMemcpyHostToDevice, c->stream));
  LCRB_CUDA(cudaEventRecord(c->staged[slot], c->stream));
  c->last_n = n;
  return launch_step(c, n);
}

extern "C" int lcr_batch_fill_kv(lcr_batch* c, int slot, int length, uint64_t seed) {
  LCRB_REQUIRE(c, LCR_ERR_INVALID, "null batch");
  LCRB_REQUIRE(slot >= 0 && slot < c->o.max_batch, LCR_ERR_INVALID, "slot %d", slot);
  LCRB_REQUIRE(length >= 0 && length <= c->o.max_seq, LCR_ERR_STATE, "length %d outside the cache", length);
  LCRB_REQUIRE((length + c->o.page_size - 1) / c->o.page_size <= c->pages_set[static_cast<size_t>(slot)],
               LCR_ERR_STATE, "slot %d: %d positions need more than its %d pages", slot, length,
               c->pages_set[static_cast<size_t>(slot)]);
  if (length == 0) return LCR_OK;
  LCRB_CUDA(cudaSetDevice(c->device));
  if (c->tables_dirty) {
    LCRB_CUDA(cudaMemcpyAsync(c->tables, c->tables_host.data(),
                              sizeof(int32_t) * static_cast<size_t>(c->o.max_batch) * c->max_pages,
                              cudaMemcpyHostToDevice, c->stream));
    c->tables_dirty = false;
  }
  FillKvArgs a = {};
  a.kpool = c->kpool;
  a.vpool = c->vpool;
  a.layer_elems = c->layer_elems;
  a.layers = c->d.num_layers;
  a.kv_heads = c->d.num_kv_heads;
  a.head_dim = c->d.head_dim;
  a.page_size = c->o.page_size;
  a.length = length;
  a.pages = c->tables + static_cast<size_t>(slot) * c->max_pages;
  a.seed = seed;
  fill_kv_kernel<<<4 * c->sms, 256, 0, c->stream>>>(a);
  return launch_status("fill_kv");
}

namespace {

// Grows the prefill activations to at least `rows` rows (a multiple of 128).
int prefill_reserve(lcr_batch* c, int rows) {
  if (rows <= c->pre_rows) return LCR_OK;
  const lcr_model_desc& d = c->d;
  const size_t R = static_cast<size_t>((rows + 127) / 128 * 128);
  const int qd = d.num_heads * d.head_dim, kvd = d.num_kv_heads * d.head_dim;
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    const size_t at = off;
    off = (off + bytes + 255) / 256 * 256;
    return at;
  };
  const size_t o_tok = carve(sizeof(int32_t) * R), o_pos = carve(sizeof(int32_t) * R);
  const size_t o_x = carve(sizeof(bf16) * R * d.hidden_size), o_xsum = carve(sizeof(float) * R * d.hidden_size);
  const size_t o_xn = carve(sizeof(bf16) * R * d.hidden_size), o_qkv = carve(sizeof(bf16) * R * (qd + 2 * kvd));
  const size_t o_attn = carve(sizeof(bf16) * R * qd), o_act = carve(sizeof(bf16) * R * d.intermediate_size);
  const size_t o_rope = carve(sizeof(float2) * R * (d.head_dim / 2));
  LCRB_CUDA(cudaStreamSynchronize(c->stream));  // the old buffers may still be in use
  cudaFree(c->pre_buf);
  c->pre_buf = nullptr;
  c->pre_rows = 0;
  LCRB_CUDA(cudaMalloc(&c->pre_buf, off));
  char* b = c->pre_buf;
  c->pre = Acts{reinterpret_cast<int32_t*>(b + o_tok), reinterpret_cast<int32_t*>(b + o_pos),
                reinterpret_cast<bf16*>(b + o_x),       reinterpret_cast<float*>(b + o_xsum),
                reinterpret_cast<bf16*>(b + o_xn),      reinterpret_cast<bf16*>(b + o_qkv),
                reinterpret_cast<bf16*>(b + o_attn),    reinterpret_cast<bf16*>(b + o_act),
                reinterpret_cast<float2*>(b + o_rope)};
  c->pre_rows = static_cast<int>(R);
  return LCR_OK;
}

}  // namespace

namespace lcrb {

cudaStream_t batch_stream(lcr_batch* c) { return c->stream; }
int make_prefill_kv_map(CUtensorMap* out, const bf16* pool, int rows, int head_dim) {
  return make_kmajor_map(out, pool, rows, head_dim, 1, kAbUnit, head_dim / 64);
}
int batch_check_status(lcr_batch* c) { return check_status(c); }

int batch_prefill_into(lcr_batch* c, const PrefillKv& kv, const int32_t* tokens, int count, int start,
                       float* logits) {
  const lcr_model_desc& d = c->d;
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_TRY(prefill_reserve(c, count));
  const Acts& v = c->pre;
  const int H = d.hidden_size, F = d.intermediate_size;
  const int qd = d.num_heads * d.head_dim, kvd = d.num_kv_heads * d.head_dim;
  // Inputs of the chunk (pageable sources are staged by the copy itself).
  std::vector<int32_t> pos(static_cast<size_t>(count));
  for (int i = 0; i < count; ++i) pos[static_cast<size_t>(i)] = start + i;
  LCRB_CUDA(cudaMemcpyAsync(v.tokens, tokens, sizeof(int32_t) * count, cudaMemcpyHostToDevice, c->stream));
  LCRB_CUDA(cudaMemcpyAsync(v.positions, pos.data(), sizeof(int32_t) * count, cudaMemcpyHostToDevice, c->stream));
  // Activation tensor maps for this chunk's batch tiles (one 64-column chunk
  // per stage), and the tile of each projection.
  const int nb = gemm_tc_batch_tile(count);
  StepMaps m, m2;
  LCRB_TRY(make_kmajor_map(&m.xn, v.xn, c->pre_rows, H, 1, nb, 1));
  LCRB_TRY(make_kmajor_map(&m.attn, v.attn, c->pre_rows, qd, 1, nb, 1));
  LCRB_TRY(make_kmajor_map(&m.act, v.act, c->pre_rows, F, 1, nb, 1));
  // 256-row tiles (persistent kernel; a third fewer shared-memory operand
  // bytes per FLOP, modelled as 1.36x the rate of 128-row tiles) where they
  // need no split-K and their last round of tiles idles no more SMs than
  // that saves.
  auto wide = [&](int weight_tiles) {
    if (nb != 128 || !c->persist_gemm) return false;
    const long long t128 = static_cast<long long>(weight_tiles) * ((count + 127) / 128);
    const long long t256 = static_cast<long long>(weight_tiles) * ((count + 255) / 256);
    if (2 * t256 <= c->sms) return false;
    const long long r128 = (t128 + c->sms - 1) / c->sms, r256 = (t256 + c->sms - 1) / c->sms;
    return r256 * 376 <= r128 * 256;
  };
  const bool wide_qkv = wide((qd + 2 * kvd + kTcTileM - 1) / kTcTileM);
  const bool wide_o = wide((H + kTcTileM - 1) / kTcTileM);
  const bool wide_gu = wide((F + 63) / 64);
  const bool wide_down = wide((H + kTcTileM - 1) / kTcTileM);
  if (wide_qkv || wide_o || wide_gu || wide_down) {
    LCRB_TRY(make_kmajor_map(&m2.xn, v.xn, c->pre_rows, H, 1, 256, 1));
    LCRB_TRY(make_kmajor_map(&m2.attn, v.attn, c->pre_rows, qd, 1, 256, 1));
    LCRB_TRY(make_kmajor_map(&m2.act, v.act, c->pre_rows, F, 1, 256, 1));
  }
  const int group = d.num_heads / d.num_kv_heads;
  const int pad_rows = (start + count + 15) / 16 * 16 - start;
  for (int l = 0; l < d.num_layers; ++l) {
    const lcr_layer_weights& w = c->layers[static_cast<size_t>(l)];
    const CUtensorMap* wm = &c->wmaps1[static_cast<size_t>(4 * l)];
    const int32_t* table = kv.table + static_cast<size_t>(l) * kv.table_layer_stride;
    LCRB_TRY(norm_launch(c, v, count, l == 0, w.input_norm));
    LCRB_TRY(gemm_node(c, v, wm[0], wide_qkv ? m2.xn : m.xn, wide_qkv ? 256 : nb, count, qd + 2 * kvd, H, EPI_ROPE,
                       v.qkv, nullptr, qd + 2 * kvd, 1));
    KvWriteArgs kw = {};
    kw.qkv = v.qkv;
    kw.qkv_stride = qd + 2 * kvd;
    kw.q_dim = qd;
    kw.kv_dim = kvd;
    kw.head_dim = d.head_dim;
    kw.kv_heads = d.num_kv_heads;
    kw.kpool = kv.kpool + static_cast<size_t>(l) * kv.layer_elems;
    kw.vpool = kv.vpool + static_cast<size_t>(l) * kv.layer_elems;
    kw.table = table;
    kw.page_size = kv.page_size;
    kw.pool_pages = kv.pool_pages;
    kw.page_stride = static_cast<long long>(d.num_kv_heads) * kv.page_size * d.head_dim;
    kw.head_stride = static_cast<long long>(kv.page_size) * d.head_dim;
    kw.start = start;
    kw.count = count;
    kw.limit = kv.limit;
    kw.status = c->status;
    LCRB_TRY(launch_kernel(kv_write_kernel, dim3(static_cast<unsigned>(pad_rows)), dim3(128), 0, c->stream, true, kw));
    PrefillAttnArgs pa = {};
    pa.qkv = v.qkv;
    pa.qkv_stride = qd + 2 * kvd;
    pa.q_dim = qd;
    pa.kv_dim = kvd;
    pa.table = table;
    pa.page_size = kv.page_size;
    pa.pool_pages = kv.pool_pages;
    pa.start = start;
    pa.count = count;
    pa.scale_log2 = (1.0f / std::sqrt(static_cast<float>(d.head_dim))) * kLog2e;
    pa.out = v.attn;
    pa.status = c->status;
    const CUtensorMap* km = kv.kvmaps + static_cast<size_t>(l) * kv.kvmap_layer_stride;
    LCRB_TRY(attn_prefill_launch(pa, km[0], km[1], d.head_dim, group, d.num_kv_heads, c->stream));
    LCRB_TRY(gemm_node(c, v, wm[1], wide_o ? m2.attn : m.attn, wide_o ? 256 : nb, count, H, qd, EPI_RESID, nullptr,
                       nullptr, H, 1));
    LCRB_TRY(norm_launch(c, v, count, false, w.post_attention_norm));
    LCRB_TRY(gemm_node(c, v, wm[2], wide_gu ? m2.xn : m.xn, wide_gu ? 256 : nb, count, F, H, EPI_SWIGLU, v.act, nullptr,
                       F, 1));
    LCRB_TRY(gemm_node(c, v, wm[3], wide_down ? m2.act : m.act, wide_down ? 256 : nb, count, H, F, EPI_RESID, nullptr,
                       nullptr, H, 1));
  }
  // The last row only: final norm, lm_head into fp32 logits.
  Acts last = v;
  last.x += static_cast<size_t>(count - 1) * H;
  last.xsum += static_cast<size_t>(count - 1) * H;
  LCRB_TRY(norm_launch(c, last, 1, false, c->final_norm));
  CUtensorMap xlast;
  LCRB_TRY(make_kmajor_map(&xlast, v.xn, c->pre_rows, H, 1, 16, c->tc_chunks));
  return gemm_node(c, last, c->wmaps.back(), xlast, 16, 1, d.vocab_size, H, EPI_STORE_F32, nullptr, logits,
                   d.vocab_size, c->tc_chunks);
}

}  // namespace lcrb

extern "C" int lcr_batch_prefill(lcr_batch* c, int slot, const int32_t* tokens, int count, int start) {
  LCRB_REQUIRE(c && tokens, LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(slot >= 0 && slot < c->o.max_batch, LCR_ERR_INVALID, "slot %d outside 0..%d", slot,
               c->o.max_batch - 1);
  LCRB_REQUIRE(count >= 1 && start >= 0 && start + count <= c->o.max_seq, LCR_ERR_STATE,
               "prefill of %d positions at %d outside the cache built for %d", count, start, c->o.max_seq);
  LCRB_REQUIRE((start + count - 1) / c->o.page_size < c->pages_set[static_cast<size_t>(slot)], LCR_ERR_STATE,
               "slot %d: no page for position %d (its table holds %d pages)", slot, start + count - 1,
               c->pages_set[static_cast<size_t>(slot)]);
  const lcr_model_desc& d = c->d;
  for (int i = 0; i < count; ++i) {
    LCRB_REQUIRE(tokens[i] >= 0 && tokens[i] < d.vocab_size, LCR_ERR_INVALID, "token %d: id %d outside the vocabulary",
                 i, tokens[i]);
  }
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_TRY(upload_slot_state(c));
  // The batch's own pools: one per layer, the slot's table shared by all layers.
  PrefillKv kv = {};
  kv.kpool = c->kpool;
  kv.vpool = c->vpool;
  kv.layer_elems = c->layer_elems;
  kv.table = c->tables + static_cast<size_t>(slot) * c->max_pages;
  kv.table_layer_stride = 0;
  kv.page_size = c->o.page_size;
  kv.pool_pages = c->o.pool_pages;
  kv.kvmaps = c->kvmaps.data();
  kv.kvmap_layer_stride = 2;
  kv.limit = c->max_pages * c->o.page_size;
  float* logits = c->logits + static_cast<size_t>(slot) * d.vocab_size;
  LCRB_TRY(batch_prefill_into(c, kv, tokens, count, start, logits));
  // Sample with this slot's parameters and Philox counter = the last position.
  SampleArgs s = {};
  s.logits = logits;
  s.row_stride = d.vocab_size;
  s.vocab = d.vocab_size;
  s.inv_temperature = c->inv_temp + slot;
  s.top_k = c->top_k + slot;
  s.top_p = c->top_p + slot;
  s.uniform = nullptr;
  s.seed = c->seed + slot;
  s.counter = c->pre.positions + (count - 1);
  s.out = c->next + slot;
  return sample_launch(s, 1, c->stream, true);
}

extern "C" int lcr_batch_read(lcr_batch* c, int32_t* next_ids, int n) {
  LCRB_REQUIRE(c && next_ids, LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(n >= 0 && n <= c->o.max_batch, LCR_ERR_INVALID, "bad count %d", n);
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_CUDA(cudaMemcpyAsync(next_ids, c->next, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, c->stream));
  return check_status(c);
}

extern "C" int lcr_batch_logits(lcr_batch* c, int slot, float* host) {
  LCRB_REQUIRE(c && host, LCR_ERR_INVALID, "null argument");
  LCRB_REQUIRE(slot >= 0 && slot < c->o.max_batch, LCR_ERR_INVALID, "slot %d", slot);
  LCRB_CUDA(cudaSetDevice(c->device));
  LCRB_CUDA(cudaMemcpyAsync(host, c->logits + static_cast<size_t>(slot) * c->d.vocab_size,
                            sizeof(float) * c->d.vocab_size, cudaMemcpyDeviceToHost, c->stream));
  return check_status(c);
}

extern "C" int lcr_batch_sync(lcr_batch* c) {
  LCRB_REQUIRE(c, LCR_ERR_INVALID, "null batch");
  LCRB_CUDA(cudaSetDevice(c->device));
  return check_status(c);
}

extern "C" lcr_stream_t lcr_batch_stream(lcr_batch* c) {
  return c ? reinterpret_cast<lcr_stream_t>(c->stream) : nullptr;
}

extern "C" int lcr_batch_step_launches(const lcr_batch* c, int n) {
  if (!c) return 0;
  const auto it = c->launches_by_n.find(n);
  return it == c->launches_by_n.end() ? 0 : it->second;
}

extern "C" int lcr_batch_time_steps(lcr_batch* c, int steps, float* ms) {
  LCRB_REQUIRE(c && ms && steps > 0 && c->last_n > 0, LCR_ERR_INVALID,
               "time_steps needs a previous lcr_batch_step and a positive count");
  LCRB_CUDA(cudaSetDevice(c->device));
  cudaEvent_t e0, e1;
  LCRB_CUDA(cudaEventCreate(&e0));
  LCRB_CUDA(cudaEventCreate(&e1));
  cudaEventRecord(e0, c->stream);
  int st = LCR_OK;
  for (int i = 0; i < steps && st == LCR_OK; ++i) st = launch_step(c, c->last_n);
  cudaEventRecord(e1, c->stream);
  cudaEventSynchronize(e1);
  float t = 0.f;
  cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (st != LCR_OK) return st;
  *ms = t;
  return check_status(c);
}
