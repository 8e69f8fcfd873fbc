// The whole decode step as ONE persistent cooperative kernel.
//
// One CTA per SM (cooperative launch guarantees they are co-resident): 8
// consumer warps, the ring producer (warp 8) and an L2 prefetcher (warp 9);
// a 6-stage x 33 KB shared-memory ring of weight (or K/V) stages. Per layer
// the step has five phases, each needing every output of the one before (a
// batch-1 step is a chain of full reductions):
//
//   QKV   rows of [q;k;v]: RMSNorm prologue (embedding row for layer 0)
//   ATTN  one (KV head, split) item per CTA: RoPE, KV write, split-K
//         online softmax over the KV pages; the splits are merged in this
//         phase (split 0 of each KV head up to 4 splits, splits 0-3 each a
//         quarter of the head group beyond; the grid-barrier form merges up
//         to 4 in the O prologue). With tensor maps of the cache (head_dim
//         64): QK^T and PV of each 16-position unit on the tensor pipe
//         (mega_attn_consume_tc); otherwise CUDA-core dot products, 8 lanes
//         per position.
//   O     rows of o_proj, residual epilogue
//   GU    gate/up row pairs: RMSNorm prologue, SwiGLU epilogue
//   DOWN  rows of down_proj, residual epilogue
//
// then the lm_head rows with the final norm and the argmax hand-off.
//
// Two arithmetic modes (template F32):
//   F32 = true   activations stay fp32 end to end, as in the fp32 host
//                evaluation: GEMV inputs are split into a bf16 pair hi + lo
//                fed to the two halves of one m16n8k16 A operand (gemv.cuh,
//                mma_x_hilo); q, k, v, the attention output, the residual
//                stream and SwiGLU stay fp32. Only the KV cache holds bf16 (the
//                reference's KvCacheView format). The ring has 5 stages: the
//                staged input's low half takes the sixth stage's shared memory.
//   F32 = false  the reference's storage rounding (src/model.cu:370-484):
//                bf16 normed inputs, qkv, roped q/k, attention output,
//                projections, residual stream and SwiGLU output, with the
//                unrounded residual sum feeding the norm.
// Between phases (template LL): by default the phases exchange their outputs
// as tagged words (ll.cuh) and each phase polls only its own inputs; the
// other instance meets at a grid barrier (an arrival counter with a bounded
// acquire spin). Both compute the same bits. The producer never waits at
// phase boundaries: it walks the same schedule -- this CTA's rows of every
// matrix, and the KV blocks of its attention item -- and keeps the ring full,
// so HBM keeps streaming the next matrices while the consumers wait. The
// arithmetic per output is that of the multi-kernel step (the same device
// functions).
#pragma once

#include "attention.cuh"
#include "attn_batch.cuh"  // ab_offset, ldmatrix_x4_trans
#include "gemv.cuh"

namespace lcrb {

constexpr int kMegaStageBytes = kGemvSlotBytes;
// Ring stages: 6, or 5 with fp32 activations.
template <bool F32>
constexpr int kMegaStages = F32 ? 5 : 6;
// 8 consumer warps, the ring producer (warp 8) and the L2 prefetcher (warp 9).
constexpr int kMegaThreads = kGemvConsumers + 64;
constexpr int kMegaWarps = kGemvConsumers / 32;

struct MegaLayer {
  const bf16* input_norm;
  const bf16* qkv;
  const bf16* o;
  const bf16* post_norm;
  const bf16* gate_up;
  const bf16* down;
};

struct MegaArgs {
  int layers, vocab, num_kv, max_seq, splits;
  float eps, scale_log2;
  const bf16* embed;
  const bf16* final_norm;
  const bf16* lm_head;
  const MegaLayer* L;  // device array [layers]
  const CUtensorMap* wmaps;  // device array: [layer * 4 + m] (qkv, o, gate/up, down), then lm_head
  const float* inv_freq;
  int32_t* state;      // [0] token, [1] position
  bf16* x;
  float* xsum;         // unrounded residual sums (with fp32 activations: the residual stream)
  bf16* qkv;
  bf16* attn;
  bf16* act;
  float* qkv_f;        // fp32 activations: q;k;v, the merged attention output, SwiGLU
  float* attn_f;
  float* act_f;
  float* logits;
  float* partials;     // [heads][splits][2 + D]
  unsigned* attn_ctr;  // [layers][num_kv]
  unsigned* bar;       // grid barrier arrivals, zero at launch
  unsigned long long* argmax_acc;
  unsigned* argmax_done;  // [2], [1] counts finished CTAs
  int32_t* history;
  int history_len;
  uint32_t* status;
  // KV cache
  bf16* kpool;
  bf16* vpool;
  const int32_t* tables;  // paged: [layers][max_pages]
  int max_pages, pool_pages, page_size;
  long long page_stride, head_stride, layer_stride;  // layer_stride: contiguous
  // Tensor maps of the cache rows ({64, 16, D / 64} boxes, 128-byte swizzle):
  // [l * kvmap_layer_stride + {0: K, 1: V}], the row of (kv head, position)
  // being (page * num_kv + kv head) * page_size + position % page_size when
  // paged, kv head * max_seq + position per layer otherwise. nullptr: the
  // CUDA-core attention phase.
  const CUtensorMap* kvmaps;
  int kvmap_layer_stride;
  // Low-latency exchange between phases (ll.cuh) instead of grid barriers
  // (the kernel instance with LL; bf16 activations with the tensor-pipe
  // attention only). Tags: epoch base + 5 layer + phase + 1; the step's last
  // CTA advances the base.
  int ll;
  uint32_t* epoch;
  uint32_t* qkv_ll;              // [QD + 2 KVD] LL32, phase 0
  unsigned long long* part_ll;   // [heads][splits][D + 4] LL64 split records, phase 1
  uint32_t* attn_ll;             // [QD] LL32 merged output (many splits), phase 1
  unsigned long long* x_ll;      // [H] LL64 residual sums, phases 2 (O) and 4 (DOWN)
  uint32_t* act_ll;              // [F] LL32, phase 3
  // qkv_ll, attn_ll, x_ll and act_ll are held in kLLCopies replicas
  // ll_copy_bytes apart: writers store every replica, CTA c reads replica
  // c % kLLCopies (fewer CTAs polling each line).
  unsigned long long ll_copy_bytes;
  unsigned long long prefetch_bytes;  // L2 prefetch lead of the producer (0: off)
  int split_positions;                // attention: cached positions per split this step aims at
  unsigned long long wait_ns;         // bound of each grid-barrier wait
  int test_skip_arrival;              // test only: CTA 0 does not arrive at the first grid barrier
                                      // (exchange: does not publish its first q/k/v rows)
  // Optional phase trace (globaltimer ns), per CTA kMegaTraceEvents slots:
  // [0] consumers start, [1 + 2k] arrival at barrier k, [2 + 2k] departure,
  // [kMegaTraceProducer + p] producer starting phase p.
  unsigned long long* trace;
};

constexpr int kMegaTraceEvents = 1024;
constexpr int kMegaTraceProducer = 256;
// SM cycles consumer thread 0 waited on full stages in GEMV phase p, and the
// producer waited on empty slots while issuing GEMV phase p.
constexpr int kMegaTraceConsumerWait = 340;
constexpr int kMegaTraceProducerWait = 424;
// Per-stage timestamps of one layer's gate/up phase: producer issue [512 + s],
// consumer thread 0 stage ready [576 + s] and released [640 + s].
constexpr int kMegaTraceStageLayer = 8;
constexpr int kMegaTraceStages = 512;


__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier over the consumer threads of every CTA. Returns false (and
// raises the abort bit so every other CTA stops waiting too) if the bounded
// wait expired or another CTA already aborted.
__device__ __forceinline__ bool mega_grid_sync(unsigned* bar, unsigned target, uint32_t* status,
                                               int* s_abort, unsigned long long* trace = nullptr,
                                               uint64_t wait_ns = kWaitLimitNs, bool arrive = true) {
  named_sync(1, kGemvConsumers);
  if (threadIdx.x == 0) {
    if (trace) trace[0] = globaltimer_ns();
    // Release at GPU scope: every write this CTA's consumers made before the
    // named barrier is visible to whoever acquires the count.
    if (arrive) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
    uint64_t start = 0;
    for (uint32_t spin = 0;; ++spin) {
      if (ld_acquire_u32(bar) >= target) break;
      if ((spin & 63u) == 63u) {
        if (__ldcg(status) & kStatusAbort) {
          *s_abort = 1;
          break;
        }
        const uint64_t now = globaltimer_ns();
        if (start == 0) {
          start = now;
        } else if (now - start > wait_ns) {
          atomicOr(status, kStatusTimeoutBarrier | kStatusAbort);
          *s_abort = 1;
          break;
        }
      }
    }
    if (trace) trace[1] = globaltimer_ns();
  }
  named_sync(1, kGemvConsumers);
  return *s_abort == 0;
}

// ---------------------------------------------------------------------------
// fp32-activation staging
// ---------------------------------------------------------------------------

// 8 fp32 values -> their bf16 pair (hi, lo = bf16(v - hi)) at chunk c.
__device__ __forceinline__ void store_hilo8(const float (&v)[8], bf16* xs, bf16* xs_lo, int c) {
  uint4 hi;
  hi.x = pack_bf2(v[0], v[1]);
  hi.y = pack_bf2(v[2], v[3]);
  hi.z = pack_bf2(v[4], v[5]);
  hi.w = pack_bf2(v[6], v[7]);
  reinterpret_cast<uint4*>(xs)[c] = hi;
  float h[8];
  unpack8(hi, h);
  uint4 lo;
  lo.x = pack_bf2(v[0] - h[0], v[1] - h[1]);
  lo.y = pack_bf2(v[2] - h[2], v[3] - h[3]);
  lo.z = pack_bf2(v[4] - h[4], v[5] - h[5]);
  lo.w = pack_bf2(v[6] - h[6], v[7] - h[7]);
  reinterpret_cast<uint4*>(xs_lo)[c] = lo;
}

// RMSNorm of the fp32 residual stream `xsum` (or, when `embed` is given, of
// the device token's embedding row, which CTA 0 also stores as the stream)
// times `gain`, staged as the bf16 pair xs + xs_lo, every value fp32 up to the
// pair's ~16 significant bits. Uses named barrier 1; complete on return.
template <int K>
__device__ __forceinline__ void mega_stage_norm_f32(const float* xsum, const bf16* embed, const int32_t* token,
                                                    int vocab, uint32_t* status, bf16* x_out, float* xsum_out,
                                                    const bf16* gain, float eps, bf16* xs, bf16* xs_lo,
                                                    float* red8) {
  constexpr int NC = K / 8;
  constexpr int PER = (NC + kGemvConsumers - 1) / kGemvConsumers;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bf16* erow = nullptr;
  if (embed != nullptr) {
    int tok = __ldcg(token);
    if (tok < 0 || tok >= vocab) {
      if (tid == 0) atomicOr(status, kStatusBadToken);
      tok = 0;
    }
    erow = embed + static_cast<size_t>(tok) * K;
  }
  float v[PER][8];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int c = tid + p * kGemvConsumers;
    if (c >= NC) break;
    if (erow != nullptr) {
      const uint4 raw = ldg_cg16(erow + c * 8);
      unpack8(raw, v[p]);
      if (blockIdx.x == 0) {
        *reinterpret_cast<uint4*>(x_out + c * 8) = raw;
        *reinterpret_cast<float4*>(xsum_out + c * 8) = make_float4(v[p][0], v[p][1], v[p][2], v[p][3]);
        *reinterpret_cast<float4*>(xsum_out + c * 8 + 4) = make_float4(v[p][4], v[p][5], v[p][6], v[p][7]);
      }
    } else {
      const float4 a0 = __ldcg(reinterpret_cast<const float4*>(xsum + c * 8));
      const float4 a1 = __ldcg(reinterpret_cast<const float4*>(xsum + c * 8 + 4));
      v[p][0] = a0.x; v[p][1] = a0.y; v[p][2] = a0.z; v[p][3] = a0.w;
      v[p][4] = a1.x; v[p][5] = a1.y; v[p][6] = a1.z; v[p][7] = a1.w;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[p][e], v[p][e], ss);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) red8[warp] = ss;
  named_sync(1, kGemvConsumers);
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kGemvConsumers / 32; ++w) total += red8[w];
  const float scale = rsqrtf(total / static_cast<float>(K) + eps);
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int c = tid + p * kGemvConsumers;
    if (c >= NC) break;
    float gf[8], n[8];
    unpack8(ldg16(gain + c * 8), gf);
#pragma unroll
    for (int e = 0; e < 8; ++e) n[e] = __fmul_rn(__fmul_rn(v[p][e], scale), gf[e]);
    store_hilo8(n, xs, xs_lo, c);
  }
  named_sync(1, kGemvConsumers);  // xs complete (and red8 free again)
}

// An fp32 vector of n values (a multiple of 8) staged as the bf16 pair
// xs + xs_lo. Uses named barrier 1; complete on return.
__device__ __forceinline__ void mega_stage_vec_f32(const float* src, int n, bf16* xs, bf16* xs_lo) {
  for (int c = threadIdx.x; c < n / 8; c += kGemvConsumers) {
    const float4 a0 = __ldcg(reinterpret_cast<const float4*>(src + c * 8));
    const float4 a1 = __ldcg(reinterpret_cast<const float4*>(src + c * 8 + 4));
    const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    store_hilo8(v, xs, xs_lo, c);
  }
  named_sync(1, kGemvConsumers);
}

// 8 fp32 dims of one head from this step's fp32 qkv row with the rotate-half
// RoPE applied from the step's cos/sin table, kept in fp32.
template <int D>
__device__ __forceinline__ void rope8f(const float* head, int lig, const float* cs, float* outv) {
  constexpr int HALF = D / 2;
  const int d0 = lig * 8;
  const int p0 = d0 < HALF ? d0 + HALF : d0 - HALF;
  const float4 s0 = __ldcg(reinterpret_cast<const float4*>(head + d0));
  const float4 s1 = __ldcg(reinterpret_cast<const float4*>(head + d0 + 4));
  const float4 o0 = __ldcg(reinterpret_cast<const float4*>(head + p0));
  const float4 o1 = __ldcg(reinterpret_cast<const float4*>(head + p0 + 4));
  const float self[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  const float other[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
  const bool lo = d0 < HALF;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int i = (d0 + e) % HALF;
    const float c = cs[i], s = cs[HALF + i];
    outv[e] = lo ? (self[e] * c - other[e] * s) : (self[e] * c + other[e] * s);
  }
}

// ---------------------------------------------------------------------------
// Attention phase
// ---------------------------------------------------------------------------

template <int D>
struct MegaAttnGeom {
  static constexpr int LPP = D / 8;            // lanes per position
  static constexpr int GPW = 32 / LPP;         // positions per warp per pass
  static constexpr int P = kMegaWarps * GPW;   // positions per pass of the 8 warps
  static constexpr int ROWB = D * 2;
  // A ring stage carries STAGE_POS positions: K in its first 16 KB, V in the
  // next, consumed in PASSES passes (128 positions at D = 64).
  static constexpr int STAGE_POS = 16384 / ROWB;
  static constexpr int PASSES = STAGE_POS / P;
  static_assert(2 * STAGE_POS * ROWB <= kMegaStageBytes, "KV stage must fit a ring stage");
  static_assert(PASSES >= 1 && STAGE_POS % P == 0, "a stage is whole passes");
};

__device__ __forceinline__ int mega_attn_chunk(int seq_len, int splits, int p) {
  const int per = (seq_len + splits - 1) / splits;
  return (per + p - 1) / p * p;
}

// Physical element offset of (kv head, position) in layer `l` of the cache.
// A page-table entry outside the pool raises kStatusBadPage and reads page 0.
template <bool PAGED>
__device__ __forceinline__ long long kv_offset(const MegaArgs& a, int l, int kvh, int pos, int D) {
  if constexpr (PAGED) {
    int page = a.tables[static_cast<size_t>(l) * a.max_pages + pos / a.page_size];
    if (page < 0 || page >= a.pool_pages) {
      atomicOr(a.status, kStatusBadPage);
      page = 0;
    }
    return static_cast<long long>(page) * a.page_stride + kvh * a.head_stride +
           static_cast<long long>(pos % a.page_size) * D;
  } else {
    return static_cast<long long>(l) * a.layer_stride + kvh * a.head_stride +
           static_cast<long long>(pos) * D;
  }
}

struct AttnItem {
  int kvh, split, splits, begin, end, cache_end, nblocks;
};

// This CTA's replica of an exchange buffer (kLLCopies of them).
template <class T>
__device__ __forceinline__ T* mega_ll_mine(const MegaArgs& a, T* p) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(p) +
                              static_cast<unsigned long long>(blockIdx.x % kLLCopies) * a.ll_copy_bytes);
}

__device__ __forceinline__ int mega_attn_splits(int seq_len, int max_splits, int per_split) {
  return max(1, min(max_splits, (seq_len + per_split - 1) / per_split));
}

// Split partial record: acc[D], m, l, two floats of padding (16-byte rows).
template <int D>
constexpr int kMegaPartStride = D + 4;
// Largest split count the persistent step uses.
constexpr int kMegaMaxMergeSplits = 32;
// Grid-barrier form: up to this many splits the O projection's prologue
// merges them (one round of L2 loads); beyond it the last split of each KV
// head to finish merges its heads once and the prologue loads the bf16
// result. The exchange form always merges in the attention phase (split 0
// of each KV head, with the prologue's arithmetic up to this count, so the
// two forms give the same bits), because every O-phase CTA polling every
// split record (80 KB per CTA per attempt) cost ~4.7 us per layer.
constexpr int kMegaPrologueMergeMax = 4;
// Exchange form, more than kMegaPrologueMergeMax splits: this many split CTAs
// per KV head share the merge.
constexpr int kMegaMergers = 4;

// Online logsumexp merge of the split records rec0[s * stride_s] for s in
// [s_begin, s_end) stepping by `step`, dims d0..d0+7, into (M, L, acc) --
// four records per round of L2 loads.
template <int D>
__device__ __forceinline__ void merge_split_records(const float* rec0, int s_begin, int s_end, int step, int d0,
                                                    float& M, float& L, float (&acc)[8]) {
  constexpr int B = 4;
  for (int s0 = s_begin; s0 < s_end; s0 += B * step) {
    float ms[B], ls[B];
    float4 lo[B], hi[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int s = s0 + b * step;
      const bool in = s < s_end;
      const float* rec = rec0 + static_cast<size_t>(in ? s : s_begin) * kMegaPartStride<D>;
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(rec + D));
      ms[b] = in ? ml.x : kNegBig;
      ls[b] = in ? ml.y : 0.f;
      lo[b] = __ldcg(reinterpret_cast<const float4*>(rec + d0));
      hi[b] = __ldcg(reinterpret_cast<const float4*>(rec + d0 + 4));
    }
    float Mn = M;
#pragma unroll
    for (int b = 0; b < B; ++b) Mn = fmaxf(Mn, ms[b]);
    const float keep = ex2_approx(M - Mn);
    L *= keep;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] *= keep;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float w = s0 + b * step < s_end ? ex2_approx(ms[b] - Mn) : 0.f;
      L += ls[b] * w;
      acc[0] += lo[b].x * w; acc[1] += lo[b].y * w; acc[2] += lo[b].z * w; acc[3] += lo[b].w * w;
      acc[4] += hi[b].x * w; acc[5] += hi[b].y * w; acc[6] += hi[b].z * w; acc[7] += hi[b].w * w;
    }
    M = Mn;
  }
}

// merge_split_records over LL64 records (the same arithmetic, so the result
// is the same bits): false if a poll gave up.
template <int D>
__device__ __forceinline__ bool merge_split_records_ll(const unsigned long long* rec0, int s_begin, int s_end,
                                                       int step, int d0, uint32_t tag, float& M, float& L,
                                                       float (&acc)[8], LLWait& w) {
  constexpr int B = 4;
  for (int s0 = s_begin; s0 < s_end; s0 += B * step) {
    float ms[B], ls[B];
    float4 lo[B], hi[B];
    // the B records' words in one poll (a missing record reads split s_begin's)
    uint4 g[5 * B];
    const bool polled = ll_poll_groups<5 * B, true>(
        [&](int i) -> const void* {
          const int s = s0 + (i / 5) * step;
          const unsigned long long* rec = rec0 + static_cast<size_t>(s < s_end ? s : s_begin) * kMegaPartStride<D>;
          return i % 5 == 4 ? rec + D : rec + d0 + 2 * (i % 5);
        },
        g, tag, w);
    if (!polled) return false;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const bool in = s0 + b * step < s_end;
      ms[b] = in ? __uint_as_float(g[5 * b + 4].y) : kNegBig;
      ls[b] = in ? __uint_as_float(g[5 * b + 4].w) : 0.f;
      lo[b] = in ? make_float4(__uint_as_float(g[5 * b].y), __uint_as_float(g[5 * b].w),
                               __uint_as_float(g[5 * b + 1].y), __uint_as_float(g[5 * b + 1].w))
                 : make_float4(0.f, 0.f, 0.f, 0.f);
      hi[b] = in ? make_float4(__uint_as_float(g[5 * b + 2].y), __uint_as_float(g[5 * b + 2].w),
                               __uint_as_float(g[5 * b + 3].y), __uint_as_float(g[5 * b + 3].w))
                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float Mn = M;
#pragma unroll
    for (int b = 0; b < B; ++b) Mn = fmaxf(Mn, ms[b]);
    const float keep = ex2_approx(M - Mn);
    L *= keep;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] *= keep;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float wgt = s0 + b * step < s_end ? ex2_approx(ms[b] - Mn) : 0.f;
      L += ls[b] * wgt;
      acc[0] += lo[b].x * wgt; acc[1] += lo[b].y * wgt; acc[2] += lo[b].z * wgt; acc[3] += lo[b].w * wgt;
      acc[4] += hi[b].x * wgt; acc[5] += hi[b].y * wgt; acc[6] += hi[b].z * wgt; acc[7] += hi[b].w * wgt;
    }
    M = Mn;
  }
  return true;
}

// 8 dims of the merged output, rounded to bf16 as the reference stores attn_out.
__device__ __forceinline__ uint4 merged_bf16x8(float L, const float (&acc)[8]) {
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint4 o;
  o.x = pack_bf2(acc[0] * inv, acc[1] * inv);
  o.y = pack_bf2(acc[2] * inv, acc[3] * inv);
  o.z = pack_bf2(acc[4] * inv, acc[5] * inv);
  o.w = pack_bf2(acc[6] * inv, acc[7] * inv);
  return o;
}

template <int D>
__device__ __forceinline__ AttnItem mega_attn_item(const MegaArgs& a, int pos) {
  using AG = MegaAttnGeom<D>;
  AttnItem it{};
  const int items = a.num_kv * a.splits;
  if (static_cast<int>(blockIdx.x) >= items || pos < 0 || pos >= a.max_seq) {
    it.nblocks = 0;
    it.kvh = -1;
    return it;
  }
  const int seq_len = pos + 1;
  // Splits this step: about split_positions cached positions each, at most
  // the configured count -- a short context is one split, and needs no merge.
  const int splits = mega_attn_splits(seq_len, a.splits, a.split_positions);
  if (static_cast<int>(blockIdx.x) >= a.num_kv * splits) {
    it.nblocks = 0;
    it.kvh = -1;
    return it;
  }
  it.splits = splits;
  it.kvh = blockIdx.x / splits;
  it.split = blockIdx.x % splits;
  const int chunk = mega_attn_chunk(seq_len, splits, AG::P);
  it.begin = it.split * chunk;
  it.end = min(seq_len, it.begin + chunk);
  it.cache_end = min(it.end, pos);
  it.nblocks = it.cache_end > it.begin ? (it.cache_end - it.begin + AG::STAGE_POS - 1) / AG::STAGE_POS : 0;
  return it;
}

template <int D, int STAGES, bool PAGED>
__device__ __forceinline__ bool mega_attn_produce(uint8_t* ring, uint64_t* full, uint64_t* empty,
                                                  int& it, const MegaArgs& a, int l, int pos) {
  using AG = MegaAttnGeom<D>;
  const AttnItem item = mega_attn_item<D>(a, pos);
  for (int blk = 0; blk < item.nblocks; ++blk, ++it) {
    const int slot = it % STAGES;
    if (it >= STAGES &&
        !mbar_wait(&empty[slot], ((it / STAGES) - 1) & 1, a.status, kStatusTimeoutEmpty)) {
      return false;
    }
    const int p0 = item.begin + blk * AG::STAGE_POS;
    // Only positions below cache_end are copied: one run for the contiguous
    // layout, one per page for the paged one.
    const int nvalid = min(AG::STAGE_POS, item.cache_end - p0);
    uint8_t* dst = ring + slot * kMegaStageBytes;
    mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nvalid) * 2 * AG::ROWB);
    for (int n = 0; n < nvalid;) {
      int run = nvalid - n;
      if constexpr (PAGED) run = min(run, a.page_size - (p0 + n) % a.page_size);
      const uint32_t bytes = static_cast<uint32_t>(run) * AG::ROWB;
      const long long off = kv_offset<PAGED>(a, l, item.kvh, p0 + n, D);
      bulk_g2s(dst + n * AG::ROWB, a.kpool + off, bytes, &full[slot]);
      bulk_g2s(dst + AG::STAGE_POS * AG::ROWB + n * AG::ROWB, a.vpool + off, bytes, &full[slot]);
      n += run;
    }
  }
  return true;
}

// Tensor-pipe attention: a stage's 128 positions as 8 units of 16, each one
// TMA tensor copy of K and one of V ([16 rows][128 bytes], 128-byte swizzle)
// out of the cache rows. Unit starts are 16-aligned (item starts are
// multiples of 32), so a unit never straddles a page of a multiple of 16
// positions; rows past cache_end that the last unit carries are masked by
// the consumers (contiguous cache: rows past a head's end belong to later
// positions of the next head, or lie past the tensor and read as zero).
constexpr int kMegaUnit = 16;

template <int D, int STAGES, bool PAGED>
__device__ __forceinline__ bool mega_attn_produce_tc(uint8_t* ring, uint64_t* full, uint64_t* empty, int& it,
                                                     const MegaArgs& a, int l, int pos, uint64_t policy) {
  using AG = MegaAttnGeom<D>;
  constexpr int UNITS = AG::STAGE_POS / kMegaUnit;
  constexpr uint32_t UNIT_BYTES = kMegaUnit * D * 2;
  const AttnItem item = mega_attn_item<D>(a, pos);
  const CUtensorMap* km = a.kvmaps + static_cast<size_t>(l) * a.kvmap_layer_stride;
  for (int blk = 0; blk < item.nblocks; ++blk, ++it) {
    const int slot = it % STAGES;
    if (it >= STAGES &&
        !mbar_wait(&empty[slot], ((it / STAGES) - 1) & 1, a.status, kStatusTimeoutEmpty)) {
      return false;
    }
    const int p0 = item.begin + blk * AG::STAGE_POS;
    const int units = min(UNITS, (item.cache_end - p0 + kMegaUnit - 1) / kMegaUnit);
    uint8_t* dst = ring + slot * kMegaStageBytes;
    mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(units) * 2 * UNIT_BYTES);
    for (int u = 0; u < units; ++u) {
      const int q0 = p0 + u * kMegaUnit;
      int row;
      if constexpr (PAGED) {
        int page = a.tables[static_cast<size_t>(l) * a.max_pages + q0 / a.page_size];
        if (page < 0 || page >= a.pool_pages) {
          atomicOr(a.status, kStatusBadPage);
          page = 0;
        }
        row = (page * a.num_kv + item.kvh) * a.page_size + q0 % a.page_size;
      } else {
        row = item.kvh * a.max_seq + q0;
      }
      tma_load_3d(dst + u * UNIT_BYTES, km, 0, row, 0, &full[slot], policy);
      tma_load_3d(dst + AG::STAGE_POS * AG::ROWB + u * UNIT_BYTES, km + 1, 0, row, 0, &full[slot], policy);
    }
  }
  return true;
}

// Publishes the item's per-warp records in `scratch` (per warp and head: m,
// l, acc[D]) as this split's (acc[D], m, l) record; the O phase merges the
// splits of every head in its prologue (mega_load_attention_merged), or, with
// many splits, the last split of the KV head to publish merges them here.
// With `ll_tag` (the low-latency exchange) the records go out as LL64 words,
// and with many splits the KV head's split 0 polls the others' records and
// merges them (no counter, no fence); false if a poll gave up.
template <int D, int G, bool F32>
__device__ __forceinline__ bool mega_attn_publish(const MegaArgs& a, int l, const AttnItem& item,
                                                  const float* scratch, int* s_last, uint32_t ll_tag = 0) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (ll_tag != 0) {
    unsigned long long* lbase = a.part_ll + static_cast<size_t>(item.kvh) * G * a.splits * kMegaPartStride<D>;
    for (int idx = tid; idx < G * D; idx += kGemvConsumers) {
      const int g = idx / D, d = idx % D;
      float M = kNegBig;
#pragma unroll
      for (int w = 0; w < kMegaWarps; ++w) M = fmaxf(M, scratch[(w * G + g) * (D + 2)]);
      float L = 0.f, A = 0.f;
#pragma unroll
      for (int w = 0; w < kMegaWarps; ++w) {
        const float* c = scratch + (w * G + g) * (D + 2);
        const float sc = ex2_approx(c[0] - M);
        L += c[1] * sc;
        A += c[2 + d] * sc;
      }
      if (item.splits == 1) {
        // One split: the record is the whole softmax, so the output is what
        // the merge of one record gives (bf16(A / L), merged_bf16x8).
        const float inv = L > 0.f ? 1.f / L : 0.f;
        ll_store_all(a.attn_ll + static_cast<size_t>(item.kvh * G + g) * D + d, ll32_word(A * inv, ll_tag),
                     a.ll_copy_bytes);
        continue;
      }
      unsigned long long* rec = lbase + (g * a.splits + item.split) * kMegaPartStride<D>;
      st_relaxed_u64(rec + d, ll64_word(A, ll_tag));
      if (d == 0) {
        st_relaxed_u64(rec + D, ll64_word(M, ll_tag));
        st_relaxed_u64(rec + D + 1, ll64_word(L, ll_tag));
      }
    }
    // Mergers: split 0 for a few splits; splits 0 .. kMegaMergers - 1 for
    // many, each merging a quarter of the head group's 8-dim chunks (a
    // quarter of the records' bytes polled per attempt).
    if (item.splits == 1 || item.split >= (item.splits <= kMegaPrologueMergeMax ? 1 : kMegaMergers)) return true;
    named_sync(1, kGemvConsumers);  // this CTA's own record is written
    LLWait wt{a.status, a.wait_ns};
    bool ok = true;
    if (item.splits <= kMegaPrologueMergeMax) {
      // Few splits: the merge the O prologue of the barrier form does
      // (merge_split_records from split 0, one thread per 8-dim chunk), so
      // both forms compute the same bits.
      for (int c = tid; c < G * D / 8; c += kGemvConsumers) {
        const int g = c * 8 / D, d0 = c * 8 % D;
        float M = kNegBig, L = 0.f;
        float acc8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (ok) {
          ok = merge_split_records_ll<D>(lbase + static_cast<size_t>(g) * a.splits * kMegaPartStride<D>, 0,
                                         item.splits, 1, d0, ll_tag, M, L, acc8, wt);
        }
        const uint4 o = merged_bf16x8(L, acc8);
        uint32_t* dst = a.attn_ll + static_cast<size_t>(item.kvh * G + g) * D + d0;
        const uint32_t t16 = ll_tag & 0xffffu;
        const uint32_t words[8] = {(o.x << 16) | t16, (o.x & 0xffff0000u) | t16, (o.y << 16) | t16,
                                   (o.y & 0xffff0000u) | t16, (o.z << 16) | t16, (o.z & 0xffff0000u) | t16,
                                   (o.w << 16) | t16, (o.w & 0xffff0000u) | t16};
#pragma unroll
        for (int e = 0; e < 8; ++e) ll_store_all(dst + e, words[e], a.ll_copy_bytes);
      }
      return ok;
    }
    const int sg = lane & 7;
    constexpr int kChunks = G * D / 8;
    const int c0 = item.split * ((kChunks + kMegaMergers - 1) / kMegaMergers);
    const int c1 = min(kChunks, c0 + (kChunks + kMegaMergers - 1) / kMegaMergers);
    for (int c = tid >> 3; c < kChunks; c += kGemvConsumers / 8) {
      const int g = c * 8 / D, d0 = c * 8 % D;
      const bool mine = c >= c0 && c < c1;  // the same for the 8 lanes of a chunk
      float M = kNegBig, L = 0.f;
      float acc8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (ok && mine) {
        ok = merge_split_records_ll<D>(lbase + static_cast<size_t>(g) * a.splits * kMegaPartStride<D>, sg,
                                       item.splits, 8, d0, ll_tag, M, L, acc8, wt);
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, M, off);
        const float ol = __shfl_xor_sync(0xffffffffu, L, off);
        const float Mn = fmaxf(M, om);
        const float ws = ex2_approx(M - Mn), wo = ex2_approx(om - Mn);
        L = L * ws + ol * wo;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float oa = __shfl_xor_sync(0xffffffffu, acc8[e], off);
          acc8[e] = acc8[e] * ws + oa * wo;
        }
        M = Mn;
      }
      if (sg == 0 && mine) {
        const float inv = L > 0.f ? 1.f / L : 0.f;
        uint32_t* dst = a.attn_ll + static_cast<size_t>(item.kvh * G + g) * D + d0;
#pragma unroll
        for (int e = 0; e < 8; ++e) ll_store_all(dst + e, ll32_word(acc8[e] * inv, ll_tag), a.ll_copy_bytes);
      }
    }
    return ok;
  }
  float* part_base = a.partials + static_cast<size_t>(item.kvh) * G * a.splits * kMegaPartStride<D>;
  for (int idx = tid; idx < G * D; idx += kGemvConsumers) {
    const int g = idx / D, d = idx % D;
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < kMegaWarps; ++w) M = fmaxf(M, scratch[(w * G + g) * (D + 2)]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kMegaWarps; ++w) {
      const float* c = scratch + (w * G + g) * (D + 2);
      const float s = ex2_approx(c[0] - M);
      L += c[1] * s;
      A += c[2 + d] * s;
    }
    float* rec = part_base + (g * a.splits + item.split) * kMegaPartStride<D>;
    rec[d] = A;
    if (d == 0) {
      rec[D] = M;
      rec[D + 1] = L;
    }
  }
  if (item.splits <= kMegaPrologueMergeMax) return true;
  // Many splits: the last split of this KV head to publish merges the head
  // group once (8 threads per 8-dim chunk, splits strided over them) and
  // writes the bf16 output; the counter resets for the next step.
  __threadfence();
  named_sync(1, kGemvConsumers);
  unsigned* ctr = a.attn_ctr + static_cast<size_t>(l) * a.num_kv + item.kvh;
  if (tid == 0) *s_last = atomicAdd(ctr, 1u) == static_cast<unsigned>(item.splits - 1);
  named_sync(1, kGemvConsumers);
  if (!*s_last) return true;
  __threadfence();
  const int sg = lane & 7;
  for (int c = tid >> 3; c < G * D / 8; c += kGemvConsumers / 8) {
    const int g = c * 8 / D, d0 = c * 8 % D;
    float M = kNegBig, L = 0.f;
    float acc8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    merge_split_records<D>(part_base + static_cast<size_t>(g) * a.splits * kMegaPartStride<D>, sg, item.splits, 8,
                           d0, M, L, acc8);
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, M, off);
      const float ol = __shfl_xor_sync(0xffffffffu, L, off);
      const float Mn = fmaxf(M, om);
      const float ws = ex2_approx(M - Mn), wo = ex2_approx(om - Mn);
      L = L * ws + ol * wo;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float oa = __shfl_xor_sync(0xffffffffu, acc8[e], off);
        acc8[e] = acc8[e] * ws + oa * wo;
      }
      M = Mn;
    }
    if (sg == 0) {
      if constexpr (F32) {
        const float inv = L > 0.f ? 1.f / L : 0.f;
        float* dst = a.attn_f + static_cast<size_t>(item.kvh * G + g) * D + d0;
        *reinterpret_cast<float4*>(dst) = make_float4(acc8[0] * inv, acc8[1] * inv, acc8[2] * inv, acc8[3] * inv);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(acc8[4] * inv, acc8[5] * inv, acc8[6] * inv, acc8[7] * inv);
      } else {
        *reinterpret_cast<uint4*>(a.attn + static_cast<size_t>(item.kvh * G + g) * D + d0) = merged_bf16x8(L, acc8);
      }
    }
  }
  if (tid == 0) *ctr = 0u;
  return true;
}

// Consumers: one (KV head, split) item -> partials (or the output when there
// is a single split); the last CTA of a KV head merges its splits.
// `cs` is the step's RoPE table, `scratch` >= kMegaWarps * G * (D + 2) floats.
template <int D, int G, int STAGES, bool PAGED, bool F32>
__device__ __forceinline__ void mega_attn_consume(const uint8_t* ring, uint64_t* full,
                                                  uint64_t* empty, int& it, const MegaArgs& a,
                                                  int l, int pos, const float* cs, float* scratch,
                                                  int* s_last, bool& failed,
                                                  unsigned long long* wait_cycles = nullptr) {
  using AG = MegaAttnGeom<D>;
  constexpr int LPP = AG::LPP, GPW = AG::GPW, P = AG::P;
  const AttnItem item = mega_attn_item<D>(a, pos);
  if (item.kvh < 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lig = lane % LPP, grp = warp * GPW + lane / LPP;
  const int heads = a.num_kv * G;
  const int qd = heads * D, kvd = a.num_kv * D;

  // The new position's K and V (this step's projection) are loaded with the
  // query, so one L2 round trip covers both.
  const bool has_new = pos >= item.begin && pos < item.end && grp == 0;
  uint4 k_self = make_uint4(0, 0, 0, 0), k_other = k_self, v_raw = k_self;
  float k_newf[8], v_newf[8];
  if (has_new) {
    if constexpr (F32) {
      rope8f<D>(a.qkv_f + qd + item.kvh * D, lig, cs, k_newf);
      const float* vh = a.qkv_f + qd + kvd + item.kvh * D + lig * 8;
      const float4 v0 = __ldcg(reinterpret_cast<const float4*>(vh));
      const float4 v1 = __ldcg(reinterpret_cast<const float4*>(vh + 4));
      v_newf[0] = v0.x; v_newf[1] = v0.y; v_newf[2] = v0.z; v_newf[3] = v0.w;
      v_newf[4] = v1.x; v_newf[5] = v1.y; v_newf[6] = v1.z; v_newf[7] = v1.w;
    } else {
      const bf16* kh = a.qkv + qd + item.kvh * D;
      k_self = ldg_cg16(kh + lig * 8);
      k_other = ldg_cg16(kh + (lig * 8 < D / 2 ? lig * 8 + D / 2 : lig * 8 - D / 2));
      v_raw = ldg_cg16(a.qkv + qd + kvd + item.kvh * D + lig * 8);
    }
  }
  float q[G][8], acc[G][8], m[G], l_[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if constexpr (F32) {
      rope8f<D>(a.qkv_f + (item.kvh * G + g) * D, lig, cs, q[g]);
    } else {
      // rotated q rounded to bf16, as the reference stores it (rope_q)
      rope8<D>(a.qkv + (item.kvh * G + g) * D, lig, cs, q[g]);
#pragma unroll
      for (int e = 0; e < 8; ++e) q[g][e] = rbf(q[g][e]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      q[g][e] *= a.scale_log2;
      acc[g][e] = 0.f;
    }
    m[g] = kNegBig;
    l_[g] = 0.f;
  }

  const bool timed = wait_cycles != nullptr && tid == 0;
  unsigned long long waited = 0;
  for (int blk = 0; blk < item.nblocks; ++blk, ++it) {
    const int slot = it % STAGES;
    const long long w0 = timed ? clock64() : 0;
    if (!failed) failed = !mbar_wait(&full[slot], (it / STAGES) & 1, a.status, kStatusTimeoutFull);
    if (timed) waited += static_cast<unsigned long long>(clock64() - w0);
    const uint8_t* kst = ring + slot * kMegaStageBytes;
    const uint8_t* vst = kst + AG::STAGE_POS * AG::ROWB;
#pragma unroll 1
    for (int pass = 0; pass < AG::PASSES; ++pass) {
      const int row = pass * P + grp;
      const int first = item.begin + blk * AG::STAGE_POS + pass * P;
      if (first >= item.cache_end) break;  // uniform across the CTA
      const bool live = !failed && first + grp < item.cache_end;
      float kf[8], vf[8];
      unpack8(*reinterpret_cast<const uint4*>(kst + row * AG::ROWB + lig * 16), kf);
      unpack8(*reinterpret_cast<const uint4*>(vst + row * AG::ROWB + lig * 16), vf);
      float sc[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(q[g][e], kf[e], s);
        sc[g] = s;
      }
#pragma unroll
      for (int off = LPP / 2; off >= 1; off >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], off, LPP);
      }
      if (live) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float mn = fmaxf(m[g], sc[g]);
          const float alpha = ex2_approx(m[g] - mn);
          const float p = ex2_approx(sc[g] - mn);
          l_[g] = l_[g] * alpha + p;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p, vf[e], acc[g][e] * alpha);
          m[g] = mn;
        }
      }
    }
    __syncwarp();
    if (lane == 0 && !failed) mbar_arrive(&empty[slot]);
  }
  if (timed) *wait_cycles = waited;

  // The new position (this step's token): rotate K, store K and V, attend.
  if (has_new) {
    // The cache holds bf16; with fp32 activations this step attends to the
    // unrounded K and V.
    float kf[8], vf[8];
    uint4 vraw;
    if constexpr (F32) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        kf[e] = k_newf[e];
        vf[e] = v_newf[e];
      }
      vraw.x = pack_bf2(vf[0], vf[1]); vraw.y = pack_bf2(vf[2], vf[3]);
      vraw.z = pack_bf2(vf[4], vf[5]); vraw.w = pack_bf2(vf[6], vf[7]);
    } else {
      rope8_from<D>(k_self, k_other, lig, cs, kf);
#pragma unroll
      for (int e = 0; e < 8; ++e) kf[e] = rbf(kf[e]);  // attends to the cache's bf16 key
      vraw = v_raw;
      unpack8(vraw, vf);
    }
    const long long off = kv_offset<PAGED>(a, l, item.kvh, pos, D);
    uint4 kw;
    kw.x = pack_bf2(kf[0], kf[1]); kw.y = pack_bf2(kf[2], kf[3]);
    kw.z = pack_bf2(kf[4], kf[5]); kw.w = pack_bf2(kf[6], kf[7]);
    *reinterpret_cast<uint4*>(a.kpool + off + lig * 8) = kw;
    *reinterpret_cast<uint4*>(a.vpool + off + lig * 8) = vraw;
    float sc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(q[g][e], kf[e], s);
      sc[g] = s;
    }
#pragma unroll
    for (int off2 = LPP / 2; off2 >= 1; off2 >>= 1) {
#pragma unroll
      for (int g = 0; g < G; ++g) sc[g] += __shfl_xor_sync(0xffffffffu >> (32 - LPP), sc[g], off2, LPP);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mn = fmaxf(m[g], sc[g]);
      const float alpha = ex2_approx(m[g] - mn);
      const float p = ex2_approx(sc[g] - mn);
      l_[g] = l_[g] * alpha + p;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p, vf[e], acc[g][e] * alpha);
      m[g] = mn;
    }
  }

  // Groups of a warp hold the same dims for other positions: combine them.
#pragma unroll
  for (int off = LPP; off < 32; off <<= 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float om = __shfl_xor_sync(0xffffffffu, m[g], off);
      const float ol = __shfl_xor_sync(0xffffffffu, l_[g], off);
      float oacc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) oacc[e] = __shfl_xor_sync(0xffffffffu, acc[g][e], off);
      softmax_merge<G>(m[g], l_[g], acc, g, om, ol, oacc);
    }
  }
  if (lane < LPP) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float* c = scratch + (warp * G + g) * (D + 2);
      if (lane == 0) {
        c[0] = m[g];
        c[1] = l_[g];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) c[2 + lane * 8 + e] = acc[g][e];
    }
  }
  named_sync(1, kGemvConsumers);
  mega_attn_publish<D, G, F32>(a, l, item, scratch, s_last);
}

// 8 fp32 values as bf16 (hi) and the bf16 of their remainders (lo).
__device__ __forceinline__ void split_hilo8(const float (&v)[8], uint4& hi, uint4& lo) {
  hi.x = pack_bf2(v[0], v[1]);
  hi.y = pack_bf2(v[2], v[3]);
  hi.z = pack_bf2(v[4], v[5]);
  hi.w = pack_bf2(v[6], v[7]);
  lo.x = pack_bf2(v[0] - bf_lo(hi.x), v[1] - bf_hi(hi.x));
  lo.y = pack_bf2(v[2] - bf_lo(hi.y), v[3] - bf_hi(hi.y));
  lo.z = pack_bf2(v[4] - bf_lo(hi.z), v[5] - bf_hi(hi.z));
  lo.w = pack_bf2(v[6] - bf_lo(hi.w), v[7] - bf_hi(hi.w));
}

// The attention phase on the tensor pipe (head_dim 64, G <= 8 query heads
// per KV head). Warp w takes unit w (16 positions) of every stage:
//   S = Q K^T   m16n8k16, the G query heads as MMA rows 0..G-1 (the rest
//               zero), bf16 q as the reference stores it after RoPE (with
//               fp32 activations: q as a bf16 pair hi + lo, two MMAs), bf16
//               K from ldmatrix of the swizzled unit, fp32 sums;
//   online softmax per head in the log2 domain, fp32, over the quad of lanes
//               holding a head's 16 scores;
//   O += P V    P as a bf16 pair hi + lo (two MMAs: the weights keep about
//               16 significant bits, as the fp32 weights of the reference's
//               decode attention), V fragments from ldmatrix.trans.
// The denominator sums the fp32 weights. The new position is folded into
// warp 0's record by lanes 0-7 after the stages (its K and V go to the
// cache), then the records are published as in mega_attn_consume. `qs` is
// shared memory for the rotated q (2 G D bf16).
template <int D, int G, int STAGES, bool PAGED, bool F32>
__device__ __forceinline__ void mega_attn_consume_tc(const uint8_t* ring, uint64_t* full, uint64_t* empty, int& it,
                                                     const MegaArgs& a, int l, int pos, const float* cs,
                                                     float* scratch, bf16* qs, int* s_last, bool& failed,
                                                     unsigned long long* wait_cycles = nullptr,
                                                     uint32_t ll_in_tag = 0, uint32_t ll_out_tag = 0) {
  using AG = MegaAttnGeom<D>;
  static_assert(D == 64 && G >= 1 && G <= 8, "tensor-pipe attention: head_dim 64, at most 8 heads per KV head");
  constexpr int UNIT_BYTES = kMegaUnit * D * 2;
  constexpr int KS = D / 16;  // k-steps of Q K^T, and pairs of P V column tiles
  constexpr int LPP = D / 8;  // lanes per position on the new position
  const AttnItem item = mega_attn_item<D>(a, pos);
  if (item.kvh < 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int heads = a.num_kv * G;
  const int qd = heads * D, kvd = a.num_kv * D;
  bf16* qlo = qs + G * D;

  // The new position's K and V (this step's projection), loaded early.
  const bool has_new = pos >= item.begin && pos < item.end;
  const bool new_lane = has_new && warp == 0 && lane < LPP;
  uint4 k_self = make_uint4(0, 0, 0, 0), k_other = k_self, v_raw = k_self;
  float k_newf[8], v_newf[8];
  LLWait wt{a.status, a.wait_ns};
  bool ll_ok = true;
  const uint32_t* qkvll = a.qkv_ll != nullptr ? mega_ll_mine(a, a.qkv_ll) : nullptr;
  if (new_lane && ll_in_tag != 0) {
    const uint32_t* kh = qkvll + qd + item.kvh * D;
    const uint32_t* ko = kh + (lane * 8 < D / 2 ? lane * 8 + D / 2 : lane * 8 - D / 2);
    const uint32_t* vh = qkvll + qd + kvd + item.kvh * D + lane * 8;
    const uint32_t* const grp[3] = {kh + lane * 8, ko, vh};
    uint4 g6[6];
    ll_ok = ll_poll_groups<6, false>([&](int i) -> const void* { return grp[i >> 1] + (i & 1) * 4; }, g6,
                                     ll_in_tag, wt);
    k_self = ll32_values8(g6[0], g6[1]);
    k_other = ll32_values8(g6[2], g6[3]);
    v_raw = ll32_values8(g6[4], g6[5]);
  } else if (new_lane) {
    if constexpr (F32) {
      rope8f<D>(a.qkv_f + qd + item.kvh * D, lane, cs, k_newf);
      const float* vh = a.qkv_f + qd + kvd + item.kvh * D + lane * 8;
      const float4 v0 = __ldcg(reinterpret_cast<const float4*>(vh));
      const float4 v1 = __ldcg(reinterpret_cast<const float4*>(vh + 4));
      v_newf[0] = v0.x; v_newf[1] = v0.y; v_newf[2] = v0.z; v_newf[3] = v0.w;
      v_newf[4] = v1.x; v_newf[5] = v1.y; v_newf[6] = v1.z; v_newf[7] = v1.w;
    } else {
      const bf16* kh = a.qkv + qd + item.kvh * D;
      k_self = ldg_cg16(kh + lane * 8);
      k_other = ldg_cg16(kh + (lane * 8 < D / 2 ? lane * 8 + D / 2 : lane * 8 - D / 2));
      v_raw = ldg_cg16(a.qkv + qd + kvd + item.kvh * D + lane * 8);
    }
  }
  // Rotated q of the group into shared memory: bf16 (and its remainder).
  if (tid < G * LPP) {
    const int g = tid / LPP, lig = tid % LPP;
    float qf[8];
    if constexpr (F32) {
      rope8f<D>(a.qkv_f + (item.kvh * G + g) * D, lig, cs, qf);
    } else {
      if (ll_in_tag != 0) {
        const uint32_t* qh = qkvll + (item.kvh * G + g) * D;
        const uint32_t* qo = qh + (lig * 8 < D / 2 ? lig * 8 + D / 2 : lig * 8 - D / 2);
        const uint32_t* const grp[2] = {qh + lig * 8, qo};
        uint4 g4[4];
        ll_ok = ll_ok && ll_poll_groups<4, false>([&](int i) -> const void* { return grp[i >> 1] + (i & 1) * 4; },
                                                  g4, ll_in_tag, wt);
        rope8_from<D>(ll32_values8(g4[0], g4[1]), ll32_values8(g4[2], g4[3]), lig, cs, qf);
      } else {
        rope8<D>(a.qkv + (item.kvh * G + g) * D, lig, cs, qf);
      }
    }
    uint4 hi, lo;
    split_hilo8(qf, hi, lo);
    *reinterpret_cast<uint4*>(qs + g * D + lig * 8) = hi;
    if constexpr (F32) *reinterpret_cast<uint4*>(qlo + g * D + lig * 8) = lo;
  }
  if (!ll_ok) failed = true;
  named_sync(1, kGemvConsumers);

  const int g = lane >> 2, qq = lane & 3;
  const bool hrow = g < G;
  uint32_t qa0[KS], qa2[KS], ql0[KS], ql2[KS];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    const bf16* qrow = qs + g * D + 16 * ks + 2 * qq;
    qa0[ks] = hrow ? *reinterpret_cast<const uint32_t*>(qrow) : 0u;
    qa2[ks] = hrow ? *reinterpret_cast<const uint32_t*>(qrow + 8) : 0u;
    if constexpr (F32) {
      ql0[ks] = hrow ? *reinterpret_cast<const uint32_t*>(qrow + G * D) : 0u;
      ql2[ks] = hrow ? *reinterpret_cast<const uint32_t*>(qrow + G * D + 8) : 0u;
    } else {
      ql0[ks] = ql2[ks] = 0u;
    }
  }
  const float sl2 = a.scale_log2;
  float m = kNegBig, lsum = 0.f;
  float o[2 * KS][4];
#pragma unroll
  for (int t = 0; t < 2 * KS; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  const int mi = lane >> 3, r8 = lane & 7;

  const bool timed = wait_cycles != nullptr && tid == 0;
  unsigned long long waited = 0;
  for (int blk = 0; blk < item.nblocks; ++blk, ++it) {
    const int slot = it % STAGES;
    const long long w0 = timed ? clock64() : 0;
    if (!failed) failed = !mbar_wait(&full[slot], (it / STAGES) & 1, a.status, kStatusTimeoutFull);
    failed = __any_sync(0xffffffffu, failed);  // the MMAs below are warp-wide
    if (timed) waited += static_cast<unsigned long long>(clock64() - w0);
    const int q0 = item.begin + blk * AG::STAGE_POS + warp * kMegaUnit;
    if (!failed && q0 < item.cache_end) {  // uniform across the warp
      const uint32_t kbase = smem_addr(ring + slot * kMegaStageBytes) + warp * UNIT_BYTES;
      const uint32_t vbase = kbase + AG::STAGE_POS * AG::ROWB;
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t kb[4];
        ldmatrix_x4(kb, kbase + ab_offset(((mi >> 1) << 3) + r8, 2 * ks + (mi & 1)));
        mma_x_rows(s0, qa0[ks], qa2[ks], kb[0], kb[1]);
        mma_x_rows(s1, qa0[ks], qa2[ks], kb[2], kb[3]);
        if constexpr (F32) {
          mma_x_rows(s0, ql0[ks], ql2[ks], kb[0], kb[1]);
          mma_x_rows(s1, ql0[ks], ql2[ks], kb[2], kb[3]);
        }
      }
      // This lane's keys: q0 + 2 qq + {0, 1} (tile 0) and + 8 (tile 1).
      const int k0 = q0 + 2 * qq;
      const float v[4] = {s0[0] * sl2, s0[1] * sl2, s1[0] * sl2, s1[1] * sl2};
      const bool in[4] = {k0 < item.cache_end, k0 + 1 < item.cache_end, k0 + 8 < item.cache_end,
                          k0 + 9 < item.cache_end};
      float mx = kNegBig;
#pragma unroll
      for (int j = 0; j < 4; ++j) mx = in[j] ? fmaxf(mx, v[j]) : mx;
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m, mx);
      const float alpha = ex2_approx(m - mn);
      float p[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) p[j] = in[j] ? ex2_approx(v[j] - mn) : 0.f;
      lsum = lsum * alpha + ((p[0] + p[1]) + (p[2] + p[3]));
      m = mn;
#pragma unroll
      for (int t = 0; t < 2 * KS; ++t) {
        o[t][0] *= alpha;
        o[t][1] *= alpha;
      }
      const uint32_t ph0 = pack_bf2(p[0], p[1]), ph2 = pack_bf2(p[2], p[3]);
      const uint32_t pl0 = pack_bf2(p[0] - bf_lo(ph0), p[1] - bf_hi(ph0));
      const uint32_t pl2 = pack_bf2(p[2] - bf_lo(ph2), p[3] - bf_hi(ph2));
#pragma unroll
      for (int c = 0; c < KS; ++c) {
        uint32_t vb[4];
        ldmatrix_x4_trans(vb, vbase + ab_offset(((mi & 1) << 3) + r8, 2 * c + (mi >> 1)));
        mma_x_rows(o[2 * c], ph0, ph2, vb[0], vb[1]);
        mma_x_rows(o[2 * c], pl0, pl2, vb[0], vb[1]);
        mma_x_rows(o[2 * c + 1], ph0, ph2, vb[2], vb[3]);
        mma_x_rows(o[2 * c + 1], pl0, pl2, vb[2], vb[3]);
      }
    }
    __syncwarp();
    if (lane == 0 && !failed) mbar_arrive(&empty[slot]);
  }
  if (timed) *wait_cycles = waited;

  // This warp's record per head: m, the quad's l, O (dims 8 t + 2 qq + {0, 1}).
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
  if (hrow) {
    float* c = scratch + (warp * G + g) * (D + 2);
    if (qq == 0) {
      c[0] = m;
      c[1] = lsum;
    }
#pragma unroll
    for (int t = 0; t < 2 * KS; ++t) {
      c[2 + 8 * t + 2 * qq] = o[t][0];
      c[3 + 8 * t + 2 * qq] = o[t][1];
    }
  }
  __syncwarp();

  // The new position (this step's token) on warp 0, lanes 0-7: rotate K,
  // store K and V, fold them into warp 0's records. Attention reads the
  // cache's bf16 K and V (with fp32 activations: the unrounded ones).
  if (new_lane) {
    float kf[8], vf[8];
    uint4 kw, vw;
    if constexpr (F32) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        kf[e] = k_newf[e];
        vf[e] = v_newf[e];
      }
      kw.x = pack_bf2(kf[0], kf[1]); kw.y = pack_bf2(kf[2], kf[3]);
      kw.z = pack_bf2(kf[4], kf[5]); kw.w = pack_bf2(kf[6], kf[7]);
      vw.x = pack_bf2(vf[0], vf[1]); vw.y = pack_bf2(vf[2], vf[3]);
      vw.z = pack_bf2(vf[4], vf[5]); vw.w = pack_bf2(vf[6], vf[7]);
    } else {
      float kr[8];
      rope8_from<D>(k_self, k_other, lane, cs, kr);
      kw.x = pack_bf2(kr[0], kr[1]); kw.y = pack_bf2(kr[2], kr[3]);
      kw.z = pack_bf2(kr[4], kr[5]); kw.w = pack_bf2(kr[6], kr[7]);
      unpack8(kw, kf);
      vw = v_raw;
      unpack8(vw, vf);
    }
    const long long off = kv_offset<PAGED>(a, l, item.kvh, pos, D);
    *reinterpret_cast<uint4*>(a.kpool + off + lane * 8) = kw;
    *reinterpret_cast<uint4*>(a.vpool + off + lane * 8) = vw;
    constexpr unsigned kLanes = 0xffffffffu >> (32 - LPP);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float qf[8];
      unpack8(*reinterpret_cast<const uint4*>(qs + h * D + lane * 8), qf);
      if constexpr (F32) {
        float ql[8];
        unpack8(*reinterpret_cast<const uint4*>(qlo + h * D + lane * 8), ql);
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[e] += ql[e];
      }
      float sc = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) sc = fmaf(qf[e], kf[e], sc);
#pragma unroll
      for (int off2 = LPP / 2; off2 >= 1; off2 >>= 1) sc += __shfl_xor_sync(kLanes, sc, off2, LPP);
      sc *= sl2;
      float* c = scratch + h * (D + 2);  // warp 0's record of head h
      const float c0 = c[0], c1 = c[1];
      const float mn = fmaxf(c0, sc);
      const float al = ex2_approx(c0 - mn), pw = ex2_approx(sc - mn);
#pragma unroll
      for (int e = 0; e < 8; ++e) c[2 + lane * 8 + e] = c[2 + lane * 8 + e] * al + pw * vf[e];
      __syncwarp(kLanes);
      if (lane == 0) {
        c[0] = mn;
        c[1] = c1 * al + pw;
      }
      __syncwarp(kLanes);
    }
  }
  named_sync(1, kGemvConsumers);
  if (!mega_attn_publish<D, G, F32>(a, l, item, scratch, s_last, ll_out_tag)) failed = true;
}

// O-phase prologue: the attention output staged in shared memory, each thread
// one 8-element chunk. With the exchange it is polled as the attention
// phase's merged LL32 words. Otherwise, up to kMegaPrologueMergeMax splits it
// is merged here
// from the split partials with the logsumexp rule (merge_split_records) and
// rounded to bf16 as the reference stores attn_out; beyond that the attention
// phase has already merged it into `attn`. Uses named barrier 1; `xs` is
// complete on return.
// With fp32 activations the output is staged unrounded, as the bf16 pair
// xs + xs_lo.
template <int QD, int D, bool F32>
__device__ __forceinline__ bool mega_stage_attention(const MegaArgs& a, int pos, bf16* xs, bf16* xs_lo,
                                                     uint32_t ll_tag = 0) {
  const int splits = mega_attn_splits(pos + 1, a.splits, a.split_positions);
  if (ll_tag != 0) {
    // The same values, merged by the attention phase (every split count)
    // and exchanged as LL32 words: 2 KB of polls per 512 outputs instead of
    // every split record.
    LLWait wt{a.status, a.wait_ns};
    bool ok = true;
    const uint32_t* attn_in = mega_ll_mine(a, a.attn_ll);
    for (int c = threadIdx.x; c < QD / 8 && ok; c += kGemvConsumers) {
      uint4 g2[2];
      ok = ll_poll_groups<2, false>([&](int i) -> const void* { return attn_in + c * 8 + 4 * i; }, g2, ll_tag, wt);
      reinterpret_cast<uint4*>(xs)[c] = ll32_values8(g2[0], g2[1]);
    }
    return !named_sync_or(1, kGemvConsumers, !ok);
  }
  for (int c = threadIdx.x; c < QD / 8; c += kGemvConsumers) {
    const int col = c * 8;
    if (splits > kMegaPrologueMergeMax) {  // merged by the attention phase
      if constexpr (F32) {
        const float4 a0 = __ldcg(reinterpret_cast<const float4*>(a.attn_f + col));
        const float4 a1 = __ldcg(reinterpret_cast<const float4*>(a.attn_f + col + 4));
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        store_hilo8(v, xs, xs_lo, c);
      } else {
        reinterpret_cast<uint4*>(xs)[c] = ldg_cg16(a.attn + col);
      }
      continue;
    }
    const int h = col / D, d0 = col % D;
    float M = kNegBig, L = 0.f;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    merge_split_records<D>(a.partials + static_cast<size_t>(h) * a.splits * kMegaPartStride<D>, 0, splits, 1, d0, M, L,
                           acc);
    if constexpr (F32) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = acc[e] * inv;
      store_hilo8(v, xs, xs_lo, c);
    } else {
      reinterpret_cast<uint4*>(xs)[c] = merged_bf16x8(L, acc);
    }
  }
  named_sync(1, kGemvConsumers);
  return true;
}

// ---------------------------------------------------------------------------
// L2 prefetch window
// ---------------------------------------------------------------------------

// Walks this CTA's weight slices in the producer's order -- per layer qkv, o,
// gate/up (gate and up rows alternating in 16 KB pieces, as the ring takes
// them), down, then the lm_head -- prefetching them into L2 with the 32 lanes
// of its own warp (warp 9), one 128-byte line per lane and instruction, on the
// load/store path: a bulk prefetch would queue in the same TMA unit as the
// ring's copies and delay them. It stays at most MegaArgs::prefetch_bytes
// ahead of the bytes the producer has issued into the ring: while the
// consumers sit in barriers, attention and the small projections and the ring
// is full, HBM keeps streaming the next matrices into L2, and the ring
// refills from there.
constexpr unsigned kMegaPrefetchChunk = 16u << 10;
// Value of the producer's progress word once it has issued everything (or
// stopped on a failed wait): the prefetcher then stops.
constexpr unsigned long long kMegaIssuedDone = ~0ull;

template <int H, int QD, int F, int D>
struct MegaPrefetch {
  const MegaArgs* a;
  int slice;                  // index into the schedule: 4 per layer, then lm_head
  const char* ptr[2];         // next byte of each range of the slice
  unsigned long long left[2]; // bytes left in each range
  int turn;                   // range the next piece comes from
  unsigned long long done;    // bytes prefetched so far

  __device__ __forceinline__ void open(int s) {
    slice = s;
    left[0] = left[1] = 0;
    turn = 0;
    const int c = blockIdx.x, n = gridDim.x;
    if (s < 4 * a->layers) {
      const MegaLayer& w = a->L[s / 4];
      const int nqkv = QD + 2 * D * a->num_kv;
      int o0, o1, K;
      const bf16* base;
      switch (s % 4) {
        case 0: o0 = gemv_share(nqkv, c, n); o1 = gemv_share(nqkv, c + 1, n); K = H; base = w.qkv; break;
        case 1: o0 = gemv_share(H, c, n); o1 = gemv_share(H, c + 1, n); K = QD; base = w.o; break;
        case 2: o0 = gemv_share(F, c, n); o1 = gemv_share(F, c + 1, n); K = H; base = w.gate_up; break;
        default: o0 = gemv_share(H, c, n); o1 = gemv_share(H, c + 1, n); K = F; base = w.down; break;
      }
      ptr[0] = reinterpret_cast<const char*>(base + static_cast<size_t>(o0) * K);
      left[0] = static_cast<unsigned long long>(o1 - o0) * K * 2;
      if (s % 4 == 2) {  // the up rows of the same outputs
        ptr[1] = reinterpret_cast<const char*>(base + (static_cast<size_t>(F) + o0) * K);
        left[1] = left[0];
      }
    } else if (s == 4 * a->layers) {
      const int o0 = gemv_share(a->vocab, c, n), o1 = gemv_share(a->vocab, c + 1, n);
      ptr[0] = reinterpret_cast<const char*>(a->lm_head + static_cast<size_t>(o0) * H);
      left[0] = static_cast<unsigned long long>(o1 - o0) * H * 2;
    }
  }

  __device__ __forceinline__ void init(const MegaArgs* args) {
    a = args;
    done = 0;
    open(0);
  }

  // Issues one piece (every lane of the warp, with identical state); false
  // once the schedule is exhausted.
  __device__ __forceinline__ bool step(int lane) {
    while (left[0] == 0 && left[1] == 0) {
      if (slice >= 4 * a->layers) return false;
      open(slice + 1);
    }
    const bool second = left[0] == 0 || (turn == 1 && left[1] != 0);
    const unsigned long long avail = second ? left[1] : left[0];
    const unsigned bytes = static_cast<unsigned>(avail < kMegaPrefetchChunk ? avail : kMegaPrefetchChunk);
    const char* p = second ? ptr[1] : ptr[0];
    for (unsigned off = static_cast<unsigned>(lane) * 128u; off < bytes; off += 32u * 128u) prefetch_line_l2(p + off);
    if (second) {
      ptr[1] += bytes;
      left[1] -= bytes;
    } else {
      ptr[0] += bytes;
      left[0] -= bytes;
    }
    done += bytes;
    turn = second ? 0 : 1;
    return true;
  }
};

// The producer's side: publishes the weight bytes issued into the ring.
struct MegaProgress {
  volatile unsigned long long* word;
  __device__ __forceinline__ void top_up(unsigned long long issued) { *word = issued; }
};

// Prefetcher loop (one whole warp, kept converged: lane 0 reads the
// producer's progress and decides, the lanes follow). Every wait is bounded:
// it gives up when the producer's progress has not moved for kWaitLimitNs.
template <int H, int QD, int F, int D>
__device__ __forceinline__ void mega_prefetch_loop(const MegaArgs& a, volatile unsigned long long* issued_word,
                                                   int lane) {
  MegaPrefetch<H, QD, F, D> pf;
  pf.init(&a);
  unsigned long long last = 0;
  uint64_t since = globaltimer_ns();
  for (;;) {
    unsigned long long issued = lane == 0 ? *issued_word : 0ull;
    issued = __shfl_sync(0xffffffffu, issued, 0);
    if (issued == kMegaIssuedDone) return;
    if (pf.done < issued + a.prefetch_bytes) {
      if (!pf.step(lane)) return;
      continue;
    }
    int give_up = 0;
    if (lane == 0) {
      if (issued != last) {
        last = issued;
        since = globaltimer_ns();
      } else if (globaltimer_ns() - since > kWaitLimitNs) {
        give_up = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, give_up, 0)) return;
    __nanosleep(256);
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------

template <int H, int QD, int F, int D, int G, bool PAGED, bool F32>
struct MegaShape {
  static constexpr int STAGES = kMegaStages<F32>;
  static constexpr int RED_FLOATS = kGemvRedFloats + 512;  // GEMV segments, attention scratch
  static_assert(kMegaWarps * G * (D + 2) <= RED_FLOATS, "attention scratch");
  static constexpr int XS = (H > F ? H : F) > QD ? (H > F ? H : F) : QD;
  static constexpr size_t SMEM = static_cast<size_t>(STAGES) * kMegaStageBytes +
                                 2 * STAGES * 8 + 64 + (RED_FLOATS + 8 + D) * 4 + 128 +
                                 static_cast<size_t>(XS) * 2 * (F32 ? 2 : 1) + 64;
};

template <int H, int QD, int F, int D, int G, bool PAGED, bool F32, bool LL = false>
__global__ void __launch_bounds__(kMegaThreads, 1) decode_step_kernel(const MegaArgs a) {
  using Shape = MegaShape<H, QD, F, D, G, PAGED, F32>;
  constexpr int STAGES = Shape::STAGES;
  constexpr int SB = kMegaStageBytes;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * SB);
  uint64_t* empty = full + STAGES;
  unsigned long long* cta_best = reinterpret_cast<unsigned long long*>(empty + STAGES);
  int* s_flags = reinterpret_cast<int*>(cta_best + 1);  // [0] abort, [1] last-CTA
  // s_flags[2..3]: the producer's issued-bytes word read by the prefetcher;
  // [4]: the exchange's epoch base, [5]: the step's token (clamped) -- kept
  // in shared memory, not in registers across the step
  volatile unsigned long long* s_issued = reinterpret_cast<volatile unsigned long long*>(s_flags + 2);
  float* red8 = reinterpret_cast<float*>(s_flags + 8);
  float* red = red8 + 8;
  float* cs = red + Shape::RED_FLOATS;  // RoPE cos/sin [D]
  bf16* xs = align_smem<bf16>(cs + D, 128);  // staged input vector [max(H, QD, F)], 16-byte access
  bf16* xs_lo = F32 ? xs + Shape::XS : nullptr;  // its low bf16 half (fp32 activations)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos = __ldcg(a.state + 1);
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMegaWarps);
    }
    *cta_best = 0ull;
    s_flags[0] = 0;
    s_flags[1] = 0;
    if constexpr (LL) {
      s_flags[4] = static_cast<int>(__ldcg(a.epoch));
      int tok = __ldcg(a.state);
      s_flags[5] = (tok < 0 || tok >= a.vocab) ? 0 : tok;
    }
    *s_issued = 0;
    mbar_fence_init();
    if (blockIdx.x == 0 && (pos < 0 || pos >= a.max_seq)) atomicOr(a.status, kStatusBadPosition);
  }
  rope_table<D>(cs, (pos >= 0 && pos < a.max_seq) ? pos : 0, a.inv_freq);
  __syncthreads();

  const int ctas = gridDim.x;
  if (warp == kMegaWarps) {
    // ---------------- producer: this CTA's share of every matrix, in order.
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      int it = 0;
      bool ok = true;
      unsigned long long* ptrace = a.trace ? a.trace + blockIdx.x * kMegaTraceEvents + kMegaTraceProducer : nullptr;
      int phase = 0;
      auto mark = [&]() {
        if (ptrace && phase < kMegaTraceEvents - kMegaTraceProducer) ptrace[phase] = globaltimer_ns();
        ++phase;
        return true;
      };
      // Per-phase producer wait (written as the phase's slot; `phase` was
      // advanced by mark(), so the current phase is phase - 1).
      auto pwait = [&]() -> unsigned long long* {
        if (!ptrace) return nullptr;
        unsigned long long* w = ptrace + (kMegaTraceProducerWait - kMegaTraceProducer) + (phase - 1);
        *w = 0;
        return w;
      };
      MegaProgress progress{s_issued};
      MegaProgress* pf = a.prefetch_bytes ? &progress : nullptr;
      unsigned long long issued = 0;
      for (int l = 0; l < a.layers && ok; ++l) {
        const MegaLayer& w = a.L[l];
        const int nqkv = QD + 2 * (D * a.num_kv);
        ok = ok && mark() && gemv_produce<H, STAGES, false>(ring, full, empty, it, a.wmaps + 4 * l, w.qkv, nqkv,
                                                     gemv_share(nqkv, blockIdx.x, ctas),
                                                     gemv_share(nqkv, blockIdx.x + 1, ctas), policy, a.status,
                                                     pf, &issued, pwait());
        if constexpr (D == 64 && G <= 8) {
          ok = ok && mark() &&
               (a.kvmaps ? mega_attn_produce_tc<D, STAGES, PAGED>(ring, full, empty, it, a, l, pos, policy)
                         : mega_attn_produce<D, STAGES, PAGED>(ring, full, empty, it, a, l, pos));
        } else {
          ok = ok && mark() && mega_attn_produce<D, STAGES, PAGED>(ring, full, empty, it, a, l, pos);
        }
        ok = ok && mark() && gemv_produce<QD, STAGES, false>(ring, full, empty, it, a.wmaps + 4 * l + 1, w.o, H,
                                                      gemv_share(H, blockIdx.x, ctas),
                                                      gemv_share(H, blockIdx.x + 1, ctas), policy, a.status,
                                                      pf, &issued, pwait());
        ok = ok && mark() && gemv_produce<H, STAGES, true>(ring, full, empty, it, a.wmaps + 4 * l + 2, w.gate_up, F,
                                                    gemv_share(F, blockIdx.x, ctas),
                                                    gemv_share(F, blockIdx.x + 1, ctas), policy, a.status,
                                                    pf, &issued, pwait(),
                                                    (ptrace && l == kMegaTraceStageLayer) ? ptrace + (kMegaTraceStages - kMegaTraceProducer) : nullptr);
        ok = ok && mark() && gemv_produce<F, STAGES, false>(ring, full, empty, it, a.wmaps + 4 * l + 3, w.down, H,
                                                     gemv_share(H, blockIdx.x, ctas),
                                                     gemv_share(H, blockIdx.x + 1, ctas), policy, a.status,
                                                     pf, &issued, pwait());
      }
      if (ok) {
        mark();
        gemv_produce<H, STAGES, false>(ring, full, empty, it, a.wmaps + 4 * a.layers, a.lm_head, a.vocab,
                                          gemv_share(a.vocab, blockIdx.x, ctas),
                                          gemv_share(a.vocab, blockIdx.x + 1, ctas), policy, a.status,
                                          pf, &issued, pwait());
      }
      *s_issued = kMegaIssuedDone;
      ring_drain<STAGES>(full, it, a.status);
    }
  } else if (warp == kMegaWarps + 1) {
    // ---------------- L2 prefetcher (a zero lead means none)
    if (a.prefetch_bytes) mega_prefetch_loop<H, QD, F, D>(a, s_issued, lane);
  } else {
    // ---------------- consumers
    int it = 0;
    bool failed = false;
    unsigned nbar = 0;
    unsigned long long best = 0ull;
    unsigned long long* ctrace = a.trace ? a.trace + blockIdx.x * kMegaTraceEvents : nullptr;
    if (ctrace && tid == 0) ctrace[0] = globaltimer_ns();
    int phase_no = 0;
    auto cwait = [&]() -> unsigned long long* {
      return ctrace ? ctrace + kMegaTraceConsumerWait + (phase_no - 1) : nullptr;
    };
    auto pro_done = [&]() {
      if (ctrace && tid == 0 && 163 + phase_no < kMegaTraceProducer - 1) ctrace[163 + phase_no] = globaltimer_ns();
      ++phase_no;
    };
    // Low-latency exchange: the phase outputs carry tags, so a phase ends
    // with a CTA-local barrier only; the next phase's prologue polls its
    // inputs. Tag of (layer l, phase p): ep0 + 5 l + p + 1.
    constexpr bool ll = LL;  // a compile-time choice: each instance carries one exchange
    auto tag = [&](int layer, int ph) -> uint32_t {
      return static_cast<uint32_t>(s_flags[4]) + 5u * static_cast<uint32_t>(layer) + ph + 1u;
    };
    auto sync = [&]() -> bool {
      ++nbar;
      unsigned long long* t = (ctrace && 2 * nbar < kMegaTraceProducer) ? ctrace + 2 * nbar - 1 : nullptr;
      if (ll) {
        if (t && tid == 0) t[0] = t[1] = globaltimer_ns();
        const bool any = named_sync_or(1, kGemvConsumers, failed);
        if (any && tid == 0) atomicOr(a.status, kStatusAbort);
        return !any;
      }
      if (failed) atomicOr(a.status, kStatusAbort);
      const bool arrive = !(a.test_skip_arrival && nbar == 1 && blockIdx.x == 0);
      return mega_grid_sync(a.bar, nbar * static_cast<unsigned>(ctas), a.status, &s_flags[0], t, a.wait_ns,
                            arrive) &&
             !failed;
    };
    // With the exchange, a CTA without rows in a phase reads none of its
    // inputs: every reader of an exchange buffer then also produces output
    // that the buffer's next writer must see first, so no word is rewritten
    // while a reader still needs its previous value (the argument holds for
    // each replica of a buffer, since every replica has the same writers):
    //   qkv_ll  read by ATTN(l); rewritten by QKV(l+1), whose writers polled
    //           every DOWN(l) residual word, written after each DOWN-row owner
    //           finished O(l), which needed the whole attention output of
    //           layer l, written after the attention reads;
    //   part_ll read by ATTN(l)'s split-0 mergers before they write attn_ll;
    //   attn_ll read by O(l); both rewritten by ATTN(l+1), whose CTAs
    //           polled q/k/v rows written after their owners' QKV(l+1)
    //           prologue, which needed every DOWN(l) word -- written after
    //           each O-row owner (the same rows as DOWN) finished O(l);
    //   x_ll    read by GU(l) (O's sums) and QKV(l+1) (DOWN's); rewritten by
    //           DOWN(l) after polling every act word of GU(l), and by
    //           O(l+1) after polling the attention output, which needed
    //           every q/k/v row of QKV(l+1);
    //   act_ll  read by DOWN(l); rewritten by GU(l+1) after polling every
    //           O(l+1) residual word, written by the DOWN-row owners after
    //           DOWN(l).
    auto hrow0 = [&]() { return gemv_share(H, blockIdx.x, ctas); };
    auto hrow1 = [&]() { return gemv_share(H, blockIdx.x + 1, ctas); };
    bool run = true;
    for (int l = 0; l < a.layers && run; ++l) {
      const MegaLayer& w = a.L[l];
      const int nqkv = QD + 2 * (D * a.num_kv);
      {  // QKV
        GemvArgs g = {};
        g.status = a.status;
        g.eps = a.eps;
        g.norm_w = w.input_norm;
        g.y = a.qkv;
        g.yf = a.qkv_f;
        const int r0 = gemv_share(nqkv, blockIdx.x, ctas), r1 = gemv_share(nqkv, blockIdx.x + 1, ctas);
        if (ll) {
          g.ll_wait_ns = a.wait_ns;
          // test switch: CTA 0 keeps its first q/k/v rows out of the exchange
          // (plain stores), so the attention phase's polls time out
          g.ll_y32 = (a.test_skip_arrival && l == 0 && blockIdx.x == 0) ? nullptr : a.qkv_ll;
          g.ll_copy_bytes = a.ll_copy_bytes;
          g.ll_out_tag = tag(l, 0);
          g.ll_x = l > 0 ? mega_ll_mine(a, a.x_ll) : nullptr;
          g.ll_in_tag = l > 0 ? tag(l - 1, 4) : 0u;
        }
        if constexpr (F32) {
          mega_stage_norm_f32<H>(a.xsum, l == 0 ? a.embed : nullptr, a.state, a.vocab, a.status, a.x, a.xsum,
                                 w.input_norm, a.eps, xs, xs_lo, red8);
        } else if (ll && r0 >= r1) {
          // no rows: nothing to stage
        } else if (l == 0) {
          g.embed = a.embed;
          g.token = a.state;
          g.vocab = a.vocab;
          g.x_out = a.x;
          g.xsum_out = a.xsum;
          gemv_stage_x<H, PRO_EMBED_NORM>(g, xs, red8);
        } else {
          g.x_in = a.x;
          g.xsum = a.xsum;
          if (!gemv_stage_x<H, PRO_NORM>(g, xs, red8)) failed = true;
        }
        pro_done();
        g.wait_cycles = cwait();
        gemv_consume<H, STAGES, F32 ? EPI_STORE_F32 : EPI_STORE, F32>(ring, full, empty, it, g, r0, r1, xs, red,
                                                                      best, failed, xs_lo);
      }
      if (!(run = sync())) break;
      pro_done();  // attention: no separate prologue
      if constexpr (D == 64 && G <= 8) {
        if (a.kvmaps) {
          mega_attn_consume_tc<D, G, STAGES, PAGED, F32>(ring, full, empty, it, a, l, pos, cs, red, xs, &s_flags[1],
                                                         failed, cwait(), ll ? tag(l, 0) : 0u,
                                                         ll ? tag(l, 1) : 0u);
        } else {
          mega_attn_consume<D, G, STAGES, PAGED, F32>(ring, full, empty, it, a, l, pos, cs, red, &s_flags[1], failed,
                                                      cwait());
        }
      } else {
        mega_attn_consume<D, G, STAGES, PAGED, F32>(ring, full, empty, it, a, l, pos, cs, red, &s_flags[1], failed,
                                                    cwait());
      }
      if (!(run = sync())) break;
      {  // O
        GemvArgs g = {};
        g.status = a.status;
        g.resid = a.x;
        g.resid_sum = a.xsum;
        g.exact_resid = F32 ? 1 : 0;
        if (ll) {
          g.ll_y64 = a.x_ll;
          g.ll_copy_bytes = a.ll_copy_bytes;
          g.ll_resid = a.x_ll;
          g.resid_embed = l == 0 ? a.embed + static_cast<size_t>(s_flags[5]) * H : nullptr;
          g.ll_out_tag = tag(l, 2);
          if (hrow0() < hrow1() && !mega_stage_attention<QD, D, F32>(a, pos, xs, xs_lo, tag(l, 1))) failed = true;
        } else {
          mega_stage_attention<QD, D, F32>(a, pos, xs, xs_lo);
        }
        pro_done();
        g.wait_cycles = cwait();
        gemv_consume<QD, STAGES, EPI_RESID, F32>(ring, full, empty, it, g, hrow0(), hrow1(), xs, red, best, failed,
                                                 xs_lo);
      }
      if (!(run = sync())) break;
      {  // GU
        GemvArgs g = {};
        g.status = a.status;
        g.eps = a.eps;
        g.x_in = a.x;
        g.xsum = a.xsum;
        g.norm_w = w.post_norm;
        g.y = a.act;
        g.yf = a.act_f;
        const int f0 = gemv_share(F, blockIdx.x, ctas), f1 = gemv_share(F, blockIdx.x + 1, ctas);
        if (ll) {
          g.ll_wait_ns = a.wait_ns;
          g.ll_x = mega_ll_mine(a, a.x_ll);
          g.ll_in_tag = tag(l, 2);
          g.ll_y32 = a.act_ll;
          g.ll_copy_bytes = a.ll_copy_bytes;
          g.ll_out_tag = tag(l, 3);
        }
        if constexpr (F32) {
          mega_stage_norm_f32<H>(a.xsum, nullptr, nullptr, 0, a.status, nullptr, nullptr, w.post_norm, a.eps, xs,
                                 xs_lo, red8);
        } else if (!ll || f0 < f1) {
          if (!gemv_stage_x<H, PRO_NORM>(g, xs, red8)) failed = true;
        }
        pro_done();
        g.wait_cycles = cwait();
        g.stage_ns = (ctrace && l == kMegaTraceStageLayer) ? ctrace + kMegaTraceStages + 64 : nullptr;
        gemv_consume<H, STAGES, F32 ? EPI_SWIGLU_F32 : EPI_SWIGLU, F32>(ring, full, empty, it, g, f0, f1, xs, red,
                                                                        best, failed, xs_lo);
      }
      if (!(run = sync())) break;
      {  // DOWN
        GemvArgs g = {};
        g.status = a.status;
        g.x_in = a.act;
        g.resid = a.x;
        g.resid_sum = a.xsum;
        g.exact_resid = F32 ? 1 : 0;
        if (ll) {
          g.ll_wait_ns = a.wait_ns;
          g.ll_v = mega_ll_mine(a, a.act_ll);
          g.ll_in_tag = tag(l, 3);
          g.ll_y64 = a.x_ll;
          g.ll_copy_bytes = a.ll_copy_bytes;
          g.ll_resid = a.x_ll;
          g.ll_out_tag = tag(l, 4);
        }
        if constexpr (F32) {
          mega_stage_vec_f32(a.act_f, F, xs, xs_lo);
        } else if (!ll || hrow0() < hrow1()) {
          if (!gemv_stage_x<F, PRO_PLAIN>(g, xs, red8)) failed = true;
        }
        pro_done();
        g.wait_cycles = cwait();
        gemv_consume<F, STAGES, EPI_RESID, F32>(ring, full, empty, it, g, hrow0(), hrow1(), xs, red, best, failed,
                                                xs_lo);
      }
      if (!(run = sync())) break;
    }
    if (run) {  // lm_head
      GemvArgs g = {};
      g.status = a.status;
      g.eps = a.eps;
      g.x_in = a.x;
      g.xsum = a.xsum;
      g.norm_w = a.final_norm;
      g.yf = a.logits;
      const int v0 = gemv_share(a.vocab, blockIdx.x, ctas), v1 = gemv_share(a.vocab, blockIdx.x + 1, ctas);
      if (ll) {
        g.ll_wait_ns = a.wait_ns;
        g.ll_x = mega_ll_mine(a, a.x_ll);
        g.ll_in_tag = tag(a.layers - 1, 4);
      }
      if constexpr (F32) {
        mega_stage_norm_f32<H>(a.xsum, nullptr, nullptr, 0, a.status, nullptr, nullptr, a.final_norm, a.eps, xs,
                               xs_lo, red8);
      } else if (!ll || v0 < v1) {
        if (!gemv_stage_x<H, PRO_NORM>(g, xs, red8)) failed = true;
      }
      pro_done();
      g.wait_cycles = cwait();
      gemv_consume<H, STAGES, EPI_LOGITS_ARGMAX, F32>(ring, full, empty, it, g, v0, v1, xs, red, best, failed,
                                                      xs_lo);
      if (best != 0ull) atomicMax(cta_best, best);
      if (ctrace && tid == 0) ctrace[kMegaTraceProducer - 1] = globaltimer_ns();
    }
    if (failed) atomicOr(a.status, kStatusAbort);
  }
  __syncthreads();
  if (tid == 0 && !(__ldcg(a.status) & kStatusAbort)) {
    GemvArgs g = {};
    g.argmax_acc = a.argmax_acc;
    g.sched = a.argmax_done;
    g.state_token = a.state;
    g.state_pos = a.state + 1;
    g.history = a.history;
    g.history_len = a.history_len;
    g.advance = 1;
    if constexpr (LL) {  // the next step's epoch base, past every tag of this one
      g.epoch = a.epoch;
      g.epoch_next = __ldcg(a.epoch) + 5u * static_cast<uint32_t>(a.layers) + 8u;
    }
    argmax_finish(g, *cta_best);
  }
}

}  // namespace lcrb
