// Split-K GQA decode attention (replaces decode_attention_kernel +
// merge_splits_kernel, src/kernels/attention.cu:110-299, and folds in the
// RoPE / cache write of rope_write_kv_kernel, src/kernels/rope.cu:58-87).
//
// Grid (splits, kv_heads, sequences); 4 consumer warps + 1 producer warp.
// One CTA covers one KV head for every query head of its group, so the cache
// is read once per group, and a contiguous run of 16-position blocks.
//
//   producer   streams each 16-position block's K and V rows (contiguous in
//              both layouts: a page holds [kv_head][slot][d]) into a ring of
//              shared-memory stages with cp.async.bulk; it needs only the
//              device position and page table, fixed for the step, so it
//              starts before griddepcontrol.wait and overlaps the QKV GEMV.
//   consumers  a group of D/8 lanes owns one position at a time, each lane 8
//              dims held as fp32: score = q.k reduced across the group, an
//              online softmax in the log2 domain (ex2 of scaled scores, the
//              reference's __expf), acc += p * v. Groups, then warps, are
//              combined with the logsumexp rule.
// FUSED mode (the decode step): q and the new key/value come straight from the
// QKV projection row; q is rotated (rotate-half pairing i <-> i + d/2, angle
// float(pos) * inv_freq[i], sincosf) and rounded to bf16 as the reference
// stores q_heads; the new key is rotated, rounded, written to the cache and
// used from registers (the copy of its block may predate the write). Splits
// publish (m, l, acc) partials and the last CTA of a (sequence, KV head) to
// finish merges them and resets its counter.
// STANDALONE mode (lcr_decode_attention): q is given already rotated, all
// seq_len positions come from the cache, and partials go to the caller's
// scratch for a separate merge launch, as in the reference.
#pragma once

#include "common.cuh"

namespace lcrb {

struct AttnArgs {
  const bf16* qkv;        // FUSED: per-sequence QKV rows
  int qkv_stride;         // elements between sequences' rows
  int q_dim, kv_dim;
  const bf16* q;          // STANDALONE: rotated q [heads][D]
  const float* inv_freq;  // [D/2]
  bf16* kpool;
  bf16* vpool;
  const int32_t* tables;  // paged: this layer's table of sequence 0
  int table_seq_stride;   // entries between sequences' tables
  int max_pages;          // entries per table
  int pool_pages;         // physical pages in the pool
  int page_size;          // positions per page (multiple of 16)
  long long page_stride;  // elements between physical pages
  long long head_stride;  // elements between KV heads (in a page / sequence)
  long long seq_stride;   // contiguous: elements between sequences
  int max_seq;
  const int32_t* positions;  // FUSED: position being decoded, per sequence
  int seq_len;               // STANDALONE: cached positions
  int splits;
  float scale_log2;          // softmax scale * log2(e)
  bf16* out;                 // [sequences][heads * D]
  float* partials;           // [sequences][heads][splits][2 + D]
  unsigned* counters;        // FUSED: [sequences][kv_heads]
  uint32_t* status;
  // attn_batch_kernel only: positions per work item (a multiple of 16), the
  // sequences of the batch, and two work counters that are zero between
  // launches (next item, finished CTAs).
  int item_pos;
  int seqs;
  unsigned* work;
};

constexpr int kAttnConsumerWarps = 4;
constexpr int kAttnThreads = (kAttnConsumerWarps + 1) * 32;
constexpr int kAttnBlock = 16;      // positions per chunk unit (split boundaries, pages)
constexpr int kAttnStagePos = 64;   // positions per ring stage

// Largest split count whose partials for one (sequence, KV head) group fit the
// stage ring, so the last CTA can merge them from shared memory.
template <int D, int STAGES>
constexpr int attn_max_staged_splits(int group) {
  return (STAGES * 2 * kAttnStagePos * D * 2) / (group * (2 + D) * 4);
}

template <int D, int STAGES>
constexpr size_t attn_smem_bytes() {
  return static_cast<size_t>(STAGES) * 2 * kAttnStagePos * D * 2 + 2 * STAGES * 8 +
         static_cast<size_t>(kAttnConsumerWarps) * 8 * (D + 2) * 4 + 64;
}

__device__ __forceinline__ int attn_chunk(int seq_len, int splits) {
  const int per = (seq_len + splits - 1) / splits;
  return (per + kAttnBlock - 1) / kAttnBlock * kAttnBlock;
}

// Loads 8 dims of one head from a bf16 row and applies the rotate-half RoPE
// for this lane's dims with the step's precomputed cos/sin table (cs[i] =
// cos, cs[HALF + i] = sin of float(pos) * inv_freq[i]), returning the
// bf16-rounded values the reference stores.
// Rotate-half RoPE (src/kernels/rope.cu:9-11) of lane `lig`'s 8 dims from
// the raw 16-byte vectors of its own dims (`self`) and their partners.
template <int D>
__device__ __forceinline__ void rope8_from(uint4 self_raw, uint4 other_raw, int lig, const float* cs,
                                           float* outv) {
  constexpr int HALF = D / 2;
  const int d0 = lig * 8;
  float self[8], other[8];
  unpack8(self_raw, self);
  unpack8(other_raw, other);
  const bool lo = d0 < HALF;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int i = (d0 + e) % HALF;
    const float c = cs[i], s = cs[HALF + i];
    const float v = lo ? (self[e] * c - other[e] * s) : (self[e] * c + other[e] * s);
    outv[e] = rbf(v);
  }
}

template <int D>
__device__ __forceinline__ void rope8(const bf16* head, int lig, const float* cs, float* outv) {
  constexpr int HALF = D / 2;
  const int d0 = lig * 8;
  const uint4 self = ldg_cg16(head + d0);
  const uint4 other = ldg_cg16(head + (d0 < HALF ? d0 + HALF : d0 - HALF));
  rope8_from<D>(self, other, lig, cs, outv);
}

// cos/sin of float(pos) * inv_freq[i] for the D/2 rotation pairs (sincosf,
// as src/kernels/rope.cu:50, 77 evaluates them), one pair per thread.
template <int D>
__device__ __forceinline__ void rope_table(float* cs, int pos, const float* inv_freq) {
  constexpr int HALF = D / 2;
  for (int i = threadIdx.x; i < HALF; i += blockDim.x) {
    float s, c;
    sincosf(static_cast<float>(pos) * inv_freq[i], &s, &c);
    cs[i] = c;
    cs[HALF + i] = s;
  }
}

template <int G>
__device__ __forceinline__ void softmax_merge(float& m, float& l, float (&acc)[G][8], int g,
                                              float om, float ol, const float* oacc) {
  const float mn = fmaxf(m, om);
  const float a = ex2_approx(m - mn), b = ex2_approx(om - mn);
  l = l * a + ol * b;
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[g][e] = acc[g][e] * a + oacc[e] * b;
  m = mn;
}

// Finishes split `split` of `splits` of one (sequence, KV head) from the
// consumer warps' (m, l, acc) records in `comb` ([warps][G][2 + D]): the
// output itself when there is one split, else this split's partial (slot
// `split` of `slots` per head), and -- FUSED, in the last CTA of the
// (sequence, KV head) to finish -- the merge of every split, staged through
// `stage` (stage_bytes of idle shared memory) when it fits, else read from
// L2. Run by the 128 consumer threads (threadIdx.x 0..127) after `comb` is
// complete; uses named barrier 1.
template <int D, int G, bool FUSED>
__device__ __forceinline__ void attn_finish(const AttnArgs& a, const float* comb, uint8_t* stage, int stage_bytes,
                                            int split, int splits, int slots, int kvh, int b, int num_kv,
                                            int* s_last) {
  const int tid = threadIdx.x;
  const int heads = num_kv * G;
  // Thread t of the 128 consumers finalises (head g, dims) pairs.
  for (int idx = tid; idx < G * D; idx += kAttnConsumerWarps * 32) {
    const int g = idx / D, d = idx % D;
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < kAttnConsumerWarps; ++w) M = fmaxf(M, comb[(w * G + g) * (D + 2)]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnConsumerWarps; ++w) {
      const float* c = comb + (w * G + g) * (D + 2);
      const float sc = ex2_approx(c[0] - M);
      L += c[1] * sc;
      A += c[2 + d] * sc;
    }
    const int h = kvh * G + g;
    if (splits == 1) {
      a.out[static_cast<size_t>(b) * heads * D + h * D + d] =
          __ushort_as_bfloat16(f2bf(L > 0.f ? A / L : 0.f));
    } else {
      float* slotp = a.partials + ((static_cast<size_t>(b) * heads + h) * slots + split) * (2 + D);
      if (d == 0) {
        slotp[0] = M;
        slotp[1] = L;
      }
      slotp[2 + d] = A;
    }
  }

  if (FUSED && splits > 1) {
    // Last CTA of this (sequence, KV head) merges every split: this
    // thread's partial is visible device-wide before the count moves.
    __threadfence();
    named_sync(1, kAttnConsumerWarps * 32);
    if (tid == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(&a.counters[b * num_kv + kvh], 1u);
      *s_last = (prev == static_cast<unsigned>(splits) - 1) ? 1 : 0;
      if (*s_last) {
        __threadfence();
        a.counters[b * num_kv + kvh] = 0u;
      }
    }
    named_sync(1, kAttnConsumerWarps * 32);
    if (*s_last) {
      // Stage the group's split partials -- one contiguous span of
      // G * splits * (2 + D) floats -- into the idle stage memory with
      // coalesced L2 loads, then merge from shared memory.
      const int span = G * slots * (2 + D);
      const float* src = a.partials + (static_cast<size_t>(b) * heads + kvh * G) * slots * (2 + D);
      float* stg = reinterpret_cast<float*>(stage);
      if (span * static_cast<int>(sizeof(float)) <= stage_bytes) {
#pragma unroll 8
        for (int i = tid; i < span; i += kAttnConsumerWarps * 32) stg[i] = __ldcg(src + i);
        named_sync(1, kAttnConsumerWarps * 32);
      } else {
        stg = nullptr;  // too many splits to stage: merge straight from L2
      }
      for (int idx = tid; idx < G * D; idx += kAttnConsumerWarps * 32) {
        const int g = idx / D, d = idx % D;
        const int h = kvh * G + g;
        const float* base = stg ? stg + g * slots * (2 + D)
                                : src + g * slots * (2 + D);
        float M = kNegBig;
        for (int s = 0; s < splits; ++s) M = fmaxf(M, stg ? base[s * (2 + D)] : __ldcg(base + s * (2 + D)));
        float L = 0.f, A = 0.f;
        for (int s = 0; s < splits; ++s) {
          const float m_s = stg ? base[s * (2 + D)] : __ldcg(base + s * (2 + D));
          const float l_s = stg ? base[s * (2 + D) + 1] : __ldcg(base + s * (2 + D) + 1);
          const float a_s = stg ? base[s * (2 + D) + 2 + d] : __ldcg(base + s * (2 + D) + 2 + d);
          const float sc = ex2_approx(m_s - M);
          L += l_s * sc;
          A += a_s * sc;
        }
        a.out[static_cast<size_t>(b) * heads * D + h * D + d] =
            __ushort_as_bfloat16(f2bf(L > 0.f ? A / L : 0.f));
      }
    }
  }
}

template <int D, int G, bool PAGED, bool FUSED, int STAGES>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
  constexpr int LPP = D / 8;                    // lanes per position
  constexpr int GPW = 32 / LPP;                 // position groups per warp
  constexpr int NG = kAttnConsumerWarps * GPW;  // groups per CTA
  constexpr int PASSES = kAttnStagePos / NG;
  constexpr int ROWB = D * 2;                   // bytes per K (or V) row
  constexpr int KB = kAttnStagePos * ROWB;      // bytes of K per stage
  static_assert(kAttnStagePos % NG == 0 && kAttnStagePos % kAttnBlock == 0, "positions per stage");

  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * 2 * KB);
  uint64_t* empty = full + STAGES;
  float* comb = reinterpret_cast<float*>(empty + STAGES);  // [warps][G][D + 2]
  __shared__ int s_last;
  __shared__ float rope_cs[D];  // cos / sin of this step's angles

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int num_kv = gridDim.y;

  int pos, seq_len;
  if constexpr (FUSED) {
    pos = a.positions[b];
    seq_len = pos + 1;
  } else {
    pos = a.seq_len;  // every position comes from the cache
    seq_len = a.seq_len;
  }
  bool valid = seq_len >= 1 && seq_len <= a.max_seq;
  if (PAGED && valid && (seq_len + a.page_size - 1) / a.page_size > a.max_pages) valid = false;
  const int chunk = attn_chunk(seq_len, a.splits);
  const int begin = split * chunk;
  const int end = valid ? min(seq_len, begin + chunk) : 0;
  const int cache_end = min(end, pos);  // positions read from the cache
  const int nblocks = cache_end > begin ? (cache_end - begin + kAttnStagePos - 1) / kAttnStagePos : 0;

  if constexpr (FUSED) {
    // The angles depend only on the position: one sincosf per pair per CTA,
    // before the wait on the QKV projection.
    rope_table<D>(rope_cs, valid ? pos : 0, a.inv_freq);
  }
  if (tid == 0) {
    if (!valid && split == 0 && kvh == 0 && a.status) atomicOr(a.status, kStatusBadPosition);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kAttnConsumerWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_launch_next();

  if (warp == kAttnConsumerWarps) {
    if (lane == 0) {
      const int32_t* table = PAGED ? a.tables + static_cast<size_t>(b) * a.table_seq_stride : nullptr;
      int issued = 0;
      for (int blk = 0; blk < nblocks; ++blk) {
        const int slot = blk % STAGES;
        if (blk >= STAGES &&
            !mbar_wait(&empty[slot], ((blk / STAGES) - 1) & 1, a.status, kStatusTimeoutEmpty)) {
          break;
        }
        const int p0 = begin + blk * kAttnStagePos;
        // Copy only positions below cache_end (the caller's cache may end
        // inside this stage), in runs that do not cross a page.
        const int nvalid = min(kAttnStagePos, cache_end - p0);
        uint8_t* dst = ring + slot * 2 * KB;
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nvalid) * 2 * ROWB);
        for (int n = 0; n < nvalid;) {
          int run = nvalid - n;
          long long off;
          const int p = p0 + n;
          if constexpr (PAGED) {
            run = min(run, a.page_size - p % a.page_size);
            int page = table[p / a.page_size];
            if (page < 0 || page >= a.pool_pages) {
              if (a.status) atomicOr(a.status, kStatusBadPage);
              page = 0;
            }
            off = static_cast<long long>(page) * a.page_stride + kvh * a.head_stride +
                  static_cast<long long>(p % a.page_size) * D;
          } else {
            off = static_cast<long long>(b) * a.seq_stride + kvh * a.head_stride + static_cast<long long>(p) * D;
          }
          const uint32_t bytes = static_cast<uint32_t>(run) * ROWB;
          bulk_g2s(dst + n * ROWB, a.kpool + off, bytes, &full[slot]);
          bulk_g2s(dst + KB + n * ROWB, a.vpool + off, bytes, &full[slot]);
          n += run;
        }
        issued = blk + 1;
      }
      // Never leave the CTA with a copy still writing its shared memory.
      for (int blk = issued > STAGES ? issued - STAGES : 0; blk < issued; ++blk) {
        mbar_wait(&full[blk % STAGES], (blk / STAGES) & 1, nullptr, 0);  // waits even after an abort
      }
    }
  } else {
    const int lig = lane % LPP;    // lane within the position group
    const int grp = warp * GPW + lane / LPP;

    float q[G][8], acc[G][8], m[G], l[G];
    pdl_wait();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int h = kvh * G + g;
      if constexpr (FUSED) {
        // rotated q rounded to bf16, as the reference stores it (rope_q)
        rope8<D>(a.qkv + static_cast<size_t>(b) * a.qkv_stride + h * D, lig, rope_cs, q[g]);
#pragma unroll
        for (int e = 0; e < 8; ++e) q[g][e] = rbf(q[g][e]);
      } else {
        unpack8(ldg16(a.q + h * D + lig * 8), q[g]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        q[g][e] *= a.scale_log2;
        acc[g][e] = 0.f;
      }
      m[g] = kNegBig;
      l[g] = 0.f;
    }

    for (int blk = 0; blk < nblocks; ++blk) {
      const int slot = blk % STAGES;
      if (!mbar_wait(&full[slot], (blk / STAGES) & 1, a.status, kStatusTimeoutFull)) break;
      const uint8_t* kst = ring + slot * 2 * KB;
      const uint8_t* vst = kst + KB;
      const int p0 = begin + blk * kAttnStagePos;
#pragma unroll
      for (int pass = 0; pass < PASSES; ++pass) {
        const int pl = pass * NG + grp;
        // Every lane runs the loads and shuffles (the stage is always in
        // bounds); only the softmax update is predicated on the position.
        const bool live = p0 + pl < cache_end;
        {
          float kf[8], vf[8];
          unpack8(*reinterpret_cast<const uint4*>(kst + pl * ROWB + lig * 16), kf);
          unpack8(*reinterpret_cast<const uint4*>(vst + pl * ROWB + lig * 16), vf);
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
              l[g] = l[g] * alpha + p;
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p, vf[e], acc[g][e] * alpha);
              m[g] = mn;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    if constexpr (FUSED) {
      // The new position: rotate K, store K and V in the cache, and attend to
      // it from registers (group 0 of warp 0).
      if (valid && pos >= begin && pos < end && grp == 0) {
        const bf16* row = a.qkv + static_cast<size_t>(b) * a.qkv_stride;
        float kf[8], vf[8];
        rope8<D>(row + a.q_dim + kvh * D, lig, rope_cs, kf);
#pragma unroll
        for (int e = 0; e < 8; ++e) kf[e] = rbf(kf[e]);  // attends to the cache's bf16 key
        unpack8(ldg_cg16(row + a.q_dim + a.kv_dim + kvh * D + lig * 8), vf);
        long long off;
        if constexpr (PAGED) {
          const int32_t* table = a.tables + static_cast<size_t>(b) * a.table_seq_stride;
          int page = table[pos / a.page_size];
          if (page < 0 || page >= a.pool_pages) page = 0;
          off = static_cast<long long>(page) * a.page_stride + kvh * a.head_stride +
                static_cast<long long>(pos % a.page_size) * D;
        } else {
          off = static_cast<long long>(b) * a.seq_stride + kvh * a.head_stride +
                static_cast<long long>(pos) * D;
        }
        uint4 kw;
        kw.x = pack_bf2(kf[0], kf[1]); kw.y = pack_bf2(kf[2], kf[3]);
        kw.z = pack_bf2(kf[4], kf[5]); kw.w = pack_bf2(kf[6], kf[7]);
        *reinterpret_cast<uint4*>(a.kpool + off + lig * 8) = kw;
        *reinterpret_cast<uint4*>(a.vpool + off + lig * 8) =
            ldg_cg16(row + a.q_dim + a.kv_dim + kvh * D + lig * 8);
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
          l[g] = l[g] * alpha + p;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p, vf[e], acc[g][e] * alpha);
          m[g] = mn;
        }
      }
    }

    // Combine the position groups of this warp (same dims, other positions).
#pragma unroll
    for (int off = LPP; off < 32; off <<= 1) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float om = __shfl_xor_sync(0xffffffffu, m[g], off);
        const float ol = __shfl_xor_sync(0xffffffffu, l[g], off);
        float oacc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) oacc[e] = __shfl_xor_sync(0xffffffffu, acc[g][e], off);
        softmax_merge<G>(m[g], l[g], acc, g, om, ol, oacc);
      }
    }
    // Then the warps, through shared memory.
    if (lane < LPP) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float* c = comb + (warp * G + g) * (D + 2);
        if (lane == 0) {
          c[0] = m[g];
          c[1] = l[g];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) c[2 + lane * 8 + e] = acc[g][e];
      }
    }
    named_sync(1, kAttnConsumerWarps * 32);
    attn_finish<D, G, FUSED>(a, comb, ring, STAGES * 2 * KB, split, a.splits, a.splits, kvh, b, num_kv, &s_last);
  }
}

// STANDALONE merge of split partials (merge_splits_kernel,
// src/kernels/attention.cu:267-299), one block per query head.
template <int D>
__global__ void attn_merge_kernel(bf16* __restrict__ out, const float* __restrict__ partials,
                                  int splits) {
  const int h = blockIdx.x;
  const float* base = partials + static_cast<size_t>(h) * splits * (2 + D);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float M = kNegBig;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, base[s * (2 + D)]);
    float L = 0.f, A = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float sc = ex2_approx(base[s * (2 + D)] - M);
      L += base[s * (2 + D) + 1] * sc;
      A += base[s * (2 + D) + 2 + d] * sc;
    }
    out[h * D + d] = __ushort_as_bfloat16(f2bf(L > 0.f ? A / L : 0.f));
  }
}

}  // namespace lcrb
