// Token selection on the device (replaces argmax_kernel, argmax_unpack_kernel
// and sample_kernel, src/kernels/sampling.cu:42-224).
//
// One 1024-thread block per sequence row of logits.
//   greedy (inv_temperature <= 0): the largest logit, ties to the lowest id,
//     through the packed (order key, ~index) maximum of sampling.cu:42-61.
//   sampling: the reference's semantics -- s = (logit - max) / T, the
//     full-vocabulary exponential sum as denominator, candidates walked in
//     descending order, cut at top_k or once the kept mass reaches top_p (the
//     crossing token kept), a pick at uniform * kept_mass -- computed exactly
//     and deterministically so a CPU restatement reproduces it bit for bit:
//       * exp is det_expf: Cody-Waite reduction + degree-7 Taylor polynomial
//         with explicit fused multiply-adds, no contraction anywhere;
//       * the denominator is a fixed tree: thread t sums i = t, t+1024, ... in
//         index order, then an xor butterfly per warp and over the 32 warps;
//       * the candidates are exactly the first M = min(top_k or V, 1024)
//         tokens in (s desc, index asc) order. A 2048-bucket histogram of -s
//         (monotone in s) names the bucket holding the M-th token; every
//         token at or above that bucket is compacted and bitonic-sorted under
//         the total order, and the first M kept. When that set exceeds
//         kMaxBucketSet (a flat distribution), a 4 x 8-bit radix select over
//         the vocabulary finds the M-th key instead, ties at it taken lowest
//         index first;
//       * the uniform is the caller's, or Philox4x32-10 (Salmon et al., SC'11)
//         of (seed, counter = position, stream 0): the top 24 bits of word 0
//         times 2^-24.
#pragma once

#include "common.cuh"

namespace lcrb {

constexpr int kSampleThreads = 1024;
constexpr int kMaxCandidates = 1024;
constexpr int kSampleBuckets = 2048;  // buckets of -s over [0, kSampleRange)
constexpr float kSampleRange = 32.0f;
constexpr int kMaxBucketSet = 2048;   // tokens the bucket path may sort
static_assert(kSampleBuckets == 2 * kSampleThreads, "two buckets per thread in the scan");

__device__ __forceinline__ float det_expf(float x) {
  if (!(x > -88.0f)) return 0.0f;
  if (x > 88.0f) return __int_as_float(0x7f800000);
  const float k = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-k, 0.693147182464599609375f, x);
  r = __fmaf_rn(-k, -1.904654299957768e-09f, r);
  float p = 1.98412698412698413e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ki = static_cast<int>(k);
  const int k1 = ki / 2, k2 = ki - k1;
  const float s1 = __int_as_float((k1 + 127) << 23);
  const float s2 = __int_as_float((k2 + 127) << 23);
  return __fmul_rn(__fmul_rn(p, s1), s2);
}

__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

__device__ __forceinline__ float philox_uniform(unsigned long long seed,
                                                unsigned long long counter, uint32_t stream) {
  uint32_t c[4] = {static_cast<uint32_t>(counter), static_cast<uint32_t>(counter >> 32), stream, 0u};
  philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  return __fmul_rn(static_cast<float>(c[0] >> 8), 1.0f / 16777216.0f);
}

__device__ __forceinline__ uint32_t sample_key(float s) {
  const uint32_t b = __float_as_uint(s);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SampleArgs {
  const float* logits;         // [rows][row_stride]
  long long row_stride;
  int vocab;
  const float* inv_temperature;  // [rows]; <= 0 means greedy
  const int* top_k;              // [rows]; <= 0 means no top-k cut
  const float* top_p;            // [rows]
  const float* uniform;          // [rows] or nullptr -> Philox
  const unsigned long long* seed;     // [rows] Philox key
  const int32_t* counter;             // [rows] Philox counter (e.g. the position)
  int32_t* out;                  // [rows]
  // Optional device-state update after the pick (single sequence):
  int32_t* state_token;
  int32_t* state_pos;
  int32_t* history;
  int history_len;
  int advance;
  // Single-row calls may pass the parameters by value instead (inline_params
  // set): nothing is read from memory, so the launch can be captured.
  int inline_params;
  float inv_temperature_v, top_p_v, uniform_v;
  int top_k_v;
};

__device__ __forceinline__ float block_max_1024(float v, float* red32) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  if (lane == 0) red32[warp] = v;
  __syncthreads();
  float w = red32[lane];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, off));
  __syncthreads();
  return w;
}

// The fixed summation tree (see the file comment).
__device__ __forceinline__ float block_tree_sum_1024(float v, float* red32) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  if (lane == 0) red32[warp] = v;
  __syncthreads();
  float w = red32[lane];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) w = __fadd_rn(w, __shfl_xor_sync(0xffffffffu, w, off));
  __syncthreads();
  return w;
}

// Bucket of a scaled logit s <= 0: non-decreasing in -s, so a lower bucket
// holds only strictly larger logits (NaN and very negative s go last).
__device__ __forceinline__ int sample_bucket(float s) {
  const float d = __fmul_rn(-s, kSampleBuckets / kSampleRange);
  return d < static_cast<float>(kSampleBuckets - 1) ? max(0, static_cast<int>(d)) : kSampleBuckets - 1;
}

// Bitonic sort of keys[0, n) (n a power of two) under (key desc, index asc).
__device__ __forceinline__ void sort_candidates(uint32_t* keys, uint32_t* idx, int n) {
  for (int span = 2; span <= n; span <<= 1) {
    for (int step = span >> 1; step > 0; step >>= 1) {
      for (int i = threadIdx.x; i < n; i += kSampleThreads) {
        const int j = i ^ step;
        if (j > i) {
          const bool i_first = (keys[i] > keys[j]) || (keys[i] == keys[j] && idx[i] < idx[j]);
          const bool ascending_block = (i & span) != 0;  // reverse order in this half
          if (ascending_block ? i_first : !i_first) {
            const uint32_t tk = keys[i], ti = idx[i];
            keys[i] = keys[j]; idx[i] = idx[j];
            keys[j] = tk; idx[j] = ti;
          }
        }
      }
      __syncthreads();
    }
  }
}

static __global__ void __launch_bounds__(kSampleThreads) sample_rows_kernel(const SampleArgs a) {
  __shared__ float red32[32];
  __shared__ unsigned long long best_s;
  __shared__ int hist[kSampleBuckets];
  __shared__ uint32_t ckey[kMaxBucketSet];
  __shared__ uint32_t cidx[kMaxBucketSet];
  __shared__ uint32_t sel_prefix, sel_want;
  __shared__ int n_gt, sel_bucket, sel_count;
  __shared__ int scan[kSampleThreads / 32];

  const int row = blockIdx.x, tid = threadIdx.x;
  pdl_wait();  // the logits come from the preceding kernel
  pdl_launch_next();
  const float* L = a.logits + static_cast<long long>(row) * a.row_stride;
  const int V = a.vocab;
  const float inv_t = a.inline_params ? a.inv_temperature_v : a.inv_temperature[row];
  int picked = 0;

  if (!(inv_t > 0.0f)) {
    unsigned long long best = 0ull;
    for (int i = tid; i < V; i += kSampleThreads) {
      const unsigned long long packed =
          (static_cast<unsigned long long>(sample_key(L[i])) << 32) |
          static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(i));
      best = best > packed ? best : packed;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = best > o ? best : o;
    }
    if (tid == 0) best_s = 0ull;
    __syncthreads();
    if ((tid & 31) == 0) atomicMax(&best_s, best);
    __syncthreads();
    picked = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(best_s & 0xFFFFFFFFull));
  } else {
    // Pass 1: the maximum logit.
    float mx = -__int_as_float(0x7f800000);
    for (int i = tid; i < V; i += kSampleThreads) mx = fmaxf(mx, L[i]);
    mx = block_max_1024(mx, red32);

    // Pass 2: the denominator and the bucket histogram.
    for (int i = tid; i < kSampleBuckets; i += kSampleThreads) hist[i] = 0;
    __syncthreads();
    float acc = 0.0f;
    for (int i = tid; i < V; i += kSampleThreads) {
      const float s = __fmul_rn(__fsub_rn(L[i], mx), inv_t);
      acc = __fadd_rn(acc, det_expf(s));
      atomicAdd(&hist[sample_bucket(s)], 1);
    }
    const float total = block_tree_sum_1024(acc, red32);  // synchronises hist too

    int k = a.inline_params ? a.top_k_v : a.top_k[row];
    int M = k > 0 ? k : V;
    M = min(M, min(kMaxCandidates, V));

    // The bucket holding the M-th token: a block-wide inclusive scan of the
    // histogram (two buckets per thread).
    {
      const int lane = tid & 31, warp = tid >> 5;
      const int h0 = hist[2 * tid], h1 = hist[2 * tid + 1];
      int incl = h0 + h1;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      if (lane == 31) scan[warp] = incl;
      if (tid == 0) {
        sel_bucket = kSampleBuckets - 1;
        sel_count = V;
      }
      __syncthreads();
      int before = 0;
      for (int w = 0; w < warp; ++w) before += scan[w];
      const int c1 = before + incl;   // tokens in buckets <= 2 tid + 1
      const int c0 = c1 - h1;         // tokens in buckets <= 2 tid
      const int prev = c0 - h0;       // tokens in buckets < 2 tid
      if (prev < M && c0 >= M) {
        sel_bucket = 2 * tid;
        sel_count = c0;
      } else if (c0 < M && c1 >= M) {
        sel_bucket = 2 * tid + 1;
        sel_count = c1;
      }
      if (tid == 0) n_gt = 0;
      __syncthreads();
    }
    const int bucket = sel_bucket, count = sel_count;

    if (count <= kMaxBucketSet) {
      // Pass 3: compact every token in buckets <= bucket, then sort them.
      for (int i = tid; i < V; i += kSampleThreads) {
        const float s = __fmul_rn(__fsub_rn(L[i], mx), inv_t);
        if (sample_bucket(s) <= bucket) {
          const int slot = atomicAdd(&n_gt, 1);
          if (slot < kMaxBucketSet) {
            ckey[slot] = sample_key(s);
            cidx[slot] = static_cast<uint32_t>(i);
          }
        }
      }
      int n = 32;
      while (n < count) n <<= 1;
      for (int i = count + tid; i < n; i += kSampleThreads) {
        ckey[i] = 0u;
        cidx[i] = 0x7fffffffu;
      }
      __syncthreads();
      sort_candidates(ckey, cidx, n);
    } else {
      // Radix select of the M-th largest key, eight bits at a time.
      uint32_t prefix = 0u, mask = 0u, want = static_cast<uint32_t>(M);
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kSampleThreads) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < V; i += kSampleThreads) {
          const uint32_t key = sample_key(__fmul_rn(__fsub_rn(L[i], mx), inv_t));
          if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
        }
        __syncthreads();
        if (tid == 0) {
          uint32_t w = want;
          int digit = 0;
          for (int d = 255; d >= 0; --d) {
            const uint32_t c = static_cast<uint32_t>(hist[d]);
            if (w <= c) {
              digit = d;
              break;
            }
            w -= c;
          }
          sel_prefix = prefix | (static_cast<uint32_t>(digit) << shift);
          sel_want = w;
        }
        __syncthreads();
        prefix = sel_prefix;
        want = sel_want;
        mask |= 255u << shift;
        __syncthreads();
      }
      const uint32_t T = prefix;       // key of the M-th candidate
      const int need_eq = static_cast<int>(want);  // ties at T to take, lowest ids first
      const int n_greater = M - need_eq;

      // Compaction: thread t scans a contiguous index range, so an exclusive
      // scan of its tie count orders ties by index.
      const int R = (V + kSampleThreads - 1) / kSampleThreads;
      const int lo = min(V, tid * R), hi = min(V, lo + R);
      int my_eq = 0;
      for (int i = lo; i < hi; ++i) {
        my_eq += sample_key(__fmul_rn(__fsub_rn(L[i], mx), inv_t)) == T;
      }
      // exclusive scan over 1024 threads
      int incl = my_eq;
      const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      if (lane == 31) scan[warp] = incl;
      __syncthreads();
      if (warp == 0) {
        int v = scan[lane];
        int vi = v;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int o = __shfl_up_sync(0xffffffffu, vi, off);
          if (lane >= off) vi += o;
        }
        scan[lane] = vi - v;  // exclusive warp offsets
      }
      __syncthreads();
      int eq_rank = scan[warp] + incl - my_eq;
      for (int i = tid; i < kMaxCandidates; i += kSampleThreads) {
        ckey[i] = 0u;
        cidx[i] = 0x7fffffffu;
      }
      __syncthreads();
      for (int i = lo; i < hi; ++i) {
        const uint32_t key = sample_key(__fmul_rn(__fsub_rn(L[i], mx), inv_t));
        if (key > T) {
          const int slot = atomicAdd(&n_gt, 1);
          if (slot < n_greater) {
            ckey[slot] = key;
            cidx[slot] = static_cast<uint32_t>(i);
          }
        } else if (key == T) {
          if (eq_rank < need_eq) {
            ckey[n_greater + eq_rank] = key;
            cidx[n_greater + eq_rank] = static_cast<uint32_t>(i);
          }
          ++eq_rank;
        }
      }
      __syncthreads();
      sort_candidates(ckey, cidx, kMaxCandidates);
    }

    // Each candidate's probability, computed in parallel; the walk below
    // adds them in candidate order, as a serial loop would.
    const float inv_total = __fdiv_rn(1.0f, total);
    float* prob = reinterpret_cast<float*>(ckey);
    for (int j = tid; j < M; j += kSampleThreads) {
      prob[j] = __fmul_rn(det_expf(key_to_float(ckey[j])), inv_total);
    }
    __syncthreads();

    if (tid == 0) {
      float u;
      if (a.inline_params) {
        u = a.uniform_v;
      } else if (a.uniform != nullptr) {
        u = a.uniform[row];
      } else {
        // Stream 0: a sequence's draws depend on its seed and position only,
        // not on the batch slot it occupies.
        u = philox_uniform(a.seed[row], static_cast<unsigned long long>(a.counter[row]), 0u);
      }
      const float top_p = a.inline_params ? a.top_p_v : a.top_p[row];
      int keep = 0;
      float kept = 0.0f;
      for (int j = 0; j < M; ++j) {
        const float p = prob[j];
        kept = __fadd_rn(kept, p);
        ++keep;
        if (top_p < 1.0f && kept >= top_p) break;
      }
      const float target = __fmul_rn(u, kept);
      float running = 0.0f;
      picked = static_cast<int>(cidx[0]);
      for (int j = 0; j < keep; ++j) {
        const float p = prob[j];
        running = __fadd_rn(running, p);
        picked = static_cast<int>(cidx[j]);
        if (running >= target) break;
      }
    }
  }

  if (tid == 0) {
    a.out[row] = picked;
    if (a.state_token != nullptr) {
      const int pos = *a.state_pos;
      *a.state_token = picked;
      if (a.history != nullptr && pos >= 0 && pos < a.history_len) a.history[pos] = picked;
      if (a.advance) *a.state_pos = pos + 1;
    }
  }
}

}  // namespace lcrb
