// The reference's standalone elementwise kernels, as sm_100a SIMT kernels for
// the per-kernel C entry points (src/kernels/elementwise.cu, rmsnorm.cu,
// rope.cu). The decode step itself does not launch these: it folds each of
// them into the neighbouring streaming GEMV or into the attention kernel.
// Storage is bf16, arithmetic fp32, with the reference's rounding points.
#pragma once

#include "common.cuh"

namespace lcrb {

constexpr int kSmallThreads = 256;

// x[t] = table[ids[t]] (elementwise.cu:25-41); bit-exact copy.
static __global__ void embedding_kernel(bf16* __restrict__ out, const bf16* __restrict__ table,
                                 const int32_t* __restrict__ ids, int dim, int vocab,
                                 uint32_t* status) {
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && status) atomicOr(status, kStatusBadToken);
    id = 0;
  }
  const bf16* src = table + static_cast<size_t>(id) * dim;
  bf16* dst = out + static_cast<size_t>(t) * dim;
  const int vecs = dim / 8;
  for (int i = threadIdx.x; i < vecs; i += blockDim.x) {
    reinterpret_cast<uint4*>(dst)[i] = ldg16(src + i * 8);
  }
  for (int i = vecs * 8 + threadIdx.x; i < dim; i += blockDim.x) dst[i] = src[i];
}

__device__ __forceinline__ float block_sum_256(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kSmallThreads / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}

// out = bf16(x * rsqrt(mean(x^2) + eps) * w) (rmsnorm.cu:21-63). When `delta`
// is given, first x = bf16(x + delta) with the sum of squares taken over the
// unrounded sums (rmsnorm.cu:68-119).
static __global__ void rmsnorm_kernel(bf16* __restrict__ out, bf16* __restrict__ x,
                               const bf16* __restrict__ delta, const bf16* __restrict__ w,
                               int dim, float eps) {
  __shared__ float red[kSmallThreads / 32];
  const size_t row = static_cast<size_t>(blockIdx.x) * dim;
  bf16* xr = x + row;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = bf2f(__bfloat16_as_ushort(xr[i]));
    if (delta != nullptr) {
      v = v + bf2f(__bfloat16_as_ushort(delta[row + i]));
      xr[i] = __ushort_as_bfloat16(f2bf(v));
    }
    ss += v * v;
  }
  const float total = block_sum_256(ss, red);
  const float scale = rsqrtf(total / static_cast<float>(dim) + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = bf2f(__bfloat16_as_ushort(xr[i]));
    out[row + i] = __ushort_as_bfloat16(
        f2bf(__fmul_rn(__fmul_rn(v, scale), bf2f(__bfloat16_as_ushort(w[i])))));
  }
}

// x += delta (elementwise.cu:43-62).
static __global__ void add_residual_kernel(bf16* __restrict__ x, const bf16* __restrict__ delta,
                                    int64_t count) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride) {
    x[i] = __ushort_as_bfloat16(f2bf(bf2f(__bfloat16_as_ushort(x[i])) +
                                     bf2f(__bfloat16_as_ushort(delta[i]))));
  }
}

__device__ __forceinline__ float silu_ref(float v) { return v / (1.0f + __expf(-v)); }

// out[t][i] = silu(gate[t*stride + i]) * up[t*stride + i] (elementwise.cu:64-121);
// stride = width for the contiguous form.
static __global__ void swiglu_kernel(bf16* __restrict__ out, const bf16* __restrict__ gate,
                              const bf16* __restrict__ up, int64_t width, int64_t stride,
                              int64_t rows) {
  const int64_t total = width * rows;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < total;
       k += step) {
    const int64_t r = k / width, i = k % width;
    const float g = bf2f(__bfloat16_as_ushort(gate[r * stride + i]));
    const float u = bf2f(__bfloat16_as_ushort(up[r * stride + i]));
    out[k] = __ushort_as_bfloat16(f2bf(silu_ref(g) * u));
  }
}

// Rotate-half RoPE (rope.cu:9-56): grid (tokens, heads). Writes head-major
// [heads][tokens][d] when head_major, else [tokens][heads][d] at dst_row_stride.
static __global__ void rope_q_kernel(bf16* __restrict__ q_heads, const bf16* __restrict__ q_proj,
                              const float* __restrict__ inv_freq, int tokens, int start,
                              int head_dim, int src_row_stride) {
  const int t = blockIdx.x, h = blockIdx.y, half = head_dim / 2;
  const size_t src = static_cast<size_t>(t) * src_row_stride + static_cast<size_t>(h) * head_dim;
  const size_t dst = (static_cast<size_t>(h) * tokens + t) * head_dim;
  const float p = static_cast<float>(start + t);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float s, c;
    sincosf(p * inv_freq[i], &s, &c);
    const float lo = bf2f(__bfloat16_as_ushort(q_proj[src + i]));
    const float hi = bf2f(__bfloat16_as_ushort(q_proj[src + i + half]));
    q_heads[dst + i] = __ushort_as_bfloat16(f2bf(lo * c - hi * s));
    q_heads[dst + i + half] = __ushort_as_bfloat16(f2bf(hi * c + lo * s));
  }
}

// RoPE on K plus the K/V cache write (rope.cu:58-87): grid (tokens, kv_heads).
static __global__ void rope_write_kv_kernel(bf16* __restrict__ keys, bf16* __restrict__ values,
                                     const int32_t* __restrict__ page_table, int page_size,
                                     long long page_stride, long long head_stride, int head_dim,
                                     const bf16* __restrict__ k_proj,
                                     const bf16* __restrict__ v_proj,
                                     const float* __restrict__ inv_freq, int start,
                                     int src_row_stride) {
  const int t = blockIdx.x, h = blockIdx.y, half = head_dim / 2;
  const int pos = start + t;
  const size_t src = static_cast<size_t>(t) * src_row_stride + static_cast<size_t>(h) * head_dim;
  long long dst;
  if (page_table != nullptr) {
    dst = static_cast<long long>(page_table[pos / page_size]) * page_stride + h * head_stride +
          static_cast<long long>(pos % page_size) * head_dim;
  } else {
    dst = h * head_stride + static_cast<long long>(pos) * head_dim;
  }
  const float p = static_cast<float>(pos);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float s, c;
    sincosf(p * inv_freq[i], &s, &c);
    const float lo = bf2f(__bfloat16_as_ushort(k_proj[src + i]));
    const float hi = bf2f(__bfloat16_as_ushort(k_proj[src + i + half]));
    keys[dst + i] = __ushort_as_bfloat16(f2bf(lo * c - hi * s));
    keys[dst + i + half] = __ushort_as_bfloat16(f2bf(hi * c + lo * s));
  }
  for (int i = threadIdx.x; i < head_dim; i += blockDim.x) values[dst + i] = v_proj[src + i];
}

// Multi-row fallback of gemm_nt for shapes the streaming kernel has no
// instantiation for: one warp per (row, output), fp32 accumulation.
static __global__ void gemm_nt_simple_kernel(void* __restrict__ y, int y_fp32, const bf16* __restrict__ x,
                                      const bf16* __restrict__ w, int rows, int in_f, int out_f) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows * out_f) return;
  const int r = warp / out_f, o = warp % out_f;
  const bf16* xr = x + static_cast<size_t>(r) * in_f;
  const bf16* wr = w + static_cast<size_t>(o) * in_f;
  float acc = 0.f;
  for (int k = lane; k < in_f; k += 32) {
    acc = fmaf(bf2f(__bfloat16_as_ushort(xr[k])), bf2f(__bfloat16_as_ushort(wr[k])), acc);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const size_t idx = static_cast<size_t>(r) * out_f + o;
    if (y_fp32) reinterpret_cast<float*>(y)[idx] = acc;
    else reinterpret_cast<bf16*>(y)[idx] = __ushort_as_bfloat16(f2bf(acc));
  }
}

// Causal softmax of prefill attention scores (attention.cu:42-100 computes the
// same distribution): row r of head h is query position start + r and sees
// keys [0, min(keys, start + r + 1)); probs = bf16(exp(s - max) / sum) there,
// 0 beyond (the buffer is reused across chunks). One CTA per (row, head),
// three passes over the row: the maximum, the exponential sum, the write.
static __global__ void causal_softmax_kernel(bf16* __restrict__ probs, const float* __restrict__ scores,
                                             int rows, int keys, int start) {
  __shared__ float red[kSmallThreads / 32];
  const int row = blockIdx.x;
  const size_t base = (static_cast<size_t>(blockIdx.y) * rows + row) * keys;
  const int limit = min(keys, start + row + 1);
  const float* sr = scores + base;
  float mx = kNegBig;
  for (int j = threadIdx.x; j < limit; j += blockDim.x) mx = fmaxf(mx, sr[j]);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < kSmallThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int j = threadIdx.x; j < limit; j += blockDim.x) sum += expf(sr[j] - mx);
  sum = block_sum_256(sum, red);
  const float inv = sum > 0.f ? 1.0f / sum : 0.f;
  bf16* pr = probs + base;
  for (int j = threadIdx.x; j < keys; j += blockDim.x) {
    pr[j] = __ushort_as_bfloat16(f2bf(j < limit ? expf(sr[j] - mx) * inv : 0.f));
  }
}

// heads[h][t][0, d) -> out[t][h * d, h * d + d) (elementwise.cu:124-143): a
// copy, 16 bytes at a time when d is a multiple of 8.
static __global__ void merge_heads_kernel(bf16* __restrict__ out, const bf16* __restrict__ heads, int tokens,
                                          int num_heads, int d) {
  const int v8 = d % 8 == 0 ? 8 : 1;
  const long long units = static_cast<long long>(tokens) * num_heads * (d / v8);
  for (long long u = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; u < units;
       u += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(u % (d / v8)) * v8;
    const long long th = u / (d / v8);
    const int h = static_cast<int>(th % num_heads);
    const long long t = th / num_heads;
    const bf16* src = heads + (static_cast<long long>(h) * tokens + t) * d + i;
    bf16* dst = out + (t * num_heads + h) * d + i;
    if (v8 == 8) {
      *reinterpret_cast<uint4*>(dst) = ldg16(src);
    } else {
      *dst = *src;
    }
  }
}

// The cache of positions [0, positions) as contiguous [kv_head][position][d]
// keys and values (attention.cu:302-316): per (position, head) the row at the
// view's offset (page_table[p / page_size] * page_stride + head * head_stride
// + (p % page_size) * d; no table: page 0, slot p). A negative table entry
// (an unmapped page) gives zero rows.
static __global__ void gather_kv_kernel(bf16* __restrict__ out_k, bf16* __restrict__ out_v, const bf16* keys,
                                        const bf16* values, const int32_t* table, int page_size,
                                        long long page_stride, long long head_stride, int d, int positions) {
  const int p = blockIdx.x, h = blockIdx.y;
  long long src;
  bool mapped = true;
  if (table != nullptr) {
    const int page = table[p / page_size];
    mapped = page >= 0;
    src = static_cast<long long>(page) * page_stride + h * head_stride + static_cast<long long>(p % page_size) * d;
  } else {
    src = h * head_stride + static_cast<long long>(p) * d;
  }
  const long long dst = (static_cast<long long>(h) * positions + p) * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const bf16 z = __ushort_as_bfloat16(0);
    out_k[dst + i] = mapped ? keys[src + i] : z;
    out_v[dst + i] = mapped ? values[src + i] : z;
  }
}

}  // namespace lcrb
