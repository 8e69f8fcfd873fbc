// Row kernels of the batched decode step (batch_ctx.cu): the RMSNorm in
// front of each projection, for every sequence of the batch at once.
#pragma once

#include "common.cuh"

namespace lcrb {

struct NormRowsArgs {
  // EMBED: the token's embedding row is the residual stream (elementwise.cu:25-41)
  const int32_t* tokens;  // [rows]
  const bf16* embed;      // [vocab][H]
  int vocab;
  bf16* x;                // [rows][H] residual stream (bf16), written when EMBED
  float* xsum;            // [rows][H] its unrounded sums, written when EMBED
  const bf16* gain;       // [H]
  float eps;
  bf16* out;              // [rows][H] bf16(x * rsqrt(mean(xsum^2) + eps) * gain)
  uint32_t* status;
  // EMBED, optional: the step's RoPE table, rope[row][half] = (cos, sin) of
  // float(positions[row]) * inv_freq[i] (sincosf, as src/kernels/rope.cu:50).
  const int32_t* positions;
  const float* inv_freq;
  float2* rope;
  int half;
};

constexpr int kNormThreads = 256;

// One CTA per row; the rounding points are those of the single-sequence
// step (rmsnorm.cu:21-119): the sum of squares over the unrounded residual
// sums, the product from the bf16 residual, rounded to bf16.
template <int H, bool EMBED>
__global__ void __launch_bounds__(kNormThreads) norm_rows_kernel(const NormRowsArgs a) {
  constexpr int CH = H / 8;                                   // 8-element chunks
  constexpr int PER = (CH + kNormThreads - 1) / kNormThreads;  // per thread
  __shared__ float red[kNormThreads / 32];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();  // the residual stream comes from the preceding projection
  pdl_launch_next();
  const size_t row = static_cast<size_t>(b) * H;
  const bf16* src = a.x + row;
  if constexpr (EMBED) {
    if (a.rope != nullptr) {
      const float p = static_cast<float>(a.positions[b]);
      for (int i = tid; i < a.half; i += kNormThreads) {
        float sn, cs;
        sincosf(p * a.inv_freq[i], &sn, &cs);
        a.rope[static_cast<size_t>(b) * a.half + i] = make_float2(cs, sn);
      }
    }
    int tok = a.tokens[b];
    if (tok < 0 || tok >= a.vocab) {
      if (tid == 0 && a.status) atomicOr(a.status, kStatusBadToken);
      tok = 0;
    }
    src = a.embed + static_cast<size_t>(tok) * H;
  }
  uint4 raw[PER], gain[PER];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int c = tid + p * kNormThreads;
    if (c < CH) {
      raw[p] = ldg_cg16(src + c * 8);
      gain[p] = ldg16(a.gain + c * 8);
      float v[8];
      if constexpr (EMBED) {
        unpack8(raw[p], v);
        *reinterpret_cast<uint4*>(a.x + row + c * 8) = raw[p];
        *reinterpret_cast<float4*>(a.xsum + row + c * 8) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(a.xsum + row + c * 8 + 4) = make_float4(v[4], v[5], v[6], v[7]);
      } else {
        const float4 s0 = __ldcg(reinterpret_cast<const float4*>(a.xsum + row + c * 8));
        const float4 s1 = __ldcg(reinterpret_cast<const float4*>(a.xsum + row + c * 8 + 4));
        v[0] = s0.x; v[1] = s0.y; v[2] = s0.z; v[3] = s0.w;
        v[4] = s1.x; v[5] = s1.y; v[6] = s1.z; v[7] = s1.w;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) total += red[w];
  const float scale = rsqrtf(total / static_cast<float>(H) + a.eps);
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int c = tid + p * kNormThreads;
    if (c < CH) {
      float xv[8], gf[8];
      unpack8(raw[p], xv);
      unpack8(gain[p], gf);
      uint4 o;
      o.x = pack_bf2(__fmul_rn(__fmul_rn(xv[0], scale), gf[0]), __fmul_rn(__fmul_rn(xv[1], scale), gf[1]));
      o.y = pack_bf2(__fmul_rn(__fmul_rn(xv[2], scale), gf[2]), __fmul_rn(__fmul_rn(xv[3], scale), gf[3]));
      o.z = pack_bf2(__fmul_rn(__fmul_rn(xv[4], scale), gf[4]), __fmul_rn(__fmul_rn(xv[5], scale), gf[5]));
      o.w = pack_bf2(__fmul_rn(__fmul_rn(xv[6], scale), gf[6]), __fmul_rn(__fmul_rn(xv[7], scale), gf[7]));
      *reinterpret_cast<uint4*>(a.out + row + c * 8) = o;
    }
  }
}

// Prefill: the chunk's rotated K rows and V rows (from the QKV projection)
// into the sequence's pages at positions start .. start + count - 1, one CTA
// per position; CTAs past the chunk, up to the next multiple of 16, zero
// those slots, so that a 16-position unit read by attn_prefill_kernel holds
// finite values everywhere (decode overwrites them later).
struct KvWriteArgs {
  const bf16* qkv;
  int qkv_stride, q_dim, kv_dim, head_dim, kv_heads;
  bf16* kpool;  // this layer's pools
  bf16* vpool;
  const int32_t* table;
  int page_size, pool_pages;
  long long page_stride, head_stride;
  int start, count;
  int limit;  // positions the cache holds: padding rows at or past it are skipped
  uint32_t* status;
};

__global__ void __launch_bounds__(128) kv_write_kernel(const KvWriteArgs a) {
  pdl_wait();  // the rows come from the preceding projection
  pdl_launch_next();
  const int r = blockIdx.x;
  const int pos = a.start + r;
  if (pos >= a.limit) return;  // a padding row past the end of the cache
  int page = a.table[pos / a.page_size];
  if (page < 0 || page >= a.pool_pages) {
    if (threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusBadPage);
    return;
  }
  const int pieces = a.head_dim / 8;
  const long long base = static_cast<long long>(page) * a.page_stride +
                         static_cast<long long>(pos % a.page_size) * a.head_dim;
  for (int i = threadIdx.x; i < a.kv_heads * pieces; i += blockDim.x) {
    const int h = i / pieces, piece = i % pieces;
    uint4 k = make_uint4(0u, 0u, 0u, 0u), v = k;
    if (r < a.count) {
      const bf16* row = a.qkv + static_cast<size_t>(r) * a.qkv_stride + a.q_dim + h * a.head_dim + piece * 8;
      k = ldg_cg16(row);
      v = ldg_cg16(row + a.kv_dim);
    }
    const long long off = base + h * a.head_stride + piece * 8;
    *reinterpret_cast<uint4*>(a.kpool + off) = k;
    *reinterpret_cast<uint4*>(a.vpool + off) = v;
  }
}

// Seeded synthetic K/V for positions [0, length) of one sequence in every
// layer: each element is an approximately standard normal value (the sum of
// four hashed uniforms, centred and scaled), rounded to bf16, written at the
// sequence's pages. Stands in for the prompt's KV when a benchmark admits a
// sequence without running its prefill.
struct FillKvArgs {
  bf16* kpool;
  bf16* vpool;
  size_t layer_elems;
  int layers, kv_heads, head_dim, page_size, length;
  const int32_t* pages;  // the slot's device page table [max_pages]
  unsigned long long seed;
};

__device__ __forceinline__ uint32_t fill_hash(uint64_t x) {
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdull;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ull;
  x ^= x >> 33;
  return static_cast<uint32_t>(x);
}

__global__ void fill_kv_kernel(const FillKvArgs a) {
  const long long per_layer = static_cast<long long>(a.length) * a.kv_heads * a.head_dim;
  const long long total = per_layer * a.layers;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int layer = static_cast<int>(i / per_layer);
    long long r = i % per_layer;
    const int pos = static_cast<int>(r / (a.kv_heads * a.head_dim));
    r %= a.kv_heads * a.head_dim;
    const int head = static_cast<int>(r / a.head_dim), dim = static_cast<int>(r % a.head_dim);
    const size_t off = static_cast<size_t>(layer) * a.layer_elems +
                       (static_cast<size_t>(a.pages[pos / a.page_size]) * a.kv_heads + head) * a.page_size * a.head_dim +
                       static_cast<size_t>(pos % a.page_size) * a.head_dim + dim;
    const uint64_t key = a.seed ^ (static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull);
    float kv[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      float u = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) u += (fill_hash(key + 4 * t + j) >> 8) * (1.0f / 16777216.0f);
      kv[t] = (u - 2.0f) * 1.7320508f;
    }
    a.kpool[off] = __float2bfloat16_rn(kv[0]);
    a.vpool[off] = __float2bfloat16_rn(kv[1]);
  }
}

}  // namespace lcrb
