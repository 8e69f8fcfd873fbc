// Causal prefill attention of one prompt chunk over a sequence's paged KV on
// the tensor pipe: the flash-style replacement of the reference's chunked
// prefill attention (cublasGemmStridedBatchedEx QK^T and PV with a
// materialised [heads][chunk][max_seq] fp32 score buffer, causal_softmax_kernel,
// gather_kv, merge_heads: src/model.cu:509-560, src/kernels/attention.cu:42-100,
// 302-316, src/kernels/elementwise.cu:124-143).
//
// The chunk's rotated K/V rows are in the cache already (kv_write_kernel), so
// every key -- the cached prefix and the chunk itself -- comes from the pool.
// Grid (kv_heads, CTAs per KV head); each consumer warp owns one (query head,
// 16-query tile) pair of the KV head's group, four pairs per CTA, heaviest
// tiles first. The producer warp streams the keys 0 .. (last query of the
// CTA) in stages of four 16-position units: K and V as 128-byte-swizzled TMA
// boxes, the layout attn_batch_kernel reads (AbGeom). Per stage a warp
// computes S = Q K^T for the stage's 64 keys (m16n8k16, 16 queries x 8 keys
// per tile, bf16 operands, fp32 sums), the causal mask and one online-softmax
// update per query row in the log2 domain, then O += P V with P rounded to
// bf16 (l sums the unrounded weights); the output is O / l.
#pragma once

#include "attn_batch.cuh"

namespace lcrb {

struct PrefillAttnArgs {
  const bf16* qkv;       // [count][qkv_stride] rotated q, k and v rows of the chunk
  int qkv_stride, q_dim, kv_dim;
  const int32_t* table;  // the sequence's page table
  int page_size, pool_pages;
  int start, count;      // chunk rows are positions start .. start + count - 1
  float scale_log2;      // softmax scale * log2(e)
  bf16* out;             // [count][q_dim]
  uint32_t* status;
};

// m16n8k16 with all four A registers (16 live rows).
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four ring stages for head_dim 64 (three CTAs share an SM: the per-stage
// softmax of 64 keys needs more than the 96 registers a thread of four
// resident CTAs gets), two for head_dim 128.
template <int D>
constexpr int attn_prefill_stages() {
  return D == 64 ? 4 : 2;
}

template <int D>
constexpr size_t attn_prefill_smem_bytes() {
  return 1024 + static_cast<size_t>(attn_prefill_stages<D>()) * AbGeom<D>::STAGE + 2 * attn_prefill_stages<D>() * 8;
}

template <int D, int G>
__global__ void __launch_bounds__(kAttnThreads, D == 64 ? 3 : 2) attn_prefill_kernel(const PrefillAttnArgs a,
                                                                    const __grid_constant__ CUtensorMap kmap,
                                                                    const __grid_constant__ CUtensorMap vmap) {
  using Geo = AbGeom<D>;
  constexpr int STAGES = attn_prefill_stages<D>();
  constexpr int UNIT = Geo::UNIT;
  constexpr int KSTEPS = D / 16;
  constexpr int NT = D / 8;
  constexpr int W = kAttnConsumerWarps;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = align_smem<uint8_t>(smem_raw, 1024);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + STAGES * Geo::STAGE);
  uint64_t* empty = full + STAGES;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // KV heads vary fastest in the grid, so every head's heaviest tiles are
  // dispatched first.
  const int kvh = blockIdx.x, num_kv = gridDim.x;
  const int tiles = (a.count + 15) / 16;
  const int pairs = tiles * G;
  // This CTA's pairs 4 * blockIdx.y + w, taken from the last query tile down.
  const int p_first = W * static_cast<int>(blockIdx.y);
  const int qt_max = tiles - 1 - p_first / G;
  const int key_end = a.start + min(a.count, (qt_max + 1) * 16);  // keys 0 .. key_end - 1
  const int units = (key_end + kAbUnit - 1) / kAbUnit;
  const int nstages = (units + W - 1) / W;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == W) {
    // Producer: pages of 32 units at a time, one lookup per lane.
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    const uint64_t policy = l2_policy_evict_first();
    pdl_wait();
    int issued = 0;
    bool ok = true;
    int row_mine = 0;
    for (int st = 0; st < nstages; ++st) {
      const int u0 = st * W;
      if (u0 % 32 == 0 && u0 + lane < units) {
        const int p = (u0 + lane) * kAbUnit;
        int page = a.table[p / a.page_size];
        if (page < 0 || page >= a.pool_pages) {
          if (a.status) atomicOr(a.status, kStatusBadPage);
          page = 0;
        }
        row_mine = (page * num_kv + kvh) * a.page_size + p % a.page_size;
      }
      const int slot = st % STAGES;
      if (lane == 0 && st >= STAGES) {
        ok = mbar_wait(&empty[slot], ((st / STAGES) - 1) & 1, a.status, kStatusTimeoutEmpty);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const int cnt = min(W, units - u0);
      int rows[W];
#pragma unroll
      for (int u = 0; u < W; ++u) rows[u] = __shfl_sync(0xffffffffu, row_mine, (u0 + u) & 31);
      if (lane == 0) {
        uint8_t* dst = ring + slot * Geo::STAGE;
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(cnt) * 2 * UNIT);
#pragma unroll
        for (int u = 0; u < W; ++u) {
          if (u < cnt) {
            tma_load_3d(dst + u * UNIT, &kmap, 0, rows[u], 0, &full[slot], policy);
            tma_load_3d(dst + (W + u) * UNIT, &vmap, 0, rows[u], 0, &full[slot], policy);
          }
        }
      }
      issued = st + 1;
    }
    pdl_launch_next();
    if (lane == 0) {
      for (int st = issued > STAGES ? issued - STAGES : 0; st < issued; ++st) {
        mbar_wait(&full[st % STAGES], (st / STAGES) & 1, nullptr, 0);  // waits even after an abort
      }
    }
    return;
  }

  // Consumer warp: query head h, queries q0 .. q0 + 15 of the chunk.
  const int pair = p_first + warp;
  const bool live_pair = pair < pairs;
  const int qt = tiles - 1 - pair / G;
  const int h = kvh * G + pair % G;
  const int q0 = qt * 16;
  const int g = lane >> 2, t = lane & 3;
  const int lrow = lane & 7, mi = lane >> 3;
  const int k_row = (mi >> 1) * 8 + lrow;
  const int v_row = (mi & 1) * 8 + lrow;
  // Rows g and g + 8 of the tile: positions, and whether they exist.
  const int qa_row = q0 + g, qb_row = q0 + g + 8;
  const bool ra = live_pair && qa_row < a.count, rb = live_pair && qb_row < a.count;
  const int pos_a = a.start + qa_row, pos_b = a.start + qb_row;
  const int warp_last = live_pair ? a.start + min(a.count, q0 + 16) - 1 : -1;  // last key this warp needs

  pdl_wait();  // q comes from the preceding projection
  uint32_t qf[KSTEPS][4];
  {
    const bf16* qa_ptr = a.qkv + static_cast<size_t>(qa_row) * a.qkv_stride + h * D;
    const bf16* qb_ptr = a.qkv + static_cast<size_t>(qb_row) * a.qkv_stride + h * D;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      qf[kk][0] = ra ? *reinterpret_cast<const uint32_t*>(qa_ptr + 16 * kk + 2 * t) : 0u;
      qf[kk][1] = rb ? *reinterpret_cast<const uint32_t*>(qb_ptr + 16 * kk + 2 * t) : 0u;
      qf[kk][2] = ra ? *reinterpret_cast<const uint32_t*>(qa_ptr + 16 * kk + 8 + 2 * t) : 0u;
      qf[kk][3] = rb ? *reinterpret_cast<const uint32_t*>(qb_ptr + 16 * kk + 8 + 2 * t) : 0u;
    }
  }
  float o[NT][4];
#pragma unroll
  for (int nn = 0; nn < NT; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
  float m_a = kNegBig, m_b = kNegBig, l_a = 0.f, l_b = 0.f;

  for (int st = 0; st < nstages; ++st) {
    const int slot = st % STAGES;
    if (!mbar_wait(&full[slot], (st / STAGES) & 1, a.status, kStatusTimeoutFull)) break;
    const int u0 = st * W;
    const int kp0 = u0 * kAbUnit;
    // Units of this stage that hold a key this warp needs (warp-uniform);
    // the rest stay untouched: their bytes may be another stage's.
    const int live = warp_last < kp0 ? 0 : min(min(W, units - u0), (warp_last - kp0) / kAbUnit + 1);
    if (live > 0) {
      const uint32_t ks = smem_addr(ring + slot * Geo::STAGE);
      const uint32_t vs = ks + W * UNIT;
      // S = Q K^T over the stage's keys: eight independent accumulator
      // chains (unit u, 8-key half j), KSTEPS deep.
      float s[W][2][4];
#pragma unroll
      for (int u = 0; u < W; ++u) {
#pragma unroll
        for (int j = 0; j < 2; ++j) s[u][j][0] = s[u][j][1] = s[u][j][2] = s[u][j][3] = 0.f;
      }
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
        for (int u = 0; u < W; ++u) {
          if (u < live) {
            uint32_t kb[4];
            ldmatrix_x4(kb, ks + u * UNIT + ab_offset(k_row, 2 * kk + (mi & 1)));
            mma_16816(s[u][0], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], kb[0], kb[1]);
            mma_16816(s[u][1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], kb[2], kb[3]);
          }
        }
      }
      // Causal mask (only a stage that reaches past the tile's first query,
      // or holds units past the keys, needs one), then one online-softmax
      // update per query row for all the stage's keys: rows g (regs 0, 1)
      // and g + 8 (2, 3). Maxima are taken on the raw scores (the scale is
      // positive) and the scale is folded into the exponent's FMA; the
      // running maximum m is kept in the scaled log2 domain.
      if (kp0 + live * kAbUnit - 1 > a.start + q0 || live < W) {
        const int lim_a = pos_a - kp0 - 2 * t, lim_b = pos_b - kp0 - 2 * t;
#pragma unroll
        for (int u = 0; u < W; ++u) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int off = kAbUnit * u + 8 * j + e;
              if (u >= live || off > lim_a) s[u][j][e] = kNegBig;
              if (u >= live || off > lim_b) s[u][j][2 + e] = kNegBig;
            }
          }
        }
      }
      float ua[W], ub[W];
#pragma unroll
      for (int u = 0; u < W; ++u) {
        ua[u] = fmaxf(fmaxf(s[u][0][0], s[u][0][1]), fmaxf(s[u][1][0], s[u][1][1]));
        ub[u] = fmaxf(fmaxf(s[u][0][2], s[u][0][3]), fmaxf(s[u][1][2], s[u][1][3]));
      }
      static_assert(W == 4, "the stage maximum below is a tree over four units");
      float mxa = fmaxf(fmaxf(ua[0], ua[1]), fmaxf(ua[2], ua[3]));
      float mxb = fmaxf(fmaxf(ub[0], ub[1]), fmaxf(ub[2], ub[3]));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
      // (every row has an unmasked key 0 in the first stage, so m is finite
      // from there on and masked scores give exp2(-huge) = 0)
      const float na = fmaxf(m_a, mxa * a.scale_log2), nb = fmaxf(m_b, mxb * a.scale_log2);
      const float alpha_a = ex2_approx(m_a - na), alpha_b = ex2_approx(m_b - nb);
      uint32_t pf[W][4];
#pragma unroll
      for (int u = 0; u < W; ++u) {
        float pa[2][2], pb[2][2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            pa[j][e] = ex2_approx(fmaf(s[u][j][e], a.scale_log2, -na));
            pb[j][e] = ex2_approx(fmaf(s[u][j][2 + e], a.scale_log2, -nb));
          }
        }
        ua[u] = (pa[0][0] + pa[0][1]) + (pa[1][0] + pa[1][1]);
        ub[u] = (pb[0][0] + pb[0][1]) + (pb[1][0] + pb[1][1]);
        pf[u][0] = pack_bf2(pa[0][0], pa[0][1]);
        pf[u][1] = pack_bf2(pb[0][0], pb[0][1]);
        pf[u][2] = pack_bf2(pa[1][0], pa[1][1]);
        pf[u][3] = pack_bf2(pb[1][0], pb[1][1]);
      }
      l_a = fmaf(l_a, alpha_a, (ua[0] + ua[1]) + (ua[2] + ua[3]));
      l_b = fmaf(l_b, alpha_b, (ub[0] + ub[1]) + (ub[2] + ub[3]));
      m_a = na;
      m_b = nb;
      // Most stages leave every row's maximum where it was: skip the
      // rescale then (warp-uniform test).
      if (__any_sync(0xffffffffu, alpha_a != 1.0f || alpha_b != 1.0f)) {
#pragma unroll
        for (int nn = 0; nn < NT; ++nn) {
          o[nn][0] *= alpha_a;
          o[nn][1] *= alpha_a;
          o[nn][2] *= alpha_b;
          o[nn][3] *= alpha_b;
        }
      }
      // O += P V, one 16-key k-step per live unit.
#pragma unroll
      for (int u = 0; u < W; ++u) {
        if (u < live) {
#pragma unroll
          for (int c = 0; c < D / 16; ++c) {
            uint32_t vb[4];
            ldmatrix_x4_trans(vb, vs + u * UNIT + ab_offset(v_row, 2 * c + (mi >> 1)));
            mma_16816(o[2 * c], pf[u][0], pf[u][1], pf[u][2], pf[u][3], vb[0], vb[1]);
            mma_16816(o[2 * c + 1], pf[u][0], pf[u][1], pf[u][2], pf[u][3], vb[2], vb[3]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float ia = l_a > 0.f ? 1.0f / l_a : 0.f, ib = l_b > 0.f ? 1.0f / l_b : 0.f;
#pragma unroll
  for (int nn = 0; nn < NT; ++nn) {
    const int d = 8 * nn + 2 * t;
    if (ra) {
      *reinterpret_cast<uint32_t*>(a.out + static_cast<size_t>(qa_row) * a.q_dim + h * D + d) =
          pack_bf2(o[nn][0] * ia, o[nn][1] * ia);
    }
    if (rb) {
      *reinterpret_cast<uint32_t*>(a.out + static_cast<size_t>(qb_row) * a.q_dim + h * D + d) =
          pack_bf2(o[nn][2] * ib, o[nn][3] * ib);
    }
  }
}

}  // namespace lcrb
