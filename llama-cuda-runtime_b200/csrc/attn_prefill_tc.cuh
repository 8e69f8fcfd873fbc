// Causal prefill attention on the 5th-generation tensor cores (tcgen05),
// head_dim 64: the same maths as attn_prefill_kernel (which stays the path
// for head_dim 128), and the same replacement of the reference's chunked
// prefill attention (src/model.cu:509-560, src/kernels/attention.cu:42-100).
//
// A CTA owns 128 query rows of one KV head: QB = 128 / G queries x the G
// query heads of the group, row r = (head in group) * QB + query. Those rows
// are the M side of every MMA, so each of the 128 softmax threads owns one
// row of S and of O in TMEM (no shuffles). Per block of 64 keys (four
// 16-position units of the paged cache, copied by TMA as 128-byte-swizzled
// boxes, the layout of the decode kernels):
//
//   S_j = Q K_j^T            m128 n64 k16 x 4, Q and K K-major, into one of
//                            two TMEM buffers (S_{j+1} runs during softmax j)
//   softmax j                tcgen05.ld of the row, causal mask on the
//                            diagonal block only, online max / sum in the log2
//                            domain, P rounded to bf16 into a swizzled K-major
//                            shared-memory tile; when a row's maximum grew by
//                            more than 8 (log2), its O row is rescaled in
//                            TMEM (ld, scale, st)
//   O += P_j V_j             m128 n64 k16 per live unit, V read in place as an
//                            MN-major operand (its rows are keys)
//
// Warps: 0 TMA producer (one lane), 1 TMEM allocation + MMA issue (one lane),
// 2-5 softmax and epilogue (warp w owns TMEM lanes 32 * (w % 4) .. + 31).
// Every wait is bounded (status bit, then the CTA drains its copies and MMAs
// and frees TMEM before returning).
#pragma once

#include "attn_prefill.cuh"
#include "gemm_tc.cuh"

namespace lcrb {

constexpr int kApTcThreads = 192;
constexpr int kApTcStages = 4;
// Of the 8 groups of 8 exponentials per row and block, this many are
// computed by exp2_fma on the FMA and integer pipes instead of ex2.approx:
// the transcendental unit was the busiest pipe (61 % of its peak, the FMA
// pipe 9 %).
constexpr int kApTcFmaGroups = 2;

// 2^x for x <= 8 without the transcendental unit: Cody-Waite reduction
// x = n + f with n = round(x) (the 1.5 * 2^23 shift leaves n in the low
// mantissa bits of t), 2^f for |f| <= 1/2 by a degree-4 polynomial, and n
// added to the exponent field (modulo 2^9, which the 32-bit add carries out
// of). The coefficients were fitted here to 2^f on [-1/2, 1/2] by
// iteratively reweighted least squares on the relative error: at most
// 2.7e-6 relative in fp32, far inside the bf16 rounding of P. Below 2^-125
// it returns 0 (ex2.approx returns a value that is 0 after the MMA's scale).
__device__ __forceinline__ float exp2_fma(float x) {
  const float t = __fadd_rn(x, 12582912.0f);
  const float f = __fsub_rn(x, __fsub_rn(t, 12582912.0f));
  float p = 0.009569993242621422f;
  p = fmaf(p, f, 0.055917542427778244f);
  p = fmaf(p, f, 0.240247443318367f);
  p = fmaf(p, f, 0.6931218504905701f);
  p = fmaf(p, f, 0.9999992847442627f);
  const int bits = __float_as_int(p) + static_cast<int>(static_cast<unsigned>(__float_as_int(t)) << 23);
  return x < -125.0f ? 0.0f : __int_as_float(bits);
}

__device__ __forceinline__ void tc_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Generic-proxy shared-memory writes become visible to the tensor cores.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Descriptor of one V unit as the MN-major B operand of O += P V: 16 key rows
// of 128 bytes (64 head dimensions, the MN extent of one 128-byte swizzle
// atom), 8-row groups 1024 bytes apart. Both byte-offset fields hold 1024:
// with a single atom along MN only the 8-row-group stride is used.
__device__ __forceinline__ uint64_t ap_vdesc(uint32_t smem_addr) {
  return static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4) | (64ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

constexpr size_t attn_prefill_tc_smem_bytes() {
  return 32768 + static_cast<size_t>(kApTcStages) * AbGeom<64>::STAGE + (2 * kApTcStages + 9) * 8 + 16;
}

template <int G>
__global__ void __launch_bounds__(kApTcThreads, 2) attn_prefill_tc_kernel(const PrefillAttnArgs a,
                                                                          const __grid_constant__ CUtensorMap kmap,
                                                                          const __grid_constant__ CUtensorMap vmap) {
  constexpr int D = 64;
  constexpr int QB = 128 / G;  // queries per CTA
  using Geo = AbGeom<D>;
  constexpr int STAGES = kApTcStages;
  constexpr int UNIT = Geo::UNIT;  // 16 positions x 128 bytes
  static_assert(Geo::STAGE == 8 * UNIT, "a stage is four K units, then four V units");
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* qs = smem;           // Q tile: 128 rows x 128 bytes, K-major SW128
  uint8_t* ps = smem + 16384;   // P tile: 128 rows x 64 keys, K-major SW128
  uint8_t* ring = smem + 32768;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + STAGES * Geo::STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* q_ready = empty + STAGES;
  uint64_t* s_full = q_ready + 1;  // [2]
  uint64_t* s_free = s_full + 2;   // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 1;
  uint64_t* drain = pv_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.x, num_kv = gridDim.x;
  const int q0 = (static_cast<int>(gridDim.y) - 1 - static_cast<int>(blockIdx.y)) * QB;  // heaviest first
  const int key_end = a.start + min(a.count, q0 + QB);  // keys 0 .. key_end - 1
  const int units = (key_end + kAbUnit - 1) / kAbUnit;
  const int nblk = (units + 3) / 4;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(q_ready, 4);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool aligned = (smem_addr(smem) & 1023u) == 0;
  if (!aligned && tid == 0 && a.status) atomicOr(a.status, kStatusBadSmem | kStatusAbort);

  if (warp == 0) {
    if (aligned) {
      // Producer: block j is units 4j .. 4j + 3 (fewer at the end); lane i
      // looks up unit 4j + i's cache row, lane 0 issues the copies.
      if (lane == 0) {
        prefetch_tensormap(&kmap);
        prefetch_tensormap(&vmap);
      }
      const uint64_t policy = l2_policy_evict_first();
      pdl_wait();
      int issued = 0;
      int row = 0;  // lane i: cache row of unit 32 * (j / 8) + i
      for (int j = 0; j < nblk; ++j) {
        const int slot = j % STAGES;
        if (j % 8 == 0) {
          row = 0;
          if (4 * j + lane < units) {
            const int p = (4 * j + lane) * kAbUnit;
            int page = a.table[p / a.page_size];
            if (page < 0 || page >= a.pool_pages) {
              if (a.status) atomicOr(a.status, kStatusBadPage);
              page = 0;
            }
            row = (page * num_kv + kvh) * a.page_size + p % a.page_size;
          }
        }
        bool ok = true;
        if (lane == 0 && j >= STAGES) ok = mbar_wait(&empty[slot], ((j / STAGES) - 1) & 1, a.status, kStatusTimeoutEmpty);
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        int rows[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) rows[u] = __shfl_sync(0xffffffffu, row, 4 * (j % 8) + u);
        if (lane == 0) {
          const int cnt = min(4, units - 4 * j);
          uint8_t* dst = ring + slot * Geo::STAGE;
          mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(cnt) * 2 * UNIT);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (u < cnt) {
              tma_load_3d(dst + u * UNIT, &kmap, 0, rows[u], 0, &full[slot], policy);
              tma_load_3d(dst + (4 + u) * UNIT, &vmap, 0, rows[u], 0, &full[slot], policy);
            }
          }
        }
        issued = j + 1;
      }
      if (lane == 0) ring_drain<STAGES>(full, issued, a.status);
    }
  } else if (warp == 1) {
    if (lane == 0 && aligned) {
      const uint32_t idesc_s = tc_idesc<64>();
      const uint32_t idesc_pv = tc_idesc<64>() | (1u << 16);  // B (V) MN-major
      const uint64_t qdesc = tc_desc_sw128(smem_addr(qs));
      const uint64_t pdesc = tc_desc_sw128(smem_addr(ps));
      bool ok = mbar_wait(q_ready, 0, a.status, kStatusTimeoutFull);
      auto do_s = [&](int j) {
        const int slot = j % STAGES;
        if (!mbar_wait(&full[slot], (j / STAGES) & 1, a.status, kStatusTimeoutFull)) return false;
        if (j >= 2 && !mbar_wait(&s_free[j & 1], ((j >> 1) - 1) & 1, a.status, kStatusTimeoutEmpty)) return false;
        tc_fence_after();
        const uint64_t kdesc = tc_desc_sw128(smem_addr(ring + slot * Geo::STAGE));
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          tc_mma(tmem + static_cast<uint32_t>((j & 1) * 64), qdesc + 2 * k, kdesc + 2 * k, idesc_s, k > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[j & 1]);
        return true;
      };
      auto do_pv = [&](int j) {
        if (!mbar_wait(p_full, j & 1, a.status, kStatusTimeoutFull)) return false;
        tc_fence_after();
        const int slot = j % STAGES;
        const int live = min(4, units - 4 * j);
        const uint32_t vbase = smem_addr(ring + slot * Geo::STAGE + 4 * UNIT);
        for (int k = 0; k < live; ++k) {
          tc_mma(tmem + 128u, pdesc + 2 * k, ap_vdesc(vbase + k * UNIT), idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&empty[slot]);
        tc_commit(pv_done);
        return true;
      };
      for (int j = 0; j < nblk && ok; ++j) {
        ok = do_s(j);
        if (ok && j > 0) ok = do_pv(j - 1);
      }
      if (ok && nblk > 0) ok = do_pv(nblk - 1);
      if (!ok && a.status) atomicOr(a.status, kStatusAbort);
      pdl_launch_next();
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);  // the MMAs in flight land even after an abort
    }
  } else if (aligned) {
    // Softmax thread: row r of the tile = TMEM lane r.
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int hl = r / QB, qrow = q0 + r % QB;
    const bool exists = qrow < a.count;
    const int pos = a.start + qrow;
    const int h = kvh * G + hl;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    pdl_wait();  // q comes from the preceding projection
    {
      const uint4* src = reinterpret_cast<const uint4*>(a.qkv + static_cast<size_t>(qrow) * a.qkv_stride + h * D);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = exists ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(qs + r * 128 + ((c ^ (r & 7)) << 4)) = v;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_ready);
    float m = kNegBig, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1, a.status, kStatusTimeoutFull));
      if (!ok) break;
      tc_fence_after();
      float s[64];
#pragma unroll
      for (int c = 0; c < 64; c += 16) {
        float t16[16];
        tc_ld16(trow + static_cast<uint32_t>((j & 1) * 64 + c), t16);
#pragma unroll
        for (int e = 0; e < 16; ++e) s[c + e] = t16[e];
      }
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[j & 1]);
      const int kp0 = j * 64;
      const int live_keys = min(64, (units - 4 * j) * kAbUnit);
      // Mask keys past this row's position, and units that were not copied
      // (their bytes may be another block's): only the diagonal and last
      // blocks have any.
      if (kp0 + 63 > a.start + q0 || live_keys < 64) {
        const int lim = min(pos - kp0, live_keys - 1);
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          if (c > lim) s[c] = kNegBig;
        }
      }
      float mx[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        mx[g] = fmaxf(fmaxf(fmaxf(s[8 * g], s[8 * g + 1]), fmaxf(s[8 * g + 2], s[8 * g + 3])),
                      fmaxf(fmaxf(s[8 * g + 4], s[8 * g + 5]), fmaxf(s[8 * g + 6], s[8 * g + 7])));
      }
      const float rmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      // The running maximum moves only when the block's maximum exceeds it by
      // more than 8 (a factor of 256): P and l use the same stale maximum, so
      // O / l is unchanged, P stays <= 256, and the rescale of O in TMEM (a
      // round trip per 16 columns) is rare instead of nearly every block.
      // (Every row has an unmasked key 0 in the first block, so m is finite
      // from there on and masked scores give exp2(-huge) = 0.)
      const bool grow = rmax * a.scale_log2 > m + 8.0f;
      const float na = grow ? rmax * a.scale_log2 : m;
      const float alpha = ex2_approx(m - na);
      uint32_t pk[32];
      float sums[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float x = fmaf(s[8 * g + e], a.scale_log2, -na);
          p[e] = g >= 8 - kApTcFmaGroups ? exp2_fma(x) : ex2_approx(x);
        }
        sums[g] = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
#pragma unroll
        for (int e = 0; e < 4; ++e) pk[4 * g + e] = pack_bf2(p[2 * e], p[2 * e + 1]);
      }
      l = fmaf(l, alpha, ((sums[0] + sums[1]) + (sums[2] + sums[3])) + ((sums[4] + sums[5]) + (sums[6] + sums[7])));
      m = na;
      if (j > 0) {
        // O += P_{j-1} V_{j-1} is complete: P's tile is free, and O may be
        // rescaled.
        ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, a.status, kStatusTimeoutFull));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int c = 0; c < 64; c += 16) {
            float o16[16];
            tc_ld16(trow + static_cast<uint32_t>(128 + c), o16);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) o16[e] *= alpha;
            tc_st16(trow + static_cast<uint32_t>(128 + c), o16);
          }
          tc_wait_st();
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        *reinterpret_cast<uint4*>(ps + r * 128 + ((c ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && nblk > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (nblk - 1) & 1, a.status, kStatusTimeoutFull));
      if (ok) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(a.out + static_cast<size_t>(qrow) * a.q_dim + h * D);
#pragma unroll
        for (int c = 0; c < 64; c += 16) {
          float o16[16];
          tc_ld16(trow + static_cast<uint32_t>(128 + c), o16);
          tc_wait_ld();
          if (exists) {
            dst[c / 8] = make_uint4(pack_bf2(o16[0] * inv, o16[1] * inv), pack_bf2(o16[2] * inv, o16[3] * inv),
                                    pack_bf2(o16[4] * inv, o16[5] * inv), pack_bf2(o16[6] * inv, o16[7] * inv));
            dst[c / 8 + 1] =
                make_uint4(pack_bf2(o16[8] * inv, o16[9] * inv), pack_bf2(o16[10] * inv, o16[11] * inv),
                           pack_bf2(o16[12] * inv, o16[13] * inv), pack_bf2(o16[14] * inv, o16[15] * inv));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
  }
}

}  // namespace lcrb
