// Batched projection y[b][n] = sum_k x[b][k] w[n][k] on the 5th-generation
// tensor cores (tcgen05): the reference's gemm_nt (src/model.cu:38-45) at
// batch >= 16 -- batched decode and prefill chunks.
//
// A tile is 128 weight rows (the UMMA M side, operand A) x NB batch rows (the
// N side, operand B), accumulated in fp32 in TMEM. Both operands stream
// through a shared-memory ring in stages of CH 64-column K chunks: TMA tensor
// copies (make_kmajor_map, box {64, rows, CH}) land each chunk K-major with
// the 128-byte swizzle, which is the canonical SW128 K-major operand layout
// of tcgen05.mma (8-row groups 1024 bytes apart), chunk after chunk. Per
// chunk the MMA thread issues four m128 x nNB x k16 MMAs, advancing both
// descriptors by 32 bytes, and commits the stage's release to its empty
// barrier. Several chunks per copy give each weight row CH x 128 contiguous
// bytes per request, which the DRAM streams far better than 128-byte pieces
// 4 KB apart.
//
// Warps: 0 TMA producer (one lane), 1 TMEM allocation + MMA issue (one lane),
// 2-5 epilogue: each reads its 32 TMEM lanes (= 32 weight rows) with
// tcgen05.ld.32x32b, so the four epilogue warps cover the 128 rows.
//
// Split-K: with splits > 1 each CTA stores its partial tile in fp32
// workspace [split][row][tile column], and gemm_tc_reduce_kernel sums the
// splits in split order and applies the epilogue -- the result does not
// depend on which CTA finishes first.
// Every wait is bounded (status bit, then the CTA drains its copies and MMAs
// and frees TMEM before returning).
#pragma once

#include "common.cuh"
#include "gemv.cuh"  // GemvEpi, order_key

namespace lcrb {

constexpr int kTcTileM = 128;        // weight rows per tile
constexpr int kTcSlabK = 64;         // K columns per chunk (128-byte swizzle span)
constexpr int kTcThreads = 192;      // 6 warps
constexpr int kTcRingBytes = 196608; // ring budget (stage count derived from it)
// 128-row batch tiles with one chunk per stage (prefill chunks) take half of
// it, so that two CTAs share an SM and one's epilogue overlaps the other's
// main loop.
constexpr int kTcRingBytesPaired = 98304;

template <int NB, int CH>
struct TcGeom {
  static_assert(NB == 16 || NB == 32 || NB == 64 || NB == 128 || NB == 256, "batch tile");
  static constexpr int W_CHUNK = kTcTileM * kTcSlabK * 2;  // 16 KB
  static constexpr int X_CHUNK = NB * kTcSlabK * 2;
  static constexpr int W_BYTES = CH * W_CHUNK;
  static constexpr int X_BYTES = CH * X_CHUNK;
  static constexpr int STAGE = W_BYTES + X_BYTES;  // a multiple of 1024
  static constexpr int RING = (NB == 128 && CH == 1) ? kTcRingBytesPaired : kTcRingBytes;
  static constexpr int STAGES = (RING / STAGE) < 8 ? (RING / STAGE) : 8;
  static constexpr int TMEM_COLS = NB < 32 ? 32 : NB;  // power of two >= 32
  static_assert(STAGE % 1024 == 0 && STAGES >= 2, "stage geometry");
};

struct TcArgs {
  int n_out;        // weight rows (SWIGLU: F, outputs; the matrix has 2F rows)
  int K;
  int rows;         // batch rows of x
  int splits;       // K slabs are split over this many CTAs per tile
  int ldy;          // row stride of y / yf / resid (elements)
  bf16* y;          // STORE / SWIGLU
  float* yf;        // STORE_F32
  bf16* resid;      // RESID: resid = bf16(resid + bf16(out)), sums kept
  float* resid_sum;
  float* work;      // splits > 1: [splits][rows][tiles_n * 128] fp32 partials
  uint32_t* status;    // device status word, or nullptr
  // ROPE: columns [0, rope_cols) are heads of head_dim (a power of two <= 128)
  // rotated with rope[row][head_dim / 2] = (cos, sin) of the row's angles.
  const float2* rope;
  int head_dim;
  int rope_cols;
  // 128-row batch tiles without split-K: run gemm_tc_persist_kernel on this
  // many CTAs (at most one per tile); 0 launches one CTA per tile instead.
  int ctas;
  // RESID with splits > 1, optional: the RMSNorm of the updated residual rows
  // into norm_out (bf16 [rows][n_out]) with gain norm_gain, fused into the
  // reduction (gemm_tc_reduce_norm_kernel).
  const bf16* norm_gain;
  float norm_eps;
  bf16* norm_out;
};

// UMMA shared-memory descriptor of a K-major, 128-byte swizzled tile whose
// 8-row groups are 1024 bytes apart (start address in 16-byte units; version 1).
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t smem_addr) {
  return static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor: bf16 A and B, fp32 accumulator, both K-major,
// M = 128, N = NB.
template <int NB>
__device__ __forceinline__ uint32_t tc_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(NB >> 3) << 17) |
         (static_cast<uint32_t>(kTcTileM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// The rotation of one RoPE pair in fp32 with explicit roundings (no
// contraction into an FMA, which the compiler may or may not do depending on
// the surroundings), so every epilogue computes the same bits: dimension d <
// head_dim / 2 gives r cos - other sin, the upper half r cos + other sin.
__device__ __forceinline__ float rope_rot(float r, float other, float2 cs, bool lower) {
  const float rc = __fmul_rn(r, cs.x), os = __fmul_rn(other, cs.y);
  return lower ? __fsub_rn(rc, os) : __fadd_rn(rc, os);
}

// One output element of the epilogue: row n of the weights, batch row b.
// `up` is SWIGLU's up-projection value, or ROPE's rotation partner (column
// n ^ head_dim / 2).
template <int EPI>
__device__ __forceinline__ void tc_store(const TcArgs& a, int b, int n, float v, float up) {
  const size_t o = static_cast<size_t>(b) * a.ldy + n;
  if constexpr (EPI == EPI_STORE) {
    a.y[o] = __ushort_as_bfloat16(f2bf(v));
  } else if constexpr (EPI == EPI_STORE_F32) {
    a.yf[o] = v;
  } else if constexpr (EPI == EPI_RESID) {
    const float s = __fadd_rn(bf2f(__ldcg(reinterpret_cast<const unsigned short*>(a.resid) + o)), rbf(v));
    a.resid[o] = __ushort_as_bfloat16(f2bf(s));
    a.resid_sum[o] = s;
  } else if constexpr (EPI == EPI_SWIGLU) {
    const float g = rbf(v);
    const float silu = g / (1.0f + __expf(-g));
    a.y[o] = __ushort_as_bfloat16(f2bf(silu * rbf(up)));
  } else if constexpr (EPI == EPI_ROPE) {
    // The projection output is rounded to bf16, then rotated in fp32 and
    // rounded again (rope_write_kv_kernel, src/kernels/rope.cu:58-87).
    float r = rbf(v);
    if (n < a.rope_cols) {
      const int half = a.head_dim >> 1;
      const int d = n & (a.head_dim - 1);
      const float2 cs = a.rope[static_cast<size_t>(b) * half + (d & (half - 1))];
      const float other = rbf(up);
      r = rbf(rope_rot(r, other, cs, d < half));
    }
    a.y[o] = __ushort_as_bfloat16(f2bf(r));
  }
}

// Outputs n .. n + 7 of batch row b (fewer at the matrix edge): one 16-byte
// access per bf16 vector where the row is 16-byte aligned, else per element.
template <int EPI>
__device__ __forceinline__ void tc_store8(const TcArgs& a, int b, int n, const float (&v)[8], const float (&aux)[8]) {
  const size_t o = static_cast<size_t>(b) * a.ldy + n;
  const bool whole = n + 8 <= a.n_out;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if constexpr (EPI == EPI_STORE || EPI == EPI_SWIGLU || EPI == EPI_ROPE) {
    if (whole && al16(a.y + o)) {
      float r[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if constexpr (EPI == EPI_STORE) {
          r[e] = v[e];
        } else if constexpr (EPI == EPI_SWIGLU) {
          const float g = rbf(v[e]);
          r[e] = (g / (1.0f + __expf(-g))) * rbf(aux[e]);
        } else {
          r[e] = rbf(v[e]);
          if (n + e < a.rope_cols) {
            const int half = a.head_dim >> 1;
            const int d = (n + e) & (a.head_dim - 1);
            const float2 cs = a.rope[static_cast<size_t>(b) * half + (d & (half - 1))];
            const float other = rbf(aux[e]);
            r[e] = rope_rot(r[e], other, cs, d < half);
          }
        }
      }
      uint4 w;
      w.x = pack_bf2(r[0], r[1]);
      w.y = pack_bf2(r[2], r[3]);
      w.z = pack_bf2(r[4], r[5]);
      w.w = pack_bf2(r[6], r[7]);
      *reinterpret_cast<uint4*>(a.y + o) = w;
      return;
    }
  } else if constexpr (EPI == EPI_STORE_F32) {
    if (whole && al16(a.yf + o)) {
      *reinterpret_cast<float4*>(a.yf + o) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(a.yf + o + 4) = make_float4(v[4], v[5], v[6], v[7]);
      return;
    }
  } else if constexpr (EPI == EPI_RESID) {
    if (whole && al16(a.resid + o) && al16(a.resid_sum + o)) {
      float x[8], s8[8];
      unpack8(ldg_cg16(a.resid + o), x);
#pragma unroll
      for (int e = 0; e < 8; ++e) s8[e] = __fadd_rn(x[e], rbf(v[e]));
      uint4 w;
      w.x = pack_bf2(s8[0], s8[1]);
      w.y = pack_bf2(s8[2], s8[3]);
      w.z = pack_bf2(s8[4], s8[5]);
      w.w = pack_bf2(s8[6], s8[7]);
      *reinterpret_cast<uint4*>(a.resid + o) = w;
      *reinterpret_cast<float4*>(a.resid_sum + o) = make_float4(s8[0], s8[1], s8[2], s8[3]);
      *reinterpret_cast<float4*>(a.resid_sum + o + 4) = make_float4(s8[4], s8[5], s8[6], s8[7]);
      return;
    }
  }
  for (int e = 0; e < 8 && n + e < a.n_out; ++e) tc_store<EPI>(a, b, n + e, v[e], aux[e]);
}

template <int NB, int EPI, int CH>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const TcArgs a, const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap) {
  using G = TcGeom<NB, CH>;
  constexpr bool SWIGLU = EPI == EPI_SWIGLU;
  constexpr int STAGES = G::STAGES;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * G::STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* drain = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles_n = SWIGLU ? (a.n_out + 63) / 64 : (a.n_out + kTcTileM - 1) / kTcTileM;
  // Batch tiles vary fastest: the CTAs of one weight tile run side by side,
  // so each weight tile leaves DRAM once however many batch tiles there are.
  const int tiles_b = (a.rows + NB - 1) / NB;
  const int tile = blockIdx.x / tiles_b;
  const int tile_b = blockIdx.x % tiles_b;
  const int split = blockIdx.y;
  const int slabs = a.K / (kTcSlabK * CH);  // ring stages over K
  const int s0 = static_cast<int>(static_cast<long long>(split) * slabs / a.splits);
  const int s1 = static_cast<int>(static_cast<long long>(split + 1) * slabs / a.splits);
  const int n0 = SWIGLU ? tile * 64 : tile * kTcTileM;
  const int b0 = tile_b * NB;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(G::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool aligned = (smem_addr(ring) & 1023u) == 0;

  if (warp == 0) {
    if (lane == 0 && aligned) {
      const uint64_t policy = l2_policy_evict_first();
      // Each weight tile walks its K range from its own starting stage, so
      // CTAs of neighbouring weight tiles read different slabs of x (not the
      // same L2 lines at once); the accumulation order is fixed per weight
      // tile, whatever the batch tiling.
      const int span = s1 - s0;
      const int rot = span > 0 ? tile % span : 0;
      auto k_stage = [&](int q) { return s0 + (q + rot < span ? q + rot : q + rot - span); };
      auto load_w = [&](int q, uint8_t* st, uint64_t* bar) {
        if constexpr (SWIGLU) {
          tma_load_4d(st, &wmap, 0, n0, 0, k_stage(q) * CH, bar, policy);
        } else {
          tma_load_3d(st, &wmap, 0, n0, k_stage(q) * CH, bar, policy);
        }
      };
      // The weights do not depend on the preceding kernel: the first ring's
      // worth streams before the wait for its output (x).
      const int pre = span < STAGES ? span : STAGES;
      for (int q = 0; q < pre; ++q) {
        mbar_arrive_expect_tx(&full[q], G::STAGE);
        load_w(q, ring + q * G::STAGE, &full[q]);
      }
      pdl_wait();
      for (int q = 0; q < pre; ++q) {
        tma_load_3d(ring + q * G::STAGE + G::W_BYTES, &xmap, 0, b0, k_stage(q) * CH, &full[q], policy);
      }
      int it = pre;
      for (int q = pre; q < span; ++q, ++it) {
        const int slot = it % STAGES;
        if (!mbar_wait(&empty[slot], ((it / STAGES) - 1) & 1, a.status, kStatusTimeoutEmpty)) break;
        uint8_t* st = ring + slot * G::STAGE;
        mbar_arrive_expect_tx(&full[slot], G::STAGE);
        load_w(q, st, &full[slot]);
        tma_load_3d(st + G::W_BYTES, &xmap, 0, b0, k_stage(q) * CH, &full[slot], policy);
      }
      ring_drain<STAGES>(full, it, a.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc_idesc<NB>();
      int it = 0;
      bool ok = aligned;
      for (int s = s0; s < s1 && ok; ++s, ++it) {
        const int slot = it % STAGES;
        if (!mbar_wait(&full[slot], (it / STAGES) & 1, a.status, kStatusTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_addr(ring + slot * G::STAGE);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const uint64_t adesc = tc_desc_sw128(st + c * G::W_CHUNK);
          const uint64_t bdesc = tc_desc_sw128(st + G::W_BYTES + c * G::X_CHUNK);
#pragma unroll
          for (int k = 0; k < kTcSlabK / 16; ++k) {
            // +32 bytes per 16 columns inside the 128-byte swizzle span
            tc_mma(tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (it > 0 || c > 0 || k > 0) ? 1u : 0u);
          }
        }
        tc_commit(&empty[slot]);
      }
      // Accumulator complete (or abandoned): the next kernel may start
      // launching; release the epilogue, and make sure no MMA is still
      // running before TMEM is freed.
      pdl_launch_next();
      tc_commit(acc_full);
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);  // the MMAs in flight land even after an abort
      if (!ok && a.status) atomicOr(a.status, kStatusAbort);
    }
  } else {
    // Epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 = tile rows.
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // tile row 0..127
    pdl_wait();  // the residual stream and RoPE table come from earlier kernels
    // (status is optional: the per-kernel entry points may pass none)
    const bool mine = mbar_wait(acc_full, 0, a.status, kStatusTimeoutFull) &&
                      !(a.status != nullptr && (__ldcg(a.status) & kStatusAbort));
    // One decision for all 128 epilogue threads (the branches below hold
    // 128-thread barriers).
    const bool have = !named_sync_or(2, 128, !mine);
    tc_fence_after();
    float v[NB];
    if (have) {
#pragma unroll
      for (int c = 0; c < NB; c += 16) {
        float t[16];
        tc_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + c, t);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[c + i] = t[i];
      }
      tc_wait_ld();
    }
    if (have && a.splits > 1) {
      // This CTA's partial; gemm_tc_reduce_kernel finishes the tile.
      const size_t m_total = static_cast<size_t>(tiles_n) * kTcTileM;
      float* part = a.work + static_cast<size_t>(split) * a.rows * m_total + static_cast<size_t>(tile) * kTcTileM + row;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b0 + b < a.rows) part[static_cast<size_t>(b0 + b) * m_total] = v[b];
      }
    }
    if (have && a.splits == 1) {
      // Transpose the tile through the idle ring (rows padded to NB + 1
      // floats), then each thread finishes 8 consecutive outputs of one
      // batch row at a time: vector loads and stores, and every epilogue
      // warp shares the work (SWIGLU: rows 0-63 gate, 64-127 up; ROPE: the
      // partner of tile row r is r ^ head_dim / 2).
      float* T = reinterpret_cast<float*>(ring);
#pragma unroll
      for (int b = 0; b < NB; ++b) T[row * (NB + 1) + b] = v[b];
      named_sync(2, 128);
      constexpr int NOUT = SWIGLU ? 64 : kTcTileM;
      for (int c = tid - 64; c < (NOUT / 8) * NB; c += 128) {
        const int n8 = c / NB, b = c % NB;
        const int nl = n8 * 8;
        if (b0 + b >= a.rows || n0 + nl >= a.n_out) continue;
        float val[8], aux[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          val[e] = T[(nl + e) * (NB + 1) + b];
          if constexpr (SWIGLU) {
            aux[e] = T[(64 + nl + e) * (NB + 1) + b];
          } else if constexpr (EPI == EPI_ROPE) {
            aux[e] = T[((nl + e) ^ (a.head_dim >> 1)) * (NB + 1) + b];
          } else {
            aux[e] = 0.f;
          }
        }
        tc_store8<EPI>(a, b0 + b, n0 + nl, val, aux);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::TMEM_COLS) : "memory");
  }
}

// Split-K epilogue: y[b][n] = EPI(sum over splits, in split order, of the
// partials). SWIGLU output n takes gate column (n / 64) * 128 + n % 64 and the
// up column 64 after it (the tile layout of gemm_tc_kernel).
template <int EPI>
__global__ void __launch_bounds__(256) gemm_tc_reduce_kernel(const TcArgs a) {
  const int tiles_n = EPI == EPI_SWIGLU ? (a.n_out + 63) / 64 : (a.n_out + kTcTileM - 1) / kTcTileM;
  const size_t m_total = static_cast<size_t>(tiles_n) * kTcTileM;
  const size_t plane = static_cast<size_t>(a.rows) * m_total;
  const size_t total = static_cast<size_t>(a.rows) * a.n_out;
  pdl_wait();
  pdl_launch_next();
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / a.n_out), n = static_cast<int>(i % a.n_out);
    const size_t col = EPI == EPI_SWIGLU ? static_cast<size_t>(n / 64) * kTcTileM + n % 64 : n;
    const float* src = a.work + static_cast<size_t>(b) * m_total + col;
    float v = 0.f, up = 0.f;
    for (int sp = 0; sp < a.splits; ++sp) {
      v = __fadd_rn(v, __ldcg(src + sp * plane));
      if constexpr (EPI == EPI_SWIGLU) up = __fadd_rn(up, __ldcg(src + sp * plane + 64));
    }
    if constexpr (EPI == EPI_ROPE) {
      if (n < a.rope_cols) {  // the partner's sum, in the same order
        const float* par = a.work + static_cast<size_t>(b) * m_total + (n ^ (a.head_dim >> 1));
        for (int sp = 0; sp < a.splits; ++sp) up = __fadd_rn(up, __ldcg(par + sp * plane));
      }
    }
    tc_store<EPI>(a, b, n, v, up);
  }
}

// Split-K residual epilogue fused with the RMSNorm that follows it: one CTA
// of 256 threads per batch row, thread t owning 8-column chunks t, t + 256,
// .. as norm_rows_kernel does. Per chunk: the split sum in split order (as
// gemm_tc_reduce_kernel), s = resid + bf16(sum), stored as bf16 and as the
// unrounded fp32 sum; then the sum of squares of the fp32 sums over the same
// tree as norm_rows_kernel, and out = bf16(bf16(s) * scale * gain) --
// bit-identical to the two launches it replaces.
template <int H>
__global__ void __launch_bounds__(256) gemm_tc_reduce_norm_kernel(const TcArgs a) {
  constexpr int CHUNKS = H / 8;
  constexpr int PER = (CHUNKS + 255) / 256;
  __shared__ float red[8];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  pdl_launch_next();
  const size_t plane = static_cast<size_t>(a.rows) * H;  // m_total = H for RESID
  const size_t row = static_cast<size_t>(b) * H;
  float xs[PER][8];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int c = tid + p * 256;
    if (c < CHUNKS) {
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int sp = 0; sp < a.splits; ++sp) {
        const float* src = a.work + sp * plane + row + c * 8;
        const float4 lo = __ldcg(reinterpret_cast<const float4*>(src));
        const float4 hi = __ldcg(reinterpret_cast<const float4*>(src + 4));
        v[0] = __fadd_rn(v[0], lo.x); v[1] = __fadd_rn(v[1], lo.y);
        v[2] = __fadd_rn(v[2], lo.z); v[3] = __fadd_rn(v[3], lo.w);
        v[4] = __fadd_rn(v[4], hi.x); v[5] = __fadd_rn(v[5], hi.y);
        v[6] = __fadd_rn(v[6], hi.z); v[7] = __fadd_rn(v[7], hi.w);
      }
      float x[8];
      unpack8(ldg_cg16(a.resid + row + c * 8), x);
      float s8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) s8[e] = __fadd_rn(x[e], rbf(v[e]));
      uint4 w;
      w.x = pack_bf2(s8[0], s8[1]);
      w.y = pack_bf2(s8[2], s8[3]);
      w.z = pack_bf2(s8[4], s8[5]);
      w.w = pack_bf2(s8[6], s8[7]);
      *reinterpret_cast<uint4*>(a.resid + row + c * 8) = w;
      *reinterpret_cast<float4*>(a.resid_sum + row + c * 8) = make_float4(s8[0], s8[1], s8[2], s8[3]);
      *reinterpret_cast<float4*>(a.resid_sum + row + c * 8 + 4) = make_float4(s8[4], s8[5], s8[6], s8[7]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ss = fmaf(s8[e], s8[e], ss);
        xs[p][e] = rbf(s8[e]);
      }
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) total += red[w];
  const float scale = rsqrtf(total / static_cast<float>(H) + a.norm_eps);
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int c = tid + p * 256;
    if (c < CHUNKS) {
      float gf[8];
      unpack8(ldg16(a.norm_gain + c * 8), gf);
      uint4 o;
      o.x = pack_bf2(__fmul_rn(__fmul_rn(xs[p][0], scale), gf[0]), __fmul_rn(__fmul_rn(xs[p][1], scale), gf[1]));
      o.y = pack_bf2(__fmul_rn(__fmul_rn(xs[p][2], scale), gf[2]), __fmul_rn(__fmul_rn(xs[p][3], scale), gf[3]));
      o.z = pack_bf2(__fmul_rn(__fmul_rn(xs[p][4], scale), gf[4]), __fmul_rn(__fmul_rn(xs[p][5], scale), gf[5]));
      o.w = pack_bf2(__fmul_rn(__fmul_rn(xs[p][6], scale), gf[6]), __fmul_rn(__fmul_rn(xs[p][7], scale), gf[7]));
      *reinterpret_cast<uint4*>(a.norm_out + row + c * 8) = o;
    }
  }
}

// Persistent form for prefill chunks (128- or 256-row batch tiles, no
// split-K). One CTA per SM walks the tiles blockIdx.x, blockIdx.x +
// gridDim.x, ... (batch tiles fastest, as in gemm_tc_kernel); the producer
// streams their stages through one ring without a break, the MMA thread
// alternates between two TMEM accumulators, and the epilogue of one tile runs
// while the next tile's MMAs do. The epilogue reads the accumulator in
// 64-column passes (batch rows), each transposed through a padded staging
// buffer T[batch row][tile row], so that a thread finishes 8 consecutive
// outputs of one batch row and a warp's stores cover whole rows. Per tile the
// K order (rotated by the weight tile's index) and the accumulation are those
// of gemm_tc_kernel<128, EPI, 1>, so the outputs do not depend on the tile
// size or on the kernel.
//
// Why 256-row tiles: an m128 x n x k16 MMA reads (128 + n) x 32 bytes of
// operands from shared memory and the ring is written with as many, so at
// n = 128 an SM moves 16 KB per 64-clock MMA -- twice what its shared memory
// delivers at the tensor pipe's full rate; n = 256 moves 24 KB per 128 clocks.
constexpr int kTcpHalf = 64;                  // batch rows per epilogue pass
constexpr int kTcpPitch = kTcTileM + 4;       // staging row pitch (floats)
constexpr int kTcpStaging = kTcpHalf * kTcpPitch * 4;
// Staging column of tile row r: r with bit 2 flipped where bit 5 is set, so
// the eight 32-byte row pieces that eight lanes read at once (m = 0, 8, .., 56)
// start in eight different 4-bank groups; a warp's writes (32 consecutive
// rows) stay a permutation of 32 consecutive words.
__device__ __forceinline__ int tcp_swz(int r) { return r ^ (((r >> 5) & 1) << 2); }
// Tile rows m .. m + 7 (m a multiple of 8) of one staging row.
__device__ __forceinline__ void tcp_ld8(const float* tr, int m, float* out) {
  const int f = ((m >> 5) & 1) << 2;
  *reinterpret_cast<float4*>(out) = *reinterpret_cast<const float4*>(tr + (m ^ f));
  *reinterpret_cast<float4*>(out + 4) = *reinterpret_cast<const float4*>(tr + ((m + 4) ^ f));
}

template <int NB>
constexpr int tcp_stages() {
  return NB == 128 ? 6 : 4;  // 192 KB of ring either way
}

template <int NB, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_persist_kernel(const TcArgs a,
                                                                        const __grid_constant__ CUtensorMap wmap,
                                                                        const __grid_constant__ CUtensorMap xmap) {
  static_assert(NB == 128 || NB == 256, "persistent batch tile");
  using G = TcGeom<NB, 1>;
  constexpr int STAGES = tcp_stages<NB>();
  constexpr bool SWIGLU = EPI == EPI_SWIGLU;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  float* T = reinterpret_cast<float*>(smem + STAGES * G::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * G::STAGE + kTcpStaging);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles_n = SWIGLU ? (a.n_out + 63) / 64 : (a.n_out + kTcTileM - 1) / kTcTileM;
  const int tiles_b = (a.rows + NB - 1) / NB;
  const int tiles = tiles_n * tiles_b;
  const int span = a.K / kTcSlabK;
  const int first = static_cast<int>(blockIdx.x), stride = static_cast<int>(gridDim.x);
  const int mine = tiles > first ? (tiles - 1 - first) / stride + 1 : 0;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(2 * NB)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool aligned = (smem_addr(ring) & 1023u) == 0;

  if (warp == 0) {
    if (lane == 0 && aligned) {
      const uint64_t policy = l2_policy_evict_first();
      // Stage q of tile t: weight rows of tile t / tiles_b, batch rows of
      // tile t % tiles_b, K slab (q + t / tiles_b) mod span.
      auto slab = [&](int t, int q) { return (q + (t / tiles_b) % span) % span; };
      auto load_w = [&](int t, int q, uint8_t* st, uint64_t* bar) {
        const int tile = t / tiles_b;
        if constexpr (SWIGLU) {
          tma_load_4d(st, &wmap, 0, tile * 64, 0, slab(t, q), bar, policy);
        } else {
          tma_load_3d(st, &wmap, 0, tile * kTcTileM, slab(t, q), bar, policy);
        }
      };
      auto load_x = [&](int t, int q, uint8_t* st, uint64_t* bar) {
        tma_load_3d(st + G::W_BYTES, &xmap, 0, (t % tiles_b) * NB, slab(t, q), bar, policy);
      };
      // The weights do not depend on the preceding kernel: the first ring's
      // worth streams before the wait for its output (x).
      const int pre = mine > 0 ? (span < STAGES ? span : STAGES) : 0;
      for (int q = 0; q < pre; ++q) {
        mbar_arrive_expect_tx(&full[q], G::STAGE);
        load_w(first, q, ring + q * G::STAGE, &full[q]);
      }
      pdl_wait();
      for (int q = 0; q < pre; ++q) load_x(first, q, ring + q * G::STAGE, &full[q]);
      int it = pre;
      bool ok = true;
      for (int i = 0; i < mine && ok; ++i) {
        const int t = first + i * stride;
        for (int q = i == 0 ? pre : 0; q < span; ++q, ++it) {
          const int slot = it % STAGES;
          if (!mbar_wait(&empty[slot], ((it / STAGES) - 1) & 1, a.status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* st = ring + slot * G::STAGE;
          mbar_arrive_expect_tx(&full[slot], G::STAGE);
          load_w(t, q, st, &full[slot]);
          load_x(t, q, st, &full[slot]);
        }
      }
      ring_drain<STAGES>(full, it, a.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc_idesc<NB>();
      int it = 0;
      bool ok = aligned;
      for (int i = 0; i < mine && ok; ++i) {
        const int buf = i & 1;
        // The epilogue has finished with this accumulator's previous tile.
        if (i >= 2 && !mbar_wait(&acc_empty[buf], ((i >> 1) - 1) & 1, a.status, kStatusTimeoutEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * NB);
        for (int q = 0; q < span; ++q, ++it) {
          const int slot = it % STAGES;
          if (!mbar_wait(&full[slot], (it / STAGES) & 1, a.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_addr(ring + slot * G::STAGE);
          const uint64_t adesc = tc_desc_sw128(st);
          const uint64_t bdesc = tc_desc_sw128(st + G::W_BYTES);
#pragma unroll
          for (int k = 0; k < kTcSlabK / 16; ++k) {
            tc_mma(d, adesc + 2 * k, bdesc + 2 * k, idesc, (q > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[slot]);
        }
        if (!ok && a.status) atomicOr(a.status, kStatusAbort);
        // Accumulator complete (or abandoned: the epilogue sees the abort).
        tc_commit(&acc_full[buf]);
      }
      pdl_launch_next();
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);  // the MMAs in flight land even after an abort
      if (!ok && a.status) atomicOr(a.status, kStatusAbort);
    }
  } else {
    // Epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 = tile rows.
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // tile row 0..127
    const int et = tid - 64;           // 0..127
    constexpr int NOUT = SWIGLU ? 64 : kTcTileM;
    constexpr int N8 = NOUT / 8;
    pdl_wait();  // the residual stream and RoPE table come from earlier kernels
    for (int i = 0; i < mine; ++i) {
      const int buf = i & 1;
      const int t = first + i * stride;
      const int n0 = SWIGLU ? (t / tiles_b) * 64 : (t / tiles_b) * kTcTileM;
      const int b0 = (t % tiles_b) * NB;
      const bool got = mbar_wait(&acc_full[buf], (i >> 1) & 1, a.status, kStatusTimeoutFull) &&
                       !(a.status != nullptr && (__ldcg(a.status) & kStatusAbort));
      // One decision for all 128 epilogue threads (the loop holds 128-thread
      // barriers).
      if (named_sync_or(2, 128, !got)) break;
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < NB / kTcpHalf; ++h) {
        float v[kTcpHalf];
#pragma unroll
        for (int c = 0; c < kTcpHalf; c += 16) {
          float t16[16];
          tc_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(buf * NB + h * kTcpHalf + c),
                  t16);
#pragma unroll
          for (int e = 0; e < 16; ++e) v[c + e] = t16[e];
        }
        tc_wait_ld();
        if (h == NB / kTcpHalf - 1) {
          // This warp is done with the accumulator: the MMA thread may reuse it.
          tc_fence_before();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
#pragma unroll
        for (int bb = 0; bb < kTcpHalf; ++bb) T[bb * kTcpPitch + tcp_swz(row)] = v[bb];
        named_sync(2, 128);
        // Item c: outputs 8 * (c % N8) .. + 7 of batch row c / N8 of the half
        // (SWIGLU: gate rows 0-63, up rows 64-127; ROPE: the partner of tile
        // row r is r ^ head_dim / 2). The global inputs of a group of items
        // (RESID: the residual rows; ROPE: the rows' angles) are loaded before
        // any of the group is stored: the stores may alias them as far as the
        // compiler knows, so a load inside the store loop would wait out a
        // whole memory latency per item.
        constexpr int ITEMS = N8 * kTcpHalf / 128;
        constexpr int GROUP = EPI == EPI_ROPE ? 4 : ITEMS;
        constexpr int PRE = EPI == EPI_ROPE ? 4 : 1;  // 16-byte inputs per item
        static_assert(ITEMS * 128 == N8 * kTcpHalf && ITEMS % GROUP == 0, "epilogue items");
#pragma unroll
        for (int g0 = 0; g0 < ITEMS; g0 += GROUP) {
          uint4 pre[GROUP][PRE];
          bool fast[GROUP];
#pragma unroll
          for (int j = 0; j < GROUP; ++j) {
            const int c = et + 128 * (g0 + j);
            const int n = n0 + (c % N8) * 8, brow = b0 + h * kTcpHalf + c / N8;
            const size_t o = static_cast<size_t>(brow) * a.ldy + n;
            const bool live = brow < a.rows && n + 8 <= a.n_out;
            fast[j] = false;
            if constexpr (EPI == EPI_RESID) {
              fast[j] = live && ((reinterpret_cast<uintptr_t>(a.resid + o) | reinterpret_cast<uintptr_t>(a.resid_sum + o)) &
                                 15u) == 0;
              if (fast[j]) pre[j][0] = ldg_cg16(a.resid + o);
            } else if constexpr (EPI == EPI_ROPE) {
              // 8 consecutive outputs of one rotated head: angles d .. d + 7
              // of the half the head's dimension d falls in.
              fast[j] = live && n + 8 <= a.rope_cols && (reinterpret_cast<uintptr_t>(a.y + o) & 15u) == 0;
              if (fast[j]) {
                const int half = a.head_dim >> 1;
                const uint4* cs = reinterpret_cast<const uint4*>(a.rope + static_cast<size_t>(brow) * half +
                                                                 (n & (half - 1)));
#pragma unroll
                for (int q = 0; q < 4; ++q) pre[j][q] = ldg_cg16(cs + q);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < GROUP; ++j) {
            const int c = et + 128 * (g0 + j);
            const int nl = (c % N8) * 8, bb = c / N8;
            const int brow = b0 + h * kTcpHalf + bb;
            if (brow >= a.rows || n0 + nl >= a.n_out) continue;
            const float* tr = T + bb * kTcpPitch;
            float val[8], aux[8];
            tcp_ld8(tr, nl, val);
            if constexpr (SWIGLU) {
              tcp_ld8(tr, 64 + nl, aux);
            } else if constexpr (EPI == EPI_ROPE) {
              const int pn = nl ^ (a.head_dim >> 1);  // 8-aligned: the partners of nl .. nl + 7 are pn .. pn + 7
              tcp_ld8(tr, pn, aux);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) aux[e] = 0.f;
            }
            const size_t o = static_cast<size_t>(brow) * a.ldy + n0 + nl;
            if constexpr (EPI == EPI_RESID) {
              if (fast[j]) {
                // tc_store8's residual update with the row loaded above
                float x[8], s8[8];
                unpack8(pre[j][0], x);
#pragma unroll
                for (int e = 0; e < 8; ++e) s8[e] = __fadd_rn(x[e], rbf(val[e]));
                uint4 w;
                w.x = pack_bf2(s8[0], s8[1]);
                w.y = pack_bf2(s8[2], s8[3]);
                w.z = pack_bf2(s8[4], s8[5]);
                w.w = pack_bf2(s8[6], s8[7]);
                *reinterpret_cast<uint4*>(a.resid + o) = w;
                *reinterpret_cast<float4*>(a.resid_sum + o) = make_float4(s8[0], s8[1], s8[2], s8[3]);
                *reinterpret_cast<float4*>(a.resid_sum + o + 4) = make_float4(s8[4], s8[5], s8[6], s8[7]);
                continue;
              }
            } else if constexpr (EPI == EPI_ROPE) {
              if (fast[j]) {
                // tc_store8's rotation with the angles loaded above
                const float2* cs = reinterpret_cast<const float2*>(pre[j]);
                const int half = a.head_dim >> 1;
                float r[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  r[e] = rbf(val[e]);
                  const int d = (n0 + nl + e) & (a.head_dim - 1);
                  const float other = rbf(aux[e]);
                  r[e] = rope_rot(r[e], other, cs[e], d < half);
                }
                uint4 w;
                w.x = pack_bf2(r[0], r[1]);
                w.y = pack_bf2(r[2], r[3]);
                w.z = pack_bf2(r[4], r[5]);
                w.w = pack_bf2(r[6], r[7]);
                *reinterpret_cast<uint4*>(a.y + o) = w;
                continue;
              }
            }
            tc_store8<EPI>(a, brow, n0 + nl, val, aux);
          }
        }
        named_sync(2, 128);  // T is read before the next half or tile overwrites it
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * NB) : "memory");
  }
}

template <int NB>
constexpr size_t gemm_tc_persist_smem_bytes() {
  return static_cast<size_t>(tcp_stages<NB>()) * TcGeom<NB, 1>::STAGE + kTcpStaging + (2 * tcp_stages<NB>() + 5) * 8 +
         16;
}

template <int NB, int CH>
constexpr size_t gemm_tc_smem_bytes() {
  using G = TcGeom<NB, CH>;
  return static_cast<size_t>(G::STAGES) * G::STAGE + (2 * G::STAGES + 2) * 8 + 16 + 1024;
}

}  // namespace lcrb
