// Weight-streaming matrix-vector kernel for batch-1 decode: y = W x with W a
// row-major bf16 [N][K] matrix read exactly once from HBM.
//
// Replaces the reference's cublasGemmEx at m = 1 (gemm_nt, src/model.cu:38-45)
// and folds the small kernels around each projection into it:
//   prologue  PLAIN        x = a bf16 vector written by the previous kernel
//             NORM         x = bf16(rmsnorm(resid) * gain)  (rmsnorm.cu:21-119)
//             EMBED_NORM   the same on the embedding row of the device token
//                          (elementwise.cu:25-41), CTA 0 storing the row
//   epilogue  STORE / STORE_F32   y as bf16 / fp32
//             RESID        resid = bf16(resid + bf16(y)), unrounded sum kept
//                          for the next norm (the fused join, rmsnorm.cu:68-119)
//             SWIGLU       act = bf16(silu(bf16(gate)) * bf16(up)) with the
//                          gate and up rows of one output in the same CTA
//                          (elementwise.cu:96-121)
//             LOGITS_ARGMAX  fp32 logits plus the packed (value, ~index)
//                          argmax of sampling.cu:42-67; the last CTA to finish
//                          writes the next token into device state
//
// Structure (288 threads per CTA):
//   warp 8, lane 0  producer: streams the CTA's contiguous share of rows into a
//                   ring of shared-memory stages, one cp.async.bulk (1-D TMA,
//                   L2 evict-first) per row segment, completing on the
//                   stage's mbarrier. Rows land at a pitch of 16 bytes more
//                   than their length, so the eight rows an ldmatrix reads
//                   sit in distinct banks.
//   warps 0-7       consumers: the dot products run on the tensor pipe as
//                   mma.sync m16n8k16 (bf16 in, fp32 accumulate): per 32
//                   columns one ldmatrix.x4 loads 8 weight rows (the B
//                   operand, B[k][n] = W[n][k]) and one loads the matching
//                   32 staged x values (A rows 0-7 all x, rows 8-15 zero);
//                   lane t then holds rows 2t and 2t+1 of the 8. Warps split
//                   a stage's columns; their partials meet in shared memory.
// Weights do not depend on the previous kernel, so the producer starts before
// griddepcontrol.wait: with programmatic dependent launch the next matrix is
// already in flight while the previous kernel drains.
#pragma once

#include "common.cuh"
#include "ll.cuh"

namespace lcrb {

enum GemvPro { PRO_PLAIN = 0, PRO_NORM = 1, PRO_EMBED_NORM = 2 };
// EPI_ROPE (tcgen05 projection only): bf16 store with the rotate-half RoPE
// applied to the q and k columns of a QKV projection.
// Persistent step only: EPI_ACC64 adds y, as a 2^-32 fixed-point integer, into
// an int64 accumulator shared by every CTA (a split-K partial; integer adds
// commute, so the sum is the same whatever order the CTAs arrive in);
// EPI_SWIGLU_F32 stores act = silu(gate) * up as fp32 (rounded through bf16
// when round_out, as the reference stores it).
enum GemvEpi { EPI_STORE = 0, EPI_STORE_F32 = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_LOGITS_ARGMAX = 4, EPI_ROPE = 5,
               EPI_ACC64 = 6, EPI_SWIGLU_F32 = 7 };

// Fixed-point scale of the split-K accumulators (EPI_ACC64): 2^32.
constexpr float kFixScale = 4294967296.0f;
constexpr double kFixInv = 1.0 / 4294967296.0;

__device__ __forceinline__ void red_add_fixed(unsigned long long* acc, float y) {
  const long long v = __float2ll_rn(y * kFixScale);
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(acc), "l"(v) : "memory");
}
__device__ __forceinline__ float fixed_to_float(unsigned long long v) {
  return static_cast<float>(static_cast<double>(static_cast<long long>(v)) * kFixInv);
}

struct GemvArgs {
  const bf16* w;      // [N][K]; SWIGLU: rows [0, F) gate, [F, 2F) up
  int n_out;          // outputs (rows; SWIGLU: F)
  unsigned* sched;    // LOGITS_ARGMAX: [2], [1] counts finished CTAs -- zero
                      //     before the first launch; the last CTA resets it
  uint32_t* status;   // device status word (bounded-wait failures)
  // prologue
  const bf16* x_in;       // PLAIN: input; NORM: residual stream (bf16)
  const float* xsum;      // NORM: unrounded residual sums (nullptr: use x_in)
  const bf16* norm_w;     // NORM / EMBED_NORM gain
  float eps;
  const bf16* embed;      // EMBED_NORM: table [vocab][K]
  const int32_t* token;   // EMBED_NORM: device token id
  int vocab;
  bf16* x_out;            // EMBED_NORM: residual stream written by CTA 0
  float* xsum_out;
  // epilogue
  bf16* y;                // STORE / SWIGLU output
  float* yf;              // STORE_F32 / LOGITS output
  bf16* resid;            // RESID: residual stream, updated in place
  float* resid_sum;       // RESID: unrounded sums
  unsigned long long* argmax_acc;  // LOGITS_ARGMAX accumulator (0 between uses)
  int32_t* state_token;   // LOGITS_ARGMAX: next token
  int32_t* state_pos;     //   position, advanced by one when `advance`
  int32_t* history;       //   history[pos] = next token (nullable)
  int history_len;
  int advance;
  unsigned long long* acc64;  // ACC64: fixed-point accumulators, indexed by output
  int round_out;              // STORE_F32 / SWIGLU_F32: round through bf16 as the reference stores
  int exact_resid;            // RESID: resid_sum += y in fp32 (resid = its bf16 copy), no bf16 rounding of y
  int32_t* state_gen;         // LOGITS_ARGMAX: step generation, advanced by one (nullable)
  unsigned long long* wait_cycles;  // trace: SM cycles thread 0 waited on full stages (nullable)
  unsigned long long* stage_ns;     // trace: [s] stage s ready, [64 + s] released (nullable)
  // Low-latency exchange (the persistent step, ll.cuh); nullptr: plain memory.
  const unsigned long long* ll_x;  // NORM input: [K] LL64 residual sums (x = their bf16)
  const uint32_t* ll_v;            // PLAIN input: [K] LL32 values
  uint32_t ll_in_tag;
  uint32_t* ll_y32;                // STORE / SWIGLU output: LL32 words
  unsigned long long* ll_y64;      // RESID output: LL64 residual sums
  const unsigned long long* ll_resid;  // RESID: the residual sums of this CTA's rows (its own words)
  const bf16* resid_embed;         // RESID at the first layer: the embedding row is the residual
  uint32_t ll_out_tag;
  uint64_t ll_wait_ns;
  uint32_t* epoch;          // LOGITS_ARGMAX: the last CTA writes epoch_next there (nullable)
  uint32_t epoch_next;
  unsigned long long ll_copy_bytes;  // ll_y32 / ll_y64: kLLCopies replicas this far apart
};

// Stores an exchange word into each of the buffer's kLLCopies replicas.
template <class T>
__device__ __forceinline__ void ll_store_all(T* p, T w, unsigned long long copy_bytes) {
#pragma unroll
  for (int r = 0; r < kLLCopies; ++r) {
    T* q = reinterpret_cast<T*>(reinterpret_cast<char*>(p) + r * copy_bytes);
    if constexpr (sizeof(T) == 8) {
      st_relaxed_u64(reinterpret_cast<unsigned long long*>(q), w);
    } else {
      st_relaxed_u32(reinterpret_cast<uint32_t*>(q), w);
    }
  }
}

// Stage geometry for a K-column matrix. A stage holds RPS rows of KC columns
// (the whole row for K <= 2048, a 2048-column segment beyond), 32 KB of
// weights; CHUNKS stages make one group of rows. A whole group arrives as one
// tensor copy per stage in the swizzled chunk-major layout of make_weight_map
// (byte (c / 64 * RPS + r) * 128 + ((c % 64 / 8) ^ (r % 8)) * 16 + c % 8 * 2
// holds row r, column c); the last, partial group of a CTA's share arrives
// as one bulk copy per row at PITCH = 2 KC + 16 bytes. In both layouts the
// eight rows of an 8x8 ldmatrix tile fall in distinct banks.
template <int K>
struct GemvGeom {
  static constexpr int KC = K < 2048 ? K : 2048;  // columns per stage
  static constexpr int CHUNKS = K / KC;           // stages per row group
  static constexpr int G8 = 2048 / KC;            // 8-row MMA tiles per stage
  static constexpr int RPS = 8 * G8;              // rows per stage
  static constexpr int WPG = 8 / G8;              // consumer warps per tile
  static constexpr int KW = KC / WPG;             // columns per warp per stage
  static constexpr int STEPS = KW / 32;           // ldmatrix.x4 pairs per warp per stage
  static constexpr int ROW_BYTES = K * 2;
  static constexpr int SEG_BYTES = KC * 2;        // bytes of one row copy
  static constexpr int PITCH = SEG_BYTES + 16;
  static constexpr int BYTES = RPS * PITCH;       // padded layout (a group's tail)
  static constexpr int TILE_BYTES = RPS * KC * 2;  // swizzled layout (whole groups)
  // Row groups per reduction segment: 2048 floats (8 KB) of warp partials.
  static constexpr int SEG = 2048 / (RPS * WPG);
  static_assert(K % 256 == 0 && (K <= 2048 || K % 2048 == 0), "K must be 256..2048 or a multiple of 2048");
  static_assert(KW == 256 && STEPS == 8, "every consumer warp covers 256 columns of a stage");
};

constexpr int kGemvConsumers = 256;
// Shared-memory row partials gathered before one cross-warp reduction and
// epilogue pass (GemvGeom::SEG stages' worth).
constexpr int kGemvRedFloats = 2048;
constexpr int kGemvThreads = kGemvConsumers + 32;
// Ring slot stride: every GemvGeom<K>::BYTES (at most 64 rows x (512 + 16)
// bytes) fits.
constexpr int kGemvSlotBytes = 33792;

__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Outputs [o0, o1) of the contiguous share CTA `cta` of `ctas` owns.
__device__ __forceinline__ int gemv_share(int n_out, int cta, int ctas) {
  return static_cast<int>(static_cast<long long>(cta) * n_out / ctas);
}

// ---------------------------------------------------------------------------
// Building blocks, shared by the standalone kernel below and the persistent
// decode kernel. A "ring" is STAGES shared-memory stages with a full and an
// empty mbarrier each; `it` is the running stage sequence number, advanced
// identically by the producer and the consumers.
// ---------------------------------------------------------------------------

// Something the producer can do while it would otherwise block on a full
// ring (the persistent kernel's L2 prefetch window); `bytes` is the weight
// volume issued into the ring so far.
struct NoPrefetch {
  __device__ __forceinline__ void top_up(unsigned long long) {}
};

// Producer: streams weight rows [o0, o1) (SWIGLU: pairs, gate and up rows) of
// a [rows][K] matrix into the ring: whole groups with one tensor copy per
// stage through `map` (make_weight_map of the same matrix), the last partial
// group one bulk copy per row from `w`. The consumers' results for rows past
// o1 are never stored. Returns false if a bounded wait expired or the ring is
// not 1024-byte aligned. `wait_cycles` (nullable) accumulates SM cycles spent
// waiting for free slots; `issue_ns` (nullable) records when each of the
// first 64 stages was issued.
template <int K, int STAGES, bool SWIGLU, class PF = NoPrefetch>
__device__ __forceinline__ bool gemv_produce(uint8_t* ring, uint64_t* full, uint64_t* empty,
                                             int& it, const CUtensorMap* map, const bf16* w, int n_out,
                                             int o0, int o1, uint64_t policy, uint32_t* status,
                                             PF* pf = nullptr, unsigned long long* issued = nullptr,
                                             unsigned long long* wait_cycles = nullptr,
                                             unsigned long long* issue_ns = nullptr, int ld = 0,
                                             int chunk0 = 0) {
  using G = GemvGeom<K>;
  constexpr int UNIT = SWIGLU ? G::RPS / 2 : G::RPS;
  constexpr int CHUNK_STEP = G::KC / 64;  // tensor-map chunk coordinate per stage
  // A column tile of a wider matrix: rows `ld` elements apart, the tile
  // starting at 64-column chunk `chunk0`.
  const size_t row_pitch = static_cast<size_t>(ld > 0 ? ld : K);
  if ((smem_addr(ring) & 1023u) != 0) {
    if (status) atomicOr(status, kStatusBadSmem);
    return false;
  }
  const char* wbase = reinterpret_cast<const char*>(w);
  for (int first = o0; first < o1; first += UNIT) {
    const int rows = min(UNIT, o1 - first);
    for (int c = 0; c < G::CHUNKS; ++c, ++it) {
      if (pf) pf->top_up(*issued);
      const int slot = it % STAGES;
      const long long w0 = wait_cycles ? clock64() : 0;
      if (it >= STAGES &&
          !mbar_wait(&empty[slot], ((it / STAGES) - 1) & 1, status, kStatusTimeoutEmpty)) {
        return false;
      }
      if (wait_cycles) *wait_cycles += static_cast<unsigned long long>(clock64() - w0);
      if (issue_ns) {
        const int k = (first - o0) / UNIT * G::CHUNKS + c;
        if (k < 64) issue_ns[k] = globaltimer_ns();
      }
      uint8_t* dst = ring + slot * kGemvSlotBytes;
      unsigned long long bytes;
      if (rows == UNIT) {
        bytes = G::TILE_BYTES;
        mbar_arrive_expect_tx(&full[slot], G::TILE_BYTES);
        if constexpr (SWIGLU) {
          tma_load_4d(dst, map, 0, first, 0, chunk0 + c * CHUNK_STEP, &full[slot], policy);
        } else {
          tma_load_3d(dst, map, 0, first, chunk0 + c * CHUNK_STEP, &full[slot], policy);
        }
      } else {
        bytes = static_cast<unsigned long long>(SWIGLU ? 2 : 1) * rows * G::SEG_BYTES;
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(bytes));
        const char* src = wbase + (static_cast<size_t>(first) * row_pitch + chunk0 * 64 + c * G::KC) * 2;
        for (int r = 0; r < rows; ++r) {
          bulk_g2s(dst + r * G::PITCH, src + static_cast<size_t>(r) * row_pitch * 2, G::SEG_BYTES,
                   &full[slot], policy);
          if constexpr (SWIGLU) {
            bulk_g2s(dst + (UNIT + r) * G::PITCH,
                     src + (static_cast<size_t>(n_out) + r) * row_pitch * 2, G::SEG_BYTES, &full[slot],
                     policy);
          }
        }
      }
      if (issued) *issued += bytes;
    }
  }
  return true;
}

// Waits (bounded) until every copy issued into the ring has landed, so a CTA
// never exits with a copy still writing its shared memory. `issued` is the
// producer's stage count; the last STAGES stages are the only ones that can
// still be in flight. It waits even after an abort (no status word: the
// abort bit does not cut it short).
template <int STAGES>
__device__ __forceinline__ void ring_drain(uint64_t* full, int issued, uint32_t*) {
  for (int k = issued > STAGES ? issued - STAGES : 0; k < issued; ++k) {
    mbar_wait(&full[k % STAGES], (k / STAGES) & 1, nullptr, 0);
  }
}

// Consumers (256 threads): the input vector, staged ONCE per CTA in shared
// memory as bf16 (`xs`, K elements; every value the GEMV multiplies is
// bf16-exact), each thread preparing 8-element chunks: a plain copy, or
// RMSNorm (sum of squares over the unrounded residual sums when given, scale
// applied to the bf16 residual, rounded to bf16 as the reference stores
// `normed`). Uses named barrier 1; `xs` is complete on return.
template <int K, int PRO>
__device__ __forceinline__ bool gemv_stage_x(const GemvArgs& a, bf16* xs, float* red8) {
  constexpr int KC = K / 8;
  constexpr int PER = (KC + kGemvConsumers - 1) / kGemvConsumers;  // chunks per thread
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  bool ok = true;
  if constexpr (PRO == PRO_PLAIN) {
    if (a.ll_v != nullptr) {
      // every chunk of this thread in one poll (KC is a multiple of the
      // thread count for the persistent step's shapes; others repeat chunks)
      LLWait wt{a.status, a.ll_wait_ns};
      uint4 v[2 * PER];
      ok = ll_poll_groups<2 * PER, false>(
          [&](int i) -> const void* { return a.ll_v + min(tid + (i >> 1) * kGemvConsumers, KC - 1) * 8 + (i & 1) * 4; },
          v, a.ll_in_tag, wt);
#pragma unroll
      for (int p = 0; p < PER; ++p) {
        const int c = tid + p * kGemvConsumers;
        if (c < KC) reinterpret_cast<uint4*>(xs)[c] = ll32_values8(v[2 * p], v[2 * p + 1]);
      }
    } else {
#pragma unroll
      for (int p = 0; p < PER; ++p) {
        const int c = tid + p * kGemvConsumers;
        if (c < KC) reinterpret_cast<uint4*>(xs)[c] = ldg_cg16(a.x_in + c * 8);
      }
    }
  } else {
    const bf16* src = a.x_in;
    if constexpr (PRO == PRO_EMBED_NORM) {
      int tok = __ldcg(a.token);
      if (tok < 0 || tok >= a.vocab) {
        if (tid == 0 && a.status) atomicOr(a.status, kStatusBadToken);
        tok = 0;
      }
      src = a.embed + static_cast<size_t>(tok) * K;
    }
    uint4 raw[PER], gain[PER];
    float ss = 0.f;
    // With the exchange: the residual sums of every chunk of this thread in
    // one poll; the residual is their bf16 (the RESID epilogue's store).
    uint4 lv[PER == 0 ? 1 : 4 * PER];
    if (PRO == PRO_NORM && a.ll_x != nullptr) {
      LLWait wt{a.status, a.ll_wait_ns};
      ok = ll_poll_groups<4 * PER, true>(
          [&](int i) -> const void* { return a.ll_x + min(tid + (i >> 2) * kGemvConsumers, KC - 1) * 8 + (i & 3) * 2; },
          lv, a.ll_in_tag, wt);
    }
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = tid + p * kGemvConsumers;
      if (c < KC) {
        gain[p] = ldg16(a.norm_w + c * 8);
        float v[8];
        if (PRO == PRO_NORM && a.ll_x != nullptr) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            v[2 * q] = __uint_as_float(lv[4 * p + q].y);
            v[2 * q + 1] = __uint_as_float(lv[4 * p + q].w);
          }
          raw[p].x = pack_bf2(v[0], v[1]);
          raw[p].y = pack_bf2(v[2], v[3]);
          raw[p].z = pack_bf2(v[4], v[5]);
          raw[p].w = pack_bf2(v[6], v[7]);
        } else if (PRO == PRO_NORM && a.xsum != nullptr) {
          raw[p] = ldg_cg16(src + c * 8);
          const float4 s0 = __ldcg(reinterpret_cast<const float4*>(a.xsum + c * 8));
          const float4 s1 = __ldcg(reinterpret_cast<const float4*>(a.xsum + c * 8 + 4));
          v[0] = s0.x; v[1] = s0.y; v[2] = s0.z; v[3] = s0.w;
          v[4] = s1.x; v[5] = s1.y; v[6] = s1.z; v[7] = s1.w;
        } else {
          raw[p] = ldg_cg16(src + c * 8);
          unpack8(raw[p], v);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
        if (PRO == PRO_EMBED_NORM && blockIdx.x == 0) {
          float xv[8];
          unpack8(raw[p], xv);
          *reinterpret_cast<uint4*>(a.x_out + c * 8) = raw[p];
          *reinterpret_cast<float4*>(a.xsum_out + c * 8) = make_float4(xv[0], xv[1], xv[2], xv[3]);
          *reinterpret_cast<float4*>(a.xsum_out + c * 8 + 4) = make_float4(xv[4], xv[5], xv[6], xv[7]);
        }
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red8[warp] = ss;
    named_sync(1, kGemvConsumers);
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) total += red8[w];
    const float scale = rsqrtf(total / static_cast<float>(K) + a.eps);
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = tid + p * kGemvConsumers;
      if (c < KC) {
        float xv[8], gf[8];
        unpack8(raw[p], xv);
        unpack8(gain[p], gf);
        uint4 o;
        o.x = pack_bf2(__fmul_rn(__fmul_rn(xv[0], scale), gf[0]), __fmul_rn(__fmul_rn(xv[1], scale), gf[1]));
        o.y = pack_bf2(__fmul_rn(__fmul_rn(xv[2], scale), gf[2]), __fmul_rn(__fmul_rn(xv[3], scale), gf[3]));
        o.z = pack_bf2(__fmul_rn(__fmul_rn(xv[4], scale), gf[4]), __fmul_rn(__fmul_rn(xv[5], scale), gf[5]));
        o.w = pack_bf2(__fmul_rn(__fmul_rn(xv[6], scale), gf[6]), __fmul_rn(__fmul_rn(xv[7], scale), gf[7]));
        reinterpret_cast<uint4*>(xs)[c] = o;
      }
    }
  }
  // xs complete (and red8 free again); false: a poll gave up (the step aborts)
  return !named_sync_or(1, kGemvConsumers, !ok);
}

// ldmatrix.x4: lane l supplies the shared address of row l % 8 of 8x8 tile
// l / 8; r[i] receives tile i's elements (lane / 4, 2 (lane % 4) .. + 1).
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// d += A B for one m16n8k16 tile, bf16 operands, fp32 accumulation; A rows
// 8-15 are zero (a1 = a3 = 0), so d[2], d[3] stay as they were.
__device__ __forceinline__ void mma_x_rows(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                           uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// d += A B with A rows 0-7 the bf16 x (high part) and rows 8-15 its bf16
// remainder x - hi (low part): d[0], d[1] collect W x_hi and d[2], d[3]
// W x_lo, so their sum is the product with x to about 16 significant bits
// at no extra MMA (the rows are otherwise zero).
__device__ __forceinline__ void mma_x_hilo(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Consumers (256 threads): dot products of the streamed rows [o0, o1) with
// the staged input `xs` (bf16 [K] in shared memory, 16-byte aligned) on the
// tensor pipe, partials of the WPG warps sharing a row tile combined through
// `red` (kGemvRedFloats floats) once per segment, then the epilogue.
// LOGITS_ARGMAX folds the packed (order key, ~index) maximum into `best`.
// Uses named barrier 1. With `xs_lo` (LO) the input is xs + xs_lo, the bf16
// pair of an fp32 vector (mma_x_hilo).
template <int K, int STAGES, int EPI, bool LO = false>
__device__ __forceinline__ void gemv_consume(const uint8_t* ring, uint64_t* full, uint64_t* empty,
                                             int& it, const GemvArgs& a, int o0, int o1,
                                             const bf16* xs, float* red, unsigned long long& best,
                                             bool& failed, const bf16* xs_lo = nullptr) {
  using G = GemvGeom<K>;
  constexpr int RPS = G::RPS, WPG = G::WPG, STEPS = G::STEPS, CHUNKS = G::CHUNKS;
  constexpr int PAIRS = RPS / 2;
  constexpr int UNIT = (EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_F32) ? PAIRS : RPS;
  constexpr int SEG = G::SEG;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = warp / WPG, ks = warp % WPG;
  // This lane's ldmatrix row addresses: weight row (tile * 8 + lane % 8) and
  // the x chunk of tile lane / 8, at the warp's first column of a stage --
  // padded layout: w_lane + 64 j for the j-th 32 columns; swizzled layout:
  // 64-column chunk ks * 4 + j / 2, 16-byte piece (j % 2) * 4 + lane / 8
  // rotated by the row.
  const int r8 = lane & 7, piece = lane >> 3;
  const uint32_t w_lane = static_cast<uint32_t>((tile * 8 + r8) * G::PITCH + (ks * G::KW + piece * 8) * 2);
  const uint32_t s_lane = static_cast<uint32_t>(((ks * 4) * G::RPS + tile * 8 + r8) * 128);
  const uint32_t s_even = static_cast<uint32_t>((piece ^ r8) << 4);
  const uint32_t s_odd = static_cast<uint32_t>(((4 + piece) ^ r8) << 4);
  const uint32_t x_lane = smem_addr(xs) + static_cast<uint32_t>((ks * G::KW + (lane >> 3) * 8) * 2);
  const uint32_t ring_base = smem_addr(ring);
  const uint32_t xl_lane = LO ? smem_addr(xs_lo) + (x_lane - smem_addr(xs)) : 0u;
  // With one stage per group the warp's x fragments never change.
  uint32_t xf[CHUNKS == 1 ? STEPS : 1][4];
  uint32_t xl[(CHUNKS == 1 && LO) ? STEPS : 1][4];
  if constexpr (CHUNKS == 1) {
#pragma unroll
    for (int j = 0; j < STEPS; ++j) {
      ldmatrix_x4(xf[j], x_lane + j * 64);
      if constexpr (LO) ldmatrix_x4(xl[j], xl_lane + j * 64);
    }
  }
  const int n_units = (o1 - o0 + UNIT - 1) / UNIT;
  const bool timed = a.wait_cycles != nullptr && tid == 0;
  unsigned long long waited = 0;
  for (int seg0 = 0; seg0 < n_units; seg0 += SEG) {
    const int seg1 = min(n_units, seg0 + SEG);
    for (int u = seg0; u < seg1; ++u) {
      float acc[4][4] = {};
      const bool whole = o1 - (o0 + u * UNIT) >= UNIT;  // tensor-copied, swizzled
#pragma unroll 1
      for (int c = 0; c < CHUNKS; ++c, ++it) {
        const int slot = it % STAGES;
        const long long w0 = timed ? clock64() : 0;
        if (!failed) failed = !mbar_wait(&full[slot], (it / STAGES) & 1, a.status, kStatusTimeoutFull);
        if (timed) waited += static_cast<unsigned long long>(clock64() - w0);
        const int sk = u * CHUNKS + c;
        if (a.stage_ns && tid == 0 && sk < 64) a.stage_ns[sk] = globaltimer_ns();
        const uint32_t st_base = ring_base + static_cast<uint32_t>(slot * kGemvSlotBytes);
#pragma unroll
        for (int j = 0; j < STEPS; ++j) {
          uint32_t wb[4], xa[4], xb[4];
          const uint32_t sw = s_lane + static_cast<uint32_t>((j >> 1) * G::RPS * 128) + ((j & 1) ? s_odd : s_even);
          ldmatrix_x4(wb, st_base + (whole ? sw : w_lane + j * 64));
          if constexpr (CHUNKS == 1) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              xa[q] = xf[j][q];
              if constexpr (LO) xb[q] = xl[j][q];
            }
          } else {
            ldmatrix_x4(xa, x_lane + static_cast<uint32_t>(c * G::KC * 2) + j * 64);
            if constexpr (LO) ldmatrix_x4(xb, xl_lane + static_cast<uint32_t>(c * G::KC * 2) + j * 64);
          }
          if constexpr (LO) {
            mma_x_hilo(acc[(2 * j) & 3], xa[0], xb[0], xa[1], xb[1], wb[0], wb[1]);
            mma_x_hilo(acc[(2 * j + 1) & 3], xa[2], xb[2], xa[3], xb[3], wb[2], wb[3]);
          } else {
            mma_x_rows(acc[(2 * j) & 3], xa[0], xa[1], wb[0], wb[1]);
            mma_x_rows(acc[(2 * j + 1) & 3], xa[2], xa[3], wb[2], wb[3]);
          }
        }
        __syncwarp();
        if (lane == 0 && !failed) mbar_arrive(&empty[slot]);
        if (a.stage_ns && tid == 0 && sk < 64) a.stage_ns[64 + sk] = globaltimer_ns();
      }
      if (lane < 4) {
        const int row = tile * 8 + 2 * lane;
        float* dst = red + ((u - seg0) * RPS + row) * WPG + ks;
        if constexpr (LO) {
          dst[0] = ((acc[0][0] + acc[1][0]) + (acc[2][0] + acc[3][0])) +
                   ((acc[0][2] + acc[1][2]) + (acc[2][2] + acc[3][2]));
          dst[WPG] = ((acc[0][1] + acc[1][1]) + (acc[2][1] + acc[3][1])) +
                     ((acc[0][3] + acc[1][3]) + (acc[2][3] + acc[3][3]));
        } else {
          dst[0] = (acc[0][0] + acc[1][0]) + (acc[2][0] + acc[3][0]);
          dst[WPG] = (acc[0][1] + acc[1][1]) + (acc[2][1] + acc[3][1]);
        }
      }
    }
    named_sync(1, kGemvConsumers);  // the segment's partials are in shared memory
    const int first = o0 + seg0 * UNIT;
    const int outs = min(o1, o0 + seg1 * UNIT) - first;
    for (int v = tid; v < outs && !failed; v += kGemvConsumers) {
      const int un = v / UNIT, r = v % UNIT;
      const float* rr = red + (un * RPS + r) * WPG;
      float y = 0.f;
#pragma unroll
      for (int w = 0; w < WPG; ++w) y += rr[w];
      const int out = first + v;
      if constexpr (EPI == EPI_STORE) {
        if (a.ll_y32 != nullptr) {
          ll_store_all(a.ll_y32 + out, ll32_word(y, a.ll_out_tag), a.ll_copy_bytes);
        } else {
          a.y[out] = __ushort_as_bfloat16(f2bf(y));
        }
      } else if constexpr (EPI == EPI_STORE_F32) {
        a.yf[out] = a.round_out ? rbf(y) : y;
      } else if constexpr (EPI == EPI_RESID) {
        if (a.ll_y64 != nullptr) {
          // the residual: the embedding row at the first layer, else the bf16
          // of this CTA's own previous sum
          const float r = a.resid_embed != nullptr
                              ? bf2f(__ldg(reinterpret_cast<const unsigned short*>(a.resid_embed) + out))
                              : rbf(ll64_value(__ldcg(a.ll_resid + out)));
          ll_store_all(a.ll_y64 + out, ll64_word(__fadd_rn(r, rbf(y)), a.ll_out_tag), a.ll_copy_bytes);
        } else {
          const float s = a.exact_resid
                              ? __fadd_rn(__ldcg(a.resid_sum + out), y)
                              : __fadd_rn(bf2f(__ldcg(reinterpret_cast<const unsigned short*>(a.resid) + out)),
                                          rbf(y));
          a.resid[out] = __ushort_as_bfloat16(f2bf(s));
          a.resid_sum[out] = s;
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
        const float* ru = red + (un * RPS + r + PAIRS) * WPG;
        float up = 0.f;
#pragma unroll
        for (int w = 0; w < WPG; ++w) up += ru[w];
        const float g = rbf(y);
        const float silu = g / (1.0f + __expf(-g));
        if (a.ll_y32 != nullptr) {
          ll_store_all(a.ll_y32 + out, ll32_word(silu * rbf(up), a.ll_out_tag), a.ll_copy_bytes);
        } else {
          a.y[out] = __ushort_as_bfloat16(f2bf(silu * rbf(up)));
        }
      } else if constexpr (EPI == EPI_SWIGLU_F32) {
        const float* ru = red + (un * RPS + r + PAIRS) * WPG;
        float up = 0.f;
#pragma unroll
        for (int w = 0; w < WPG; ++w) up += ru[w];
        if (a.round_out) {
          const float g = rbf(y);
          a.yf[out] = rbf(g / (1.0f + __expf(-g)) * rbf(up));
        } else {
          a.yf[out] = y / (1.0f + __expf(-y)) * up;
        }
      } else if constexpr (EPI == EPI_ACC64) {
        red_add_fixed(a.acc64 + out, y);
      } else if constexpr (EPI == EPI_LOGITS_ARGMAX) {
        a.yf[out] = y;
        const unsigned long long packed =
            (static_cast<unsigned long long>(order_key(y)) << 32) |
            static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(out));
        best = best > packed ? best : packed;
      }
    }
    named_sync(1, kGemvConsumers);  // the next segment may overwrite `red`
  }
  if (timed) *a.wait_cycles = waited;
}

// Argmax hand-off after the lm_head: the CTA maximum into the global
// accumulator, and the last CTA to finish writes the next token, the history
// entry and the advanced position, then resets for the next step.
__device__ __forceinline__ void argmax_finish(const GemvArgs& a, unsigned long long cta_best) {
  atomicMax(a.argmax_acc, cta_best);
  __threadfence();
  const unsigned prev = atomicAdd(&a.sched[1], 1u);
  if (prev == gridDim.x - 1) {
    __threadfence();
    atomicExch(&a.sched[1], 0u);
    const unsigned long long packed = atomicExch(a.argmax_acc, 0ull);
    const int next = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(packed & 0xFFFFFFFFull));
    const int pos = __ldcg(a.state_pos);
    *a.state_token = next;
    if (a.history != nullptr && pos >= 0 && pos < a.history_len) a.history[pos] = next;
    if (a.advance) *a.state_pos = pos + 1;
    if (a.state_gen) *a.state_gen += 1;
    if (a.epoch) *a.epoch = a.epoch_next;
  }
}

template <int K, int STAGES, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1)
    gemv_stream_kernel(const GemvArgs a, const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kGemvSlotBytes);
  uint64_t* empty = full + STAGES;
  unsigned long long* cta_best = reinterpret_cast<unsigned long long*>(empty + STAGES);
  float* red8 = reinterpret_cast<float*>(cta_best + 1);   // [8]
  float* red = red8 + 8;                                    // [kGemvRedFloats]
  bf16* xs = align_smem<bf16>(red + kGemvRedFloats, 128);  // [K], 16-byte vector access

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int o0 = gemv_share(a.n_out, blockIdx.x, gridDim.x);
  const int o1 = gemv_share(a.n_out, blockIdx.x + 1, gridDim.x);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvConsumers / 32);
    }
    *cta_best = 0ull;
    mbar_fence_init();
  }
  __syncthreads();
  pdl_launch_next();

  if (warp == kGemvConsumers / 32) {
    // Weights do not depend on the previous kernel: stream before the wait.
    if (lane == 0) {
      int it = 0;
      gemv_produce<K, STAGES, EPI == EPI_SWIGLU>(ring, full, empty, it, &wmap, a.w, a.n_out, o0, o1,
                                              l2_policy_evict_first(), a.status);
      ring_drain<STAGES>(full, it, a.status);
    }
  } else {
    pdl_wait();
    gemv_stage_x<K, PRO>(a, xs, red8);
    int it = 0;
    unsigned long long best = 0ull;
    bool failed = false;
    gemv_consume<K, STAGES, EPI>(ring, full, empty, it, a, o0, o1, xs, red, best, failed);
    if constexpr (EPI == EPI_LOGITS_ARGMAX) {
      if (best != 0ull) atomicMax(cta_best, best);
    }
  }
  __syncthreads();
  if constexpr (EPI == EPI_LOGITS_ARGMAX) {
    if (tid == 0) argmax_finish(a, *cta_best);
  }
}

template <int K, int STAGES>
constexpr size_t gemv_smem_bytes() {
  return static_cast<size_t>(STAGES) * kGemvSlotBytes + 2 * STAGES * sizeof(uint64_t) + 8 +
         (8 + kGemvRedFloats) * sizeof(float) + 128 + static_cast<size_t>(K) * 2 + 64;
}

}  // namespace lcrb
