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
// Structure (one CTA per SM by default, 288 threads):
//   warp 8, lane 0  producer: takes the next chunk of rows from a global
//                   counter (dynamic scheduling, so CTAs that start late or
//                   share an SM still balance; the allocation-free standalone
//                   entry uses a fixed strided schedule instead), and streams
//                   it into a ring of
//                   shared-memory stages with cp.async.bulk (TMA, 1-D, L2
//                   evict-first), completing on the stage's mbarrier.
//   warps 0-7       consumers: each thread owns CPT 16-byte column chunks of
//                   the input vector in registers for the whole kernel; per
//                   stage it forms RPT row partials, the warp reduces them with
//                   a transposing butterfly, warps combine through shared memory.
// Weights do not depend on the previous kernel, so the producer starts before
// griddepcontrol.wait: with programmatic dependent launch the next matrix is
// already in flight while the previous kernel drains.
#pragma once

#include "common.cuh"

namespace lcrb {

enum GemvPro { PRO_PLAIN = 0, PRO_NORM = 1, PRO_EMBED_NORM = 2 };
enum GemvEpi { EPI_STORE = 0, EPI_STORE_F32 = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_LOGITS_ARGMAX = 4 };

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
};

template <int K, int STAGE_BYTES>
struct GemvGeom {
  static constexpr int KC = K / 8;                       // 16-byte chunks per row
  // A warp per row up to K = 2048 (64 elements a lane), more warps beyond, so
  // the reduction is amortised over many multiply-adds.
  static constexpr int TPR = (K / 64) > 32 ? (K / 64) : 32;  // threads per row
  static constexpr int CPT = KC / TPR;                   // chunks per thread (<= 8)
  static constexpr int SLOTS = 256 / TPR;                // rows in flight per pass
  static constexpr int WPR = TPR / 32;                   // warps per row
  static constexpr int ROW_BYTES = K * 2;
  static constexpr int RPS = STAGE_BYTES / ROW_BYTES;    // rows per stage
  static constexpr int RPT = RPS / SLOTS;                // rows per thread per stage
  // Stages per reduction segment: 2048 floats (8 KB) of row partials.
  static constexpr int SEG = 2048 / (RPS * WPR) > 0 ? 2048 / (RPS * WPR) : 1;
  static_assert(K % 256 == 0 && KC % 32 == 0, "K must be a multiple of 256");
  static_assert(TPR * CPT == KC && CPT <= 8, "K/8 must split evenly over the row's threads");
  static_assert(TPR <= 256 && 256 % TPR == 0, "rows must split the 8 consumer warps");
  static_assert(RPS >= SLOTS && RPS % SLOTS == 0, "stage too small for this K");
  static_assert(RPT == 1 || RPT == 2 || RPT == 4 || RPT == 8 || RPT == 16, "RPT");
};

constexpr int kGemvConsumers = 256;
// Shared-memory row partials gathered before one cross-warp reduction and
// epilogue pass (GemvGeom::SEG stages' worth).
constexpr int kGemvRedFloats = 2048;
constexpr int kGemvThreads = kGemvConsumers + 32;

__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Transposing butterfly: each lane enters with RPT row partials, and leaves
// holding the warp total of row warp_row_of_lane() (lanes whose low bits are
// zero are the unique holders).
template <int RPT>
__device__ __forceinline__ float warp_reduce_rows(float (&v)[RPT], int lane) {
  int n = RPT;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (n > 1) {
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < RPT / 2; ++i) {
        if (i < n / 2) {
          const float send = upper ? v[i] : v[i + n / 2];
          const float keep = upper ? v[i + n / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      n >>= 1;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
  return v[0];
}

template <int RPT>
__device__ __forceinline__ int warp_row_of_lane(int lane) {
  // Halving step k (offset 16 >> k) sends the lane with that bit set to the
  // upper half of the remaining rows.
  int r = 0;
#pragma unroll
  for (int k = 0, n = RPT; n > 1; ++k, n >>= 1) r += ((lane >> (4 - k)) & 1) * (n >> 1);
  return r;
}

template <int RPT>
__device__ __forceinline__ bool warp_row_owner(int lane) {
  constexpr int m = (RPT >= 16) ? 4 : (RPT >= 8) ? 3 : (RPT >= 4) ? 2 : (RPT >= 2) ? 1 : 0;
  return (lane & ((1 << (5 - m)) - 1)) == 0;
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
// a [rows][K] matrix into the ring. Returns false if a bounded wait expired.
template <int K, int STAGE_BYTES, int STAGES, bool SWIGLU, class PF = NoPrefetch>
__device__ __forceinline__ bool gemv_produce(uint8_t* ring, uint64_t* full, uint64_t* empty,
                                             int& it, const bf16* w, int n_out, int o0, int o1,
                                             uint64_t policy, uint32_t* status,
                                             PF* pf = nullptr, unsigned long long* issued = nullptr) {
  using G = GemvGeom<K, STAGE_BYTES>;
  constexpr int PAIRS = G::RPS / 2;
  constexpr int UNIT = SWIGLU ? PAIRS : G::RPS;
  const char* wbase = reinterpret_cast<const char*>(w);
  for (int first = o0; first < o1; first += UNIT, ++it) {
    if (pf) pf->top_up(*issued);
    const int slot = it % STAGES;
    if (it >= STAGES &&
        !mbar_wait(&empty[slot], ((it / STAGES) - 1) & 1, status, kStatusTimeoutEmpty)) {
      return false;
    }
    uint8_t* dst = ring + slot * STAGE_BYTES;
    const uint32_t bytes = static_cast<uint32_t>(min(UNIT, o1 - first)) * G::ROW_BYTES;
    if constexpr (SWIGLU) {
      mbar_arrive_expect_tx(&full[slot], 2 * bytes);
      bulk_g2s(dst, wbase + static_cast<size_t>(first) * G::ROW_BYTES, bytes, &full[slot], policy);
      bulk_g2s(dst + PAIRS * G::ROW_BYTES, wbase + static_cast<size_t>(n_out + first) * G::ROW_BYTES,
               bytes, &full[slot], policy);
    } else {
      mbar_arrive_expect_tx(&full[slot], bytes);
      bulk_g2s(dst, wbase + static_cast<size_t>(first) * G::ROW_BYTES, bytes, &full[slot], policy);
    }
    if (issued) *issued += (SWIGLU ? 2ull : 1ull) * bytes;
  }
  return true;
}

// Waits (bounded) until every copy issued into the ring has landed, so a CTA
// never exits with a copy still writing its shared memory. `issued` is the
// producer's stage count; the last STAGES stages are the only ones that can
// still be in flight.
template <int STAGES>
__device__ __forceinline__ void ring_drain(uint64_t* full, int issued, uint32_t* status) {
  for (int k = issued > STAGES ? issued - STAGES : 0; k < issued; ++k) {
    mbar_wait(&full[k % STAGES], (k / STAGES) & 1, status, kStatusTimeoutFull);
  }
}

// Consumers (256 threads): the input vector, staged ONCE per CTA in shared
// memory as bf16 (`xs`, K elements; every value the GEMV multiplies is
// bf16-exact), each thread preparing 8-element chunks: a plain copy, or
// RMSNorm (sum of squares over the unrounded residual sums when given, scale
// applied to the bf16 residual, rounded to bf16 as the reference stores
// `normed`). Uses named barrier 1; `xs` is complete on return.
template <int K, int PRO>
__device__ __forceinline__ void gemv_stage_x(const GemvArgs& a, bf16* xs, float* red8) {
  constexpr int KC = K / 8;
  constexpr int PER = (KC + kGemvConsumers - 1) / kGemvConsumers;  // chunks per thread
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if constexpr (PRO == PRO_PLAIN) {
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = tid + p * kGemvConsumers;
      if (c < KC) reinterpret_cast<uint4*>(xs)[c] = ldg_cg16(a.x_in + c * 8);
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
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = tid + p * kGemvConsumers;
      if (c < KC) {
        gain[p] = ldg16(a.norm_w + c * 8);
        raw[p] = ldg_cg16(src + c * 8);
        float v[8];
        if (PRO == PRO_NORM && a.xsum != nullptr) {
          const float4 s0 = __ldcg(reinterpret_cast<const float4*>(a.xsum + c * 8));
          const float4 s1 = __ldcg(reinterpret_cast<const float4*>(a.xsum + c * 8 + 4));
          v[0] = s0.x; v[1] = s0.y; v[2] = s0.z; v[3] = s0.w;
          v[4] = s1.x; v[5] = s1.y; v[6] = s1.z; v[7] = s1.w;
        } else {
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
  named_sync(1, kGemvConsumers);  // xs complete (and red8 free again)
}

// Each thread's column chunks of the staged input vector, widened to fp32.
template <int K, int STAGE_BYTES>
__device__ __forceinline__ void gemv_x_regs(const bf16* xs,
                                            float (&xr)[GemvGeom<K, STAGE_BYTES>::CPT][8]) {
  using G = GemvGeom<K, STAGE_BYTES>;
  const int ci = threadIdx.x % G::TPR;
#pragma unroll
  for (int j = 0; j < G::CPT; ++j) unpack8(reinterpret_cast<const uint4*>(xs)[ci + j * G::TPR], xr[j]);
}

template <int K, int STAGE_BYTES, int PRO>
__device__ __forceinline__ void gemv_load_x(const GemvArgs& a,
                                            float (&xr)[GemvGeom<K, STAGE_BYTES>::CPT][8],
                                            bf16* xs, float* red8) {
  gemv_stage_x<K, PRO>(a, xs, red8);
  gemv_x_regs<K, STAGE_BYTES>(xs, xr);
}

// Consumers (256 threads): dot products of the streamed rows [o0, o1) with
// the register-resident x, segmented cross-warp reduction in `red`
// (kGemvRedFloats floats) and the epilogue. LOGITS_ARGMAX folds the
// packed (order key, ~index) maximum into `best`. Uses named barrier 1.
template <int K, int STAGE_BYTES, int STAGES, int EPI>
__device__ __forceinline__ void gemv_consume(const uint8_t* ring, uint64_t* full, uint64_t* empty,
                                             int& it, const GemvArgs& a, int o0, int o1,
                                             const float (&xr)[GemvGeom<K, STAGE_BYTES>::CPT][8],
                                             float* red, unsigned long long& best, bool& failed) {
  using G = GemvGeom<K, STAGE_BYTES>;
  constexpr int RPS = G::RPS, RPT = G::RPT, CPT = G::CPT, TPR = G::TPR, WPR = G::WPR;
  constexpr int PAIRS = RPS / 2;
  constexpr int UNIT = (EPI == EPI_SWIGLU) ? PAIRS : RPS;
  constexpr int SEG = G::SEG;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int slotrow = tid / TPR, ci = tid % TPR;
  const int n_stages = (o1 - o0 + UNIT - 1) / UNIT;
  for (int seg0 = 0; seg0 < n_stages; seg0 += SEG) {
    const int seg1 = min(n_stages, seg0 + SEG);
    for (int st = seg0; st < seg1; ++st, ++it) {
      const int slot = it % STAGES;
      if (!failed) failed = !mbar_wait(&full[slot], (it / STAGES) & 1, a.status, kStatusTimeoutFull);
      const uint8_t* stage = ring + slot * STAGE_BYTES;
      float part[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int row = slotrow * RPT + r;
        // Packed fp32x2 multiply-adds (sm_100 FFMA2), two accumulator pairs.
        float2 a0 = make_float2(0.f, 0.f), a1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
          const uint4 wv = *reinterpret_cast<const uint4*>(stage + row * G::ROW_BYTES + (ci + j * TPR) * 16);
          a0 = __ffma2_rn(make_float2(bf_lo(wv.x), bf_hi(wv.x)), make_float2(xr[j][0], xr[j][1]), a0);
          a1 = __ffma2_rn(make_float2(bf_lo(wv.y), bf_hi(wv.y)), make_float2(xr[j][2], xr[j][3]), a1);
          a0 = __ffma2_rn(make_float2(bf_lo(wv.z), bf_hi(wv.z)), make_float2(xr[j][4], xr[j][5]), a0);
          a1 = __ffma2_rn(make_float2(bf_lo(wv.w), bf_hi(wv.w)), make_float2(xr[j][6], xr[j][7]), a1);
        }
        part[r] = (a0.x + a1.x) + (a0.y + a1.y);
      }
      __syncwarp();
      if (lane == 0 && !failed) mbar_arrive(&empty[slot]);
      const float wsum = warp_reduce_rows<RPT>(part, lane);
      if (warp_row_owner<RPT>(lane)) {
        const int row = slotrow * RPT + warp_row_of_lane<RPT>(lane);
        red[((st - seg0) * RPS + row) * WPR + (warp % WPR)] = wsum;
      }
    }
    named_sync(1, kGemvConsumers);  // the segment's partials are in shared memory
    const int first = o0 + seg0 * UNIT;
    const int outs = min(o1, o0 + seg1 * UNIT) - first;
    for (int u = tid; u < outs && !failed; u += kGemvConsumers) {
      const int st = u / UNIT, r = u % UNIT;
      const float* rr = red + (st * RPS + r) * WPR;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < WPR; ++w) v += rr[w];
      const int out = first + u;
      if constexpr (EPI == EPI_STORE) {
        a.y[out] = __ushort_as_bfloat16(f2bf(v));
      } else if constexpr (EPI == EPI_STORE_F32) {
        a.yf[out] = v;
      } else if constexpr (EPI == EPI_RESID) {
        const float s = __fadd_rn(bf2f(__ldcg(reinterpret_cast<const unsigned short*>(a.resid) + out)), rbf(v));
        a.resid[out] = __ushort_as_bfloat16(f2bf(s));
        a.resid_sum[out] = s;
      } else if constexpr (EPI == EPI_SWIGLU) {
        const float* ru = red + (st * RPS + r + PAIRS) * WPR;
        float up = 0.f;
#pragma unroll
        for (int w = 0; w < WPR; ++w) up += ru[w];
        const float g = rbf(v);
        const float silu = g / (1.0f + __expf(-g));
        a.y[out] = __ushort_as_bfloat16(f2bf(silu * rbf(up)));
      } else if constexpr (EPI == EPI_LOGITS_ARGMAX) {
        a.yf[out] = v;
        const unsigned long long packed =
            (static_cast<unsigned long long>(order_key(v)) << 32) |
            static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(out));
        best = best > packed ? best : packed;
      }
    }
    named_sync(1, kGemvConsumers);  // the next segment may overwrite `red`
  }
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
  }
}

template <int K, int STAGE_BYTES, int STAGES, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_stream_kernel(const GemvArgs a) {
  using G = GemvGeom<K, STAGE_BYTES>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
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
      gemv_produce<K, STAGE_BYTES, STAGES, EPI == EPI_SWIGLU>(ring, full, empty, it, a.w, a.n_out, o0, o1,
                                                          l2_policy_evict_first(), a.status);
      ring_drain<STAGES>(full, it, a.status);
    }
  } else {
    float xr[G::CPT][8];
    pdl_wait();
    gemv_load_x<K, STAGE_BYTES, PRO>(a, xr, xs, red8);
    int it = 0;
    unsigned long long best = 0ull;
    bool failed = false;
    gemv_consume<K, STAGE_BYTES, STAGES, EPI>(ring, full, empty, it, a, o0, o1, xr, red, best, failed);
    if constexpr (EPI == EPI_LOGITS_ARGMAX) {
      if (best != 0ull) atomicMax(cta_best, best);
    }
  }
  __syncthreads();
  if constexpr (EPI == EPI_LOGITS_ARGMAX) {
    if (tid == 0) argmax_finish(a, *cta_best);
  }
}

template <int K, int STAGE_BYTES, int STAGES>
constexpr size_t gemv_smem_bytes() {
  return static_cast<size_t>(STAGES) * STAGE_BYTES + 2 * STAGES * sizeof(uint64_t) + 8 +
         (8 + kGemvRedFloats) * sizeof(float) + 128 + static_cast<size_t>(K) * 2 + 64;
}

}  // namespace lcrb
