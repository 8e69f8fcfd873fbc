// Batched paged decode attention on the tensor pipe: the attention node of
// the continuous-batching step (batch_ctx.cu), replacing
// decode_attention_kernel + merge_splits_kernel (src/kernels/attention.cu:
// 110-299) and the cache write of rope_write_kv_kernel (src/kernels/rope.cu:
// 58-87). q and the new key arrive already rotated (the QKV projection's
// RoPE epilogue); the new K/V row is written to the cache at each sequence's
// position and attention runs over positions 0..position.
//
// Persistent CTAs (as many as fit) take work items -- up to item_pos
// positions of one (sequence, KV head) -- from a counter in global memory.
// Warps:
//   producer   (warp 4) per stage, four 16-position units of K and of V, each
//              one TMA tensor copy of a {64, 16, D / 64} box out of the
//              layer's pool viewed as rows of D elements (row = (page *
//              kv_heads + kv_head) * page_size + slot), landing [D / 64][16]
//              [128 bytes] with the 128-byte swizzle, so ldmatrix rows fall in
//              distinct banks. With an item's first stage it also copies the
//              group's q (G x D, contiguous in the QKV row) into the stage's
//              q slot.
//   consumers  (warps 0-3) warp w owns unit w of every stage. The G query
//              heads of the group are MMA rows 0..G-1 (rows G..15 are zero):
//                S = Q K^T       m16n8k16, bf16 q (rotated and rounded as the
//                                reference stores it) x bf16 K, fp32 sums
//                online softmax  per head in the log2 domain, fp32
//                O += P V        P rounded to bf16 (weights in [0, 1]); the
//                                denominator sums the same rounded weights
//              V fragments come from ldmatrix.trans of the [position][dim]
//              rows. The unit holding the new position is patched in shared
//              memory after its copy lands (key, value, zeroed rows past the
//              sequence), and its key/value go to the cache. At an
//              item's end each warp hands its (m, l, O) record to the
//              finisher through a double-buffered record area.
//   finisher   (warp 5) combines the four records (the logsumexp rule) and
//              writes the item's output, or its split partial, so the
//              consumers never wait on global memory.
// Sequences whose cache spans several items are finished by
// attn_batch_merge_kernel, launched next, which merges each head's split
// partials (merge_splits_kernel, src/kernels/attention.cu:267-299).
#pragma once

#include "attention.cuh"
#include "gemv.cuh"  // ldmatrix_x4, mma_x_rows

namespace lcrb {

constexpr int kAbUnit = 16;  // positions per tensor copy and per warp per stage

template <int D>
struct AbGeom {
  static_assert(D % 64 == 0, "head_dim in 128-byte chunks");
  static constexpr int CHUNK = kAbUnit * 128;                 // [16 rows][128 bytes]
  static constexpr int UNIT = kAbUnit * D * 2;                // one K (or V) unit
  static constexpr int STAGE = 2 * kAttnConsumerWarps * UNIT;  // K units, then V units
  static constexpr int STAGES = D == 64 ? 4 : 2;
  static constexpr int RING = STAGES * STAGE;
};

// Ring, barriers, stage records (32 bytes each), rotated q, warp records.

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// Byte offset of 16-byte piece `piece` (0 .. D/8 - 1) of row `r` in a unit.
__device__ __forceinline__ uint32_t ab_offset(int r, int piece) {
  return static_cast<uint32_t>((piece >> 3) * (kAbUnit * 128) + r * 128 + (((piece & 7) ^ (r & 7)) << 4));
}

// The sequence's new position, row r of the unit in kst / vst: write its
// (already rotated) key and its value to the cache and into the unit, and
// zero the value rows past it so that their zero weights meet finite values.
// One warp.
template <int D>
__device__ __forceinline__ void ab_new_position(const AttnArgs& a, int b, int kvh, int pos, int r, uint8_t* kst,
                                                uint8_t* vst, int lane) {
  constexpr int PIECES = D / 8;
  const bf16* row = a.qkv + static_cast<size_t>(b) * a.qkv_stride;
  const int32_t* table = a.tables + static_cast<size_t>(b) * a.table_seq_stride;
  int page = table[pos / a.page_size];
  if (page < 0 || page >= a.pool_pages) page = 0;  // flagged by the producer
  const long long off = static_cast<long long>(page) * a.page_stride + kvh * a.head_stride +
                        static_cast<long long>(pos % a.page_size) * D;
  for (int piece = lane; piece < PIECES; piece += 32) {
    const uint4 kw = ldg_cg16(row + a.q_dim + kvh * D + piece * 8);
    const uint4 vw = ldg_cg16(row + a.q_dim + a.kv_dim + kvh * D + piece * 8);
    *reinterpret_cast<uint4*>(a.kpool + off + piece * 8) = kw;
    *reinterpret_cast<uint4*>(a.vpool + off + piece * 8) = vw;
    *reinterpret_cast<uint4*>(kst + ab_offset(r, piece)) = kw;
    *reinterpret_cast<uint4*>(vst + ab_offset(r, piece)) = vw;
  }
  for (int i = lane; i < (kAbUnit - 1 - r) * PIECES; i += 32) {
    *reinterpret_cast<uint4*>(vst + ab_offset(r + 1 + i / PIECES, i % PIECES)) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// One ring stage's work, written by the producer before it arrives on the
// stage's full barrier.
struct AbMeta {
  int item;   // sequence | kv_head << 8 | split << 16 | splits << 24
  int p0;     // first position of the stage
  int units;  // 16-position units in the stage (1..4); 0: no more work
  int flags;  // kAbFirst / kAbLast: the item's first / last stage
};
constexpr int kAbFirst = 1, kAbLast = 2;
constexpr int kAbMaxSeqs = 256;   // sequences per launch (8-bit field)
constexpr int kAbMaxSplits = 127; // partial slots per head (7-bit field)
constexpr int kAbWarps = kAttnConsumerWarps + 2;  // + producer, finisher
constexpr int kAbThreads = kAbWarps * 32;

// Shared memory of attn_batch_kernel from its 1024-byte aligned base; the
// per-sequence tables at the end are sized by the launch's sequence count.
template <int D, int G>
struct AbSmem {
  using Geo = AbGeom<D>;
  static constexpr int S = Geo::STAGES;
  static constexpr int REC = G * (D + 2);  // one warp's record: per head m, l, O[D]
  static constexpr size_t BARS = Geo::RING;                       // full[S], empty[S], rec_full[2], rec_empty[2]
  static constexpr size_t META = BARS + (2 * S + 4) * 8;          // AbMeta[S]
  static constexpr size_t QS = META + S * sizeof(AbMeta);         // bf16 [S][G][D]
  static constexpr size_t RECS = QS + static_cast<size_t>(S) * G * D * 2;  // float [2][warps][REC]
  static constexpr size_t INFO = RECS + 2 * kAttnConsumerWarps * REC * 4;   // int [2]: packed item, or -1
  static constexpr size_t CUM = INFO + 16;                        // int [n + 1], then int [n] positions
  static_assert(QS % 16 == 0 && RECS % 16 == 0, "16-byte aligned q slots and records");
};

template <int D, int G>
constexpr size_t attn_batch_smem_bytes(int seqs) {
  return AbSmem<D, G>::CUM + (2 * static_cast<size_t>(seqs) + 1) * 4;
}

template <int D, int G>
__global__ void __launch_bounds__(kAbThreads, D == 64 ? 3 : 1)
    attn_batch_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap) {
  using Geo = AbGeom<D>;
  using L = AbSmem<D, G>;
  constexpr int STAGES = Geo::STAGES;
  constexpr int UNIT = Geo::UNIT;
  constexpr int KSTEPS = D / 16;
  constexpr int NT = D / 8;  // n-tiles of the output
  constexpr int REC = L::REC;
  static_assert(G >= 1 && G <= 8, "the group's query heads are MMA rows 0..7");

  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BARS);
  uint64_t* empty = full + STAGES;
  uint64_t* rec_full = empty + STAGES;
  uint64_t* rec_empty = rec_full + 2;
  AbMeta* meta = reinterpret_cast<AbMeta*>(smem + L::META);
  bf16* qslots = reinterpret_cast<bf16*>(smem + L::QS);
  float* recs = reinterpret_cast<float*>(smem + L::RECS);
  int* info = reinterpret_cast<int*>(smem + L::INFO);
  const int n = a.seqs;
  int* cum = reinterpret_cast<int*>(smem + L::CUM);
  int* pos_s = cum + n + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int num_kv = a.kv_dim / D;

  if ((smem_addr(smem) & 1023u) != 0) {
    // Swizzled tensor copies need a 1024-byte aligned ring: report, and still
    // count this CTA out so that the work counters are rearmed.
    if (tid == 0) {
      if (a.status) atomicOr(a.status, kStatusBadSmem);
      if (atomicAdd(&a.work[1], 1u) == gridDim.x - 1) {
        a.work[0] = 0u;
        a.work[1] = 0u;
      }
    }
    return;
  }

  if (warp == 0) {
    // Items per sequence: kv_heads x ceil((position + 1) / item_pos); an
    // exclusive scan over the batch (each lane a contiguous run).
    const int per = (n + 31) / 32;
    const int s0 = min(n, lane * per), s1 = min(n, s0 + per);
    int sum = 0;
    for (int q = s0; q < s1; ++q) {
      const int p = a.positions[q];
      const bool ok = p >= 0 && p < a.max_seq && p / a.page_size < a.max_pages;
      if (!ok && blockIdx.x == 0 && a.status) atomicOr(a.status, kStatusBadPosition);
      pos_s[q] = ok ? p : -1;
      sum += ok ? (p + a.item_pos) / a.item_pos * num_kv : 0;
    }
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int run = incl - sum;
    for (int q = s0; q < s1; ++q) {
      cum[q] = run;
      run += pos_s[q] >= 0 ? (pos_s[q] + a.item_pos) / a.item_pos * num_kv : 0;
    }
    if (lane == 31) cum[n] = incl;
    if (lane == 0) {
      for (int q = 0; q < STAGES; ++q) {
        mbar_init(&full[q], 1);
        mbar_init(&empty[q], kAttnConsumerWarps);
      }
      for (int q = 0; q < 2; ++q) {
        mbar_init(&rec_full[q], kAttnConsumerWarps);
        mbar_init(&rec_empty[q], 1);
      }
      mbar_fence_init();
    }
  }
  __syncthreads();
  const int total = cum[n];

  if (warp == kAttnConsumerWarps) {
    // ---------------------------------------------------------------- producer
    // Items come from the shared counter, the next index fetched while the
    // current item issues. Pages of 32 units are looked up at a time (one
    // per lane); lane 0 waits for slots and issues the copies.
    pdl_wait();  // q comes from the preceding projection
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    const uint64_t policy = l2_policy_evict_first();
    unsigned nxt = 0;
    if (lane == 0) nxt = atomicAdd(&a.work[0], 1u);
    int cur = __shfl_sync(0xffffffffu, static_cast<int>(nxt), 0);
    int st = 0;
    bool ok = true;
    while (ok && cur < total) {
      if (lane == 0) nxt = atomicAdd(&a.work[0], 1u);
      int lo = 0, hi = n;  // the sequence: last b with cum[b] <= cur
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (cum[mid] <= cur) lo = mid;
        else hi = mid;
      }
      const int b = lo;
      const int pos = pos_s[b];
      const int splits = (pos + a.item_pos) / a.item_pos;
      const int r = cur - cum[b];
      const int kvh = r / splits, split = r % splits;
      const int begin = split * a.item_pos;
      const int units = (min(pos + 1, begin + a.item_pos) - begin + kAbUnit - 1) / kAbUnit;
      const int nst = (units + kAttnConsumerWarps - 1) / kAttnConsumerWarps;
      const int32_t* table = a.tables + static_cast<size_t>(b) * a.table_seq_stride;
      int row_mine = 0;
      for (int k = 0; k < nst; ++k, ++st) {
        const int u0 = k * kAttnConsumerWarps;
        if (u0 % 32 == 0 && u0 + lane < units) {
          const int p = begin + (u0 + lane) * kAbUnit;  // a multiple of 16: the unit lies in one page
          int page = table[p / a.page_size];
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
        const int cnt = min(kAttnConsumerWarps, units - u0);
        int rows[kAttnConsumerWarps];
#pragma unroll
        for (int u = 0; u < kAttnConsumerWarps; ++u) rows[u] = __shfl_sync(0xffffffffu, row_mine, (u0 + u) & 31);
        if (lane == 0) {
          AbMeta& m = meta[slot];
          m.item = b | (kvh << 8) | (split << 16) | (splits << 24);
          m.p0 = begin + u0 * kAbUnit;
          m.units = cnt;
          m.flags = (k == 0 ? kAbFirst : 0) | (k == nst - 1 ? kAbLast : 0);
          uint8_t* dst = ring + slot * Geo::STAGE;
          constexpr uint32_t QBYTES = G * D * 2;
          mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(cnt) * 2 * UNIT + (k == 0 ? QBYTES : 0u));
          if (k == 0) {  // the group's q heads, contiguous in the QKV row
            bulk_g2s(qslots + static_cast<size_t>(slot) * G * D,
                     a.qkv + static_cast<size_t>(b) * a.qkv_stride + kvh * G * D, QBYTES, &full[slot]);
          }
#pragma unroll
          for (int u = 0; u < kAttnConsumerWarps; ++u) {
            if (u < cnt) {
              tma_load_3d(dst + u * UNIT, &kmap, 0, rows[u], 0, &full[slot], policy);
              tma_load_3d(dst + (kAttnConsumerWarps + u) * UNIT, &vmap, 0, rows[u], 0, &full[slot], policy);
            }
          }
        }
      }
      cur = __shfl_sync(0xffffffffu, static_cast<int>(nxt), 0);
    }
    pdl_launch_next();  // the merge kernel may start launching
    if (ok) {  // the end-of-work stage: no copies, a plain arrive
      const int slot = st % STAGES;
      if (lane == 0 && st >= STAGES) {
        ok = mbar_wait(&empty[slot], ((st / STAGES) - 1) & 1, a.status, kStatusTimeoutEmpty);
      }
      if (lane == 0 && ok) {
        meta[slot].units = 0;
        mbar_arrive(&full[slot]);
      }
      ++st;
    }
    if (lane == 0) {
      // Never leave the CTA with a copy still writing its shared memory.
      for (int q = st > STAGES ? st - STAGES : 0; q < st; ++q) {
        mbar_wait(&full[q % STAGES], (q / STAGES) & 1, nullptr, 0);  // waits even after an abort
      }
      // The last CTA to finish rearms the counters for the next launch.
      __threadfence();
      if (atomicAdd(&a.work[1], 1u) == gridDim.x - 1) {
        a.work[0] = 0u;
        a.work[1] = 0u;
      }
    }
    return;
  }

  if (warp == kAttnConsumerWarps + 1) {
    // ---------------------------------------------------------------- finisher
    const int heads = num_kv * G;
    pdl_wait();  // its outputs are read by kernels that ran before this one
    for (int k = 0;; ++k) {
      const int buf = k & 1;
      if (!mbar_wait(&rec_full[buf], (k >> 1) & 1, a.status, kStatusTimeoutFull)) break;
      const int item = info[buf];
      if (item < 0) break;
      const int b = item & 255, kvh = (item >> 8) & 255, split = (item >> 16) & 255, splits = item >> 24;
      const float* rec = recs + buf * kAttnConsumerWarps * REC;
      for (int idx = lane; idx < G * D; idx += 32) {
        const int g = idx / D, d = idx % D;
        float M = kNegBig;
#pragma unroll
        for (int w = 0; w < kAttnConsumerWarps; ++w) M = fmaxf(M, rec[w * REC + g * (D + 2)]);
        float Lsum = 0.f, A = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnConsumerWarps; ++w) {
          const float* c = rec + w * REC + g * (D + 2);
          const float sc = ex2_approx(c[0] - M);
          Lsum += c[1] * sc;
          A += c[2 + d] * sc;
        }
        const int h = kvh * G + g;
        if (splits == 1) {
          a.out[static_cast<size_t>(b) * heads * D + h * D + d] =
              __ushort_as_bfloat16(f2bf(Lsum > 0.f ? A / Lsum : 0.f));
        } else {
          float* slotp = a.partials + ((static_cast<size_t>(b) * heads + h) * a.splits + split) * (2 + D);
          if (d == 0) {
            slotp[0] = M;
            slotp[1] = Lsum;
          }
          slotp[2 + d] = A;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rec_empty[buf]);
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  // Each warp runs on its own: its waits are on mbarriers, never on a
  // barrier shared with the other consumer warps.
  const int g = lane >> 2, t = lane & 3;  // MMA row (query head) and column pair
  // ldmatrix lane roles: tile mi = lane / 8, row lane % 8 of that tile.
  const int lrow = lane & 7, mi = lane >> 3;
  const int k_row = (mi >> 1) * 8 + lrow;  // K: tiles (pos 0-7, lo), (0-7, hi), (8-15, lo), (8-15, hi)
  const int v_row = (mi & 1) * 8 + lrow;   // V: tiles (pos 0-7, dims c), (8-15, c), (0-7, c+1), (8-15, c+1)
  uint32_t qa0[KSTEPS], qa2[KSTEPS];  // A fragments of q (rows 8-15 are zero)
  float o[NT][4];
  float m_run = kNegBig, l_run = 0.f;
  int pos = 0, items = 0;
  pdl_wait();  // the new key / value rows come from the QKV projection

  for (int st = 0;; ++st) {
    const int slot = st % STAGES;
    const bool got = mbar_wait(&full[slot], (st / STAGES) & 1, a.status, kStatusTimeoutFull);
    const AbMeta m = meta[slot];
    if (!got || m.units == 0) {
      // No more work: tell the finisher.
      const int buf = items & 1;
      if (items < 2 || mbar_wait(&rec_empty[buf], ((items >> 1) - 1) & 1, a.status, kStatusTimeoutEmpty)) {
        if (lane == 0) {
          info[buf] = -1;
          mbar_arrive(&rec_full[buf]);
        }
      }
      break;
    }
    const int b = m.item & 255, kvh = (m.item >> 8) & 255;
    if (m.flags & kAbFirst) {
      pos = pos_s[b];
      const bf16* qd = qslots + static_cast<size_t>(slot) * G * D;
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        qa0[kk] = g < G ? *reinterpret_cast<const uint32_t*>(qd + g * D + 16 * kk + 2 * t) : 0u;
        qa2[kk] = g < G ? *reinterpret_cast<const uint32_t*>(qd + g * D + 16 * kk + 8 + 2 * t) : 0u;
      }
#pragma unroll
      for (int nn = 0; nn < NT; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
      m_run = kNegBig;
      l_run = 0.f;
    }
    if (warp < m.units) {
      const int p0 = m.p0 + warp * kAbUnit;
      uint8_t* kst = ring + slot * Geo::STAGE + warp * UNIT;
      uint8_t* vst = kst + kAttnConsumerWarps * UNIT;
      const int nvalid = min(kAbUnit, pos + 1 - p0);
      if (pos >= p0 && pos < p0 + kAbUnit) {
        ab_new_position<D>(a, b, kvh, pos, pos - p0, kst, vst, lane);
        __syncwarp();
      }
      const uint32_t ks = smem_addr(kst), vs = smem_addr(vst);
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        uint32_t kb[4];
        ldmatrix_x4(kb, ks + ab_offset(k_row, 2 * kk + (mi & 1)));
        mma_x_rows(s[0], qa0[kk], qa2[kk], kb[0], kb[1]);
        mma_x_rows(s[1], qa0[kk], qa2[kk], kb[2], kb[3]);
      }
      // Row g's scores at unit positions 8 j + 2 t + e.
      float sc[2][2];
      float mx = kNegBig;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool live = 8 * j + 2 * t + e < nvalid;
          sc[j][e] = live ? s[j][e] * a.scale_log2 : kNegBig;
          mx = fmaxf(mx, sc[j][e]);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m_run, mx);
      const float alpha = ex2_approx(m_run - mn);
      float pr[2][2];
      float psum = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool live = 8 * j + 2 * t + e < nvalid;
          pr[j][e] = live ? rbf(ex2_approx(sc[j][e] - mn)) : 0.f;
          psum += pr[j][e];
        }
      }
      l_run = l_run * alpha + psum;
      m_run = mn;
#pragma unroll
      for (int nn = 0; nn < NT; ++nn) {
        o[nn][0] *= alpha;
        o[nn][1] *= alpha;
      }
      const uint32_t pa0 = pack_bf2(pr[0][0], pr[0][1]), pa2 = pack_bf2(pr[1][0], pr[1][1]);
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        uint32_t vb[4];
        ldmatrix_x4_trans(vb, vs + ab_offset(v_row, 2 * c + (mi >> 1)));
        mma_x_rows(o[2 * c], pa0, pa2, vb[0], vb[1]);
        mma_x_rows(o[2 * c + 1], pa0, pa2, vb[2], vb[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);

    if (m.flags & kAbLast) {
      // This warp's record (the quad holds row g's columns 2 t, 2 t + 1 of
      // each tile) to the finisher.
      float l_q = l_run + __shfl_xor_sync(0xffffffffu, l_run, 1);
      l_q += __shfl_xor_sync(0xffffffffu, l_q, 2);
      const int buf = items & 1;
      const bool free_ok =
          items < 2 || mbar_wait(&rec_empty[buf], ((items >> 1) - 1) & 1, a.status, kStatusTimeoutEmpty);
      if (free_ok) {
        float* c = recs + (buf * kAttnConsumerWarps + warp) * REC;
        if (g < G) {
          c += g * (D + 2);
          if (t == 0) {
            c[0] = m_run;
            c[1] = l_q;
          }
#pragma unroll
          for (int nn = 0; nn < NT; ++nn) {
            c[2 + 8 * nn + 2 * t] = o[nn][0];
            c[2 + 8 * nn + 2 * t + 1] = o[nn][1];
          }
        }
        if (lane == 0) info[buf] = m.item;
        __syncwarp();
        if (lane == 0) mbar_arrive(&rec_full[buf]);
      }
      ++items;
    }
  }
}

// Merges the split partials of every (sequence, query head) whose cache
// spans more than one work item; one CTA of D threads per pair.
template <int D>
__global__ void __launch_bounds__(D) attn_batch_merge_kernel(const AttnArgs a) {
  const int heads = (a.q_dim / D);
  const int b = blockIdx.x / heads, h = blockIdx.x % heads, d = threadIdx.x;
  pdl_wait();
  pdl_launch_next();
  const int p = a.positions[b];
  if (!(p >= 0 && p < a.max_seq && p / a.page_size < a.max_pages)) return;
  const int splits = (p + a.item_pos) / a.item_pos;
  if (splits == 1) return;
  const float* base = a.partials + (static_cast<size_t>(b) * heads + h) * a.splits * (2 + D);
  float M = kNegBig;
#pragma unroll 4
  for (int q = 0; q < splits; ++q) M = fmaxf(M, base[q * (2 + D)]);
  float Lsum = 0.f, A = 0.f;
#pragma unroll 4
  for (int q = 0; q < splits; ++q) {
    const float sc = ex2_approx(base[q * (2 + D)] - M);
    Lsum += base[q * (2 + D) + 1] * sc;
    A += base[q * (2 + D) + 2 + d] * sc;
  }
  a.out[static_cast<size_t>(b) * heads * D + h * D + d] = __ushort_as_bfloat16(f2bf(Lsum > 0.f ? A / Lsum : 0.f));
}

}  // namespace lcrb
