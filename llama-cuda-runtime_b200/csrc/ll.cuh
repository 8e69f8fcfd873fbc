// Low-latency exchange words for the persistent decode step.
//
// Between the phases of a step every CTA needs vectors that other CTAs
// produced (the q/k/v rows, the attention records, the residual sums, the
// SwiGLU output). Instead of storing them and meeting at a grid barrier --
// whose release fence waits for the SM's outstanding memory traffic, about a
// microsecond under the weight stream -- each value travels with a tag in the
// same single-copy-atomic word:
//
//   LL32  bits 31..16 the bf16 value, bits 15..0 the low 16 bits of the tag
//   LL64  bits 63..32 the fp32 value, bits 31..0 the tag
//
// The tag is the exchange's epoch (a per-step base plus the layer and phase),
// so a reader that sees the expected tag in a word has that word's value, and
// nothing else has to be ordered: writers use relaxed stores, readers poll
// with relaxed loads (16-byte vectors, each 32- or 64-bit element atomic on
// its own). A word is rewritten every layer, so the tag of a stale value is
// always a few epochs behind the expected one (16-bit tags wrap only after
// 65536 epochs). Every poll is bounded: after `wait_ns` it raises
// kStatusTimeoutBarrier | kStatusAbort and gives up, and it gives up at once
// when another CTA has raised kStatusAbort.
#pragma once

#include "common.cuh"

namespace lcrb {

__device__ __forceinline__ void st_relaxed_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_relaxed_v4(const void* p) {
  uint4 r;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}

__device__ __forceinline__ uint32_t ll32_word(float v, uint32_t tag) {
  return (static_cast<uint32_t>(f2bf(v)) << 16) | (tag & 0xffffu);
}
__device__ __forceinline__ unsigned long long ll64_word(float v, uint32_t tag) {
  return (static_cast<unsigned long long>(__float_as_uint(v)) << 32) | tag;
}
__device__ __forceinline__ float ll64_value(unsigned long long w) {
  return __uint_as_float(static_cast<uint32_t>(w >> 32));
}

// Replicas of each exchange buffer: writers store every replica and CTA c
// polls replica c % kLLCopies, so each line is polled by a quarter of the
// CTAs (with one replica the bs1 step measured 4-5 % slower).
constexpr int kLLCopies = 4;

// Bounded wait bookkeeping shared by the polls: true to keep waiting.
struct LLWait {
  uint32_t* status;
  uint64_t wait_ns;
  uint64_t start = 0;
  uint32_t spin = 0;
  __device__ __forceinline__ bool again() {
    if ((++spin & 31u) != 0u) return true;
    if (__ldcg(status) & kStatusAbort) return false;
    const uint64_t now = globaltimer_ns();
    if (start == 0) {
      start = now;
    } else if (now - start > wait_ns) {
      atomicOr(status, kStatusTimeoutBarrier | kStatusAbort);
      return false;
    }
    return true;
  }
};

// N 16-byte groups of words at addr(0) .. addr(N - 1), loaded together (one
// round trip when they are all there) until every word carries the tag:
// LL32 groups (four words) or, with W64, LL64 groups (two words: x, z the
// tags, y, w the values). `addr` recomputes the addresses on each attempt
// rather than holding N pointers in registers.
template <int N, bool W64, class Addr>
__device__ __forceinline__ bool ll_poll_groups(Addr addr, uint4 (&v)[N], uint32_t tag, LLWait& w) {
  const uint32_t t = tag & 0xffffu;
  for (;;) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = ld_relaxed_v4(addr(i));
    bool ok = true;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      if constexpr (W64) {
        ok &= (v[i].x == tag) & (v[i].z == tag);
      } else {
        ok &= ((v[i].x & 0xffffu) == t) & ((v[i].y & 0xffffu) == t) & ((v[i].z & 0xffffu) == t) &
              ((v[i].w & 0xffffu) == t);
      }
    }
    if (ok) return true;
    if (!w.again()) return false;
  }
}

// The bf16 values of two LL32 groups (8 words) as 8 packed bf16.
__device__ __forceinline__ uint4 ll32_values8(const uint4& a, const uint4& b) {
  uint4 out;
  out.x = (a.x >> 16) | (a.y & 0xffff0000u);
  out.y = (a.z >> 16) | (a.w & 0xffff0000u);
  out.z = (b.x >> 16) | (b.y & 0xffff0000u);
  out.w = (b.z >> 16) | (b.w & 0xffff0000u);
  return out;
}

}  // namespace lcrb
