// Shared device helpers for the sm_100a kernels: bf16 conversions, the
// mbarrier / bulk-copy (TMA, non-tensor) / programmatic-dependent-launch PTX
// wrappers, bounded waits, and host-side status plumbing for the C ABI.
#pragma once

#include <cuda.h>  // CUtensorMap (type only; the encoder is reached through cudart)
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "lcr_b200.h"

namespace lcrb {

// ---------------------------------------------------------------------------
// Host status plumbing
// ---------------------------------------------------------------------------

// Records a formatted message for lcr_last_error_string() on this thread and
// returns `status`, so call sites read `return fail(LCR_ERR_SHAPE, ...)`.
int fail(int status, const char* fmt, ...);
// cudaGetLastError() after a launch -> LCR_OK or LCR_ERR_CUDA.
int launch_status(const char* what);

#define LCRB_REQUIRE(cond, status, ...)                 \
  do {                                                  \
    if (!(cond)) return ::lcrb::fail((status), __VA_ARGS__); \
  } while (0)

#define LCRB_CUDA(expr)                                                     \
  do {                                                                      \
    cudaError_t e_ = (expr);                                                \
    if (e_ != cudaSuccess)                                                  \
      return ::lcrb::fail(LCR_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,     \
                          cudaGetErrorString(e_), __FILE__, __LINE__);      \
  } while (0)

// Whether `p` is memory that device `device` may read: device memory of that
// device (or managed / host-mapped memory). Weights on another GPU would
// otherwise surface as an illegal access inside the first kernel.
inline bool on_device(const void* p, int device) {
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (attr.type == cudaMemoryTypeDevice) return attr.device == device;
  return attr.type == cudaMemoryTypeManaged || attr.type == cudaMemoryTypeHost;
}

#define LCRB_TRY(expr)            \
  do {                            \
    int s_ = (expr);              \
    if (s_ != LCR_OK) return s_;  \
  } while (0)

// Device status word bits (written with atomicOr, read by the host).
enum : uint32_t {
  kStatusTimeoutFull = 1u << 0,   // consumer gave up waiting for a stage
  kStatusTimeoutEmpty = 1u << 1,  // producer gave up waiting for a free slot
  kStatusBadToken = 1u << 2,      // token id outside the vocabulary
  kStatusBadPosition = 1u << 3,   // position outside the cache
  kStatusBadPage = 1u << 4,       // page table entry outside the pool
  kStatusTimeoutBarrier = 1u << 5,  // a grid barrier gave up
  kStatusBadSmem = 1u << 6,       // ring not 1024-byte aligned for swizzled tensor copies
  kStatusAbort = 1u << 8,         // a CTA stopped; the others stop at their next wait
};

// ---------------------------------------------------------------------------
// bf16
// ---------------------------------------------------------------------------

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
// Round through bf16 and back: the value a bf16 store would hold.
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  return static_cast<uint32_t>(f2bf(lo)) | (static_cast<uint32_t>(f2bf(hi)) << 16);
}

// Eight bf16 from a 16-byte word, widened to fp32.
__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  f[0] = bf_lo(v.x); f[1] = bf_hi(v.x);
  f[2] = bf_lo(v.y); f[3] = bf_hi(v.y);
  f[4] = bf_lo(v.z); f[5] = bf_hi(v.z);
  f[6] = bf_lo(v.w); f[7] = bf_hi(v.w);
}

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// Plain 16-byte load.
__device__ __forceinline__ uint4 ldg16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}
// 16-byte load cached in L2 only: for activations other CTAs of the same
// kernel may have rewritten since this SM last read them (L1 is not coherent).
__device__ __forceinline__ uint4 ldg_cg16(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}

// ---------------------------------------------------------------------------
// Shared memory, mbarriers, bulk copies
// ---------------------------------------------------------------------------

// Rounds a shared-memory pointer up to `align` bytes (a power of two): every
// region read with 16-byte vector accesses starts on such a boundary.
template <typename T>
__device__ __forceinline__ T* align_smem(void* p, uintptr_t align) {
  return reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(p) + align - 1) & ~(align - 1));
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}
// Makes initialised mbarriers visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bound on every device-side wait. A wait that has not completed after this
// long reports through the status word and the kernel unwinds instead of
// spinning forever.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Waits for an mbarrier phase; false (and a status bit) if the bound expired,
// or -- without a new bit -- once another CTA raised the abort bit (a
// stopped step then unwinds at once instead of waiting out every bound).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status,
                                          uint32_t code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255u) == 255u) {
      if (status && (__ldcg(status) & (1u << 8))) return false;  // kStatusAbort
      if (globaltimer_ns() - start > kWaitLimitNs) {
        if (status) atomicOr(status, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 1-D bulk copy global -> shared (the TMA engine, no tensor map), completing
// on an mbarrier's transaction count. dst, src and bytes must be 16-byte
// aligned / multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Tiled tensor copies global -> shared (TMA with a tensor map in global or
// param memory), completing on an mbarrier's transaction count, L2 hint as
// for bulk_g2s. No cluster multicast. The innermost coordinate is always 0
// here (whole 64-element chunks), so every copy starts 16-byte aligned.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// One 128-byte L2 line through the load/store path (not the TMA queue).
__device__ __forceinline__ void prefetch_line_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch
// ---------------------------------------------------------------------------

// Blocks until the grid this kernel depends on has completed and its memory
// is visible. Everything before it may only touch data the previous kernel
// does not write (weights, the KV history, device state fixed for the step).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream start launching its CTAs.
__device__ __forceinline__ void pdl_launch_next() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launches kernel<<<grid, block, smem, stream>>>(args) -- with programmatic
// stream serialization when `pdl`, so that the kernel may start while its
// predecessor finishes (it must pdl_wait() before touching that
// predecessor's outputs, or anything a still-running kernel writes).
template <class... Params, class... Args>
inline int launch_kernel(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                         Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  return e == cudaSuccess ? LCR_OK : fail(LCR_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
}

// Named barrier over the first `threads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Barrier over the first `threads` threads that also ORs a predicate across them.
__device__ __forceinline__ bool named_sync_or(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred p, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;
// Online-softmax identity (the reference's kSoftmaxNegInf, reduce.cuh:15):
// -FLT_MAX subtracts from itself to zero and exponentiates to zero.
constexpr float kNegBig = -3.402823466e+38f;

}  // namespace lcrb
