// Decode attention that allocates nothing: the split partials live in a
// file-scope device array instead of caller scratch. It runs the same kernels
// as lcr_decode_attention (attention kernel + split merge) on that array.
//
// Set-up: the first call on each device (with that device current) looks the
// array's address up with cudaGetSymbolAddress, which may load this library's
// device code; make that first call before any stream capture. Later calls
// read the cached address and then launch exactly what lcr_decode_attention
// launches.
//
// The cached address belongs to the device's context at the time of the
// first call: after cudaDeviceReset (or anything else that destroys and
// re-creates that context) the library's device code is loaded again and the
// array may move, so do not use this entry point across a reset.
//
// Sharing: every call on a device uses the same array. Each split writes its
// whole (m, l, acc) record before the merge reads it, so nothing has to start
// at zero, but two calls whose kernels can overlap (different streams, or
// different host threads on one stream without ordering) race on the array.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "lcr_b200.h"

namespace {

constexpr int kMaxDevices = 64;

// num_heads x splits x (head_dim + 2) floats: 2 MiB, e.g. 32 heads x 64
// splits at head_dim 128, or 32 heads x 64 splits x 66 at head_dim 64.
static __device__ __align__(256) float g_partials[LCR_NOALLOC_ATTENTION_SCRATCH_FLOATS];

std::mutex g_mutex;
float* g_address[kMaxDevices] = {};

int partials_address(float** out) {
  int dev = -1;
  LCRB_CUDA(cudaGetDevice(&dev));
  LCRB_REQUIRE(dev >= 0 && dev < kMaxDevices, LCR_ERR_INVALID,
               "decode attention without allocation supports device ordinals below %d, got %d",
               kMaxDevices, dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_address[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_partials);
    if (e != cudaSuccess || !p) {
      return lcrb::fail(LCR_ERR_CUDA, "cudaGetSymbolAddress of the static attention partials "
                                      "on device %d failed: %s", dev, cudaGetErrorString(e));
    }
    g_address[dev] = static_cast<float*>(p);
  }
  *out = g_address[dev];
  return LCR_OK;
}

}  // namespace

extern "C" int lcr_decode_attention_noalloc(void* out, const void* q, const lcr_kv_view* view,
                                            int num_heads, int heads_per_kv, int seq_len,
                                            float scale, int paged, int splits,
                                            lcr_stream_t stream) {
  LCRB_REQUIRE(view != nullptr, LCR_ERR_INVALID, "decode attention: null pointer");
  LCRB_REQUIRE(seq_len > 0, LCR_ERR_INVALID, "decode attention needs at least one cached position");
  LCRB_REQUIRE(splits >= 1, LCR_ERR_INVALID, "split count must be positive, got %d", splits);
  LCRB_REQUIRE(num_heads > 0 && view->head_dim > 0, LCR_ERR_INVALID,
               "decode attention: %d heads of dimension %d", num_heads, view->head_dim);
  // The split count lcr_decode_attention actually launches: no split shorter
  // than one 16-position block.
  const long long used = std::min<long long>(splits, (seq_len + 15) / 16);
  const long long need = used > 1 ? static_cast<long long>(num_heads) * used * (2 + view->head_dim) : 0;
  LCRB_REQUIRE(need <= LCR_NOALLOC_ATTENTION_SCRATCH_FLOATS, LCR_ERR_SHAPE,
               "decode attention without allocation: %d heads x %lld splits x (head_dim %d + 2) = "
               "%lld partial floats exceeds the static %d; use fewer splits or "
               "lcr_decode_attention with caller scratch",
               num_heads, used, view->head_dim, need, LCR_NOALLOC_ATTENTION_SCRATCH_FLOATS);
  float* partials = nullptr;
  LCRB_TRY(partials_address(&partials));
  return lcr_decode_attention(out, q, view, num_heads, heads_per_kv, seq_len, scale, paged, splits,
                              partials, stream);
}
