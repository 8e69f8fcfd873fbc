// Instantiations and launch of the causal prefill attention.
#include "attn_prefill.h"
#include "attn_prefill_tc.cuh"

namespace lcrb {
namespace {

template <int D, int G>
int launch_t(const PrefillAttnArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap, int kv_heads,
             cudaStream_t s) {
  auto kernel = attn_prefill_kernel<D, G>;
  constexpr size_t smem = attn_prefill_smem_bytes<D>();
  LCRB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  const int pairs = (a.count + 15) / 16 * G;
  const dim3 grid(static_cast<unsigned>(kv_heads),
                  static_cast<unsigned>((pairs + kAttnConsumerWarps - 1) / kAttnConsumerWarps));
  return launch_kernel(kernel, grid, dim3(kAttnThreads), smem, s, true, a, kmap, vmap);
}

// head_dim 64: the tcgen05 kernel, 128 query rows (128 / G queries x G heads)
// per CTA, heaviest blocks first.
template <int G>
int launch_tc(const PrefillAttnArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap, int kv_heads,
              cudaStream_t s) {
  auto kernel = attn_prefill_tc_kernel<G>;
  constexpr size_t smem = attn_prefill_tc_smem_bytes();
  LCRB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  constexpr int QB = 128 / G;
  const dim3 grid(static_cast<unsigned>(kv_heads), static_cast<unsigned>((a.count + QB - 1) / QB));
  return launch_kernel(kernel, grid, dim3(kApTcThreads), smem, s, true, a, kmap, vmap);
}

template <int D>
int by_group(const PrefillAttnArgs& a, const CUtensorMap& k, const CUtensorMap& v, int group, int kv_heads,
             cudaStream_t s) {
  switch (group) {
    case 1: return launch_t<D, 1>(a, k, v, kv_heads, s);
    case 2: return launch_t<D, 2>(a, k, v, kv_heads, s);
    case 4: return launch_t<D, 4>(a, k, v, kv_heads, s);
    case 8: return launch_t<D, 8>(a, k, v, kv_heads, s);
    default:
      return fail(LCR_ERR_SHAPE,
                  "prefill attention is compiled for 1, 2, 4 or 8 query heads per KV head, this model has %d",
                  group);
  }
}

}  // namespace

int attn_prefill_launch(const PrefillAttnArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap, int head_dim,
                        int group, int kv_heads, cudaStream_t s) {
  // Keys are fetched 16 positions at a time from the page of the first, so
  // pages hold a multiple of 16 -- except a single page holding every
  // position (a contiguous cache): its last fetch may run past the page, into
  // rows of keys after every query (masked) or past the pool (zero fill).
  const bool one_page = a.pool_pages == 1 && a.start + a.count <= a.page_size;
  LCRB_REQUIRE(a.count >= 1 && a.start >= 0 && (a.page_size % kAbUnit == 0 || one_page), LCR_ERR_SHAPE,
               "prefill attention: unsupported chunk (%d rows at %d, page size %d)", a.count, a.start, a.page_size);
  if (head_dim == 64) {
    switch (group) {
      case 1: return launch_tc<1>(a, kmap, vmap, kv_heads, s);
      case 2: return launch_tc<2>(a, kmap, vmap, kv_heads, s);
      case 4: return launch_tc<4>(a, kmap, vmap, kv_heads, s);
      case 8: return launch_tc<8>(a, kmap, vmap, kv_heads, s);
      default: return by_group<64>(a, kmap, vmap, group, kv_heads, s);
    }
  }
  if (head_dim == 128) return by_group<128>(a, kmap, vmap, group, kv_heads, s);
  return fail(LCR_ERR_SHAPE, "prefill attention is compiled for head_dim 64 or 128, this model has %d", head_dim);
}

}  // namespace lcrb
