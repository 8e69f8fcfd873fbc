// Host launcher of the causal prefill attention (attn_prefill.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "attn_prefill.cuh"

namespace lcrb {

// Attention of a prompt chunk (a.count rows at positions a.start ..) over
// the sequence's pages, keys 0 .. a.start + a.count - 1 all read from the
// cache (the chunk's own rows written first by kv_write_kernel): kmap / vmap
// as for attn_batch_launch; page_size a multiple of 16. One programmatic
// launch.
int attn_prefill_launch(const PrefillAttnArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap, int head_dim,
                        int group, int kv_heads, cudaStream_t s);

}  // namespace lcrb
