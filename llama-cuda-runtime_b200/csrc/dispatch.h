// Host launchers of the decode-attention and sampling kernels
// (attention_dispatch.cu).
#pragma once

#include <cuda_runtime.h>

#include "attention.cuh"
#include "sampling.cuh"

namespace lcrb {

constexpr int kAttnStages = 4;

int attn_launch(const AttnArgs& a, bool fused, int head_dim, int group, bool paged, int kv_heads,
                int seqs, cudaStream_t s, bool pdl);
int attn_merge_launch(bf16* out, const float* partials, int heads, int head_dim, int splits,
                      cudaStream_t s);
int sample_launch(const SampleArgs& a, int rows, cudaStream_t s, bool pdl);

}  // namespace lcrb
