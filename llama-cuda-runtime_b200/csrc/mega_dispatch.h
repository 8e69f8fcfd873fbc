// Host launcher of the persistent decode kernel (mega_dispatch.cu).
#pragma once

#include <cuda_runtime.h>

#include "megakernel.cuh"

namespace lcrb {

// True when a persistent-kernel instantiation exists for this geometry.
bool mega_supported(int hidden, int q_dim, int ffn, int head_dim, int group);
// Largest attention split count the persistent kernel accepts (one
// (KV head, split) item per CTA, `ctas` CTAs).
int mega_max_splits(int ctas, int num_kv);
// Zeroes the barrier counter and launches the kernel cooperatively on `ctas`
// CTAs (one per SM); `f32` selects fp32 activations, else the reference's
// bf16 storage rounding.
int mega_launch(const MegaArgs& a, int hidden, int q_dim, int ffn, int head_dim, int group,
                bool paged, bool f32, int ctas, cudaStream_t stream);

}  // namespace lcrb
