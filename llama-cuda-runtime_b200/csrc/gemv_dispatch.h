// Host-side launcher of the streaming GEMV instantiations (gemv_dispatch.cu).
#pragma once

#include <cuda_runtime.h>

#include "gemv.cuh"
#include "tmap.h"

namespace lcrb {

// Three ring slots (kGemvSlotBytes each): small enough that the next
// kernel's CTA fits beside this one on an SM, so programmatic dependent
// launch overlaps them.
constexpr int kGemvStages = 3;

bool gemv_supported(int K, int pro, int epi);
// Outputs (rows, or SWIGLU pairs) per chunk of one stage.
int gemv_outputs_per_chunk(int K, int epi);
size_t gemv_smem(int K);
// Launches y = W x with the given prologue / epilogue on `ctas` CTAs, each
// streaming a contiguous share of the outputs; `map` is make_weight_map of
// a.w (with swiglu for EPI_SWIGLU). `pdl` sets programmatic stream
// serialization.
int gemv_launch(const GemvArgs& a, const CUtensorMap& map, int K, int pro, int epi, int ctas,
                cudaStream_t stream, bool pdl);

}  // namespace lcrb
