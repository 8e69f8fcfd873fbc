// Host-side launcher of the tcgen05 batched projection (gemm_tc.cu).
#pragma once

#include <cuda_runtime.h>

#include "gemm_tc.cuh"

namespace lcrb {

// Smallest supported batch tile covering `rows` (16, 32, 64 or 128; larger
// batches take several tiles of 128).
int gemm_tc_batch_tile(int rows);
// Largest chunks per stage gemm_tc_launch takes with batch tile nb.
int gemm_tc_max_chunks(int nb);
size_t gemm_tc_work_floats(int rows, int n_out, int epi, int splits);
// Launches y = x w^T for `a.rows` batch rows, each ring stage carrying `ch`
// 64-column K chunks: wmap = make_kmajor_map(w, n_out (2F for SWIGLU as two
// halves), K, halves, 128 (64 for SWIGLU), ch), xmap = make_kmajor_map(x,
// rows, K, 1, nb, ch). One CTA per (weight tile, batch tile, split); a.splits
// > 1 needs a.work of gemm_tc_work_floats() floats and adds a second launch
// (gemm_tc_reduce_kernel; for RESID with a.norm_out, the reduction fused
// with the RMSNorm of the updated rows). nb = 128 with ch = 1, a.splits = 1
// and a.ctas > 0 runs gemm_tc_persist_kernel on min(tiles, a.ctas) CTAs;
// nb = 256 (prefill chunks) runs only there. With `pdl` the kernels launch
// programmatically: the first ring's weights stream before the wait for the
// preceding kernel.
int gemm_tc_launch(const TcArgs& a, const CUtensorMap& wmap, const CUtensorMap& xmap, int nb, int epi, int ch,
                   cudaStream_t stream, bool pdl);

}  // namespace lcrb
