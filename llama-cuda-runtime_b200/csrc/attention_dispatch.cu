// Instantiations of the decode-attention and sampling kernels.
#include "dispatch.h"

namespace lcrb {
namespace {

// ---------------------------------------------------------------------------
// Attention dispatch
// ---------------------------------------------------------------------------

template <int D, int G, bool PAGED, bool FUSED>
int attn_launch_t(const AttnArgs& a, int kv_heads, int seqs, cudaStream_t stream, bool pdl) {
  auto kernel = attn_decode_kernel<D, G, PAGED, FUSED, kAttnStages>;
  constexpr size_t smem = attn_smem_bytes<D, kAttnStages>();
  // Per device and cheap; set on every launch so multi-GPU processes work.
  LCRB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.splits), static_cast<unsigned>(kv_heads),
                     static_cast<unsigned>(seqs));
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  LCRB_CUDA(cudaLaunchKernelEx(&cfg, kernel, a));
  return LCR_OK;
}

template <int D, bool PAGED, bool FUSED>
int attn_by_group(const AttnArgs& a, int group, int kv_heads, int seqs, cudaStream_t s, bool pdl) {
  switch (group) {
    case 1: return attn_launch_t<D, 1, PAGED, FUSED>(a, kv_heads, seqs, s, pdl);
    case 2: return attn_launch_t<D, 2, PAGED, FUSED>(a, kv_heads, seqs, s, pdl);
    case 4: return attn_launch_t<D, 4, PAGED, FUSED>(a, kv_heads, seqs, s, pdl);
    case 8: return attn_launch_t<D, 8, PAGED, FUSED>(a, kv_heads, seqs, s, pdl);
    default:
      return fail(LCR_ERR_SHAPE,
                  "decode attention is compiled for 1, 2, 4, or 8 query heads per key/value "
                  "head, this model has %d",
                  group);
  }
}

template <bool FUSED>
int attn_launch_impl(const AttnArgs& a, int head_dim, int group, bool paged, int kv_heads, int seqs,
                cudaStream_t s, bool pdl) {
  if (head_dim == 64) {
    return paged ? attn_by_group<64, true, FUSED>(a, group, kv_heads, seqs, s, pdl)
                 : attn_by_group<64, false, FUSED>(a, group, kv_heads, seqs, s, pdl);
  }
  if (head_dim == 128) {
    return paged ? attn_by_group<128, true, FUSED>(a, group, kv_heads, seqs, s, pdl)
                 : attn_by_group<128, false, FUSED>(a, group, kv_heads, seqs, s, pdl);
  }
  return fail(LCR_ERR_SHAPE, "decode attention is compiled for head_dim 64 or 128, this model has %d",
              head_dim);
}


}  // namespace

int attn_launch(const AttnArgs& a, bool fused, int head_dim, int group, bool paged, int kv_heads,
                int seqs, cudaStream_t s, bool pdl) {
  return fused ? attn_launch_impl<true>(a, head_dim, group, paged, kv_heads, seqs, s, pdl)
               : attn_launch_impl<false>(a, head_dim, group, paged, kv_heads, seqs, s, pdl);
}

int attn_merge_launch(bf16* out, const float* partials, int heads, int head_dim, int splits,
                      cudaStream_t s) {
  if (head_dim == 64) {
    attn_merge_kernel<64><<<heads, 64, 0, s>>>(out, partials, splits);
  } else {
    attn_merge_kernel<128><<<heads, 128, 0, s>>>(out, partials, splits);
  }
  return launch_status("decode attention merge");
}

int sample_launch(const SampleArgs& a, int rows, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows));
  cfg.blockDim = dim3(kSampleThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  LCRB_CUDA(cudaLaunchKernelEx(&cfg, sample_rows_kernel, a));
  return LCR_OK;
}

}  // namespace lcrb
