// Instantiations and launch of the batched tensor-pipe decode attention.
#include "attn_batch.h"

namespace lcrb {
namespace {

template <int D, int G>
int launch_t(const AttnArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap, int ctas, cudaStream_t s) {
  auto kernel = attn_batch_kernel<D, G>;
  const size_t smem = attn_batch_smem_bytes<D, G>(a.seqs);
  LCRB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  LCRB_TRY(launch_kernel(kernel, dim3(ctas), dim3(kAbThreads), smem, s, true, a, kmap, vmap));
  return launch_kernel(attn_batch_merge_kernel<D>, dim3(a.seqs * (a.q_dim / D)), dim3(D), 0, s, true, a);
}

template <int D, int G>
int ctas_t(int seqs, int sms, int* ctas) {
  auto kernel = attn_batch_kernel<D, G>;
  const size_t smem = attn_batch_smem_bytes<D, G>(seqs);
  LCRB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  int per_sm = 0;
  LCRB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kAbThreads, smem));
  *ctas = (per_sm > 0 ? per_sm : 1) * sms;
  return LCR_OK;
}

int bad_group(int group) {
  return fail(LCR_ERR_SHAPE,
              "batched decode attention is compiled for 1, 2, 4 or 8 query heads per KV head, this model has %d",
              group);
}

template <int D>
int ctas_d(int group, int seqs, int sms, int* ctas) {
  switch (group) {
    case 1: return ctas_t<D, 1>(seqs, sms, ctas);
    case 2: return ctas_t<D, 2>(seqs, sms, ctas);
    case 4: return ctas_t<D, 4>(seqs, sms, ctas);
    case 8: return ctas_t<D, 8>(seqs, sms, ctas);
    default: return bad_group(group);
  }
}

template <int D>
int launch_d(const AttnArgs& a, const CUtensorMap& k, const CUtensorMap& v, int group, int ctas, cudaStream_t s) {
  switch (group) {
    case 1: return launch_t<D, 1>(a, k, v, ctas, s);
    case 2: return launch_t<D, 2>(a, k, v, ctas, s);
    case 4: return launch_t<D, 4>(a, k, v, ctas, s);
    case 8: return launch_t<D, 8>(a, k, v, ctas, s);
    default: return bad_group(group);
  }
}

}  // namespace

int attn_batch_ctas(int head_dim, int group, int seqs, int sms, int* ctas) {
  if (head_dim == 64) return ctas_d<64>(group, seqs, sms, ctas);
  if (head_dim == 128) return ctas_d<128>(group, seqs, sms, ctas);
  return fail(LCR_ERR_SHAPE, "batched decode attention is compiled for head_dim 64 or 128, this model has %d",
              head_dim);
}

int attn_batch_launch(const AttnArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap, int head_dim,
                      int group, int ctas, cudaStream_t s) {
  LCRB_REQUIRE(a.page_size % kAbUnit == 0 && a.item_pos % kAbUnit == 0 && a.item_pos > 0 && a.work &&
                   a.seqs >= 1 && a.seqs <= kAbMaxSeqs && a.splits <= kAbMaxSplits &&
                   static_cast<long long>(a.splits) * a.item_pos >= a.max_seq && ctas >= 1,
               LCR_ERR_SHAPE, "batched decode attention: unsupported configuration");
  if (head_dim == 64) return launch_d<64>(a, kmap, vmap, group, ctas, s);
  if (head_dim == 128) return launch_d<128>(a, kmap, vmap, group, ctas, s);
  return fail(LCR_ERR_SHAPE, "batched decode attention is compiled for head_dim 64 or 128, this model has %d",
              head_dim);
}

}  // namespace lcrb
