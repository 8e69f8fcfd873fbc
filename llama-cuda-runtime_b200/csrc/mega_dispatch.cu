// Instantiations and cooperative launch of the persistent decode kernel.
#include "mega_dispatch.h"

namespace lcrb {
namespace {

template <int H, int QD, int F, int D, int G, bool PAGED, bool F32, bool LL = false>
int launch_t(const MegaArgs& a, int ctas, cudaStream_t stream) {
  auto kernel = decode_step_kernel<H, QD, F, D, G, PAGED, F32, LL>;
  constexpr size_t smem = MegaShape<H, QD, F, D, G, PAGED, F32>::SMEM;
  LCRB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)));
  int per_sm = 0;
  LCRB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kMegaThreads, smem));
  LCRB_REQUIRE(per_sm >= 1, LCR_ERR_SHAPE, "persistent decode kernel does not fit an SM");
  LCRB_CUDA(cudaMemsetAsync(a.bar, 0, sizeof(unsigned), stream));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas));
  cfg.blockDim = dim3(kMegaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA co-resident: grid barriers are safe
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  LCRB_CUDA(cudaLaunchKernelEx(&cfg, kernel, a));
  return LCR_OK;
}

template <int H, int QD, int F, int D, int G>
int launch_g(const MegaArgs& a, bool paged, bool f32, int ctas, cudaStream_t stream) {
  // Three instances per layout: fp32 activations; bf16 activations with grid
  // barriers; bf16 activations with the tagged-word exchange (a.ll).
  if (paged) {
    if (f32) return launch_t<H, QD, F, D, G, true, true>(a, ctas, stream);
    return a.ll ? launch_t<H, QD, F, D, G, true, false, true>(a, ctas, stream)
                : launch_t<H, QD, F, D, G, true, false>(a, ctas, stream);
  }
  if (f32) return launch_t<H, QD, F, D, G, false, true>(a, ctas, stream);
  return a.ll ? launch_t<H, QD, F, D, G, false, false, true>(a, ctas, stream)
              : launch_t<H, QD, F, D, G, false, false>(a, ctas, stream);
}

}  // namespace

bool mega_supported(int hidden, int q_dim, int ffn, int head_dim, int group) {
  return (hidden == 2048 && q_dim == 2048 && ffn == 8192 && head_dim == 64 && group == 4) ||
         (hidden == 256 && q_dim == 256 && ffn == 1024 && head_dim == 64 && group == 2);
}

int mega_max_splits(int ctas, int num_kv) { return ctas / num_kv; }

int mega_launch(const MegaArgs& a, int hidden, int q_dim, int ffn, int head_dim, int group,
                bool paged, bool f32, int ctas, cudaStream_t stream) {
  LCRB_REQUIRE(a.num_kv * a.splits <= ctas, LCR_ERR_SHAPE,
               "%d KV heads x %d splits exceed %d persistent CTAs", a.num_kv, a.splits, ctas);
  if (hidden == 2048 && q_dim == 2048 && ffn == 8192 && head_dim == 64 && group == 4) {
    return launch_g<2048, 2048, 8192, 64, 4>(a, paged, f32, ctas, stream);
  }
  if (hidden == 256 && q_dim == 256 && ffn == 1024 && head_dim == 64 && group == 2) {
    return launch_g<256, 256, 1024, 64, 2>(a, paged, f32, ctas, stream);
  }
  return fail(LCR_ERR_SHAPE, "no persistent decode kernel for hidden %d / q_dim %d / ffn %d", hidden,
              q_dim, ffn);
}

}  // namespace lcrb
