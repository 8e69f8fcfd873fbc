// Instantiations and dispatch of the streaming GEMV kernel.
#include "gemv_dispatch.h"

#include <algorithm>

namespace lcrb {
namespace {

template <int K, int PRO, int EPI>
int launch_one(const GemvArgs& a, const CUtensorMap& map, int ctas, cudaStream_t stream, bool pdl) {
  auto kernel = gemv_stream_kernel<K, kGemvStages, PRO, EPI>;
  constexpr size_t smem = gemv_smem_bytes<K, kGemvStages>();
  // Per device and cheap; set on every launch so multi-GPU processes work.
  LCRB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas));
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  LCRB_CUDA(cudaLaunchKernelEx(&cfg, kernel, a, map));
  return LCR_OK;
}

template <int K, int PRO, int EPI>
int launch_k(const GemvArgs& a, const CUtensorMap& map, int ctas, cudaStream_t s, bool pdl) {
  return launch_one<K, PRO, EPI>(a, map, ctas, s, pdl);
}

template <int K>
int launch_pe(const GemvArgs& a, const CUtensorMap& map, int pro, int epi, int ctas, cudaStream_t s,
              bool pdl) {
  if (pro == PRO_PLAIN && epi == EPI_STORE) return launch_k<K, PRO_PLAIN, EPI_STORE>(a, map, ctas, s, pdl);
  if (pro == PRO_PLAIN && epi == EPI_STORE_F32) return launch_k<K, PRO_PLAIN, EPI_STORE_F32>(a, map, ctas, s, pdl);
  if (pro == PRO_PLAIN && epi == EPI_RESID) return launch_k<K, PRO_PLAIN, EPI_RESID>(a, map, ctas, s, pdl);
  if (pro == PRO_NORM && epi == EPI_STORE) return launch_k<K, PRO_NORM, EPI_STORE>(a, map, ctas, s, pdl);
  if (pro == PRO_EMBED_NORM && epi == EPI_STORE) return launch_k<K, PRO_EMBED_NORM, EPI_STORE>(a, map, ctas, s, pdl);
  if (pro == PRO_NORM && epi == EPI_STORE_F32) return launch_k<K, PRO_NORM, EPI_STORE_F32>(a, map, ctas, s, pdl);
  if (pro == PRO_NORM && epi == EPI_LOGITS_ARGMAX) return launch_k<K, PRO_NORM, EPI_LOGITS_ARGMAX>(a, map, ctas, s, pdl);
  if (pro == PRO_NORM && epi == EPI_SWIGLU) return launch_k<K, PRO_NORM, EPI_SWIGLU>(a, map, ctas, s, pdl);
  return fail(LCR_ERR_SHAPE, "streaming GEMV has no prologue %d / epilogue %d variant for K=%d", pro, epi, K);
}

}  // namespace

bool gemv_supported(int K, int pro, int epi) {
  const bool k_ok = K == 256 || K == 512 || K == 1024 || K == 2048 || K == 4096 || K == 8192;
  if (!k_ok) return false;
  if (epi == EPI_SWIGLU) return pro == PRO_NORM;
  return true;
}

int gemv_outputs_per_chunk(int K, int epi) {
  const int rps = 8 * (2048 / std::min(K, 2048));  // GemvGeom<K>::RPS
  return epi == EPI_SWIGLU ? rps / 2 : rps;
}

size_t gemv_smem(int K) {
  switch (K) {
    case 256: return gemv_smem_bytes<256, kGemvStages>();
    case 512: return gemv_smem_bytes<512, kGemvStages>();
    case 1024: return gemv_smem_bytes<1024, kGemvStages>();
    case 2048: return gemv_smem_bytes<2048, kGemvStages>();
    case 4096: return gemv_smem_bytes<4096, kGemvStages>();
    case 8192: return gemv_smem_bytes<8192, kGemvStages>();
    default: return 0;
  }
}

int gemv_launch(const GemvArgs& a, const CUtensorMap& map, int K, int pro, int epi, int ctas,
                cudaStream_t stream, bool pdl) {
  LCRB_REQUIRE(gemv_supported(K, pro, epi), LCR_ERR_SHAPE,
               "streaming GEMV: unsupported K=%d (prologue %d, epilogue %d)", K, pro, epi);
  LCRB_REQUIRE(ctas > 0, LCR_ERR_INVALID, "streaming GEMV needs at least one CTA");
  switch (K) {
    case 256: return launch_pe<256>(a, map, pro, epi, ctas, stream, pdl);
    case 512: return launch_pe<512>(a, map, pro, epi, ctas, stream, pdl);
    case 1024: return launch_pe<1024>(a, map, pro, epi, ctas, stream, pdl);
    case 2048: return launch_pe<2048>(a, map, pro, epi, ctas, stream, pdl);
    case 4096: return launch_pe<4096>(a, map, pro, epi, ctas, stream, pdl);
    case 8192: return launch_pe<8192>(a, map, pro, epi, ctas, stream, pdl);
    default: return fail(LCR_ERR_SHAPE, "streaming GEMV: unsupported K=%d", K);
  }
}

}  // namespace lcrb
