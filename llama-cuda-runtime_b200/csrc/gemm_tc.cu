// Instantiations and launch of the tcgen05 batched projection.
#include "gemm_tc.h"

#include <algorithm>

namespace lcrb {
namespace {

template <int NB, int EPI>
int launch_persist(const TcArgs& a, const CUtensorMap& wmap, const CUtensorMap& xmap, cudaStream_t s, bool pdl) {
  auto kernel = gemm_tc_persist_kernel<NB, EPI>;
  constexpr size_t smem = gemm_tc_persist_smem_bytes<NB>();
  LCRB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  const int tiles_n = EPI == EPI_SWIGLU ? (a.n_out + 63) / 64 : (a.n_out + kTcTileM - 1) / kTcTileM;
  const int tiles = tiles_n * ((a.rows + NB - 1) / NB);
  return launch_kernel(kernel, dim3(static_cast<unsigned>(std::min(tiles, a.ctas))), dim3(kTcThreads), smem, s, pdl,
                       a, wmap, xmap);
}

template <int NB, int EPI, int CH>
int launch_t(const TcArgs& a, const CUtensorMap& wmap, const CUtensorMap& xmap, cudaStream_t s, bool pdl) {
  if constexpr (NB == 128 && CH == 1) {
    if (a.splits == 1 && a.ctas > 0) return launch_persist<128, EPI>(a, wmap, xmap, s, pdl);
  }
  auto kernel = gemm_tc_kernel<NB, EPI, CH>;
  constexpr size_t smem = gemm_tc_smem_bytes<NB, CH>();
  LCRB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  const int tiles_n = EPI == EPI_SWIGLU ? (a.n_out + 63) / 64 : (a.n_out + kTcTileM - 1) / kTcTileM;
  const int tiles_b = (a.rows + NB - 1) / NB;
  dim3 grid(static_cast<unsigned>(tiles_n * tiles_b), static_cast<unsigned>(a.splits));
  LCRB_TRY(launch_kernel(kernel, grid, dim3(kTcThreads), smem, s, pdl, a, wmap, xmap));
  if (a.splits > 1) {
    if constexpr (EPI == EPI_RESID) {
      if (a.norm_out != nullptr) {
        void (*fused)(TcArgs) = a.n_out == 2048   ? gemm_tc_reduce_norm_kernel<2048>
                                : a.n_out == 256  ? gemm_tc_reduce_norm_kernel<256>
                                : a.n_out == 4096 ? gemm_tc_reduce_norm_kernel<4096>
                                                  : nullptr;
        LCRB_REQUIRE(fused != nullptr, LCR_ERR_SHAPE, "fused residual RMSNorm has no kernel for width %d", a.n_out);
        return launch_kernel(fused, dim3(static_cast<unsigned>(a.rows)), dim3(256), 0, s, pdl, a);
      }
    }
    const long long total = static_cast<long long>(a.rows) * a.n_out;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 4096));
    LCRB_TRY(launch_kernel(gemm_tc_reduce_kernel<EPI>, dim3(blocks), dim3(256), 0, s, pdl, a));
  }
  return LCR_OK;
}

template <int NB, int CH>
int by_epi(const TcArgs& a, const CUtensorMap& w, const CUtensorMap& x, int epi, cudaStream_t s, bool pdl) {
  switch (epi) {
    case EPI_STORE: return launch_t<NB, EPI_STORE, CH>(a, w, x, s, pdl);
    case EPI_STORE_F32: return launch_t<NB, EPI_STORE_F32, CH>(a, w, x, s, pdl);
    case EPI_RESID: return launch_t<NB, EPI_RESID, CH>(a, w, x, s, pdl);
    case EPI_SWIGLU: return launch_t<NB, EPI_SWIGLU, CH>(a, w, x, s, pdl);
    case EPI_ROPE: return launch_t<NB, EPI_ROPE, CH>(a, w, x, s, pdl);
    default: return fail(LCR_ERR_SHAPE, "tcgen05 projection: no epilogue %d", epi);
  }
}

template <int NB>
int by_chunks(const TcArgs& a, const CUtensorMap& w, const CUtensorMap& x, int epi, int ch, cudaStream_t s,
              bool pdl) {
  switch (ch) {
    case 1: return by_epi<NB, 1>(a, w, x, epi, s, pdl);
    case 2: return by_epi<NB, 2>(a, w, x, epi, s, pdl);
    case 4:
      if constexpr (NB <= 64) return by_epi<NB, 4>(a, w, x, epi, s, pdl);
      [[fallthrough]];
    default: return fail(LCR_ERR_SHAPE, "tcgen05 projection: %d chunks per stage with batch tile %d", ch, NB);
  }
}

}  // namespace

int gemm_tc_batch_tile(int rows) {
  if (rows <= 16) return 16;
  if (rows <= 32) return 32;
  if (rows <= 64) return 64;
  return 128;
}

int gemm_tc_max_chunks(int nb) { return nb <= 64 ? 4 : 2; }

size_t gemm_tc_work_floats(int rows, int n_out, int epi, int splits) {
  const int tiles_n = epi == EPI_SWIGLU ? (n_out + 63) / 64 : (n_out + kTcTileM - 1) / kTcTileM;
  return splits > 1 ? static_cast<size_t>(splits) * rows * tiles_n * kTcTileM : 0;
}

int gemm_tc_launch(const TcArgs& a, const CUtensorMap& wmap, const CUtensorMap& xmap, int nb, int epi, int ch,
                   cudaStream_t stream, bool pdl) {
  LCRB_REQUIRE(ch >= 1 && a.K % (kTcSlabK * ch) == 0 && a.n_out > 0 && a.rows > 0, LCR_ERR_SHAPE,
               "tcgen05 projection: unsupported %d x %d x %d (%d chunks per stage)", a.rows, a.n_out, a.K, ch);
  LCRB_REQUIRE(a.splits >= 1 && a.splits <= a.K / (kTcSlabK * ch), LCR_ERR_INVALID,
               "tcgen05 projection: %d splits", a.splits);
  LCRB_REQUIRE(epi != EPI_ROPE || (a.rope && (a.head_dim == 64 || a.head_dim == 128) && a.rope_cols % a.head_dim == 0),
               LCR_ERR_SHAPE, "tcgen05 projection: RoPE epilogue needs a table and head_dim 64 or 128");
  LCRB_REQUIRE(a.splits == 1 || a.work, LCR_ERR_INVALID, "tcgen05 projection: split-K needs workspace");
  switch (nb) {
    case 16: return by_chunks<16>(a, wmap, xmap, epi, ch, stream, pdl);
    case 32: return by_chunks<32>(a, wmap, xmap, epi, ch, stream, pdl);
    case 64: return by_chunks<64>(a, wmap, xmap, epi, ch, stream, pdl);
    case 128: return by_chunks<128>(a, wmap, xmap, epi, ch, stream, pdl);
    case 256:
      // Persistent kernel only (one 64-column chunk per stage, no split-K).
      LCRB_REQUIRE(ch == 1 && a.splits == 1 && a.ctas > 0, LCR_ERR_SHAPE,
                   "tcgen05 projection: 256-row batch tiles run persistent, one chunk per stage, without split-K");
      switch (epi) {
        case EPI_STORE: return launch_persist<256, EPI_STORE>(a, wmap, xmap, stream, pdl);
        case EPI_STORE_F32: return launch_persist<256, EPI_STORE_F32>(a, wmap, xmap, stream, pdl);
        case EPI_RESID: return launch_persist<256, EPI_RESID>(a, wmap, xmap, stream, pdl);
        case EPI_SWIGLU: return launch_persist<256, EPI_SWIGLU>(a, wmap, xmap, stream, pdl);
        case EPI_ROPE: return launch_persist<256, EPI_ROPE>(a, wmap, xmap, stream, pdl);
        default: return fail(LCR_ERR_SHAPE, "tcgen05 projection: no epilogue %d", epi);
      }
    default: return fail(LCR_ERR_SHAPE, "tcgen05 projection: batch tile %d", nb);
  }
}

}  // namespace lcrb
