// Tensor-map encoding through the driver entry point cudart exposes, so the
// library needs no link against libcuda.
#include "tmap.h"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace lcrb {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_once;

void load_encoder() {
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  void* fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess) {
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
}

}  // namespace

int make_kmajor_map(CUtensorMap* out, const void* base, int rows, int K, int halves, int box_rows,
                    int box_chunks) {
  std::call_once(g_once, load_encoder);
  LCRB_REQUIRE(g_encode != nullptr, LCR_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  LCRB_REQUIRE(K % 64 == 0 && rows > 0 && (halves == 1 || halves == 2), LCR_ERR_SHAPE,
               "tensor map: unsupported %d x %d matrix", rows, K);
  LCRB_REQUIRE(box_rows >= 1 && box_rows <= 256 && box_chunks >= 1 && box_chunks <= K / 64, LCR_ERR_SHAPE,
               "tensor map: unsupported box %d x %d", box_rows, box_chunks);
  LCRB_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15u) == 0, LCR_ERR_SHAPE,
               "tensor map: the matrix must be 16-byte aligned");
  const cuuint32_t elem_strides[4] = {1, 1, 1, 1};
  CUresult r;
  if (halves == 1) {
    const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(K / 64)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K) * 2, 128};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), static_cast<cuuint32_t>(box_chunks)};
    r = g_encode(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                 elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(rows), 2, static_cast<cuuint64_t>(K / 64)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(K) * 2, static_cast<cuuint64_t>(rows) * K * 2, 128};
    const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows), 2, static_cast<cuuint32_t>(box_chunks)};
    r = g_encode(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                 elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  LCRB_REQUIRE(r == CUDA_SUCCESS, LCR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for a %d x %d matrix",
               static_cast<int>(r), rows, K);
  return LCR_OK;
}

int make_weight_map(CUtensorMap* out, const void* w, int rows, int K, bool swiglu) {
  LCRB_REQUIRE(K % 256 == 0 && (K <= 2048 || K % 2048 == 0) && rows > 0, LCR_ERR_SHAPE,
               "streaming GEMV tensor map: unsupported %d x %d matrix", rows, K);
  const int kc = std::min(K, 2048);
  const int rps = 8 * (2048 / kc);
  return swiglu ? make_kmajor_map(out, w, rows, K, 2, rps / 2, kc / 64)
                : make_kmajor_map(out, w, rows, K, 1, rps, kc / 64);
}

}  // namespace lcrb
