// Host-side tensor maps for the weight-streaming GEMV (tmap.cu).
#pragma once

#include <cuda.h>

namespace lcrb {

// Encodes the tensor map one GEMV stage is copied with: the row-major
// [rows][K] bf16 matrix at `w` viewed as {64 columns, rows, K / 64 chunks}
// (chunk stride 128 bytes) with a {64, RPS, KC / 64} box and 128-byte
// swizzle, so that a stage lands chunk-major -- [chunk][row][128 bytes] --
// and row r's 16-byte pieces are rotated by r % 8. With `swiglu`, rows
// [0, rows) and [rows, 2 rows) are the gate and up halves and the view gains
// a half index: {64, rows, 2, K / 64}, box {64, RPS / 2, 2, KC / 64}.
// Returns an lcr_status; LCR_ERR_CUDA if the driver encoder is missing or
// refuses the map.
int make_weight_map(CUtensorMap* out, const void* w, int rows, int K, bool swiglu);

// The general form: the same {64 columns, rows, [2 halves,] K / 64 chunks}
// view (halves = 2: rows [0, rows) and [rows, 2 rows) of the matrix) with a
// {64, box_rows, [2,] box_chunks} box. The tcgen05 GEMM uses box_chunks = 1:
// one 64-column K-major slab, 128-byte swizzled, per copy.
int make_kmajor_map(CUtensorMap* out, const void* base, int rows, int K, int halves, int box_rows,
                    int box_chunks);

}  // namespace lcrb
