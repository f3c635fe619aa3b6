// Tensor maps (TMA descriptors) for the tile-contiguous expert banks and for activation rows,
// shared by the tcgen05 GEMM and the TMA-fed decode GEMV.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>

namespace lm {

// rank 2: activation rows, dims {K, rows}, box {64, box_rows}.
// rank 3: weight tiles, dims {64, 128, n_tiles} with strides {128 B, 16 KiB},
//         box {64, box_rows, box_depth} (box_depth consecutive tiles: K blocks kb, kb+1, ...).
// Both with 128-byte swizzle (the K-major SW128 layout of the UMMA descriptors). Cached by
// (pointer, dims, box); returns LM_OK or an LM_ERR_* code.
int make_map(CUtensorMap* out, const void* ptr, int rank, uint64_t d0, uint64_t d1,
             int box_rows = 128, int box_depth = 1);

}  // namespace lm
