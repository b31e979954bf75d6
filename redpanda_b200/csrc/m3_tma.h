// Host-side construction of TMA tensor maps (cuTensorMapEncodeTiled, looked up
// once from the driver through the runtime; no link against libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <stddef.h>

namespace m3 {

// cuTensorMapEncodeTiled, or null when the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// A row-major (rows, cols) matrix of 2-byte (bf16) or 4-byte (fp32) elements as
// a 2D tensor map with a (box_cols x box_rows) box, no swizzle, zero fill out of
// bounds.  The base must be 16-byte aligned and cols * esize a multiple of 16.
bool encode_rows_map(CUtensorMap* map, const void* base, int esize, size_t rows, size_t cols,
                     int box_cols, int box_rows);

}  // namespace m3
