// Host-side helpers shared by the entry points of the C ABI.
#pragma once

#include <cuda.h>

#include <cstdint>

namespace ksw {

// Encodes a 2-D row-major tensor map with 128-byte swizzling.
// inner = columns (contiguous), rows = number of rows, row_stride_elems =
// elements between consecutive rows, box = (box_inner columns, box_rows rows).
int encode_tma_2d(CUtensorMap* tm, CUtensorMapDataType dtype, int elem_bytes,
                  const void* base, uint64_t inner, uint64_t rows,
                  uint64_t row_stride_elems, uint32_t box_inner,
                  uint32_t box_rows);

}  // namespace ksw
