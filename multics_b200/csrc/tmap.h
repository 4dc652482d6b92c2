// TMA tensor-map construction shared by the kernel launchers.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace hier {

// 2-D bf16 tensor map with 128-byte swizzle over a row-major matrix of
// `rows` x `cols` elements (row stride in elements), box = box_cols x box_rows.
int make_tmap_bf16_2d(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows,
                      uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows);

}  // namespace hier
