// Tensor maps (TMA descriptors) over the attention path's row-major f32
// buffers, shared by the tensor-core kernels.
#pragma once

#include <cuda.h>

#include <cstdint>

namespace kattn {

// The first H*d columns of a [B*T][ld] f32 buffer as a 3-D tensor
// {H*d columns, T rows, B}, boxes of `box_cols` columns x `box_rows` rows of
// one batch entry; rows past T are out of bounds and read as zeros.  `base`
// is 16-byte aligned and ld a multiple of 4 (checked at the C ABI).  False
// when the driver entry point is missing or the encoding is refused.
bool encode_rows(CUtensorMap* map, const float* base, long ld, int B, int T, int H, int d, int box_cols, int box_rows,
                 CUtensorMapSwizzle swizzle);

// A row-major f32 matrix of `rows` rows x `cols` columns (row stride ld
// elements) as a 2-D tensor {cols (innermost), rows}, boxes of box_cols x
// box_rows with no swizzle; elements past either extent read as zeros.
bool encode_2d(CUtensorMap* map, const float* base, long cols, long rows, long ld, int box_cols, int box_rows);

// The same over a row-major bf16 matrix (ld a multiple of 8 elements), with
// the given swizzle of the box in shared memory.
bool encode_2d_bf16(CUtensorMap* map, const uint16_t* base, long cols, long rows, long ld, int box_cols, int box_rows,
                    CUtensorMapSwizzle swizzle);

}  // namespace kattn
