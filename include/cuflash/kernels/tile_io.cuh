// Tile load / store primitives of the reference's primitive API
// (include/cuflash/kernels/tile_io.cuh there), same declarations.
//   load_tile<R,C>   dst[R*C] (dense fp32) = the R x C window of a row-major
//                    matrix [max_rows, max_cols] (row stride in elements)
//                    starting at (row_start, col_start); elements outside the
//                    matrix read as 0.  half sources are widened exactly.
//   store_tile<R,C>  writes a dense R x C fp32 tile into that window, skipping
//                    elements outside the matrix; half destinations round to
//                    nearest even.
//   load_store_tile_roundtrip<R,C>  load then store: copies the window's
//                    in-matrix elements from src to dst (same stride).
// Null pointers return NULL_POINTER; non-positive max_rows / max_cols /
// stride, or a start outside the matrix, INVALID_DIMENSION.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "cuflash/export.h"
#include "cuflash/flash_attention.h"

namespace cuflash {
namespace kernels {

template <int BLOCK_ROWS, int BLOCK_COLS>
CUFLASH_EXPORT FlashAttentionError load_tile(const float* src, float* dst, int row_start,
                                             int col_start, int max_rows, int max_cols,
                                             int src_stride, cudaStream_t stream = 0);
template <int BLOCK_ROWS, int BLOCK_COLS>
CUFLASH_EXPORT FlashAttentionError load_tile(const half* src, float* dst, int row_start,
                                             int col_start, int max_rows, int max_cols,
                                             int src_stride, cudaStream_t stream = 0);

template <int BLOCK_ROWS, int BLOCK_COLS>
CUFLASH_EXPORT FlashAttentionError store_tile(const float* src, float* dst, int row_start,
                                              int col_start, int max_rows, int max_cols,
                                              int dst_stride, cudaStream_t stream = 0);
template <int BLOCK_ROWS, int BLOCK_COLS>
CUFLASH_EXPORT FlashAttentionError store_tile(const float* src, half* dst, int row_start,
                                              int col_start, int max_rows, int max_cols,
                                              int dst_stride, cudaStream_t stream = 0);

template <int BLOCK_ROWS, int BLOCK_COLS>
CUFLASH_EXPORT FlashAttentionError load_store_tile_roundtrip(const float* src, float* dst,
                                                             int row_start, int col_start,
                                                             int max_rows, int max_cols,
                                                             int stride, cudaStream_t stream = 0);

}  // namespace kernels
}  // namespace cuflash
