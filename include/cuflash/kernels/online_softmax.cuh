// Online-softmax primitives of the reference's primitive API
// (include/cuflash/kernels/online_softmax.cuh there), same declarations.
// Row states are (m, l): running maximum and sum of exp(x - m).
//   init      m = -inf, l = 0
//   update    merges a block's (max, sum): m' = max(m, b_max),
//             l' = l exp(m - m') + b_sum exp(b_max - m')
//   finalize  logsumexp = m + log(l), normalizer = 1 / l
//   forward   softmax of each row of a [rows, cols] fp32 matrix and its
//             logsumexp; block_size (> 0) is accepted for compatibility, the
//             rows are reduced in one streaming pass
// Null pointers return NULL_POINTER, non-positive sizes INVALID_DIMENSION.
#pragma once

#include <cuda_runtime.h>

#include "cuflash/export.h"
#include "cuflash/flash_attention.h"

namespace cuflash {
namespace kernels {

CUFLASH_EXPORT FlashAttentionError online_softmax_init(float* state_m, float* state_l, int rows,
                                                       cudaStream_t stream = 0);

CUFLASH_EXPORT FlashAttentionError online_softmax_update(const float* block_max,
                                                         const float* block_sum, float* state_m,
                                                         float* state_l, int rows,
                                                         cudaStream_t stream = 0);

CUFLASH_EXPORT FlashAttentionError online_softmax_finalize(const float* state_m,
                                                           const float* state_l, float* logsumexp,
                                                           float* normalizer, int rows,
                                                           cudaStream_t stream = 0);

CUFLASH_EXPORT FlashAttentionError online_softmax_forward(const float* input, float* output,
                                                          float* logsumexp, int rows, int cols,
                                                          int block_size, cudaStream_t stream = 0);

// Warp-wide butterfly reductions for kernels that include this header.
__device__ __forceinline__ float warp_reduce_max(float val) {
    for (int lane_mask = 16; lane_mask >= 1; lane_mask >>= 1)
        val = fmaxf(val, __shfl_xor_sync(0xffffffffu, val, lane_mask));
    return val;
}

__device__ __forceinline__ float warp_reduce_sum(float val) {
    for (int lane_mask = 16; lane_mask >= 1; lane_mask >>= 1)
        val += __shfl_xor_sync(0xffffffffu, val, lane_mask);
    return val;
}

}  // namespace kernels
}  // namespace cuflash
