// Tile-level fp32 matrix products of the reference's primitive API
// (include/cuflash/kernels/matmul.cuh there): one thread block computes the
// whole product of small row-major matrices in global memory.  Declarations
// are identical to the reference's, so programs built against its header link
// against this library; the explicit instantiations below
// (cuflash-attn_b200/csrc/primitives.cu) are the reference's eight shapes.
//
// Every element is a k-ordered fp32 fused multiply-add chain from 0, times
// scale (accumulating forms add that product into C with one more fused
// multiply-add).  Only null pointers are rejected (NULL_POINTER).
#pragma once

#include <cuda_runtime.h>

#include "cuflash/export.h"
#include "cuflash/flash_attention.h"

namespace cuflash {
namespace kernels {

// C[M,N] = scale * A[M,K] B[N,K]^T   (S = Q K^T)
template <int M, int N, int K>
CUFLASH_EXPORT FlashAttentionError matmul_ABt(const float* A, const float* B, float* C,
                                              float scale, cudaStream_t stream = 0);

// C[M,N] = scale * A[M,K] B[K,N]     (O = P V)
template <int M, int N, int K>
CUFLASH_EXPORT FlashAttentionError matmul_AB(const float* A, const float* B, float* C,
                                             float scale, cudaStream_t stream = 0);

// C[M,N] += scale * A[M,K] B[K,N]
template <int M, int N, int K>
CUFLASH_EXPORT FlashAttentionError matmul_AB_acc(const float* A, const float* B, float* C,
                                                 float scale, cudaStream_t stream = 0);

// C[M,N] = scale * A[K,M]^T B[K,N]   (dV = P^T dO, dK = dS^T Q)
template <int M, int N, int K>
CUFLASH_EXPORT FlashAttentionError matmul_AtB(const float* A, const float* B, float* C,
                                              float scale, cudaStream_t stream = 0);

}  // namespace kernels
}  // namespace cuflash
