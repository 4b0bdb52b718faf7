// The reference's primitive kernel API (cuflash::kernels::*), re-exported so
// that this library carries every symbol of the reference's shared library:
//   matmul_{ABt,AB,AB_acc,AtB}<M,N,K>     src/kernels/matmul.cu:154-319
//   online_softmax_{init,update,finalize,forward}
//                                          src/kernels/online_softmax.cu:168-245
//   load_tile / store_tile / load_store_tile_roundtrip<R,C>
//                                          src/kernels/tile_io.cu (instantiations
//                                          as declared in include/cuflash/kernels/tile_io.cuh:41-90)
// These are single-block fp32 operations on small tiles (the reference's test
// layer), not part of the attention path; they are written as plain SIMT
// kernels:
//  * matmul: one 256-thread block; both operands staged k-major in shared
//    memory, each thread owns an (M/16) x (N/16) register tile and runs, per
//    output element, the same k-ordered fused multiply-add chain from 0 as the
//    reference, so results are bit-identical to it;
//  * online softmax: element-wise state kernels with the reference's merge
//    algebra (src/kernels/impl/online_softmax.cuh:21-37); the row softmax runs
//    one warp per row in a single streaming pass of per-lane (max, sum) states
//    merged with shuffles, then a normalising pass;
//  * tile I/O: one block, one thread per element, bounds-checked, 64-bit
//    addressing.

#include <cmath>

#include "common.cuh"
#include "cuflash/kernels/matmul.cuh"
#include "cuflash/kernels/online_softmax.cuh"
#include "cuflash/kernels/tile_io.cuh"

namespace cuflash {
namespace kernels {

namespace {

constexpr int kPrimThreads = 256;

FlashAttentionError launch_status() {
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

// ------------------------------------------------------------------ matmul

enum class MmForm { kABt, kAB, kABacc, kAtB };

template <int M, int N, int K, MmForm F>
__global__ void __launch_bounds__(kPrimThreads)
    tile_mm_kernel(const float* __restrict__ A, const float* __restrict__ B, float* C,
                   float scale) {
    static_assert(M % 16 == 0 && N % 16 == 0, "tile shape");
    constexpr int TM = M / 16;
    constexpr int TN = N / 16;
    extern __shared__ __align__(16) float smem_f[];
    float* sA = smem_f;        // A(m, k) at sA[k * M + m]
    float* sB = sA + K * M;    // B(k, n) at sB[k * N + n]
    const int tid = threadIdx.x;
    for (int e = tid; e < M * K; e += kPrimThreads) {
        if constexpr (F == MmForm::kAtB) {
            sA[e] = A[e];  // A is [K, M]
        } else {
            const int m = e / K, k = e - (e / K) * K;
            sA[k * M + m] = A[e];  // A is [M, K]
        }
    }
    for (int e = tid; e < K * N; e += kPrimThreads) {
        if constexpr (F == MmForm::kABt) {
            const int n = e / K, k = e - (e / K) * K;
            sB[k * N + n] = B[e];  // B is [N, K]
        } else {
            sB[e] = B[e];  // B is [K, N]
        }
    }
    __syncthreads();
    const int m0 = (tid / 16) * TM;
    const int n0 = (tid % 16) * TN;
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
#pragma unroll 4
    for (int k = 0; k < K; ++k) {
        float a[TM], b[TN];
#pragma unroll
        for (int i = 0; i < TM; ++i) a[i] = sA[k * M + m0 + i];
#pragma unroll
        for (int j = 0; j < TN; ++j) b[j] = sB[k * N + n0 + j];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            float* c = C + (m0 + i) * N + n0 + j;
            if constexpr (F == MmForm::kABacc)
                *c = fmaf(acc[i][j], scale, *c);
            else
                *c = acc[i][j] * scale;
        }
}

template <int M, int N, int K, MmForm F>
FlashAttentionError tile_mm(const float* A, const float* B, float* C, float scale,
                            cudaStream_t stream) {
    if (!A || !B || !C) return FlashAttentionError::NULL_POINTER;
    constexpr size_t smem = static_cast<size_t>(K) * (M + N) * sizeof(float);
    auto kern = tile_mm_kernel<M, N, K, F>;
    if (!detail::ensure_smem_attr(reinterpret_cast<const void*>(kern), static_cast<int>(smem)))
        return FlashAttentionError::CUDA_ERROR;
    kern<<<1, kPrimThreads, smem, stream>>>(A, B, C, scale);
    return launch_status();
}

// ------------------------------------------------------------ online softmax

__global__ void softmax_state_init_kernel(float* m, float* l, int rows) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows) {
        m[r] = -INFINITY;
        l[r] = 0.f;
    }
}

__global__ void softmax_state_update_kernel(const float* __restrict__ bmax,
                                            const float* __restrict__ bsum, float* m, float* l,
                                            int rows) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows) {
        const float mo = m[r], bm = bmax[r];
        const float mx = fmaxf(mo, bm);
        l[r] = fmaf(l[r], expf(mo - mx), bsum[r] * expf(bm - mx));
        m[r] = mx;
    }
}

__global__ void softmax_state_finalize_kernel(const float* __restrict__ m,
                                              const float* __restrict__ l, float* lse, float* norm,
                                              int rows) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows) {
        lse[r] = m[r] + logf(l[r]);
        norm[r] = 1.0f / l[r];
    }
}

// Merge of two (max, sum-of-exp) states; empty states (max = -inf) add nothing.
__device__ __forceinline__ void state_merge(float& m, float& l, float m2, float l2) {
    const float mx = fmaxf(m, m2);
    const float a = m == -INFINITY ? 0.f : l * expf(m - mx);
    const float b = m2 == -INFINITY ? 0.f : l2 * expf(m2 - mx);
    l = a + b;
    m = mx;
}

constexpr int kRowsPerBlock = kPrimThreads / 32;

__global__ void __launch_bounds__(kPrimThreads)
    softmax_rows_kernel(const float* __restrict__ in, float* __restrict__ out,
                        float* __restrict__ lse, int rows, int cols) {
    const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* x = in + static_cast<size_t>(row) * cols;
    float m = -INFINITY, l = 0.f;
    for (int c = lane; c < cols; c += 32) {
        const float v = x[c];
        if (v > m) {
            l = (m == -INFINITY ? 0.f : l * expf(m - v)) + 1.f;
            m = v;
        } else if (v != -INFINITY) {
            l += expf(v - m);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
        state_merge(m, l, m2, l2);
    }
    const float inv = 1.0f / l;
    float* y = out + static_cast<size_t>(row) * cols;
    for (int c = lane; c < cols; c += 32) y[c] = expf(x[c] - m) * inv;
    if (lane == 0) lse[row] = m + logf(l);
}

// ----------------------------------------------------------------- tile I/O

FlashAttentionError check_window(int row_start, int col_start, int max_rows, int max_cols,
                                 int stride) {
    if (max_rows <= 0 || max_cols <= 0 || stride <= 0) return FlashAttentionError::INVALID_DIMENSION;
    if (row_start < 0 || col_start < 0 || row_start >= max_rows || col_start >= max_cols)
        return FlashAttentionError::INVALID_DIMENSION;
    return FlashAttentionError::SUCCESS;
}

__device__ __forceinline__ float widen(float v) { return v; }
__device__ __forceinline__ float widen(half v) { return __half2float(v); }
__device__ __forceinline__ void narrow_store(float* p, float v) { *p = v; }
__device__ __forceinline__ void narrow_store(half* p, float v) { *p = __float2half_rn(v); }

template <int R, int C, typename S>
__global__ void __launch_bounds__(kPrimThreads)
    tile_load_kernel(const S* __restrict__ src, float* __restrict__ dst, int r0, int c0, int nr,
                     int nc, int stride) {
    for (int e = threadIdx.x; e < R * C; e += kPrimThreads) {
        const int gr = r0 + e / C, gc = c0 + e % C;
        dst[e] = (gr < nr && gc < nc) ? widen(src[static_cast<size_t>(gr) * stride + gc]) : 0.f;
    }
}

template <int R, int C, typename D>
__global__ void __launch_bounds__(kPrimThreads)
    tile_store_kernel(const float* __restrict__ src, D* __restrict__ dst, int r0, int c0, int nr,
                      int nc, int stride) {
    for (int e = threadIdx.x; e < R * C; e += kPrimThreads) {
        const int gr = r0 + e / C, gc = c0 + e % C;
        if (gr < nr && gc < nc) narrow_store(dst + static_cast<size_t>(gr) * stride + gc, src[e]);
    }
}

template <int R, int C>
__global__ void __launch_bounds__(kPrimThreads)
    tile_copy_kernel(const float* __restrict__ src, float* __restrict__ dst, int r0, int c0,
                     int nr, int nc, int stride) {
    for (int e = threadIdx.x; e < R * C; e += kPrimThreads) {
        const int gr = r0 + e / C, gc = c0 + e % C;
        if (gr < nr && gc < nc) {
            const size_t i = static_cast<size_t>(gr) * stride + gc;
            dst[i] = src[i];
        }
    }
}

}  // namespace

// ------------------------------------------------------------------ entries

template <int M, int N, int K>
FlashAttentionError matmul_ABt(const float* A, const float* B, float* C, float scale,
                               cudaStream_t stream) {
    return tile_mm<M, N, K, MmForm::kABt>(A, B, C, scale, stream);
}
template <int M, int N, int K>
FlashAttentionError matmul_AB(const float* A, const float* B, float* C, float scale,
                              cudaStream_t stream) {
    return tile_mm<M, N, K, MmForm::kAB>(A, B, C, scale, stream);
}
template <int M, int N, int K>
FlashAttentionError matmul_AB_acc(const float* A, const float* B, float* C, float scale,
                                  cudaStream_t stream) {
    return tile_mm<M, N, K, MmForm::kABacc>(A, B, C, scale, stream);
}
template <int M, int N, int K>
FlashAttentionError matmul_AtB(const float* A, const float* B, float* C, float scale,
                               cudaStream_t stream) {
    return tile_mm<M, N, K, MmForm::kAtB>(A, B, C, scale, stream);
}

#define CUFLASH_MM_SHAPE(M, N, K)                                                                  \
    template FlashAttentionError matmul_ABt<M, N, K>(const float*, const float*, float*, float,   \
                                                     cudaStream_t);                               \
    template FlashAttentionError matmul_AB<M, N, K>(const float*, const float*, float*, float,    \
                                                    cudaStream_t);                                \
    template FlashAttentionError matmul_AB_acc<M, N, K>(const float*, const float*, float*,       \
                                                        float, cudaStream_t);                     \
    template FlashAttentionError matmul_AtB<M, N, K>(const float*, const float*, float*, float,   \
                                                     cudaStream_t);
// the reference's shapes (src/kernels/matmul.cu:241-319)
CUFLASH_MM_SHAPE(64, 64, 32)
CUFLASH_MM_SHAPE(32, 32, 32)
CUFLASH_MM_SHAPE(64, 64, 64)
CUFLASH_MM_SHAPE(32, 32, 128)
CUFLASH_MM_SHAPE(64, 64, 128)
CUFLASH_MM_SHAPE(32, 64, 32)
CUFLASH_MM_SHAPE(32, 64, 64)
CUFLASH_MM_SHAPE(64, 32, 64)
#undef CUFLASH_MM_SHAPE

FlashAttentionError online_softmax_init(float* state_m, float* state_l, int rows,
                                        cudaStream_t stream) {
    if (!state_m || !state_l) return FlashAttentionError::NULL_POINTER;
    if (rows <= 0) return FlashAttentionError::INVALID_DIMENSION;
    softmax_state_init_kernel<<<(rows + kPrimThreads - 1) / kPrimThreads, kPrimThreads, 0,
                                stream>>>(state_m, state_l, rows);
    return launch_status();
}

FlashAttentionError online_softmax_update(const float* block_max, const float* block_sum,
                                          float* state_m, float* state_l, int rows,
                                          cudaStream_t stream) {
    if (!block_max || !block_sum || !state_m || !state_l) return FlashAttentionError::NULL_POINTER;
    if (rows <= 0) return FlashAttentionError::INVALID_DIMENSION;
    softmax_state_update_kernel<<<(rows + kPrimThreads - 1) / kPrimThreads, kPrimThreads, 0,
                                  stream>>>(block_max, block_sum, state_m, state_l, rows);
    return launch_status();
}

FlashAttentionError online_softmax_finalize(const float* state_m, const float* state_l,
                                            float* logsumexp, float* normalizer, int rows,
                                            cudaStream_t stream) {
    if (!state_m || !state_l || !logsumexp || !normalizer) return FlashAttentionError::NULL_POINTER;
    if (rows <= 0) return FlashAttentionError::INVALID_DIMENSION;
    softmax_state_finalize_kernel<<<(rows + kPrimThreads - 1) / kPrimThreads, kPrimThreads, 0,
                                    stream>>>(state_m, state_l, logsumexp, normalizer, rows);
    return launch_status();
}

FlashAttentionError online_softmax_forward(const float* input, float* output, float* logsumexp,
                                           int rows, int cols, int block_size,
                                           cudaStream_t stream) {
    if (!input || !output || !logsumexp) return FlashAttentionError::NULL_POINTER;
    if (rows <= 0 || cols <= 0 || block_size <= 0) return FlashAttentionError::INVALID_DIMENSION;
    const int blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
    softmax_rows_kernel<<<blocks, kPrimThreads, 0, stream>>>(input, output, logsumexp, rows, cols);
    return launch_status();
}

template <int R, int C>
FlashAttentionError load_tile(const float* src, float* dst, int row_start, int col_start,
                              int max_rows, int max_cols, int src_stride, cudaStream_t stream) {
    if (!src || !dst) return FlashAttentionError::NULL_POINTER;
    const FlashAttentionError e = check_window(row_start, col_start, max_rows, max_cols, src_stride);
    if (e != FlashAttentionError::SUCCESS) return e;
    tile_load_kernel<R, C, float><<<1, kPrimThreads, 0, stream>>>(src, dst, row_start, col_start,
                                                                  max_rows, max_cols, src_stride);
    return launch_status();
}
template <int R, int C>
FlashAttentionError load_tile(const half* src, float* dst, int row_start, int col_start,
                              int max_rows, int max_cols, int src_stride, cudaStream_t stream) {
    if (!src || !dst) return FlashAttentionError::NULL_POINTER;
    const FlashAttentionError e = check_window(row_start, col_start, max_rows, max_cols, src_stride);
    if (e != FlashAttentionError::SUCCESS) return e;
    tile_load_kernel<R, C, half><<<1, kPrimThreads, 0, stream>>>(src, dst, row_start, col_start,
                                                                 max_rows, max_cols, src_stride);
    return launch_status();
}
template <int R, int C>
FlashAttentionError store_tile(const float* src, float* dst, int row_start, int col_start,
                               int max_rows, int max_cols, int dst_stride, cudaStream_t stream) {
    if (!src || !dst) return FlashAttentionError::NULL_POINTER;
    const FlashAttentionError e = check_window(row_start, col_start, max_rows, max_cols, dst_stride);
    if (e != FlashAttentionError::SUCCESS) return e;
    tile_store_kernel<R, C, float><<<1, kPrimThreads, 0, stream>>>(src, dst, row_start, col_start,
                                                                   max_rows, max_cols, dst_stride);
    return launch_status();
}
template <int R, int C>
FlashAttentionError store_tile(const float* src, half* dst, int row_start, int col_start,
                               int max_rows, int max_cols, int dst_stride, cudaStream_t stream) {
    if (!src || !dst) return FlashAttentionError::NULL_POINTER;
    const FlashAttentionError e = check_window(row_start, col_start, max_rows, max_cols, dst_stride);
    if (e != FlashAttentionError::SUCCESS) return e;
    tile_store_kernel<R, C, half><<<1, kPrimThreads, 0, stream>>>(src, dst, row_start, col_start,
                                                                  max_rows, max_cols, dst_stride);
    return launch_status();
}
template <int R, int C>
FlashAttentionError load_store_tile_roundtrip(const float* src, float* dst, int row_start,
                                              int col_start, int max_rows, int max_cols,
                                              int stride, cudaStream_t stream) {
    if (!src || !dst) return FlashAttentionError::NULL_POINTER;
    const FlashAttentionError e = check_window(row_start, col_start, max_rows, max_cols, stride);
    if (e != FlashAttentionError::SUCCESS) return e;
    tile_copy_kernel<R, C><<<1, kPrimThreads, 0, stream>>>(src, dst, row_start, col_start,
                                                           max_rows, max_cols, stride);
    return launch_status();
}

#define CUFLASH_TILE_SHAPE(R, C)                                                                  \
    template FlashAttentionError load_tile<R, C>(const float*, float*, int, int, int, int, int,  \
                                                 cudaStream_t);                                  \
    template FlashAttentionError load_tile<R, C>(const half*, float*, int, int, int, int, int,   \
                                                 cudaStream_t);                                  \
    template FlashAttentionError store_tile<R, C>(const float*, float*, int, int, int, int, int, \
                                                  cudaStream_t);                                 \
    template FlashAttentionError store_tile<R, C>(const float*, half*, int, int, int, int, int,  \
                                                  cudaStream_t);
CUFLASH_TILE_SHAPE(64, 64)
CUFLASH_TILE_SHAPE(32, 32)
CUFLASH_TILE_SHAPE(64, 32)
CUFLASH_TILE_SHAPE(32, 64)
CUFLASH_TILE_SHAPE(64, 128)
CUFLASH_TILE_SHAPE(32, 128)
#undef CUFLASH_TILE_SHAPE
template FlashAttentionError load_store_tile_roundtrip<64, 64>(const float*, float*, int, int, int,
                                                               int, int, cudaStream_t);

}  // namespace kernels
}  // namespace cuflash
