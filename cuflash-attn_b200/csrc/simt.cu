// Warp-per-row CUDA-core attention backward, computed in fp32: the fp32
// backward of the library (the reference's fp32 backward is
// src/backward/flash_attention_backward_typed.cu:13-288).
//
// D_i = rowsum(dO_i * O_i) (as the reference's compute_D_kernel),
// then a warp per query row accumulates dQ and a warp per key row
// accumulates dK and dV, each recomputing P_ij = exp(scale q_i.k_j - L_i).

#include <cmath>

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
    if constexpr (std::is_same<T, float>::value)
        return *p;
    else
        return DType<T>::to_float(*p);
}

template <typename T>
__device__ __forceinline__ void st_f(T* p, float v) {
    if constexpr (std::is_same<T, float>::value)
        *p = v;
    else
        *p = DType<T>::from_float(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

constexpr int kRowsPerCta = 4;

template <typename T, int D>
__global__ void __launch_bounds__(128)
    bwd_dvec_kernel(const T* __restrict__ O, const T* __restrict__ dO, float* __restrict__ Dv,
                    long long rows) {
    constexpr int E = D / 32;
    const int lane = threadIdx.x & 31;
    const long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e)
        acc = fmaf(ld_f(O + r * D + lane + 32 * e), ld_f(dO + r * D + lane + 32 * e), acc);
    acc = warp_sum(acc);
    if (lane == 0) Dv[r] = acc;
}

template <typename T, int D>
__global__ void __launch_bounds__(128)
    bwd_dq_simt_kernel(const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V,
                       const float* __restrict__ L, const T* __restrict__ dO,
                       const float* __restrict__ Dv, T* __restrict__ dQ, int N, float scale,
                       int causal) {
    constexpr int E = D / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // one-dimensional grid: (b,h) major, row block minor (no 65535 bound on b*h)
    const int nrb = (N + kRowsPerCta - 1) / kRowsPerCta;
    const long long bh = blockIdx.x / nrb;
    const int i = static_cast<int>(blockIdx.x - bh * nrb) * kRowsPerCta + warp;
    if (i >= N) return;
    const long long rowQ = (bh * N + i) * D;
    float q[E], g[E], acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        q[e] = ld_f(Q + rowQ + lane + 32 * e);
        g[e] = ld_f(dO + rowQ + lane + 32 * e);
        acc[e] = 0.f;
    }
    const float Li = L[bh * N + i];
    const float Di = Dv[bh * N + i];
    const int jend = causal ? i + 1 : N;
    for (int j = 0; j < jend; ++j) {
        const long long rowK = (bh * N + j) * D;
        float s = 0.f, dp = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            s = fmaf(q[e], ld_f(K + rowK + lane + 32 * e), s);
            dp = fmaf(g[e], ld_f(V + rowK + lane + 32 * e), dp);
        }
        s = warp_sum(s);
        dp = warp_sum(dp);
        const float pr = expf(s * scale - Li);
        const float ds = pr * (dp - Di);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] = fmaf(ds, ld_f(K + rowK + lane + 32 * e), acc[e]);
    }
#pragma unroll
    for (int e = 0; e < E; ++e) st_f(dQ + rowQ + lane + 32 * e, acc[e] * scale);
}

template <typename T, int D>
__global__ void __launch_bounds__(128)
    bwd_dkdv_simt_kernel(const T* __restrict__ Q, const T* __restrict__ K,
                         const T* __restrict__ V, const float* __restrict__ L,
                         const T* __restrict__ dO, const float* __restrict__ Dv,
                         T* __restrict__ dK, T* __restrict__ dV, int N, float scale, int causal) {
    constexpr int E = D / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nrb = (N + kRowsPerCta - 1) / kRowsPerCta;
    const long long bh = blockIdx.x / nrb;
    const int j = static_cast<int>(blockIdx.x - bh * nrb) * kRowsPerCta + warp;
    if (j >= N) return;
    const long long rowK = (bh * N + j) * D;
    float k[E], v[E], ak[E], av[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        k[e] = ld_f(K + rowK + lane + 32 * e);
        v[e] = ld_f(V + rowK + lane + 32 * e);
        ak[e] = 0.f;
        av[e] = 0.f;
    }
    for (int i = causal ? j : 0; i < N; ++i) {
        const long long rowQ = (bh * N + i) * D;
        float s = 0.f, dp = 0.f;
        float q[E], g[E];
#pragma unroll
        for (int e = 0; e < E; ++e) {
            q[e] = ld_f(Q + rowQ + lane + 32 * e);
            g[e] = ld_f(dO + rowQ + lane + 32 * e);
            s = fmaf(q[e], k[e], s);
            dp = fmaf(g[e], v[e], dp);
        }
        s = warp_sum(s);
        dp = warp_sum(dp);
        const float pr = expf(s * scale - L[bh * N + i]);
        const float ds = pr * (dp - Dv[bh * N + i]);
#pragma unroll
        for (int e = 0; e < E; ++e) {
            ak[e] = fmaf(ds, q[e], ak[e]);
            av[e] = fmaf(pr, g[e], av[e]);
        }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
        st_f(dK + rowK + lane + 32 * e, ak[e] * scale);
        st_f(dV + rowK + lane + 32 * e, av[e]);
    }
}

template <typename T, int D>
FlashAttentionError bwd_simt_typed(const T* Q, const T* K, const T* V, const T* O, const float* L,
                                   const T* dO, T* dQ, T* dK, T* dV, int BH, int N, float scale,
                                   bool causal, cudaStream_t stream) {
    const long long rows = static_cast<long long>(BH) * N;
    const long long nblk = static_cast<long long>((N + kRowsPerCta - 1) / kRowsPerCta) * BH;
    if (nblk > 0x7fffffffLL) return FlashAttentionError::INVALID_DIMENSION;
    void* ws = nullptr;
    const FlashAttentionError werr =
        workspace_alloc(&ws, static_cast<size_t>(rows) * sizeof(float), stream);
    if (werr != FlashAttentionError::SUCCESS) return werr;
    float* dvec = static_cast<float*>(ws);
    bwd_dvec_kernel<T, D><<<static_cast<unsigned>((rows * 32 + 127) / 128), 128, 0, stream>>>(
        O, dO, dvec, rows);
    cudaError_t e1 = cudaGetLastError();
    const dim3 grid(static_cast<unsigned>(nblk));
    bwd_dq_simt_kernel<T, D><<<grid, 32 * kRowsPerCta, 0, stream>>>(Q, K, V, L, dO, dvec, dQ, N,
                                                                    scale, causal ? 1 : 0);
    cudaError_t e2 = cudaGetLastError();
    bwd_dkdv_simt_kernel<T, D><<<grid, 32 * kRowsPerCta, 0, stream>>>(
        Q, K, V, L, dO, dvec, dK, dV, N, scale, causal ? 1 : 0);
    cudaError_t e3 = cudaGetLastError();
    workspace_free(ws, stream);
    return (e1 == cudaSuccess && e2 == cudaSuccess && e3 == cudaSuccess)
               ? FlashAttentionError::SUCCESS
               : FlashAttentionError::CUDA_ERROR;
}

}  // namespace

template <typename T>
FlashAttentionError launch_bwd_simt(const T* Q, const T* K, const T* V, const T* O,
                                    const float* L, const T* dO, T* dQ, T* dK, T* dV, int B,
                                    int H, int N, int D, float scale, bool causal,
                                    cudaStream_t stream) {
    const int BH = B * H;
    switch (D) {
        case 32:
            return bwd_simt_typed<T, 32>(Q, K, V, O, L, dO, dQ, dK, dV, BH, N, scale, causal,
                                         stream);
        case 64:
            return bwd_simt_typed<T, 64>(Q, K, V, O, L, dO, dQ, dK, dV, BH, N, scale, causal,
                                         stream);
        case 128:
            return bwd_simt_typed<T, 128>(Q, K, V, O, L, dO, dQ, dK, dV, BH, N, scale, causal,
                                          stream);
        default:
            return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
}

#define CUFLASH_SIMT_INSTANTIATE(T)                                                          \
    template FlashAttentionError launch_bwd_simt<T>(const T*, const T*, const T*, const T*,   \
                                                    const float*, const T*, T*, T*, T*, int,  \
                                                    int, int, int, float, bool, cudaStream_t);
CUFLASH_SIMT_INSTANTIATE(float)
CUFLASH_SIMT_INSTANTIATE(half)
CUFLASH_SIMT_INSTANTIATE(__nv_bfloat16)
#undef CUFLASH_SIMT_INSTANTIATE

FlashAttentionError launch_bwd_f32(const float* Q, const float* K, const float* V,
                                   const float* O, const float* L, const float* dO, float* dQ,
                                   float* dK, float* dV, int B, int H, int N, int D, float scale,
                                   bool causal, cudaStream_t stream) {
    return launch_bwd_simt<float>(Q, K, V, O, L, dO, dQ, dK, dV, B, H, N, D, scale, causal,
                                  stream);
}

}  // namespace detail
}  // namespace cuflash
