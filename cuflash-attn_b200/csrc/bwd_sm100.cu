// Backward attention for fp16/bf16 on sm_100a.
//
// Replaces the reference's three backward kernels
// (src/backward/flash_attention_backward_typed.cu:13-288).

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {
__device__ int g_bwd_status;
}  // namespace

template <typename T>
FlashAttentionError launch_bwd_sm100(const T* Q, const T* K, const T* V, const T* O,
                                     const float* L, const T* dO, T* dQ, T* dK, T* dV, int B,
                                     int H, int N, int D, float scale, bool causal,
                                     cudaStream_t stream) {
    return launch_bwd_simt<T>(Q, K, V, O, L, dO, dQ, dK, dV, B, H, N, D, scale, causal, stream);
}

template FlashAttentionError launch_bwd_sm100<half>(const half*, const half*, const half*,
                                                    const half*, const float*, const half*, half*,
                                                    half*, half*, int, int, int, int, float, bool,
                                                    cudaStream_t);
template FlashAttentionError launch_bwd_sm100<__nv_bfloat16>(
    const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
    const float*, const __nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16*, int, int,
    int, int, float, bool, cudaStream_t);

int bwd_sm100_status() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_bwd_status, sizeof(int)) != cudaSuccess) return -1;
    if (v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_bwd_status, &zero, sizeof(int));
    }
    return v;
}

}  // namespace detail
}  // namespace cuflash
