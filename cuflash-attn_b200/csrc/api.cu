// Public API: argument validation, the C++ overloads and the C ABI.
//
// Mirrors the reference's src/api/flash_attention_api.cu:
//   * error strings byte-identical to :21-42 (pinned by the reference's
//     tests/unit/test_error_handling.cu:236-254);
//   * validation order of validate_common_params (:45-66): null pointer,
//     non-positive dimension, unsupported head_dim, non-finite or negative
//     scale (scale == 0 is accepted);
//   * backward checks dO/dQ/dK/dV for null before the common checks (:69-79);
//   * no CUDA call happens before validation succeeds, so invalid arguments
//     are reported on a machine without a GPU.
// Dispatch differs: fp16/bf16 go to the tcgen05 kernels, fp32 to the fp32
// kernels; there is no CPU path.

#include <cmath>
#include <initializer_list>

#include "common.cuh"

namespace cuflash {

namespace {

using detail::launch_bwd_f32;
using detail::launch_bwd_sm100;
using detail::launch_fwd_f32;
using detail::launch_fwd_sm100;

inline bool supported_head_dim(int d) { return d == 32 || d == 64 || d == 128; }

FlashAttentionError validate_common(const void* Q, const void* K, const void* V, const void* O,
                                    const void* L, int batch_size, int num_heads, int seq_len,
                                    int head_dim, float scale) {
    if (!Q || !K || !V || !O || !L) return FlashAttentionError::NULL_POINTER;
    if (batch_size <= 0 || num_heads <= 0 || seq_len <= 0 || head_dim <= 0)
        return FlashAttentionError::INVALID_DIMENSION;
    if (!supported_head_dim(head_dim)) return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    if (!std::isfinite(scale) || scale < 0.0f) return FlashAttentionError::INVALID_DIMENSION;
    return FlashAttentionError::SUCCESS;
}

FlashAttentionError validate_backward(const void* Q, const void* K, const void* V, const void* O,
                                      const void* L, const void* dO, const void* dQ,
                                      const void* dK, const void* dV, int batch_size,
                                      int num_heads, int seq_len, int head_dim, float scale) {
    if (!dO || !dQ || !dK || !dV) return FlashAttentionError::NULL_POINTER;
    return validate_common(Q, K, V, O, L, batch_size, num_heads, seq_len, head_dim, scale);
}

// The launchers index with 32-bit grid coordinates over batch*heads.
bool fits_grid(int batch_size, int num_heads) {
    return static_cast<long long>(batch_size) * num_heads <= 0x7fffffffLL;
}

template <typename T>
FlashAttentionError forward_lowp(const T* Q, const T* K, const T* V, T* O, float* L, int B, int H,
                                 int N, int D, float scale, bool causal, cudaStream_t stream) {
    FlashAttentionError e = validate_common(Q, K, V, O, L, B, H, N, D, scale);
    if (e != FlashAttentionError::SUCCESS) return e;
    if (!fits_grid(B, H)) return FlashAttentionError::INVALID_DIMENSION;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return launch_fwd_sm100<T>(Q, K, V, O, L, B, H, N, N, D, scale, causal, 0, 0, false, stream);
}

template <typename T>
FlashAttentionError backward_lowp(const T* Q, const T* K, const T* V, const T* O, const float* L,
                                  const T* dO, T* dQ, T* dK, T* dV, int B, int H, int N, int D,
                                  float scale, bool causal, cudaStream_t stream) {
    FlashAttentionError e = validate_backward(Q, K, V, O, L, dO, dQ, dK, dV, B, H, N, D, scale);
    if (e != FlashAttentionError::SUCCESS) return e;
    if (!fits_grid(B, H)) return FlashAttentionError::INVALID_DIMENSION;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return launch_bwd_sm100<T>(Q, K, V, O, L, dO, dQ, dK, dV, B, H, N, D, scale, causal, stream);
}

}  // namespace

const char* get_error_string(FlashAttentionError error) {
    switch (error) {
        case FlashAttentionError::SUCCESS:
            return "Success";
        case FlashAttentionError::INVALID_DIMENSION:
            return "Invalid dimension: dimensions must be positive";
        case FlashAttentionError::DIMENSION_MISMATCH:
            return "Dimension mismatch: Q, K, V tensors have incompatible shapes";
        case FlashAttentionError::NULL_POINTER:
            return "Null pointer: input or output pointer is null";
        case FlashAttentionError::CUDA_ERROR:
            return "CUDA error occurred";
        case FlashAttentionError::OUT_OF_MEMORY:
            return "Out of memory: insufficient GPU memory";
        case FlashAttentionError::UNSUPPORTED_HEAD_DIM:
            return "Unsupported head_dim: must be 32, 64, or 128";
        case FlashAttentionError::UNSUPPORTED_DTYPE:
            return "Unsupported data type";
        default:
            return "Unknown error";
    }
}

FlashAttentionError flash_attention_forward(const float* Q, const float* K, const float* V,
                                            float* O, float* L, int batch_size, int num_heads,
                                            int seq_len, int head_dim, float scale, bool causal,
                                            cudaStream_t stream) {
    FlashAttentionError e =
        validate_common(Q, K, V, O, L, batch_size, num_heads, seq_len, head_dim, scale);
    if (e != FlashAttentionError::SUCCESS) return e;
    if (!fits_grid(batch_size, num_heads)) return FlashAttentionError::INVALID_DIMENSION;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return launch_fwd_f32(Q, K, V, O, L, batch_size, num_heads, seq_len, head_dim, scale, causal,
                          stream);
}

FlashAttentionError flash_attention_forward(const half* Q, const half* K, const half* V, half* O,
                                            float* L, int batch_size, int num_heads, int seq_len,
                                            int head_dim, float scale, bool causal,
                                            cudaStream_t stream) {
    return forward_lowp<half>(Q, K, V, O, L, batch_size, num_heads, seq_len, head_dim, scale,
                              causal, stream);
}

FlashAttentionError flash_attention_forward(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                            const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                            int batch_size, int num_heads, int seq_len,
                                            int head_dim, float scale, bool causal,
                                            cudaStream_t stream) {
    return forward_lowp<__nv_bfloat16>(Q, K, V, O, L, batch_size, num_heads, seq_len, head_dim,
                                       scale, causal, stream);
}

FlashAttentionError flash_attention_backward(const float* Q, const float* K, const float* V,
                                             const float* O, const float* L, const float* dO,
                                             float* dQ, float* dK, float* dV, int batch_size,
                                             int num_heads, int seq_len, int head_dim, float scale,
                                             bool causal, cudaStream_t stream) {
    FlashAttentionError e = validate_backward(Q, K, V, O, L, dO, dQ, dK, dV, batch_size,
                                              num_heads, seq_len, head_dim, scale);
    if (e != FlashAttentionError::SUCCESS) return e;
    if (!fits_grid(batch_size, num_heads)) return FlashAttentionError::INVALID_DIMENSION;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return launch_bwd_f32(Q, K, V, O, L, dO, dQ, dK, dV, batch_size, num_heads, seq_len,
                          head_dim, scale, causal, stream);
}

FlashAttentionError flash_attention_backward(const half* Q, const half* K, const half* V,
                                             const half* O, const float* L, const half* dO,
                                             half* dQ, half* dK, half* dV, int batch_size,
                                             int num_heads, int seq_len, int head_dim, float scale,
                                             bool causal, cudaStream_t stream) {
    return backward_lowp<half>(Q, K, V, O, L, dO, dQ, dK, dV, batch_size, num_heads, seq_len,
                               head_dim, scale, causal, stream);
}

FlashAttentionError flash_attention_backward(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                             const __nv_bfloat16* V, const __nv_bfloat16* O,
                                             const float* L, const __nv_bfloat16* dO,
                                             __nv_bfloat16* dQ, __nv_bfloat16* dK,
                                             __nv_bfloat16* dV, int batch_size, int num_heads,
                                             int seq_len, int head_dim, float scale, bool causal,
                                             cudaStream_t stream) {
    return backward_lowp<__nv_bfloat16>(Q, K, V, O, L, dO, dQ, dK, dV, batch_size, num_heads,
                                        seq_len, head_dim, scale, causal, stream);
}

}  // namespace cuflash

namespace {

using cuflash::FlashAttentionError;

template <typename T>
FlashAttentionError decode_impl(const T* Q, const T* K, const T* V, T* O, float* L, int B, int H,
                                int kv_len, int D, float scale, int num_splits,
                                cudaStream_t stream) {
    if (!Q || !K || !V || !O || !L) return FlashAttentionError::NULL_POINTER;
    if (B <= 0 || H <= 0 || kv_len <= 0 || D <= 0) return FlashAttentionError::INVALID_DIMENSION;
    if (!(D == 32 || D == 64 || D == 128)) return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    if (!std::isfinite(scale) || scale < 0.0f) return FlashAttentionError::INVALID_DIMENSION;
    if (num_splits < 0 || num_splits > 64) return FlashAttentionError::INVALID_DIMENSION;
    if (static_cast<long long>(B) * H > 0x7fffffffLL) return FlashAttentionError::INVALID_DIMENSION;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return cuflash::detail::launch_decode<T>(Q, K, V, O, L, B, H, kv_len, D, scale, num_splits,
                                             stream);
}

template <typename T>
FlashAttentionError decode_gqa_impl(const T* Q, const T* K, const T* V, T* O, float* L, int B,
                                    int Hq, int Hkv, int kv_len, int D, float scale,
                                    int num_splits, const int* block_table, const int* seq_lens,
                                    int page_size, int max_pages, int num_pages,
                                    cudaStream_t stream) {
    const bool paged = block_table != nullptr || seq_lens != nullptr;
    if (!Q || !K || !V || !O || !L) return FlashAttentionError::NULL_POINTER;
    if (paged && (!block_table || !seq_lens)) return FlashAttentionError::NULL_POINTER;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0) return FlashAttentionError::INVALID_DIMENSION;
    if (!paged && kv_len <= 0) return FlashAttentionError::INVALID_DIMENSION;
    if (paged && (page_size <= 0 || (page_size & (page_size - 1)) != 0 || max_pages <= 0 ||
                  num_pages <= 0 || static_cast<long long>(max_pages) * page_size > 0x7fffffffLL))
        return FlashAttentionError::INVALID_DIMENSION;
    if (Hq % Hkv != 0) return FlashAttentionError::DIMENSION_MISMATCH;
    if (!(D == 32 || D == 64 || D == 128)) return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    if (!std::isfinite(scale) || scale < 0.0f) return FlashAttentionError::INVALID_DIMENSION;
    if (num_splits < 0 || num_splits > 64) return FlashAttentionError::INVALID_DIMENSION;
    if (static_cast<long long>(B) * Hq > 0x7fffffffLL) return FlashAttentionError::INVALID_DIMENSION;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return cuflash::detail::launch_decode_gqa<T>(Q, K, V, O, L, B, Hq, Hkv, kv_len, D, scale,
                                                 num_splits, block_table, seq_lens, page_size,
                                                 max_pages, num_pages, stream);
}

template <typename T>
FlashAttentionError partial_impl(const T* Q, const T* K, const T* V, float* O, float* L, int B,
                                 int H, int seq_q, int seq_k, int D, float scale,
                                 long long q_offset, long long k_offset, bool causal,
                                 cudaStream_t stream) {
    if (!Q || !K || !V || !O || !L) return FlashAttentionError::NULL_POINTER;
    if (B <= 0 || H <= 0 || seq_q <= 0 || seq_k <= 0 || D <= 0)
        return FlashAttentionError::INVALID_DIMENSION;
    if (!(D == 32 || D == 64 || D == 128)) return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    if (!std::isfinite(scale) || scale < 0.0f) return FlashAttentionError::INVALID_DIMENSION;
    if (q_offset < 0 || k_offset < 0) return FlashAttentionError::INVALID_DIMENSION;
    if (static_cast<long long>(B) * H > 0x7fffffffLL) return FlashAttentionError::INVALID_DIMENSION;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return cuflash::detail::launch_fwd_sm100<T>(Q, K, V, O, L, B, H, seq_q, seq_k, D, scale,
                                                causal, q_offset, k_offset, true, stream);
}

// Grouped-query / unequal-length checks, in the reference's order (null
// pointers, dimensions, head_dim, scale) plus the head-group relation.
FlashAttentionError validate_gqa(std::initializer_list<const void*> ptrs, int B, int Hq, int Hkv,
                                 int Nq, int Nk, int D, float scale) {
    for (const void* ptr : ptrs)
        if (!ptr) return FlashAttentionError::NULL_POINTER;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Nq <= 0 || Nk <= 0 || D <= 0)
        return FlashAttentionError::INVALID_DIMENSION;
    if (Hq % Hkv != 0) return FlashAttentionError::DIMENSION_MISMATCH;
    if (!(D == 32 || D == 64 || D == 128)) return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    if (!std::isfinite(scale) || scale < 0.0f) return FlashAttentionError::INVALID_DIMENSION;
    if (static_cast<long long>(B) * Hq > 0x7fffffffLL) return FlashAttentionError::INVALID_DIMENSION;
    return FlashAttentionError::SUCCESS;
}

template <typename T>
FlashAttentionError fwd_gqa_impl(const T* Q, const T* K, const T* V, T* O, float* L, int B, int Hq,
                                 int Hkv, int Nq, int Nk, int D, float scale, bool causal,
                                 cudaStream_t stream) {
    const FlashAttentionError e = validate_gqa({Q, K, V, O, L}, B, Hq, Hkv, Nq, Nk, D, scale);
    if (e != FlashAttentionError::SUCCESS) return e;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return cuflash::detail::launch_fwd_gqa_sm100<T>(Q, K, V, O, L, B, Hq, Hkv, Nq, Nk, D, scale,
                                                    causal, stream);
}

template <typename T>
FlashAttentionError bwd_gqa_impl(const T* Q, const T* K, const T* V, const T* O, const float* L,
                                 const T* dO, T* dQ, T* dK, T* dV, int B, int Hq, int Hkv, int Nq,
                                 int Nk, int D, float scale, bool causal, cudaStream_t stream) {
    const FlashAttentionError e =
        validate_gqa({dO, dQ, dK, dV, Q, K, V, O, L}, B, Hq, Hkv, Nq, Nk, D, scale);
    if (e != FlashAttentionError::SUCCESS) return e;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return cuflash::detail::launch_bwd_gqa_sm100<T>(Q, K, V, O, L, dO, dQ, dK, dV, B, Hq, Hkv, Nq,
                                                    Nk, D, scale, causal, stream);
}

template <typename T>
FlashAttentionError cp_step_impl(const T* Q, const T* K, const T* V, float* O_acc, float* L_acc,
                                 int nq, int nk, int B, int H, int C, int D, float scale,
                                 bool causal, int num_pairs, const int* q_slot, const int* kv_slot,
                                 const long long* q_off, const long long* kv_off, int reserve_sms,
                                 cudaStream_t stream) {
    if (!Q || !K || !V || !O_acc || !L_acc || !q_slot || !kv_slot || !q_off || !kv_off)
        return FlashAttentionError::NULL_POINTER;
    if (nq <= 0 || nk <= 0 || B <= 0 || H <= 0 || C <= 0 || D <= 0)
        return FlashAttentionError::INVALID_DIMENSION;
    if (!(D == 32 || D == 64 || D == 128)) return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    if (!std::isfinite(scale) || scale < 0.0f) return FlashAttentionError::INVALID_DIMENSION;
    if (num_pairs < 1 || num_pairs > 4 || reserve_sms < 0)
        return FlashAttentionError::INVALID_DIMENSION;
    if (static_cast<long long>(B) * H * (nq > nk ? nq : nk) > 0x7fffffffLL)
        return FlashAttentionError::INVALID_DIMENSION;
    for (int i = 0; i < num_pairs; ++i) {
        if (q_slot[i] < 0 || q_slot[i] >= nq || kv_slot[i] < 0 || kv_slot[i] >= nk ||
            q_off[i] < 0 || kv_off[i] < 0)
            return FlashAttentionError::INVALID_DIMENSION;
        for (int k = 0; k < i; ++k)  // the merge writes each query slot once per launch
            if (q_slot[k] == q_slot[i]) return FlashAttentionError::INVALID_DIMENSION;
    }
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return cuflash::detail::launch_fwd_cp_step_sm100<T>(Q, K, V, O_acc, L_acc, nq, nk, B, H, C, D,
                                                        scale, causal, num_pairs, q_slot, kv_slot,
                                                        q_off, kv_off, reserve_sms, stream);
}

FlashAttentionError cp_dims_check(int nq, int B, int H, int C, int D) {
    if (nq <= 0 || B <= 0 || H <= 0 || C <= 0 || D <= 0)
        return FlashAttentionError::INVALID_DIMENSION;
    if (!(D == 32 || D == 64 || D == 128)) return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    if (static_cast<long long>(B) * H * nq > 0x7fffffffLL) return FlashAttentionError::INVALID_DIMENSION;
    return FlashAttentionError::SUCCESS;
}

template <typename T>
FlashAttentionError cp_bwd_prepare_impl(const T* O, const T* dO, const float* L, void* ws, int nq,
                                        int B, int H, int C, int D, cudaStream_t stream) {
    if (!O || !dO || !L || !ws) return FlashAttentionError::NULL_POINTER;
    const FlashAttentionError e = cp_dims_check(nq, B, H, C, D);
    if (e != FlashAttentionError::SUCCESS) return e;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return cuflash::detail::launch_bwd_cp_prepare_sm100<T>(O, dO, L, ws, nq, B * H, C, D, stream);
}

template <typename T>
FlashAttentionError cp_bwd_step_impl(const T* Q, const T* dO, const T* K, const T* V, void* ws,
                                     float* dK_acc, float* dV_acc, int nq, int nk, int B, int H,
                                     int C, int D, float scale, bool causal, int num_pairs,
                                     const int* q_slot, const int* kv_slot,
                                     const long long* q_off, const long long* kv_off,
                                     int reserve_sms, cudaStream_t stream) {
    if (!Q || !dO || !K || !V || !ws || !dK_acc || !dV_acc || !q_slot || !kv_slot || !q_off ||
        !kv_off)
        return FlashAttentionError::NULL_POINTER;
    FlashAttentionError e = cp_dims_check(nq, B, H, C, D);
    if (e == FlashAttentionError::SUCCESS) e = cp_dims_check(nk, B, H, C, D);
    if (e != FlashAttentionError::SUCCESS) return e;
    if (!std::isfinite(scale) || scale < 0.0f) return FlashAttentionError::INVALID_DIMENSION;
    if (num_pairs < 1 || num_pairs > 4 || reserve_sms < 0)
        return FlashAttentionError::INVALID_DIMENSION;
    for (int i = 0; i < num_pairs; ++i) {
        if (q_slot[i] < 0 || q_slot[i] >= nq || kv_slot[i] < 0 || kv_slot[i] >= nk ||
            q_off[i] < 0 || kv_off[i] < 0)
            return FlashAttentionError::INVALID_DIMENSION;
        // a repeated (query slot, K/V slot) pair would add its gradients twice
        for (int k = 0; k < i; ++k)
            if (q_slot[k] == q_slot[i] && kv_slot[k] == kv_slot[i])
                return FlashAttentionError::INVALID_DIMENSION;
    }
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return cuflash::detail::launch_bwd_cp_step_sm100<T>(Q, dO, K, V, ws, dK_acc, dV_acc, nq, nk,
                                                        B * H, C, D, scale, causal, num_pairs,
                                                        q_slot, kv_slot, q_off, kv_off,
                                                        reserve_sms, stream);
}

template <typename T>
FlashAttentionError cp_bwd_finish_impl(const void* ws, T* dQ, int nq, int B, int H, int C, int D,
                                       float scale, cudaStream_t stream) {
    if (!ws || !dQ) return FlashAttentionError::NULL_POINTER;
    const FlashAttentionError e = cp_dims_check(nq, B, H, C, D);
    if (e != FlashAttentionError::SUCCESS) return e;
    if (!std::isfinite(scale) || scale < 0.0f) return FlashAttentionError::INVALID_DIMENSION;
    if (cuflash::detail::sticky_failure()) return FlashAttentionError::CUDA_ERROR;
    return cuflash::detail::launch_bwd_cp_finish_sm100<T>(ws, dQ, nq, B * H, C, D, scale, stream);
}

}  // namespace

extern "C" {

int cuflash_attention_forward_f32(const float* Q, const float* K, const float* V, float* O,
                                  float* L, int batch_size, int num_heads, int seq_len,
                                  int head_dim, float scale, bool causal, cudaStream_t stream) {
    return static_cast<int>(cuflash::flash_attention_forward(
        Q, K, V, O, L, batch_size, num_heads, seq_len, head_dim, scale, causal, stream));
}

int cuflash_attention_backward_f32(const float* Q, const float* K, const float* V, const float* O,
                                   const float* L, const float* dO, float* dQ, float* dK, float* dV,
                                   int batch_size, int num_heads, int seq_len, int head_dim,
                                   float scale, bool causal, cudaStream_t stream) {
    return static_cast<int>(cuflash::flash_attention_backward(Q, K, V, O, L, dO, dQ, dK, dV,
                                                              batch_size, num_heads, seq_len,
                                                              head_dim, scale, causal, stream));
}

int cuflash_attention_forward_f16(const half* Q, const half* K, const half* V, half* O, float* L,
                                  int batch_size, int num_heads, int seq_len, int head_dim,
                                  float scale, bool causal, cudaStream_t stream) {
    return static_cast<int>(cuflash::flash_attention_forward(
        Q, K, V, O, L, batch_size, num_heads, seq_len, head_dim, scale, causal, stream));
}

int cuflash_attention_backward_f16(const half* Q, const half* K, const half* V, const half* O,
                                   const float* L, const half* dO, half* dQ, half* dK, half* dV,
                                   int batch_size, int num_heads, int seq_len, int head_dim,
                                   float scale, bool causal, cudaStream_t stream) {
    return static_cast<int>(cuflash::flash_attention_backward(Q, K, V, O, L, dO, dQ, dK, dV,
                                                              batch_size, num_heads, seq_len,
                                                              head_dim, scale, causal, stream));
}

int cuflash_attention_forward_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                   const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                   int batch_size, int num_heads, int seq_len, int head_dim,
                                   float scale, bool causal, cudaStream_t stream) {
    return static_cast<int>(cuflash::flash_attention_forward(
        Q, K, V, O, L, batch_size, num_heads, seq_len, head_dim, scale, causal, stream));
}

int cuflash_attention_backward_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                    const __nv_bfloat16* V, const __nv_bfloat16* O, const float* L,
                                    const __nv_bfloat16* dO, __nv_bfloat16* dQ, __nv_bfloat16* dK,
                                    __nv_bfloat16* dV, int batch_size, int num_heads, int seq_len,
                                    int head_dim, float scale, bool causal, cudaStream_t stream) {
    return static_cast<int>(cuflash::flash_attention_backward(Q, K, V, O, L, dO, dQ, dK, dV,
                                                              batch_size, num_heads, seq_len,
                                                              head_dim, scale, causal, stream));
}

const char* cuflash_error_string(int error_code) {
    return cuflash::get_error_string(static_cast<cuflash::FlashAttentionError>(error_code));
}

int cuflash_attention_decode_f16(const half* Q, const half* K, const half* V, half* O, float* L,
                                 int batch_size, int num_heads, int kv_len, int head_dim,
                                 float scale, int num_splits, cudaStream_t stream) {
    return static_cast<int>(decode_impl<half>(Q, K, V, O, L, batch_size, num_heads, kv_len,
                                              head_dim, scale, num_splits, stream));
}

int cuflash_attention_decode_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                  const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                  int batch_size, int num_heads, int kv_len, int head_dim,
                                  float scale, int num_splits, cudaStream_t stream) {
    return static_cast<int>(decode_impl<__nv_bfloat16>(Q, K, V, O, L, batch_size, num_heads,
                                                       kv_len, head_dim, scale, num_splits,
                                                       stream));
}

int cuflash_attention_forward_partial_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                           const __nv_bfloat16* V, float* O_part, float* L_part,
                                           int batch_size, int num_heads, int seq_q, int seq_k,
                                           int head_dim, float scale, long long q_offset,
                                           long long k_offset, bool causal, cudaStream_t stream) {
    return static_cast<int>(partial_impl<__nv_bfloat16>(Q, K, V, O_part, L_part, batch_size,
                                                        num_heads, seq_q, seq_k, head_dim, scale,
                                                        q_offset, k_offset, causal, stream));
}

int cuflash_attention_forward_partial_f16(const half* Q, const half* K, const half* V,
                                          float* O_part, float* L_part, int batch_size,
                                          int num_heads, int seq_q, int seq_k, int head_dim,
                                          float scale, long long q_offset, long long k_offset,
                                          bool causal, cudaStream_t stream) {
    return static_cast<int>(partial_impl<half>(Q, K, V, O_part, L_part, batch_size, num_heads,
                                               seq_q, seq_k, head_dim, scale, q_offset, k_offset,
                                               causal, stream));
}

int cuflash_attention_decode_gqa_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                      const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                      int batch_size, int num_q_heads, int num_kv_heads,
                                      int kv_len, int head_dim, float scale, int num_splits,
                                      cudaStream_t stream) {
    return static_cast<int>(decode_gqa_impl<__nv_bfloat16>(
        Q, K, V, O, L, batch_size, num_q_heads, num_kv_heads, kv_len, head_dim, scale,
        num_splits, nullptr, nullptr, 0, 0, 0, stream));
}

int cuflash_attention_decode_gqa_f16(const half* Q, const half* K, const half* V, half* O,
                                     float* L, int batch_size, int num_q_heads, int num_kv_heads,
                                     int kv_len, int head_dim, float scale, int num_splits,
                                     cudaStream_t stream) {
    return static_cast<int>(decode_gqa_impl<half>(Q, K, V, O, L, batch_size, num_q_heads,
                                                  num_kv_heads, kv_len, head_dim, scale,
                                                  num_splits, nullptr, nullptr, 0, 0, 0, stream));
}

int cuflash_attention_decode_paged_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K_cache,
                                        const __nv_bfloat16* V_cache, const int* block_table,
                                        const int* seq_lens, __nv_bfloat16* O, float* L,
                                        int batch_size, int num_q_heads, int num_kv_heads,
                                        int head_dim, int page_size, int max_pages_per_seq,
                                        int num_pages, float scale, int num_splits,
                                        cudaStream_t stream) {
    return static_cast<int>(decode_gqa_impl<__nv_bfloat16>(
        Q, K_cache, V_cache, O, L, batch_size, num_q_heads, num_kv_heads, 0, head_dim, scale,
        num_splits, block_table, seq_lens, page_size, max_pages_per_seq, num_pages, stream));
}

int cuflash_attention_decode_paged_f16(const half* Q, const half* K_cache, const half* V_cache,
                                       const int* block_table, const int* seq_lens, half* O,
                                       float* L, int batch_size, int num_q_heads,
                                       int num_kv_heads, int head_dim, int page_size,
                                       int max_pages_per_seq, int num_pages, float scale,
                                       int num_splits, cudaStream_t stream) {
    return static_cast<int>(decode_gqa_impl<half>(
        Q, K_cache, V_cache, O, L, batch_size, num_q_heads, num_kv_heads, 0, head_dim, scale,
        num_splits, block_table, seq_lens, page_size, max_pages_per_seq, num_pages, stream));
}

int cuflash_attention_forward_gqa_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                       const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                       int batch_size, int num_q_heads, int num_kv_heads,
                                       int seq_len_q, int seq_len_k, int head_dim, float scale,
                                       bool causal, cudaStream_t stream) {
    return static_cast<int>(fwd_gqa_impl<__nv_bfloat16>(Q, K, V, O, L, batch_size, num_q_heads,
                                                        num_kv_heads, seq_len_q, seq_len_k,
                                                        head_dim, scale, causal, stream));
}

int cuflash_attention_forward_gqa_f16(const half* Q, const half* K, const half* V, half* O,
                                      float* L, int batch_size, int num_q_heads, int num_kv_heads,
                                      int seq_len_q, int seq_len_k, int head_dim, float scale,
                                      bool causal, cudaStream_t stream) {
    return static_cast<int>(fwd_gqa_impl<half>(Q, K, V, O, L, batch_size, num_q_heads,
                                               num_kv_heads, seq_len_q, seq_len_k, head_dim,
                                               scale, causal, stream));
}

int cuflash_attention_backward_gqa_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                        const __nv_bfloat16* V, const __nv_bfloat16* O,
                                        const float* L, const __nv_bfloat16* dO,
                                        __nv_bfloat16* dQ, __nv_bfloat16* dK, __nv_bfloat16* dV,
                                        int batch_size, int num_q_heads, int num_kv_heads,
                                        int seq_len_q, int seq_len_k, int head_dim, float scale,
                                        bool causal, cudaStream_t stream) {
    return static_cast<int>(bwd_gqa_impl<__nv_bfloat16>(
        Q, K, V, O, L, dO, dQ, dK, dV, batch_size, num_q_heads, num_kv_heads, seq_len_q,
        seq_len_k, head_dim, scale, causal, stream));
}

int cuflash_attention_backward_gqa_f16(const half* Q, const half* K, const half* V, const half* O,
                                       const float* L, const half* dO, half* dQ, half* dK,
                                       half* dV, int batch_size, int num_q_heads, int num_kv_heads,
                                       int seq_len_q, int seq_len_k, int head_dim, float scale,
                                       bool causal, cudaStream_t stream) {
    return static_cast<int>(bwd_gqa_impl<half>(Q, K, V, O, L, dO, dQ, dK, dV, batch_size,
                                               num_q_heads, num_kv_heads, seq_len_q, seq_len_k,
                                               head_dim, scale, causal, stream));
}

int cuflash_attention_forward_cp_step_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                           const __nv_bfloat16* V, float* O_acc, float* L_acc,
                                           int num_q_slots, int num_kv_slots, int batch_size,
                                           int num_heads, int chunk_len, int head_dim, float scale,
                                           bool causal, int num_pairs, const int* q_slot,
                                           const int* kv_slot, const long long* q_offset,
                                           const long long* kv_offset, int reserve_sms,
                                           cudaStream_t stream) {
    return static_cast<int>(cp_step_impl<__nv_bfloat16>(
        Q, K, V, O_acc, L_acc, num_q_slots, num_kv_slots, batch_size, num_heads, chunk_len,
        head_dim, scale, causal, num_pairs, q_slot, kv_slot, q_offset, kv_offset, reserve_sms,
        stream));
}

int cuflash_attention_forward_cp_step_f16(const half* Q, const half* K, const half* V,
                                          float* O_acc, float* L_acc, int num_q_slots,
                                          int num_kv_slots, int batch_size, int num_heads,
                                          int chunk_len, int head_dim, float scale, bool causal,
                                          int num_pairs, const int* q_slot, const int* kv_slot,
                                          const long long* q_offset, const long long* kv_offset,
                                          int reserve_sms, cudaStream_t stream) {
    return static_cast<int>(cp_step_impl<half>(Q, K, V, O_acc, L_acc, num_q_slots, num_kv_slots,
                                               batch_size, num_heads, chunk_len, head_dim, scale,
                                               causal, num_pairs, q_slot, kv_slot, q_offset,
                                               kv_offset, reserve_sms, stream));
}

long long cuflash_attention_backward_cp_workspace_size(int num_q_slots, int batch_size,
                                                       int num_heads, int chunk_len,
                                                       int head_dim) {
    if (cp_dims_check(num_q_slots, batch_size, num_heads, chunk_len, head_dim) !=
        FlashAttentionError::SUCCESS)
        return 0;
    return cuflash::detail::bwd_cp_workspace_bytes(num_q_slots, batch_size * num_heads, chunk_len,
                                                   head_dim);
}

#define CUFLASH_CP_BWD_ENTRIES(SUFFIX, T)                                                        \
    int cuflash_attention_backward_cp_prepare_##SUFFIX(                                          \
        const T* O, const T* dO, const float* L, void* workspace, int num_q_slots,               \
        int batch_size, int num_heads, int chunk_len, int head_dim, cudaStream_t stream) {       \
        return static_cast<int>(cp_bwd_prepare_impl<T>(O, dO, L, workspace, num_q_slots,         \
                                                       batch_size, num_heads, chunk_len,         \
                                                       head_dim, stream));                       \
    }                                                                                            \
    int cuflash_attention_backward_cp_step_##SUFFIX(                                             \
        const T* Q, const T* dO, const T* K, const T* V, void* workspace, float* dK_acc,         \
        float* dV_acc, int num_q_slots, int num_kv_slots, int batch_size, int num_heads,         \
        int chunk_len, int head_dim, float scale, bool causal, int num_pairs, const int* q_slot, \
        const int* kv_slot, const long long* q_offset, const long long* kv_offset,               \
        int reserve_sms, cudaStream_t stream) {                                                  \
        return static_cast<int>(cp_bwd_step_impl<T>(                                             \
            Q, dO, K, V, workspace, dK_acc, dV_acc, num_q_slots, num_kv_slots, batch_size,       \
            num_heads, chunk_len, head_dim, scale, causal, num_pairs, q_slot, kv_slot, q_offset, \
            kv_offset, reserve_sms, stream));                                                    \
    }                                                                                            \
    int cuflash_attention_backward_cp_finish_##SUFFIX(const void* workspace, T* dQ,              \
                                                      int num_q_slots, int batch_size,           \
                                                      int num_heads, int chunk_len,              \
                                                      int head_dim, float scale,                 \
                                                      cudaStream_t stream) {                     \
        return static_cast<int>(cp_bwd_finish_impl<T>(workspace, dQ, num_q_slots, batch_size,    \
                                                      num_heads, chunk_len, head_dim, scale,     \
                                                      stream));                                  \
    }
CUFLASH_CP_BWD_ENTRIES(bf16, __nv_bfloat16)
CUFLASH_CP_BWD_ENTRIES(f16, half)
#undef CUFLASH_CP_BWD_ENTRIES

int cuflash_accumulate_f32(float* dst, float* src, long long count, bool zero_src,
                           cudaStream_t stream) {
    if (!dst || !src) return static_cast<int>(FlashAttentionError::NULL_POINTER);
    if (count <= 0 || count % 4 != 0 || (reinterpret_cast<uintptr_t>(dst) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(src) & 15u) != 0)
        return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    if (cuflash::detail::sticky_failure())
        return static_cast<int>(FlashAttentionError::CUDA_ERROR);
    return static_cast<int>(
        cuflash::detail::launch_accumulate_f32(dst, src, count, zero_src, stream));
}

int cuflash_lse_merge_f32(float* O_acc, float* L_acc, const float* O_part, const float* L_part,
                          long long rows, int head_dim, cudaStream_t stream) {
    if (!O_acc || !L_acc || !O_part || !L_part)
        return static_cast<int>(FlashAttentionError::NULL_POINTER);
    if (rows <= 0 || head_dim <= 0) return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    if (cuflash::detail::sticky_failure())
        return static_cast<int>(FlashAttentionError::CUDA_ERROR);
    return static_cast<int>(
        cuflash::detail::launch_lse_merge(O_acc, L_acc, O_part, L_part, rows, head_dim, stream));
}

int cuflash_convert_f32_to_bf16(const float* src, __nv_bfloat16* dst, long long count,
                                cudaStream_t stream) {
    if (!src || !dst) return static_cast<int>(FlashAttentionError::NULL_POINTER);
    if (count <= 0) return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    if (cuflash::detail::sticky_failure())
        return static_cast<int>(FlashAttentionError::CUDA_ERROR);
    return static_cast<int>(
        cuflash::detail::launch_convert_f32<__nv_bfloat16>(src, dst, count, stream));
}

int cuflash_convert_f32_to_f16(const float* src, half* dst, long long count,
                               cudaStream_t stream) {
    if (!src || !dst) return static_cast<int>(FlashAttentionError::NULL_POINTER);
    if (count <= 0) return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    if (cuflash::detail::sticky_failure())
        return static_cast<int>(FlashAttentionError::CUDA_ERROR);
    return static_cast<int>(cuflash::detail::launch_convert_f32<half>(src, dst, count, stream));
}

int cuflash_attention_decode_bf16_noalloc(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                          const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                          int batch_size, int num_heads, int kv_len, int head_dim,
                                          float scale, int num_splits, cudaStream_t stream) {
    if (!Q || !K || !V || !O || !L) return static_cast<int>(FlashAttentionError::NULL_POINTER);
    if (batch_size <= 0 || num_heads <= 0 || kv_len <= 0 || head_dim <= 0)
        return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    if (!(head_dim == 32 || head_dim == 64 || head_dim == 128))
        return static_cast<int>(FlashAttentionError::UNSUPPORTED_HEAD_DIM);
    if (!std::isfinite(scale) || scale < 0.0f || num_splits < 0 || num_splits > 64)
        return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    if (static_cast<long long>(batch_size) * num_heads > 0x7fffffffLL)
        return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    if (cuflash::detail::sticky_failure())
        return static_cast<int>(FlashAttentionError::CUDA_ERROR);
    return static_cast<int>(cuflash::detail::launch_decode_bf16_noalloc(
        Q, K, V, O, L, batch_size, num_heads, kv_len, head_dim, scale, num_splits, stream));
}

int cuflash_device_status(void) { return cuflash::detail::read_and_clear_device_status(); }

int cuflash_profile_main_kernels(int num_launches) {
    if (num_launches < 0) return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    return static_cast<int>(cuflash::detail::profile_main_kernels(num_launches) == 0
                                ? FlashAttentionError::SUCCESS
                                : FlashAttentionError::CUDA_ERROR);
}

int cuflash_profile_read_ms(float* ms, int max_launches) {
    if (ms == nullptr) return -static_cast<int>(FlashAttentionError::NULL_POINTER);
    if (max_launches < 0) return -static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    const int n = cuflash::detail::profile_read_ms(ms, max_launches);
    return n >= 0 ? n : -static_cast<int>(FlashAttentionError::CUDA_ERROR);
}

int cuflash_set_option(const char* name, int value) {
    if (name == nullptr) return static_cast<int>(FlashAttentionError::NULL_POINTER);
    return static_cast<int>(cuflash::detail::set_option(name, value)
                                ? FlashAttentionError::SUCCESS
                                : FlashAttentionError::INVALID_DIMENSION);
}

}  // extern "C"
