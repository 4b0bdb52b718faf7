#pragma once

// Shared host/device helpers: dtype traits, tensor-map encoding, per-device
// launch attributes and the internal launcher declarations used by api.cu.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "cuflash/flash_attention.h"
#include "sm100.cuh"

namespace cuflash {
namespace detail {

template <typename T>
struct DType;

template <>
struct DType<__nv_bfloat16> {
    static constexpr uint32_t kMmaFmt = sm100::kFmtBF16;
    static constexpr CUtensorMapDataType kTmaType = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    __device__ static __forceinline__ uint32_t pack2(float lo, float hi) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __device__ static __forceinline__ float2 unpack2(uint32_t u) {
        __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
        return __bfloat1622float2(v);
    }
    __device__ static __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
    __device__ static __forceinline__ __nv_bfloat16 from_float(float x) {
        return __float2bfloat16_rn(x);
    }
};

template <>
struct DType<half> {
    static constexpr uint32_t kMmaFmt = sm100::kFmtF16;
    static constexpr CUtensorMapDataType kTmaType = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    __device__ static __forceinline__ uint32_t pack2(float lo, float hi) {
        __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __device__ static __forceinline__ float2 unpack2(uint32_t u) {
        __half2 v = *reinterpret_cast<__half2*>(&u);
        return __half22float2(v);
    }
    __device__ static __forceinline__ float to_float(half x) { return __half2float(x); }
    __device__ static __forceinline__ half from_float(float x) { return __float2half_rn(x); }
};

// Encodes a 3-D tiled tensor map over a [outer, rows, inner] row-major
// tensor: dim0 = inner (contiguous, `inner` elements), dim1 = rows,
// dim2 = outer.  Box = {box_inner, box_rows, 1}.  Out-of-bounds reads return
// zeros.  Returns false if the driver rejects the map (for example a base
// address that is not 16-byte aligned).
bool encode_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                    uint64_t inner, uint64_t rows, uint64_t outer, uint32_t box_inner,
                    uint32_t box_rows, CUtensorMapSwizzle swizzle);
// Same with explicit dimensions {inner, mid, outer}, byte strides of mid and
// outer, and box {inner, mid, outer}.
bool encode_tmap_3d_strided(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                            const uint64_t dims[3], const uint64_t stride_bytes[2],
                            const uint32_t box[3], CUtensorMapSwizzle swizzle);

// Raises the dynamic shared memory limit of `kernel` to `bytes` on the
// current device once (thread-safe, per device and kernel).  Returns false
// if the device cannot provide that much.
bool ensure_smem_attr(const void* kernel, int bytes);

int current_sm_count();
int persistent_grid(long long units, int waves);
// Value of a process-wide option (initialised once from the environment
// variable of the same name, changed by cuflash_set_option), or dflt when
// it is not set.
int env_int(const char* name, int dflt);
bool set_option(const char* name, int value);

// Stream-ordered workspace from a library-private memory pool on the current
// device (created on first use; freed blocks stay cached in the pool so
// repeated calls do not remap memory).  Returns OUT_OF_MEMORY when the pool
// cannot grow.  The option CUFLASH_FAULT_WORKSPACE_OOM=1 makes every request
// fail with OUT_OF_MEMORY before any CUDA call (host-side fault injection for
// tests).
FlashAttentionError workspace_alloc(void** ptr, size_t bytes, cudaStream_t stream);
void workspace_free(void* ptr, cudaStream_t stream);

// Non-blocking side stream i (< kNumSideStreams) of the current device,
// created on first use and kept for the life of the process; a launcher runs
// independent kernels there, forked from and joined back into the caller's
// stream with events.  nullptr if it cannot be created.
constexpr int kNumSideStreams = 2;
cudaStream_t side_stream(int i);

// Launchers (defined in the kernel .cu files).  All pointers are device
// pointers; validation has already happened.
template <typename T>
FlashAttentionError launch_fwd_sm100(const T* Q, const T* K, const T* V, void* O, float* L, int B,
                                     int H, int seq_q, int seq_k, int D, float scale, bool causal,
                                     long long q_offset, long long k_offset, bool out_f32_partial,
                                     cudaStream_t stream);

// Grouped-query split-KV decode.  Contiguous cache (block_table == nullptr):
// K, V [B, Hkv, kv_len, D].  Paged cache: K, V [num_pages, page_size, Hkv, D],
// block_table [B, max_pages] and seq_lens [B] in device memory, page_size a
// power of two.  Q, O [B, Hq, 1, D], L [B, Hq].
template <typename T>
FlashAttentionError launch_decode_gqa(const T* Q, const T* K, const T* V, T* O, float* L, int B,
                                      int Hq, int Hkv, int kv_len, int D, float scale,
                                      int num_splits, const int* block_table,
                                      const int* seq_lens, int page_size, int max_pages,
                                      int num_pages, cudaStream_t stream);

// Grouped-query backward, same layout and mask conventions as the forward.
template <typename T>
FlashAttentionError launch_bwd_gqa_sm100(const T* Q, const T* K, const T* V, const T* O,
                                         const float* L, const T* dO, T* dQ, T* dK, T* dV, int B,
                                         int Hq, int Hkv, int seq_q, int seq_k, int D, float scale,
                                         bool causal, cudaStream_t stream);

// Grouped-query forward: Q, O [B,Hq,seq_q,D], K, V [B,Hkv,seq_k,D], query head
// h reads K/V head h / (Hq/Hkv); causal is aligned bottom-right.
template <typename T>
FlashAttentionError launch_fwd_gqa_sm100(const T* Q, const T* K, const T* V, T* O, float* L, int B,
                                         int Hq, int Hkv, int seq_q, int seq_k, int D, float scale,
                                         bool causal, cudaStream_t stream);

// One context-parallel ring step: num_pairs (<= 4) partial forwards of query
// slot q_slot[i] against K/V slot k_slot[i] (global offsets q_off/k_off), each
// merged in place into O_acc / L_acc of its query slot; one launch that keeps
// reserve_sms SMs free.
template <typename T>
FlashAttentionError launch_fwd_cp_step_sm100(const T* Q, const T* K, const T* V, float* O_acc,
                                             float* L_acc, int nq, int nk, int B, int H, int C,
                                             int D, float scale, bool causal, int num_pairs,
                                             const int* q_slot, const int* k_slot,
                                             const long long* q_off, const long long* k_off,
                                             int reserve_sms, cudaStream_t stream);

// Context-parallel backward.  The workspace (bwd_cp_workspace_bytes) holds
// the fp32 dQ accumulator and the per-query -L*log2(e) / -rowsum(dO*O) of nq
// query slots; prepare fills it, each ring step adds its dQ into it and its
// dK (scaled) / dV into fp32 accumulators [nk][BH][C][D], finish writes
// dQ = scale * dQ_acc.
long long bwd_cp_workspace_bytes(int nq, int BH, int C, int D);
template <typename T>
FlashAttentionError launch_bwd_cp_prepare_sm100(const T* O, const T* dO, const float* L, void* ws,
                                                int nq, int BH, int C, int D,
                                                cudaStream_t stream);
template <typename T>
FlashAttentionError launch_bwd_cp_step_sm100(const T* Q, const T* dO, const T* K, const T* V,
                                             void* ws, float* dk_acc, float* dv_acc, int nq,
                                             int nk, int BH, int C, int D, float scale,
                                             bool causal, int num_pairs, const int* q_slot,
                                             const int* kv_slot, const long long* q_off,
                                             const long long* kv_off, int reserve_sms,
                                             cudaStream_t stream);
template <typename T>
FlashAttentionError launch_bwd_cp_finish_sm100(const void* ws, T* dQ, int nq, int BH, int C, int D,
                                               float scale, cudaStream_t stream);
// dst += src over count floats (count a multiple of 4, both 16-byte aligned);
// zero_src also clears src.
FlashAttentionError launch_accumulate_f32(float* dst, float* src, long long count, bool zero_src,
                                          cudaStream_t stream);

template <typename T>
FlashAttentionError launch_bwd_sm100(const T* Q, const T* K, const T* V, const T* O,
                                     const float* L, const T* dO, T* dQ, T* dK, T* dV, int B,
                                     int H, int N, int D, float scale, bool causal,
                                     cudaStream_t stream);

FlashAttentionError launch_fwd_f32(const float* Q, const float* K, const float* V, float* O,
                                   float* L, int B, int H, int N, int D, float scale, bool causal,
                                   cudaStream_t stream);

FlashAttentionError launch_bwd_f32(const float* Q, const float* K, const float* V,
                                   const float* O, const float* L, const float* dO, float* dQ,
                                   float* dK, float* dV, int B, int H, int N, int D, float scale,
                                   bool causal, cudaStream_t stream);

template <typename T>
FlashAttentionError launch_decode(const T* Q, const T* K, const T* V, T* O, float* L, int B, int H,
                                  int kv_len, int D, float scale, int num_splits,
                                  cudaStream_t stream);

// Split-KV decode whose partials live in a fixed device buffer (no
// allocation); see decode_sm100.cu.
FlashAttentionError launch_decode_bf16_noalloc(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                               const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                               int B, int H, int kv_len, int D, float scale,
                                               int num_splits, cudaStream_t stream);

FlashAttentionError launch_lse_merge(float* O_acc, float* L_acc, const float* O_part,
                                     const float* L_part, long long rows, int D,
                                     cudaStream_t stream);

template <typename T>
FlashAttentionError launch_convert_f32(const float* src, T* dst, long long count,
                                       cudaStream_t stream);

// Failure reporting.  Each kernel family keeps a sm100::StatusWord in device
// memory; bind_status_word (called by the family's launchers before every
// launch; cheap after the first call per device) points its `host` field at
// the device's host-mapped word, shared by all families, which host_status()
// reads for the current device without synchronising.  Non-zero means a
// kernel on that device abandoned a bounded wait (or met a misaligned
// buffer) since the last read_and_clear_device_status() there: the entry
// points then refuse new work on that device with CUDA_ERROR.  The binding
// is skipped while `stream` is being captured.
bool bind_status_word(const void* symbol, cudaStream_t stream);
int host_status();
inline bool sticky_failure() { return host_status() != 0; }
// Synchronises the device, reads and clears every family's status word and
// the host word; returns the first non-zero code.
int read_and_clear_device_status();

// Profiling hook: after profile_main_kernels(n) the next n backward main
// kernels (fp16/bf16) on the same device get an event pair recorded around
// them on their stream (profile_record before / after the launch);
// profile_read_ms returns how many were recorded and their durations.
int profile_main_kernels(int n);
void profile_record(bool after, cudaStream_t stream);
int profile_read_ms(float* ms, int max_n);
int fwd_sm100_status();
int bwd_sm100_status();
int dec_sm100_status();
int f32_sm100_status();
int bwd_f32_sm100_status();

}  // namespace detail
}  // namespace cuflash
