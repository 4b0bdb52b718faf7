#pragma once

// cuflash B200: public API.
//
// The first half of this header is the drop-in surface of the reference
// library (AICL-Lab/cuflash-attn, include/cuflash/flash_attention.h:10-118):
// the same enum, the same C++ overloads with the same default stream
// argument, and the same extern "C" entry points with the same argument
// order and meaning.  A program built against the reference header links
// against this library unchanged.
//
// The second half declares additive entry points that the reference does not
// have (split-KV decode, the partial forward used by context parallelism and
// the log-sum-exp merge).  They follow the same conventions: caller-owned
// device buffers, fp32 log-sum-exp, int return code, stream last.
//
// Layout of every Q/K/V/O/dO/dQ/dK/dV tensor: contiguous row-major
// [batch, heads, seq, head_dim]; element (b,h,i,d) lives at
// ((b*H + h)*N + i)*D + d.  L is [batch, heads, seq] fp32 and holds
// L_i = log(sum_j exp(scale * q_i.k_j)) over the unmasked keys (natural log).
// Causal masking is top-left aligned: key j is masked for query i iff j > i.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "cuflash/export.h"

#ifdef __cplusplus
namespace cuflash {

// Reference: include/cuflash/flash_attention.h:12-21 (values and order kept).
enum class FlashAttentionError {
    SUCCESS = 0,
    INVALID_DIMENSION,
    DIMENSION_MISMATCH,
    NULL_POINTER,
    CUDA_ERROR,
    OUT_OF_MEMORY,
    UNSUPPORTED_HEAD_DIM,
    UNSUPPORTED_DTYPE
};

// Reference: flash_attention.h:24.  Strings are byte-identical to the
// reference's src/api/flash_attention_api.cu:21-42.
CUFLASH_EXPORT const char* get_error_string(FlashAttentionError error);

// Reference: flash_attention.h:30-34 (fp32 forward).
CUFLASH_EXPORT FlashAttentionError flash_attention_forward(const float* Q, const float* K,
                                                           const float* V, float* O, float* L,
                                                           int batch_size, int num_heads,
                                                           int seq_len, int head_dim, float scale,
                                                           bool causal, cudaStream_t stream = 0);

// Reference: flash_attention.h:37-40 (fp32 backward).
CUFLASH_EXPORT FlashAttentionError flash_attention_backward(
    const float* Q, const float* K, const float* V, const float* O, const float* L, const float* dO,
    float* dQ, float* dK, float* dV, int batch_size, int num_heads, int seq_len, int head_dim,
    float scale, bool causal, cudaStream_t stream = 0);

// Reference: flash_attention.h:48-57 (fp16).  L stays fp32.
CUFLASH_EXPORT FlashAttentionError flash_attention_forward(const half* Q, const half* K,
                                                           const half* V, half* O, float* L,
                                                           int batch_size, int num_heads,
                                                           int seq_len, int head_dim, float scale,
                                                           bool causal, cudaStream_t stream = 0);

CUFLASH_EXPORT FlashAttentionError flash_attention_backward(
    const half* Q, const half* K, const half* V, const half* O, const float* L, const half* dO,
    half* dQ, half* dK, half* dV, int batch_size, int num_heads, int seq_len, int head_dim,
    float scale, bool causal, cudaStream_t stream = 0);

// Reference: flash_attention.h:60-71 (bf16).  L stays fp32.
CUFLASH_EXPORT FlashAttentionError flash_attention_forward(const __nv_bfloat16* Q,
                                                           const __nv_bfloat16* K,
                                                           const __nv_bfloat16* V, __nv_bfloat16* O,
                                                           float* L, int batch_size, int num_heads,
                                                           int seq_len, int head_dim, float scale,
                                                           bool causal, cudaStream_t stream = 0);

CUFLASH_EXPORT FlashAttentionError flash_attention_backward(
    const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V, const __nv_bfloat16* O,
    const float* L, const __nv_bfloat16* dO, __nv_bfloat16* dQ, __nv_bfloat16* dK,
    __nv_bfloat16* dV, int batch_size, int num_heads, int seq_len, int head_dim, float scale,
    bool causal, cudaStream_t stream = 0);

}  // namespace cuflash
#endif  // __cplusplus

#ifdef __cplusplus
extern "C" {
#else
#include <stdbool.h>
#endif

// ---------------------------------------------------------------------------
// Reference C ABI (flash_attention.h:81-118).  Return value: integer value of
// cuflash::FlashAttentionError.  Validation happens before any CUDA call, so
// invalid arguments are reported on machines without a GPU.
// ---------------------------------------------------------------------------

// Replaces flash_attention.h:81-84.
CUFLASH_EXPORT int cuflash_attention_forward_f32(const float* Q, const float* K, const float* V,
                                                 float* O, float* L, int batch_size, int num_heads,
                                                 int seq_len, int head_dim, float scale,
                                                 bool causal, cudaStream_t stream);

// Replaces flash_attention.h:86-90.
CUFLASH_EXPORT int cuflash_attention_backward_f32(const float* Q, const float* K, const float* V,
                                                  const float* O, const float* L, const float* dO,
                                                  float* dQ, float* dK, float* dV, int batch_size,
                                                  int num_heads, int seq_len, int head_dim,
                                                  float scale, bool causal, cudaStream_t stream);

// Replaces flash_attention.h:92-95.
CUFLASH_EXPORT int cuflash_attention_forward_f16(const half* Q, const half* K, const half* V,
                                                 half* O, float* L, int batch_size, int num_heads,
                                                 int seq_len, int head_dim, float scale,
                                                 bool causal, cudaStream_t stream);

// Replaces flash_attention.h:97-101.
CUFLASH_EXPORT int cuflash_attention_backward_f16(const half* Q, const half* K, const half* V,
                                                  const half* O, const float* L, const half* dO,
                                                  half* dQ, half* dK, half* dV, int batch_size,
                                                  int num_heads, int seq_len, int head_dim,
                                                  float scale, bool causal, cudaStream_t stream);

// Replaces flash_attention.h:103-107.
CUFLASH_EXPORT int cuflash_attention_forward_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                                  const __nv_bfloat16* V, __nv_bfloat16* O,
                                                  float* L, int batch_size, int num_heads,
                                                  int seq_len, int head_dim, float scale,
                                                  bool causal, cudaStream_t stream);

// Replaces flash_attention.h:109-115.
CUFLASH_EXPORT int cuflash_attention_backward_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                                   const __nv_bfloat16* V, const __nv_bfloat16* O,
                                                   const float* L, const __nv_bfloat16* dO,
                                                   __nv_bfloat16* dQ, __nv_bfloat16* dK,
                                                   __nv_bfloat16* dV, int batch_size, int num_heads,
                                                   int seq_len, int head_dim, float scale,
                                                   bool causal, cudaStream_t stream);

// Replaces flash_attention.h:118.
CUFLASH_EXPORT const char* cuflash_error_string(int error_code);

// ---------------------------------------------------------------------------
// Additive entry points (no reference counterpart; the reference lists
// split-KV decoding as future work in ROADMAP.md:22-26 and has no
// multi-GPU code).  Same conventions as above.
// ---------------------------------------------------------------------------

// Split-KV decode: one query token per (batch, head) against a KV cache of
// length kv_len.  Q, O: [B,H,1,D]; K, V: [B,H,kv_len,D]; L: [B,H] fp32.
// num_splits: 0 picks a split count from the problem size, 1..64 forces it;
// anything else returns INVALID_DIMENSION.  The split partials live in a
// stream-ordered workspace allocated and freed inside the call.
CUFLASH_EXPORT int cuflash_attention_decode_f16(const half* Q, const half* K, const half* V,
                                                half* O, float* L, int batch_size, int num_heads,
                                                int kv_len, int head_dim, float scale,
                                                int num_splits, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_decode_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                                 const __nv_bfloat16* V, __nv_bfloat16* O,
                                                 float* L, int batch_size, int num_heads,
                                                 int kv_len, int head_dim, float scale,
                                                 int num_splits, cudaStream_t stream);

// Split-KV decode (bf16) that allocates nothing.  No counterpart in the
// reference library.  For callers that must not have device memory
// allocated behind their back: serving engines that reserve nearly all of
// HBM for their KV cache and hand memory out only through their own
// allocator, and decode loops that keep allocation calls off the per-token
// path.  Same arguments and results as cuflash_attention_decode_bf16; the
// split partials go to a fixed 8 MiB device buffer that every GPU loading the
// library holds until exit (batch*heads*splits*(head_dim+1) fp32 values must
// fit: with num_splits = 0 the split count is capped to fit, an explicit
// num_splits that does not fit returns OUT_OF_MEMORY without launching).
// The first call on a device looks up the buffer's device address (make that
// first call before any stream capture on that device).  All calls share the
// buffer: calls whose kernels may overlap on the GPU race and must be
// serialised by the caller (one stream, or events between streams).
CUFLASH_EXPORT int cuflash_attention_decode_bf16_noalloc(
    const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V, __nv_bfloat16* O,
    float* L, int batch_size, int num_heads, int kv_len, int head_dim, float scale,
    int num_splits, cudaStream_t stream);

// Partial forward for context parallelism: queries [B,H,seq_q,D] at global
// positions q_offset.., keys/values [B,H,seq_k,D] at global positions
// k_offset...  With causal, key g_k is masked for query g_q iff g_k > g_q.
// Writes a normalised partial result: O_part fp32 [B,H,seq_q,D] divided by
// its own row sum, and L_part fp32 [B,H,seq_q] (natural log; -inf for a row
// whose keys are all masked, with O_part = 0).
CUFLASH_EXPORT int cuflash_attention_forward_partial_bf16(
    const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V, float* O_part,
    float* L_part, int batch_size, int num_heads, int seq_q, int seq_k, int head_dim, float scale,
    long long q_offset, long long k_offset, bool causal, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_forward_partial_f16(
    const half* Q, const half* K, const half* V, float* O_part, float* L_part, int batch_size,
    int num_heads, int seq_q, int seq_k, int head_dim, float scale, long long q_offset,
    long long k_offset, bool causal, cudaStream_t stream);

// Grouped-query split-KV decode (no reference counterpart): one query token
// per (batch, query head) against a contiguous cache K, V [B, num_kv_heads,
// kv_len, D]; Q, O [B, num_q_heads, 1, D], L fp32 [B, num_q_heads].  Query
// head h reads K/V head h / (num_q_heads / num_kv_heads); one CTA serves up
// to 8 query heads of a group, so every cache row is read once for them.
// num_splits: 0 = automatic, 1..64.
CUFLASH_EXPORT int cuflash_attention_decode_gqa_bf16(
    const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V, __nv_bfloat16* O,
    float* L, int batch_size, int num_q_heads, int num_kv_heads, int kv_len, int head_dim,
    float scale, int num_splits, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_decode_gqa_f16(const half* Q, const half* K, const half* V,
                                                    half* O, float* L, int batch_size,
                                                    int num_q_heads, int num_kv_heads,
                                                    int kv_len, int head_dim, float scale,
                                                    int num_splits, cudaStream_t stream);

// Split-KV decode over a paged KV cache (no reference counterpart).  K_cache,
// V_cache [num_pages, page_size, num_kv_heads, D]; block_table int32
// [B, max_pages_per_seq] and seq_lens int32 [B] in device memory: token t of
// sequence b sits in page block_table[b][t / page_size], slot t % page_size.
// page_size must be a power of two; page indices outside [0, num_pages) are
// clamped (a bad table reads a wrong page instead of faulting); a sequence of
// length 0 gets O = 0 and L = -inf.  Heads, Q / O / L and num_splits as in
// cuflash_attention_decode_gqa_*; splits are planned over
// max_pages_per_seq * page_size tokens.
CUFLASH_EXPORT int cuflash_attention_decode_paged_bf16(
    const __nv_bfloat16* Q, const __nv_bfloat16* K_cache, const __nv_bfloat16* V_cache,
    const int* block_table, const int* seq_lens, __nv_bfloat16* O, float* L, int batch_size,
    int num_q_heads, int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq,
    int num_pages, float scale, int num_splits, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_decode_paged_f16(
    const half* Q, const half* K_cache, const half* V_cache, const int* block_table,
    const int* seq_lens, half* O, float* L, int batch_size, int num_q_heads, int num_kv_heads,
    int head_dim, int page_size, int max_pages_per_seq, int num_pages, float scale,
    int num_splits, cudaStream_t stream);

// Grouped-query (GQA / MQA) attention with separate query and key lengths
// (no reference counterpart: the reference API has one seq_len and equal
// head counts).  Q, O, dO, dQ [B, num_q_heads, seq_len_q, D]; K, V, dK, dV
// [B, num_kv_heads, seq_len_k, D]; L fp32 [B, num_q_heads, seq_len_q].
// num_q_heads must be a multiple of num_kv_heads (else DIMENSION_MISMATCH);
// query head h reads K/V head h / (num_q_heads / num_kv_heads), and dK / dV
// of a K/V head sum over its query heads.  causal aligns the mask
// bottom-right: query i sees key j iff j <= i + seq_len_k - seq_len_q (the
// KV-cache convention; with equal lengths it is the reference's top-left
// mask).  Queries that see no key get O = 0 and L = -inf.  Validation order
// and codes otherwise follow the reference entry points.
CUFLASH_EXPORT int cuflash_attention_forward_gqa_bf16(
    const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V, __nv_bfloat16* O,
    float* L, int batch_size, int num_q_heads, int num_kv_heads, int seq_len_q, int seq_len_k,
    int head_dim, float scale, bool causal, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_forward_gqa_f16(const half* Q, const half* K, const half* V,
                                                     half* O, float* L, int batch_size,
                                                     int num_q_heads, int num_kv_heads,
                                                     int seq_len_q, int seq_len_k, int head_dim,
                                                     float scale, bool causal,
                                                     cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_backward_gqa_bf16(
    const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
    const __nv_bfloat16* O, const float* L, const __nv_bfloat16* dO, __nv_bfloat16* dQ,
    __nv_bfloat16* dK, __nv_bfloat16* dV, int batch_size, int num_q_heads, int num_kv_heads,
    int seq_len_q, int seq_len_k, int head_dim, float scale, bool causal, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_backward_gqa_f16(
    const half* Q, const half* K, const half* V, const half* O, const float* L, const half* dO,
    half* dQ, half* dK, half* dV, int batch_size, int num_q_heads, int num_kv_heads,
    int seq_len_q, int seq_len_k, int head_dim, float scale, bool causal, cudaStream_t stream);

// One ring step of context-parallel attention in a single launch (no
// reference counterpart: the reference has no multi-GPU path).  Q and the
// running result hold num_q_slots query chunks stacked as [slot][B][H][C][D]
// (O_acc fp32, L_acc fp32 [slot][B][H][C]); K and V hold num_kv_slots chunks
// the same way.  For each of num_pairs (1..4) pairs i it runs the partial
// forward of query slot q_slot[i] (global positions q_offset[i]..) against
// K/V slot kv_slot[i] (global positions kv_offset[i]..), causal on global
// positions when causal is set, and folds the result into O_acc / L_acc of
// that slot with the log-sum-exp merge of cuflash_lse_merge_f32.  The pairs
// of one call must name distinct query slots.  O_acc / L_acc start as 0 /
// -inf; the slot-index and offset arrays are host memory.  reserve_sms (>= 0)
// SMs are left out of the launch's persistent grid, for kernels that run at
// the same time (a ring's NCCL transfer); 0 uses every SM.
CUFLASH_EXPORT int cuflash_attention_forward_cp_step_bf16(
    const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V, float* O_acc,
    float* L_acc, int num_q_slots, int num_kv_slots, int batch_size, int num_heads,
    int chunk_len, int head_dim, float scale, bool causal, int num_pairs, const int* q_slot,
    const int* kv_slot, const long long* q_offset, const long long* kv_offset, int reserve_sms,
    cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_forward_cp_step_f16(
    const half* Q, const half* K, const half* V, float* O_acc, float* L_acc, int num_q_slots,
    int num_kv_slots, int batch_size, int num_heads, int chunk_len, int head_dim, float scale,
    bool causal, int num_pairs, const int* q_slot, const int* kv_slot,
    const long long* q_offset, const long long* kv_offset, int reserve_sms,
    cudaStream_t stream);

// Context-parallel backward, the ring counterpart of the step above (no
// reference counterpart).  Per query slot q the caller holds the forward's
// final O and L (natural-log LSE) and dO, stacked [slot][B][H][C][D] like Q.
//   workspace_size  bytes of the workspace kept across the steps (0 for
//                   invalid arguments);
//   prepare         fills it from O, dO, L: -L*log2(e), -rowsum(dO*O) and a
//                   zeroed fp32 dQ accumulator;
//   step            for each of num_pairs (1..4) pairs i, the backward of query
//                   slot q_slot[i] against K/V slot kv_slot[i] (global offsets
//                   as in the forward step): dQ of the query slot is added into
//                   the workspace, scale*dK and dV of the K/V slot are ADDED
//                   into dK_acc / dV_acc, fp32 [kv slot][B][H][C][D].  Pairs
//                   may share query or K/V slots, but a (query slot, K/V
//                   slot) pair may not repeat (INVALID_DIMENSION);
//                   reserve_sms as in the forward step;
//   finish          writes dQ = scale * (accumulated dQ) for all query slots.
// The slot-index and offset arrays are host memory.  dK_acc / dV_acc travel
// the ring with the K/V they belong to; the final dK / dV are their values
// converted to 16 bits (cuflash_convert_f32_to_*).
CUFLASH_EXPORT long long cuflash_attention_backward_cp_workspace_size(int num_q_slots,
                                                                      int batch_size,
                                                                      int num_heads,
                                                                      int chunk_len,
                                                                      int head_dim);
CUFLASH_EXPORT int cuflash_attention_backward_cp_prepare_bf16(
    const __nv_bfloat16* O, const __nv_bfloat16* dO, const float* L, void* workspace,
    int num_q_slots, int batch_size, int num_heads, int chunk_len, int head_dim,
    cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_backward_cp_prepare_f16(
    const half* O, const half* dO, const float* L, void* workspace, int num_q_slots,
    int batch_size, int num_heads, int chunk_len, int head_dim, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_backward_cp_step_bf16(
    const __nv_bfloat16* Q, const __nv_bfloat16* dO, const __nv_bfloat16* K,
    const __nv_bfloat16* V, void* workspace, float* dK_acc, float* dV_acc, int num_q_slots,
    int num_kv_slots, int batch_size, int num_heads, int chunk_len, int head_dim, float scale,
    bool causal, int num_pairs, const int* q_slot, const int* kv_slot,
    const long long* q_offset, const long long* kv_offset, int reserve_sms,
    cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_backward_cp_step_f16(
    const half* Q, const half* dO, const half* K, const half* V, void* workspace, float* dK_acc,
    float* dV_acc, int num_q_slots, int num_kv_slots, int batch_size, int num_heads,
    int chunk_len, int head_dim, float scale, bool causal, int num_pairs, const int* q_slot,
    const int* kv_slot, const long long* q_offset, const long long* kv_offset, int reserve_sms,
    cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_backward_cp_finish_bf16(const void* workspace,
                                                             __nv_bfloat16* dQ, int num_q_slots,
                                                             int batch_size, int num_heads,
                                                             int chunk_len, int head_dim,
                                                             float scale, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_backward_cp_finish_f16(const void* workspace, half* dQ,
                                                            int num_q_slots, int batch_size,
                                                            int num_heads, int chunk_len,
                                                            int head_dim, float scale,
                                                            cudaStream_t stream);
// dst += src over count fp32 values (count a multiple of 4, both pointers
// 16-byte aligned); with zero_src, src is cleared as it is read.
CUFLASH_EXPORT int cuflash_accumulate_f32(float* dst, float* src, long long count, bool zero_src,
                                          cudaStream_t stream);

// Log-sum-exp merge of a partial result into a running one, row by row:
//   L = log(exp(L_acc) + exp(L_part));
//   O_acc = exp(L_acc - L) * O_acc + exp(L_part - L) * O_part;  L_acc = L.
// O_acc/O_part fp32 [rows, head_dim]; L_acc/L_part fp32 [rows].  -inf rows
// contribute nothing.  Same algebra as the reference's online-softmax state
// merge (src/kernels/impl/online_softmax.cuh:16-59).
CUFLASH_EXPORT int cuflash_lse_merge_f32(float* O_acc, float* L_acc, const float* O_part,
                                         const float* L_part, long long rows, int head_dim,
                                         cudaStream_t stream);

// Converts a merged fp32 result to the storage dtype (round to nearest).
CUFLASH_EXPORT int cuflash_convert_f32_to_bf16(const float* src, __nv_bfloat16* dst,
                                               long long count, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_convert_f32_to_f16(const float* src, half* dst, long long count,
                                              cudaStream_t stream);

// Failure status.  Every kernel with a bounded wait (mbarrier polling)
// records a non-zero code instead of hanging when a wait runs out (1), or
// when it meets a shared-memory layout it cannot use (2); the code goes to a
// device word (later kernels of the same family skip their work) and to a
// host-mapped word of that device that every entry point reads, without
// synchronising, after validating its arguments: while it is set, calls on
// that device return CUDA_ERROR and launch nothing (a sticky error, as
// CUDA's own).  This call synchronises the current device, returns its code
// (0: no failure) and clears it, after which the library works again there.
CUFLASH_EXPORT int cuflash_device_status(void);

// Profiling hook (no reference counterpart).  After
// cuflash_profile_main_kernels(n), the next n launches of the fp16/bf16
// backward's main kernel on the current device each get a pair of CUDA
// events recorded right before and right after the launch, on the call's
// stream, so that the kernel alone can be timed apart from the backward's
// preprocess and dQ conversion kernels; n = 0 ends profiling.
// cuflash_profile_read_ms waits for the recorded launches and writes their
// durations (ms) into ms[0..k); it returns k, or minus an error code.
CUFLASH_EXPORT int cuflash_profile_main_kernels(int num_launches);
CUFLASH_EXPORT int cuflash_profile_read_ms(float* ms, int max_launches);

// Process-wide tuning and test options (no reference counterpart).  Each
// option starts from the environment variable of the same name, read once
// when the library first needs an option; this call changes it afterwards
// (thread-safe; launches already enqueued keep the value they saw).  A
// negative value returns the option to its built-in default.  Options:
//   CUFLASH_RESERVE_SMS          SMs left out of every persistent launch
//                                (for collectives that run concurrently);
//   CUFLASH_FWD_WAVES, CUFLASH_BWD_WAVES, CUFLASH_CP_WAVES
//                                persistent grid size in waves of SMs;
//   CUFLASH_DECODE_GQA_TC        0 routes grouped-query decode to the SIMT
//                                kernel instead of the tensor-core one;
//   CUFLASH_FAULT_WORKSPACE_OOM  1 makes every workspace request fail with
//                                OUT_OF_MEMORY (host-side fault injection);
//   CUFLASH_TEST_WAIT_LIMIT_MS   bounded-wait limit of the fp16/bf16 forward
//                                in ms (default 4000);
//   CUFLASH_TEST_SKIP_K_LOAD     1 makes the fp16/bf16 forward's first CTA
//                                leave out one K load, so that one of its
//                                waits runs out (tests of the timeout path).
// Returns SUCCESS, NULL_POINTER, or INVALID_DIMENSION for an unknown name.
CUFLASH_EXPORT int cuflash_set_option(const char* name, int value);

#ifdef __cplusplus
}
#endif
