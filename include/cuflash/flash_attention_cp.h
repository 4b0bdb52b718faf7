#pragma once

// cuflash B200: context-parallel attention over NCCL (libcuflash_attn_cp.so).
//
// No counterpart in the reference library, which has no multi-GPU code.  The
// entry points follow the reference's C-ABI conventions
// (include/cuflash/flash_attention.h:81-118 of the reference): int return
// value of cuflash::FlashAttentionError, caller-owned device buffers, stream
// last, and argument validation before any CUDA or NCCL call
// (src/api/flash_attention_api.cu:45-79 of the reference).  This target links
// NCCL and libcuflash_attn.so; the core library itself does not depend on
// NCCL.
//
// Sharding ("zigzag"): a causal sequence of seq_len tokens is cut into
// 2 * world chunks of C = seq_len / (2 * world) tokens; rank r holds global
// chunks r and 2 * world - 1 - r, which gives every rank the same amount of
// causal work.  A rank's shard of a [B, H, seq_len, D] tensor is passed as
// [2][B][H][C][D] (slot 0 = chunk r, slot 1 = chunk 2 * world - 1 - r), and of
// L [B, H, seq_len] as [2][B][H][C].
//
// Each rank keeps its query chunks and, at step s, computes with the K/V
// chunks of rank (r - s) mod world while the next ones travel, on
// library-owned streams overlapped with the step's attention kernels on the
// caller's stream; every chunk is in local device memory before a kernel
// reads it.  Two transports (cuflash_cp_set_transport, below): copy-engine
// copies between CUDA-IPC-shared buffers (the default; the backward pushes
// its fp32 dK/dV straight to the chunks' owner), or a ring of grouped
// ncclSend / ncclRecv (rank r sends to r + 1, receives from r - 1; the
// backward carries fp32 dK/dV accumulators with their K/V).  All ranks of
// `comm` must make the same call with the same shapes; a rank that does not
// leaves the others waiting in the per-call all-reduce (or the NCCL
// transfers), as with any NCCL collective (callers that need to recover use
// ncclCommAbort from a watchdog).  The communicator must be a blocking one
// (NCCL's default) of at most 256 ranks.  An NCCL failure returns CUDA_ERROR
// and leaves the communicator in an unknown state.
//
// reserve_sms: SMs each step kernel leaves free for what runs beside it;
// -1 picks the default: 2 with the copy-engine transport (its one-thread
// flag kernels), 16 with NCCL (its transfer kernels; measured best on 8
// B200s at B1 H32 N131072 D128); 0 uses every SM.  With world == 1 no
// transfer runs and comm may be NULL.
//
// Workspace (accumulators) is allocated stream-ordered inside the call and
// freed before it returns (as the reference's backward does); OUT_OF_MEMORY
// if that fails.  The copy-engine transport also keeps one cudaMalloc
// allocation per communicator (exports, pull slots, receive slots) until
// cuflash_cp_nccl_comm_destroy.

#include <nccl.h>

#include "cuflash/flash_attention.h"

#ifdef __cplusplus
extern "C" {
#endif

// Causal (or full, causal = false) attention forward of a zigzag shard.
// Q, K, V, O: [2][B][H][C][D]; L: [2][B][H][C] fp32 (natural-log LSE, as the
// single-GPU forward).  seq_len is the GLOBAL sequence length, a multiple of
// 2 * world.  Validation: NULL_POINTER (tensors; comm when world > 1),
// INVALID_DIMENSION (non-positive sizes, seq_len not divisible by 2 * world,
// world above 256, rank outside [0, world), reserve_sms < -1),
// UNSUPPORTED_HEAD_DIM, then
// scale as in the reference; DIMENSION_MISMATCH if comm's size or rank
// differs from world / rank.
CUFLASH_EXPORT int cuflash_attention_forward_cp_bf16(
    const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V, __nv_bfloat16* O,
    float* L, int batch_size, int num_heads, int seq_len, int head_dim, float scale, bool causal,
    ncclComm_t comm, int rank, int world, int reserve_sms, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_forward_cp_f16(const half* Q, const half* K, const half* V,
                                                    half* O, float* L, int batch_size,
                                                    int num_heads, int seq_len, int head_dim,
                                                    float scale, bool causal, ncclComm_t comm,
                                                    int rank, int world, int reserve_sms,
                                                    cudaStream_t stream);

// Backward of the forward above over the same ring: O and L are that
// forward's outputs, dO the output gradient (all in the shard layout); writes
// dQ, dK, dV of this rank's chunks.  dQ accumulates locally in fp32; the
// fp32 dK / dV of each K/V chunk travel the ring with it (one more hop after
// the last step brings them home) and are rounded once, at the end.
// Validation as in the forward, with dO, dQ, dK, dV checked for null first
// (the reference's backward order).
CUFLASH_EXPORT int cuflash_attention_backward_cp_bf16(
    const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
    const __nv_bfloat16* O, const float* L, const __nv_bfloat16* dO, __nv_bfloat16* dQ,
    __nv_bfloat16* dK, __nv_bfloat16* dV, int batch_size, int num_heads, int seq_len,
    int head_dim, float scale, bool causal, ncclComm_t comm, int rank, int world,
    int reserve_sms, cudaStream_t stream);
CUFLASH_EXPORT int cuflash_attention_backward_cp_f16(
    const half* Q, const half* K, const half* V, const half* O, const float* L, const half* dO,
    half* dQ, half* dK, half* dV, int batch_size, int num_heads, int seq_len, int head_dim,
    float scale, bool causal, ncclComm_t comm, int rank, int world, int reserve_sms,
    cudaStream_t stream);

// The ring schedule both entry points follow, as a host function (no CUDA or
// NCCL call).  At step `step` (0 <= step < world) rank `rank` holds the K/V
// chunks of rank *kv_owner = (rank - step) mod world.  It writes the
// *num_pairs (0..4) visible (query slot, K/V slot) pairs of that step, in
// launch order, into the four-element arrays: local slots, global chunk
// indices, and the forward launch each pair belongs to (a forward launch
// merges every query slot at most once; the backward runs all of a step's
// pairs in one launch).  Returns SUCCESS, NULL_POINTER or INVALID_DIMENSION.
CUFLASH_EXPORT int cuflash_cp_ring_schedule(int rank, int world, int step, bool causal,
                                            int* kv_owner, int* num_pairs, int* q_slot,
                                            int* kv_slot, int* q_chunk, int* kv_chunk,
                                            int* fwd_launch);

// Communicator helpers for callers without an NCCL binding of their own
// (ctypes, for instance); they use the same NCCL library as the entry points.
// unique_id: NCCL_UNIQUE_ID_BYTES bytes, made on one rank and given to all.
// comm_init runs ncclCommInitRank on the current device; comm_init_config
// creates the same blocking communicator with ncclCommInitRankConfig and, for
// max_ctas > 0, caps the CTAs (channels) NCCL's kernels use at max_ctas, so
// that they fit in the SMs the step kernels leave free (reserve_sms); 0 keeps
// NCCL's default.  NCCL failures return CUDA_ERROR.
CUFLASH_EXPORT int cuflash_cp_nccl_unique_id(void* unique_id, int nbytes);
CUFLASH_EXPORT int cuflash_cp_nccl_comm_init(ncclComm_t* comm, int world, const void* unique_id,
                                             int rank);
CUFLASH_EXPORT int cuflash_cp_nccl_comm_init_config(ncclComm_t* comm, int world,
                                                    const void* unique_id, int rank,
                                                    int max_ctas);
CUFLASH_EXPORT int cuflash_cp_nccl_comm_destroy(ncclComm_t comm);

// Transport of the ring entry points (process-wide; every rank of a
// communicator must use the same one, else the entry points return
// DIMENSION_MISMATCH on every rank):
//   0  copy engine over CUDA IPC (the default): each rank exports its K/V
//      chunks, the others pull them with copy-engine copies over NVLink and
//      push their dK/dV contributions straight to the owner; no SMs go to the
//      transfers (the step kernels leave 2 free for one-thread flag kernels).
//      The communicator is used for set-up and a small all-reduce per call;
//      ranks whose processes cannot open each other's memory (CUDA IPC) fall
//      back to NCCL together.
//   1  NCCL send/recv ring (the step kernels leave 16 SMs free by default).
// The environment variable CUFLASH_CP_TRANSPORT=nccl selects 1 at start-up.
// comm_destroy releases the communicator's copy-engine context: call it on
// every rank once every rank's ring calls have completed (for instance after
// a device synchronisation and a barrier), since peers write into the
// context's memory.
CUFLASH_EXPORT int cuflash_cp_set_transport(int transport);

// Waits of the copy-engine transport for another rank give up after 60 s
// (CUFLASH_CP_WAIT_LIMIT_MS), so that a rank that left does not hang the
// others: the entry points then return CUDA_ERROR, on every rank of the
// communicator, until this function (which reads and clears the status, 1 =
// a wait gave up) has been called on the ranks where a wait gave up.
CUFLASH_EXPORT int cuflash_cp_transport_status(void);

#ifdef __cplusplus
}
#endif
