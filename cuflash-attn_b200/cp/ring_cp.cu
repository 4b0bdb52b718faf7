// Context-parallel attention: the ring drivers behind
// cuflash_attention_{forward,backward}_cp_{bf16,f16} (libcuflash_attn_cp.so),
// over either transport: copy-engine copies between CUDA-IPC-shared buffers
// (the default; drivers forward_cp_peer / backward_cp_peer below, transport
// in peer_ring.cu) or NCCL send/recv (forward_cp / backward_cp).
//
// The reference library is single-device; this file has no counterpart
// there.  It keeps the reference's C-ABI conventions (validation before any
// CUDA or NCCL call, src/api/flash_attention_api.cu:45-79; stream-ordered
// workspace, src/backward/flash_attention_backward_typed.cu:373-394) and runs
// every step's attention through libcuflash_attn.so's one-launch ring-step
// entry points; the only kernel here fills the running log-sum-exp with -inf.
//
// Streams (NCCL transport).  The caller's stream runs the step kernels; a
// library-owned stream per device (comm) runs the NCCL groups and, in the
// backward, the fp32 adds of the travelling dK/dV accumulators.  K/V of step s (X_s) is the caller's
// K/V for s = 0 and ring buffer (s - 1) % 2 afterwards; the group of step s
// sends X_s to rank + 1 and receives X_{s+1} from rank - 1 into the buffer
// that X_{s-1} used, after step s - 1's kernels have read it.  Step s + 1's
// kernels wait for that receive.  Every rank issues the same NCCL groups in
// the same order (forward: one K/V group per step but the last; backward: a
// K/V group per step but the last and an accumulator group after every
// step), so the pairing of sends and receives is the same on all ranks.

#include <cuda_runtime.h>
#include <nccl.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "cuflash/flash_attention.h"
#include "cuflash/flash_attention_cp.h"
#include "peer_ring.h"

namespace {

using cuflash::FlashAttentionError;
using cuflash_cp::PeerCtx;

constexpr int kMaxDevices = 64;
constexpr int kDefaultReserveSms = 16;
constexpr int kMaxWorld = 256;  // ranks of one ring (bounds the events of a call)

// ------------------------------------------------------------------ schedule

struct StepPlan {
    int owner = 0;
    int n = 0;
    int q_slot[4] = {};
    int kv_slot[4] = {};
    int q_chunk[4] = {};
    int kv_chunk[4] = {};
    int launch[4] = {};
    int num_launches = 0;
};

void zigzag(int rank, int world, int out[2]) {
    out[0] = rank;
    out[1] = 2 * world - 1 - rank;
}

// Pairs (query slot qi, K/V slot ki) in the order qi-major; a pair is visible
// unless causal masking hides the whole K/V chunk (it lies after the query
// chunk).  Forward launches: each pair joins the first launch that does not
// yet merge its query slot.
StepPlan plan_step(int rank, int world, int step, bool causal) {
    StepPlan p;
    p.owner = ((rank - step) % world + world) % world;
    int qc[2], kc[2];
    zigzag(rank, world, qc);
    zigzag(p.owner, world, kc);
    bool used[4][2] = {};
    for (int qi = 0; qi < 2; ++qi)
        for (int ki = 0; ki < 2; ++ki) {
            if (causal && kc[ki] > qc[qi]) continue;
            const int i = p.n++;
            p.q_slot[i] = qi;
            p.kv_slot[i] = ki;
            p.q_chunk[i] = qc[qi];
            p.kv_chunk[i] = kc[ki];
            int l = 0;
            while (used[l][qi]) ++l;
            used[l][qi] = true;
            p.launch[i] = l;
            if (l + 1 > p.num_launches) p.num_launches = l + 1;
        }
    return p;
}

// ------------------------------------------------------------ device state

// Stream-ordered workspace from a library-private pool per device (freed
// blocks stay cached, so repeated calls do not remap memory).
FlashAttentionError ws_alloc(void** ptr, size_t bytes, cudaStream_t stream) {
    static std::mutex mu;
    static cudaMemPool_t pools[kMaxDevices] = {};
    *ptr = nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return FlashAttentionError::CUDA_ERROR;
    cudaMemPool_t pool;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (pools[dev] == nullptr) {
            cudaMemPoolProps props = {};
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = dev;
            cudaMemPool_t p = nullptr;
            if (cudaMemPoolCreate(&p, &props) != cudaSuccess) return FlashAttentionError::CUDA_ERROR;
            uint64_t keep = ~0ull;
            cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
            pools[dev] = p;
        }
        pool = pools[dev];
    }
    const cudaError_t err = cudaMallocFromPoolAsync(ptr, bytes, pool, stream);
    if (err != cudaSuccess) {
        cudaGetLastError();
        *ptr = nullptr;
        return err == cudaErrorMemoryAllocation ? FlashAttentionError::OUT_OF_MEMORY
                                                : FlashAttentionError::CUDA_ERROR;
    }
    return FlashAttentionError::SUCCESS;
}

// The comm stream of the current device (non-blocking, kept for the life of
// the process).
cudaStream_t comm_stream() {
    static std::mutex mu;
    static cudaStream_t streams[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (streams[dev] == nullptr) {
        cudaStream_t st = nullptr;
        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
        streams[dev] = st;
    }
    return streams[dev];
}

__global__ void fill_f32_kernel(float* __restrict__ dst, float value, long long n) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride)
        dst[i] = value;
}

FlashAttentionError fill_f32(float* dst, float value, long long n, cudaStream_t stream) {
    long long blocks = (n + 255) / 256;
    if (blocks > 1184) blocks = 1184;
    if (blocks < 1) blocks = 1;
    fill_f32_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(dst, value, n);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

// Events of one call, destroyed when the call returns (an event destroyed
// while its record is pending is released once it completes).
struct Events {
    std::vector<cudaEvent_t> ev;
    cudaEvent_t make() {
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
        ev.push_back(e);
        return e;
    }
    ~Events() {
        for (cudaEvent_t e : ev) cudaEventDestroy(e);
    }
};

// `waiter` waits for the work enqueued on `producer` so far.
bool join(Events& evs, cudaStream_t waiter, cudaStream_t producer) {
    cudaEvent_t e = evs.make();
    return e != nullptr && cudaEventRecord(e, producer) == cudaSuccess &&
           cudaStreamWaitEvent(waiter, e, 0) == cudaSuccess;
}

// --------------------------------------------------------------- dtype glue

template <typename T>
struct CpOps;

template <>
struct CpOps<__nv_bfloat16> {
    using T = __nv_bfloat16;
    static int step(const T* Q, const T* K, const T* V, float* O, float* L, int B, int H, int C,
                    int D, float s, bool causal, int n, const int* qs, const int* ks,
                    const long long* qo, const long long* ko, int reserve, cudaStream_t st) {
        return cuflash_attention_forward_cp_step_bf16(Q, K, V, O, L, 2, 2, B, H, C, D, s, causal,
                                                      n, qs, ks, qo, ko, reserve, st);
    }
    static int convert(const float* src, T* dst, long long n, cudaStream_t st) {
        return cuflash_convert_f32_to_bf16(src, dst, n, st);
    }
    static int bwd_prepare(const T* O, const T* dO, const float* L, void* ws, int B, int H, int C,
                           int D, cudaStream_t st) {
        return cuflash_attention_backward_cp_prepare_bf16(O, dO, L, ws, 2, B, H, C, D, st);
    }
    static int bwd_step(const T* Q, const T* dO, const T* K, const T* V, void* ws, float* dk,
                        float* dv, int B, int H, int C, int D, float s, bool causal, int n,
                        const int* qs, const int* ks, const long long* qo, const long long* ko,
                        int reserve, cudaStream_t st) {
        return cuflash_attention_backward_cp_step_bf16(Q, dO, K, V, ws, dk, dv, 2, 2, B, H, C, D,
                                                       s, causal, n, qs, ks, qo, ko, reserve, st);
    }
    static int bwd_finish(const void* ws, T* dQ, int B, int H, int C, int D, float s,
                          cudaStream_t st) {
        return cuflash_attention_backward_cp_finish_bf16(ws, dQ, 2, B, H, C, D, s, st);
    }
};

template <>
struct CpOps<half> {
    using T = half;
    static int step(const T* Q, const T* K, const T* V, float* O, float* L, int B, int H, int C,
                    int D, float s, bool causal, int n, const int* qs, const int* ks,
                    const long long* qo, const long long* ko, int reserve, cudaStream_t st) {
        return cuflash_attention_forward_cp_step_f16(Q, K, V, O, L, 2, 2, B, H, C, D, s, causal,
                                                     n, qs, ks, qo, ko, reserve, st);
    }
    static int convert(const float* src, T* dst, long long n, cudaStream_t st) {
        return cuflash_convert_f32_to_f16(src, dst, n, st);
    }
    static int bwd_prepare(const T* O, const T* dO, const float* L, void* ws, int B, int H, int C,
                           int D, cudaStream_t st) {
        return cuflash_attention_backward_cp_prepare_f16(O, dO, L, ws, 2, B, H, C, D, st);
    }
    static int bwd_step(const T* Q, const T* dO, const T* K, const T* V, void* ws, float* dk,
                        float* dv, int B, int H, int C, int D, float s, bool causal, int n,
                        const int* qs, const int* ks, const long long* qo, const long long* ko,
                        int reserve, cudaStream_t st) {
        return cuflash_attention_backward_cp_step_f16(Q, dO, K, V, ws, dk, dv, 2, 2, B, H, C, D, s,
                                                      causal, n, qs, ks, qo, ko, reserve, st);
    }
    static int bwd_finish(const void* ws, T* dQ, int B, int H, int C, int D, float s,
                          cudaStream_t st) {
        return cuflash_attention_backward_cp_finish_f16(ws, dQ, 2, B, H, C, D, s, st);
    }
};

FlashAttentionError code(int c) { return static_cast<FlashAttentionError>(c); }

// -------------------------------------------------------------- validation

FlashAttentionError validate(const void* const* ptrs, int nptrs, int B, int H, int N, int D,
                             float scale, ncclComm_t comm, int rank, int world, int reserve_sms) {
    for (int i = 0; i < nptrs; ++i)
        if (ptrs[i] == nullptr) return FlashAttentionError::NULL_POINTER;
    if (B <= 0 || H <= 0 || N <= 0 || D <= 0 || world <= 0 || world > kMaxWorld || rank < 0 ||
        rank >= world || reserve_sms < -1)
        return FlashAttentionError::INVALID_DIMENSION;
    if (N % (2 * world) != 0) return FlashAttentionError::INVALID_DIMENSION;
    if (static_cast<long long>(B) * H * 2 > 0x7fffffffLL)
        return FlashAttentionError::INVALID_DIMENSION;
    if (!(D == 32 || D == 64 || D == 128)) return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    if (!std::isfinite(scale) || scale < 0.0f) return FlashAttentionError::INVALID_DIMENSION;
    if (world > 1 && comm == nullptr) return FlashAttentionError::NULL_POINTER;
    return FlashAttentionError::SUCCESS;
}

// After validation: the communicator must match the ranks the caller names.
FlashAttentionError check_comm(ncclComm_t comm, int rank, int world) {
    if (world == 1 && comm == nullptr) return FlashAttentionError::SUCCESS;
    int n = 0, r = 0;
    if (ncclCommCount(comm, &n) != ncclSuccess || ncclCommUserRank(comm, &r) != ncclSuccess)
        return FlashAttentionError::CUDA_ERROR;
    if (n != world || r != rank) return FlashAttentionError::DIMENSION_MISMATCH;
    return FlashAttentionError::SUCCESS;
}

// One ring hop of a K/V pair (and nothing else) in one NCCL group.
bool exchange(const void* send_k, const void* send_v, void* recv_k, void* recv_v, size_t bytes,
              int rank, int world, ncclComm_t comm, cudaStream_t st) {
    const int next = (rank + 1) % world, prev = (rank - 1 + world) % world;
    bool ok = ncclGroupStart() == ncclSuccess;
    ok = ok && ncclSend(send_k, bytes, ncclUint8, next, comm, st) == ncclSuccess;
    ok = ok && ncclSend(send_v, bytes, ncclUint8, next, comm, st) == ncclSuccess;
    ok = ok && ncclRecv(recv_k, bytes, ncclUint8, prev, comm, st) == ncclSuccess;
    ok = ok && ncclRecv(recv_v, bytes, ncclUint8, prev, comm, st) == ncclSuccess;
    return (ncclGroupEnd() == ncclSuccess) && ok;
}

bool exchange_one(const void* send, void* recv, size_t bytes, int rank, int world,
                  ncclComm_t comm, cudaStream_t st) {
    const int next = (rank + 1) % world, prev = (rank - 1 + world) % world;
    bool ok = ncclGroupStart() == ncclSuccess;
    ok = ok && ncclSend(send, bytes, ncclUint8, next, comm, st) == ncclSuccess;
    ok = ok && ncclRecv(recv, bytes, ncclUint8, prev, comm, st) == ncclSuccess;
    return (ncclGroupEnd() == ncclSuccess) && ok;
}

// SMs the step kernels leave free by default: NCCL's send/recv kernels need
// about 16 to keep up with the steps; the copy-engine transport only runs
// one-thread flag kernels beside them.
constexpr int kDefaultReserveSmsPeer = 2;

int effective_reserve(int reserve_sms, int world, bool peer) {
    if (world == 1) return 0;  // no transfer runs beside the kernels
    if (reserve_sms >= 0) return reserve_sms;
    return peer ? kDefaultReserveSmsPeer : kDefaultReserveSms;
}

// ------------------------------------------------ copy-engine transport drivers
//
// Step s of rank r computes with X_s, the K/V of owner (r - s) mod W (X_0 is
// the caller's).  Each rank first copies its K and V into its export E (on
// the comm stream, once the readers of the previous call's E are done), then
// pulls X_s from the owner's E into pull slot s % 2 on the comm stream: X_1
// and X_2 right away, X_{s+2} once step s's kernels (the slot's previous
// readers) are done.  Step s's kernels wait for their pull.  The backward
// pushes step s's dK/dV (s >= 1) into its owner's slot for this rank and,
// at the end, sums its own and the W - 1 received contributions.

// A copy between GPUs (or into the export), on the comm stream: one
// copy-engine copy.  (Splitting it over several streams and engines was
// measured: no change at 8 GPUs, the copies are not the limiter.)
bool peer_copy(void* dst, const void* src, size_t bytes, cudaStream_t cs) {
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, cs) == cudaSuccess;
}

template <typename T>
struct PullPlan {
    PeerCtx* ctx;
    int rank, world;
    long long k;  // this call's number
    size_t kv_bytes;
    // pull slot of step s: [K pair][V pair]
    char* slot(int s) const { return ctx->pull_slot(s % 2); }
    int owner(int s) const { return ((rank - s) % world + world) % world; }
};

// Export this rank's K/V and signal it (comm stream).
template <typename T>
bool export_kv(const PullPlan<T>& pp, const T* K, const T* V, cudaStream_t cs) {
    PeerCtx& c = *pp.ctx;
    // readers of the previous call's export are done (their flags on this rank)
    bool ok = cuflash_cp::wait_all_geq(c.flags + 2 + 2 * pp.world, pp.world, pp.rank, c.calls, cs);
    ok = ok && peer_copy(c.mem, K, pp.kv_bytes, cs);
    ok = ok && peer_copy(c.mem + pp.kv_bytes, V, pp.kv_bytes, cs);
    if (cuflash_cp::test_skip_export_signal()) return ok || cuflash_cp::debug_fail("export");
    return (ok && cuflash_cp::signal(c.flags + 0, pp.k, cs)) || cuflash_cp::debug_fail("export");
}

// Pull X_s into slot s % 2 (comm stream); `prev_reader` (may be null) is the
// event of the step that last read the slot.
template <typename T>
bool pull_kv(const PullPlan<T>& pp, int s, cudaEvent_t prev_reader, Events& evs, cudaStream_t cs,
             cudaEvent_t* done) {
    PeerCtx& c = *pp.ctx;
    const int o = pp.owner(s);
    bool ok = prev_reader == nullptr || cudaStreamWaitEvent(cs, prev_reader, 0) == cudaSuccess;
    ok = ok && cuflash_cp::wait_geq(c.fl(o) + 0, pp.k, cs);
    ok = ok && peer_copy(pp.slot(s), c.e(o), 2 * pp.kv_bytes, cs);
    // this rank is done reading o's export
    ok = ok && cuflash_cp::signal(c.fl(o) + 2 + 2 * pp.world + pp.rank, pp.k, cs);
    *done = ok ? evs.make() : nullptr;
    return (ok && *done != nullptr && cudaEventRecord(*done, cs) == cudaSuccess) ||
           cuflash_cp::debug_fail("pull");
}

template <typename T>
FlashAttentionError forward_cp_peer(PeerCtx& ctx, const T* Q, const T* K, const T* V, T* O,
                                    float* L, int B, int H, int C, int D, float scale, bool causal,
                                    int rank, int world, int reserve, cudaStream_t stream,
                                    cudaStream_t cs) {
    const long long elems = 2LL * B * H * C * D;
    const size_t kv_bytes = static_cast<size_t>(elems) * sizeof(T);
    const size_t oacc_bytes = static_cast<size_t>(elems) * sizeof(float);
    void* ws = nullptr;
    FlashAttentionError e = ws_alloc(&ws, oacc_bytes, stream);
    if (e != FlashAttentionError::SUCCESS) return e;
    float* O_acc = static_cast<float*>(ws);
    const PullPlan<T> pp{&ctx, rank, world, ctx.calls + 1, kv_bytes};
    Events evs;
    cudaEvent_t recv[kMaxWorld] = {};
    cudaEvent_t comp[kMaxWorld] = {};
    bool ok = cudaMemsetAsync(O_acc, 0, oacc_bytes, stream) == cudaSuccess;
    if (ok) e = fill_f32(L, -INFINITY, elems / D, stream);
    ok = ok && e == FlashAttentionError::SUCCESS;
    ok = ok && join(evs, cs, stream);  // K, V, the workspace and the last call's readers
    // the previous call's kernels, on whatever stream, are done with the slots
    ok = ok && cudaStreamWaitEvent(cs, ctx.last_use, 0) == cudaSuccess;
    ok = ok && export_kv(pp, K, V, cs);
    for (int s = 1; ok && s < world && s <= 2; ++s) ok = pull_kv(pp, s, nullptr, evs, cs, &recv[s]);
    for (int s = 0; ok && s < world; ++s) {
        const StepPlan p = plan_step(rank, world, s, causal);
        const T* ck = s == 0 ? K : reinterpret_cast<const T*>(pp.slot(s));
        const T* cv = s == 0 ? V : reinterpret_cast<const T*>(pp.slot(s) + kv_bytes);
        if (s >= 1) ok = cudaStreamWaitEvent(stream, recv[s], 0) == cudaSuccess;
        for (int l = 0; ok && l < p.num_launches; ++l) {
            int qs[4], ks[4], n = 0;
            long long qo[4], ko[4];
            for (int i = 0; i < p.n; ++i) {
                if (p.launch[i] != l) continue;
                qs[n] = p.q_slot[i];
                ks[n] = p.kv_slot[i];
                qo[n] = static_cast<long long>(p.q_chunk[i]) * C;
                ko[n] = static_cast<long long>(p.kv_chunk[i]) * C;
                ++n;
            }
            e = code(CpOps<T>::step(Q, ck, cv, O_acc, L, B, H, C, D, scale, causal, n, qs, ks, qo,
                                    ko, reserve, stream));
            ok = e == FlashAttentionError::SUCCESS || cuflash_cp::debug_fail("forward step");
        }
        if (ok && s >= 1 && s + 2 < world) {
            comp[s] = evs.make();
            ok = comp[s] != nullptr && cudaEventRecord(comp[s], stream) == cudaSuccess;
            ok = ok && pull_kv(pp, s + 2, comp[s], evs, cs, &recv[s + 2]);
        }
    }
    if (ok) {
        e = code(CpOps<T>::convert(O_acc, O, elems, stream));
        ok = e == FlashAttentionError::SUCCESS;
    }
    join(evs, stream, cs);
    cudaEventRecord(ctx.last_use, stream);
    cudaFreeAsync(ws, stream);
    ++ctx.calls;  // every rank counts every call, failed or not
    if (!ok) return e != FlashAttentionError::SUCCESS ? e : FlashAttentionError::CUDA_ERROR;
    return FlashAttentionError::SUCCESS;
}

template <typename T>
FlashAttentionError backward_cp_peer(PeerCtx& ctx, const T* Q, const T* K, const T* V, const T* O,
                                     const float* L, const T* dO, T* dQ, T* dK, T* dV, int B,
                                     int H, int C, int D, float scale, bool causal, int rank,
                                     int world, int reserve, cudaStream_t stream,
                                     cudaStream_t cs) {
    const long long elems = 2LL * B * H * C * D;
    const size_t kv_bytes = static_cast<size_t>(elems) * sizeof(T);
    const size_t acc_bytes = 2 * static_cast<size_t>(elems) * sizeof(float);  // dK, dV
    const long long bwd_ws = cuflash_attention_backward_cp_workspace_size(2, B, H, C, D);
    if (bwd_ws <= 0) return FlashAttentionError::INVALID_DIMENSION;
    const size_t bwd_bytes = (static_cast<size_t>(bwd_ws) + 255) & ~static_cast<size_t>(255);
    void* ws = nullptr;
    FlashAttentionError e = ws_alloc(&ws, bwd_bytes + acc_bytes, stream);
    if (e != FlashAttentionError::SUCCESS) return e;
    char* base = static_cast<char*>(ws);
    void* ws_bwd = base;
    float* own = reinterpret_cast<float*>(base + bwd_bytes);  // this rank's chunks (step 0)
    float* part[2] = {ctx.part(0), ctx.part(1)};  // pushed from: in the peer allocation
    const PullPlan<T> pp{&ctx, rank, world, ctx.calls + 1, kv_bytes};
    const long long k = pp.k;
    Events evs;
    cudaEvent_t recv[kMaxWorld] = {};
    cudaEvent_t comp[kMaxWorld] = {};
    cudaEvent_t pushed[kMaxWorld] = {};
    e = code(CpOps<T>::bwd_prepare(O, dO, L, ws_bwd, B, H, C, D, stream));
    bool ok = e == FlashAttentionError::SUCCESS;
    ok = ok && cudaMemsetAsync(own, 0, acc_bytes, stream) == cudaSuccess;
    ok = ok && join(evs, cs, stream);
    ok = ok && cudaStreamWaitEvent(cs, ctx.last_use, 0) == cudaSuccess;
    // the part buffers are written on `stream`: after the previous call too
    ok = ok && cudaStreamWaitEvent(stream, ctx.last_use, 0) == cudaSuccess;
    ok = ok && export_kv(pp, K, V, cs);
    for (int s = 1; ok && s < world && s <= 2; ++s) ok = pull_kv(pp, s, nullptr, evs, cs, &recv[s]);
    for (int s = 0; ok && s < world; ++s) {
        const StepPlan p = plan_step(rank, world, s, causal);
        const T* ck = s == 0 ? K : reinterpret_cast<const T*>(pp.slot(s));
        const T* cv = s == 0 ? V : reinterpret_cast<const T*>(pp.slot(s) + kv_bytes);
        float* target = s == 0 ? own : part[s % 2];
        if (s >= 1) {
            ok = cudaStreamWaitEvent(stream, recv[s], 0) == cudaSuccess;
            // the part buffer's previous contents (step s - 2) have been pushed
            if (ok && s >= 3) ok = cudaStreamWaitEvent(stream, pushed[s - 2], 0) == cudaSuccess;
            ok = ok && cudaMemsetAsync(target, 0, acc_bytes, stream) == cudaSuccess;
        }
        if (ok && p.n > 0) {
            int qs[4], ks[4];
            long long qo[4], ko[4];
            for (int i = 0; i < p.n; ++i) {
                qs[i] = p.q_slot[i];
                ks[i] = p.kv_slot[i];
                qo[i] = static_cast<long long>(p.q_chunk[i]) * C;
                ko[i] = static_cast<long long>(p.kv_chunk[i]) * C;
            }
            e = code(CpOps<T>::bwd_step(Q, dO, ck, cv, ws_bwd, target, target + elems, B, H, C, D,
                                        scale, causal, p.n, qs, ks, qo, ko, reserve, stream));
            ok = e == FlashAttentionError::SUCCESS || cuflash_cp::debug_fail("backward step");
        }
        if (!ok || s == 0) continue;
        comp[s] = evs.make();
        ok = comp[s] != nullptr && cudaEventRecord(comp[s], stream) == cudaSuccess;
        // push this step's dK/dV to the owner of X_s, once the owner has summed
        // this rank's contribution of the last backward call (only backward
        // calls advance that flag)
        const int o = pp.owner(s);
        ok = ok && cudaStreamWaitEvent(cs, comp[s], 0) == cudaSuccess;
        ok = ok && cuflash_cp::wait_geq(ctx.flags + 2 + world + o, ctx.last_bwd, cs);
        ok = ok && peer_copy(ctx.r_slot(o, rank), target, acc_bytes, cs);
        ok = ok && cuflash_cp::signal(ctx.fl(o) + 2 + rank, k, cs);
        pushed[s] = ok ? evs.make() : nullptr;
        ok = (ok && pushed[s] != nullptr && cudaEventRecord(pushed[s], cs) == cudaSuccess) ||
             cuflash_cp::debug_fail("push");
        if (ok && s + 2 < world) ok = pull_kv(pp, s + 2, comp[s], evs, cs, &recv[s + 2]);
    }
    ok = ok && join(evs, stream, cs);
    // every other rank's contribution to this rank's chunks has landed
    ok = ok && cuflash_cp::wait_all_geq(ctx.flags + 2, world, rank, k, stream);
    if (ok) {
        e = code(CpOps<T>::bwd_finish(ws_bwd, dQ, B, H, C, D, scale, stream));
        ok = e == FlashAttentionError::SUCCESS;
    }
    ok = ok && cuflash_cp::sum_contributions<T>(ctx, own, dK, dV, elems, stream);
    // the senders may overwrite their slots on this rank in the next call
    ok = ok && cuflash_cp::signal_peers(ctx, 2 + world + rank, k, stream);
    if (!ok) join(evs, stream, cs);
    cudaEventRecord(ctx.last_use, stream);
    cudaFreeAsync(ws, stream);
    ++ctx.calls;
    ctx.last_bwd = k;
    if (!ok) return e != FlashAttentionError::SUCCESS ? e : FlashAttentionError::CUDA_ERROR;
    return FlashAttentionError::SUCCESS;
}

// The transport of a call with world > 1: sets *ctx for the copy-engine
// transport, leaves it null for NCCL.
FlashAttentionError pick_transport(ncclComm_t comm, int rank, int world, size_t e_bytes,
                                   size_t r_bytes, cudaStream_t cs, PeerCtx** ctx) {
    *ctx = nullptr;
    return cuflash_cp::peer_acquire(comm, rank, world, e_bytes, r_bytes, cs, ctx);
}

// ------------------------------------------------------------------ forward

template <typename T>
FlashAttentionError forward_cp(const T* Q, const T* K, const T* V, T* O, float* L, int B, int H,
                               int N, int D, float scale, bool causal, ncclComm_t comm, int rank,
                               int world, int reserve_sms, cudaStream_t stream) {
    const void* ptrs[] = {Q, K, V, O, L};
    FlashAttentionError e = validate(ptrs, 5, B, H, N, D, scale, comm, rank, world, reserve_sms);
    if (e != FlashAttentionError::SUCCESS) return e;
    e = check_comm(comm, rank, world);
    if (e != FlashAttentionError::SUCCESS) return e;

    const int C = N / (2 * world);
    const long long elems = 2LL * B * H * C * D;  // both slots of one tensor
    const size_t kv_bytes = static_cast<size_t>(elems) * sizeof(T);
    const size_t oacc_bytes = static_cast<size_t>(elems) * sizeof(float);
    const size_t ws_bytes = oacc_bytes + (world > 1 ? 4 * kv_bytes : 0);
    cudaStream_t cs = world > 1 ? comm_stream() : nullptr;
    if (world > 1 && cs == nullptr) return FlashAttentionError::CUDA_ERROR;
    if (world > 1) {
        PeerCtx* ctx = nullptr;
        e = pick_transport(comm, rank, world, 2 * kv_bytes, 0, cs, &ctx);
        if (e != FlashAttentionError::SUCCESS) return e;
        if (ctx != nullptr)
            return forward_cp_peer<T>(*ctx, Q, K, V, O, L, B, H, C, D, scale, causal, rank, world,
                                      effective_reserve(reserve_sms, world, true), stream, cs);
    }
    const int reserve = effective_reserve(reserve_sms, world, false);

    void* ws = nullptr;
    e = ws_alloc(&ws, ws_bytes, stream);
    if (e != FlashAttentionError::SUCCESS) return e;
    float* O_acc = static_cast<float*>(ws);
    T* buf_k[2] = {nullptr, nullptr};
    T* buf_v[2] = {nullptr, nullptr};
    if (world > 1) {
        char* b = static_cast<char*>(ws) + oacc_bytes;
        for (int i = 0; i < 2; ++i) {
            buf_k[i] = reinterpret_cast<T*>(b + (2 * i) * kv_bytes);
            buf_v[i] = reinterpret_cast<T*>(b + (2 * i + 1) * kv_bytes);
        }
    }
    Events evs;
    bool ok = cudaMemsetAsync(O_acc, 0, oacc_bytes, stream) == cudaSuccess;
    if (ok) e = fill_f32(L, -INFINITY, elems / D, stream);
    ok = ok && e == FlashAttentionError::SUCCESS;
    if (ok && world > 1) ok = join(evs, cs, stream);  // K, V and the workspace are ready

    const T* cur_k = K;
    const T* cur_v = V;
    cudaEvent_t comp_prev = nullptr;  // step s-1's kernels have been enqueued up to here
    for (int s = 0; ok && s < world; ++s) {
        const StepPlan p = plan_step(rank, world, s, causal);
        cudaEvent_t recv_done = nullptr;
        if (s + 1 < world) {
            T* nk = buf_k[s % 2];
            T* nv = buf_v[s % 2];
            // the buffer receiving X_{s+1} held X_{s-1}: step s-1 must have read it
            if (s >= 2) ok = cudaStreamWaitEvent(cs, comp_prev, 0) == cudaSuccess;
            ok = ok && exchange(cur_k, cur_v, nk, nv, kv_bytes, rank, world, comm, cs);
            recv_done = evs.make();
            ok = ok && recv_done != nullptr && cudaEventRecord(recv_done, cs) == cudaSuccess;
        }
        for (int l = 0; ok && l < p.num_launches; ++l) {
            int qs[4], ks[4], n = 0;
            long long qo[4], ko[4];
            for (int i = 0; i < p.n; ++i) {
                if (p.launch[i] != l) continue;
                qs[n] = p.q_slot[i];
                ks[n] = p.kv_slot[i];
                qo[n] = static_cast<long long>(p.q_chunk[i]) * C;
                ko[n] = static_cast<long long>(p.kv_chunk[i]) * C;
                ++n;
            }
            e = code(CpOps<T>::step(Q, cur_k, cur_v, O_acc, L, B, H, C, D, scale, causal, n, qs,
                                    ks, qo, ko, reserve, stream));
            ok = e == FlashAttentionError::SUCCESS;
        }
        if (ok && s + 1 < world) {
            comp_prev = evs.make();
            ok = comp_prev != nullptr && cudaEventRecord(comp_prev, stream) == cudaSuccess;
            ok = ok && cudaStreamWaitEvent(stream, recv_done, 0) == cudaSuccess;
            cur_k = buf_k[s % 2];
            cur_v = buf_v[s % 2];
        }
    }
    if (ok) {
        e = code(CpOps<T>::convert(O_acc, O, elems, stream));
        ok = e == FlashAttentionError::SUCCESS;
    }
    // the comm stream has no work left past the last receive the caller's
    // stream waited for, so the workspace can go back to the pool
    if (world > 1 && !ok) join(evs, stream, cs);
    cudaFreeAsync(ws, stream);
    if (!ok) return e != FlashAttentionError::SUCCESS ? e : FlashAttentionError::CUDA_ERROR;
    return FlashAttentionError::SUCCESS;
}

// ----------------------------------------------------------------- backward

template <typename T>
FlashAttentionError backward_cp(const T* Q, const T* K, const T* V, const T* O, const float* L,
                                const T* dO, T* dQ, T* dK, T* dV, int B, int H, int N, int D,
                                float scale, bool causal, ncclComm_t comm, int rank, int world,
                                int reserve_sms, cudaStream_t stream) {
    if (!dO || !dQ || !dK || !dV) return FlashAttentionError::NULL_POINTER;
    const void* ptrs[] = {Q, K, V, O, L};
    FlashAttentionError e = validate(ptrs, 5, B, H, N, D, scale, comm, rank, world, reserve_sms);
    if (e != FlashAttentionError::SUCCESS) return e;
    e = check_comm(comm, rank, world);
    if (e != FlashAttentionError::SUCCESS) return e;

    const int C = N / (2 * world);
    const long long elems = 2LL * B * H * C * D;
    const size_t kv_bytes = static_cast<size_t>(elems) * sizeof(T);
    const long long bwd_ws = cuflash_attention_backward_cp_workspace_size(2, B, H, C, D);
    if (bwd_ws <= 0) return FlashAttentionError::INVALID_DIMENSION;
    const size_t bwd_bytes = (static_cast<size_t>(bwd_ws) + 255) & ~static_cast<size_t>(255);
    // one accumulator = dK and dV of both K/V slots, fp32
    const size_t acc_bytes = 2 * static_cast<size_t>(elems) * sizeof(float);
    const int n_acc = world > 1 ? 2 : 1;
    const int n_part = world > 1 ? 2 : 0;
    const size_t ws_bytes =
        bwd_bytes + (n_acc + n_part) * acc_bytes + (world > 1 ? 4 * kv_bytes : 0);
    cudaStream_t cs = world > 1 ? comm_stream() : nullptr;
    if (world > 1 && cs == nullptr) return FlashAttentionError::CUDA_ERROR;
    if (world > 1) {
        PeerCtx* ctx = nullptr;
        e = pick_transport(comm, rank, world, 2 * kv_bytes, acc_bytes, cs, &ctx);
        if (e != FlashAttentionError::SUCCESS) return e;
        if (ctx != nullptr)
            return backward_cp_peer<T>(*ctx, Q, K, V, O, L, dO, dQ, dK, dV, B, H, C, D, scale,
                                       causal, rank, world,
                                       effective_reserve(reserve_sms, world, true), stream, cs);
    }
    const int reserve = effective_reserve(reserve_sms, world, false);

    void* ws = nullptr;
    e = ws_alloc(&ws, ws_bytes, stream);
    if (e != FlashAttentionError::SUCCESS) return e;
    char* base = static_cast<char*>(ws);
    void* ws_bwd = base;
    float* acc[2] = {nullptr, nullptr};
    float* part[2] = {nullptr, nullptr};
    char* b = base + bwd_bytes;
    for (int i = 0; i < n_acc; ++i, b += acc_bytes) acc[i] = reinterpret_cast<float*>(b);
    for (int i = 0; i < n_part; ++i, b += acc_bytes) part[i] = reinterpret_cast<float*>(b);
    T* buf_k[2] = {nullptr, nullptr};
    T* buf_v[2] = {nullptr, nullptr};
    if (world > 1)
        for (int i = 0; i < 2; ++i) {
            buf_k[i] = reinterpret_cast<T*>(b + (2 * i) * kv_bytes);
            buf_v[i] = reinterpret_cast<T*>(b + (2 * i + 1) * kv_bytes);
        }
    // dK of both slots, then dV of both slots
    auto dk_of = [&](float* a) { return a; };
    auto dv_of = [&](float* a) { return a + elems; };

    Events evs;
    e = code(CpOps<T>::bwd_prepare(O, dO, L, ws_bwd, B, H, C, D, stream));
    bool ok = e == FlashAttentionError::SUCCESS;
    ok = ok && cudaMemsetAsync(acc[0], 0, acc_bytes, stream) == cudaSuccess;
    for (int i = 0; ok && i < n_part; ++i)
        ok = cudaMemsetAsync(part[i], 0, acc_bytes, stream) == cudaSuccess;
    if (ok && world > 1) ok = join(evs, cs, stream);

    const T* cur_k = K;
    const T* cur_v = V;
    cudaEvent_t comp_prev = nullptr;
    cudaEvent_t part_free[2] = {nullptr, nullptr};  // part buffer cleared by its add
    int acc_cur = 0;
    for (int s = 0; ok && s < world; ++s) {
        const StepPlan p = plan_step(rank, world, s, causal);
        cudaEvent_t recv_done = nullptr;
        if (s + 1 < world) {
            if (s >= 2) ok = cudaStreamWaitEvent(cs, comp_prev, 0) == cudaSuccess;
            ok = ok && exchange(cur_k, cur_v, buf_k[s % 2], buf_v[s % 2], kv_bytes, rank, world,
                                comm, cs);
            recv_done = evs.make();
            ok = ok && recv_done != nullptr && cudaEventRecord(recv_done, cs) == cudaSuccess;
        }
        float* target = s == 0 ? acc[0] : part[s % 2];
        if (ok && s >= 2 && part_free[s % 2] != nullptr)
            ok = cudaStreamWaitEvent(stream, part_free[s % 2], 0) == cudaSuccess;
        if (ok && p.n > 0) {
            int qs[4], ks[4];
            long long qo[4], ko[4];
            for (int i = 0; i < p.n; ++i) {
                qs[i] = p.q_slot[i];
                ks[i] = p.kv_slot[i];
                qo[i] = static_cast<long long>(p.q_chunk[i]) * C;
                ko[i] = static_cast<long long>(p.kv_chunk[i]) * C;
            }
            e = code(CpOps<T>::bwd_step(Q, dO, cur_k, cur_v, ws_bwd, dk_of(target), dv_of(target),
                                        B, H, C, D, scale, causal, p.n, qs, ks, qo, ko, reserve,
                                        stream));
            ok = e == FlashAttentionError::SUCCESS;
        }
        if (ok && world > 1) {
            comp_prev = evs.make();
            ok = comp_prev != nullptr && cudaEventRecord(comp_prev, stream) == cudaSuccess;
            ok = ok && cudaStreamWaitEvent(cs, comp_prev, 0) == cudaSuccess;
            if (ok && s > 0) {
                // the accumulator of this step's K/V owner arrived in the
                // previous group; add this step's part into it and clear the part
                e = code(cuflash_accumulate_f32(acc[acc_cur], target, 2 * elems, true, cs));
                ok = e == FlashAttentionError::SUCCESS;
                part_free[s % 2] = evs.make();
                ok = ok && part_free[s % 2] != nullptr &&
                     cudaEventRecord(part_free[s % 2], cs) == cudaSuccess;
            }
            ok = ok && exchange_one(acc[acc_cur], acc[1 - acc_cur], acc_bytes, rank, world, comm,
                                    cs);
            acc_cur = 1 - acc_cur;
        }
        if (ok && s + 1 < world) {
            ok = cudaStreamWaitEvent(stream, recv_done, 0) == cudaSuccess;
            cur_k = buf_k[s % 2];
            cur_v = buf_v[s % 2];
        }
    }
    // this rank's own accumulator came in with the last group
    if (ok && world > 1) ok = join(evs, stream, cs);
    float* final_acc = acc[world > 1 ? acc_cur : 0];
    if (ok) {
        e = code(CpOps<T>::bwd_finish(ws_bwd, dQ, B, H, C, D, scale, stream));
        ok = e == FlashAttentionError::SUCCESS;
    }
    if (ok) {
        e = code(CpOps<T>::convert(dk_of(final_acc), dK, elems, stream));
        ok = e == FlashAttentionError::SUCCESS;
    }
    if (ok) {
        e = code(CpOps<T>::convert(dv_of(final_acc), dV, elems, stream));
        ok = e == FlashAttentionError::SUCCESS;
    }
    if (world > 1 && !ok) join(evs, stream, cs);
    cudaFreeAsync(ws, stream);
    if (!ok) return e != FlashAttentionError::SUCCESS ? e : FlashAttentionError::CUDA_ERROR;
    return FlashAttentionError::SUCCESS;
}

}  // namespace

extern "C" {

int cuflash_attention_forward_cp_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                      const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                      int batch_size, int num_heads, int seq_len, int head_dim,
                                      float scale, bool causal, ncclComm_t comm, int rank,
                                      int world, int reserve_sms, cudaStream_t stream) {
    return static_cast<int>(forward_cp<__nv_bfloat16>(Q, K, V, O, L, batch_size, num_heads,
                                                      seq_len, head_dim, scale, causal, comm,
                                                      rank, world, reserve_sms, stream));
}

int cuflash_attention_forward_cp_f16(const half* Q, const half* K, const half* V, half* O,
                                     float* L, int batch_size, int num_heads, int seq_len,
                                     int head_dim, float scale, bool causal, ncclComm_t comm,
                                     int rank, int world, int reserve_sms, cudaStream_t stream) {
    return static_cast<int>(forward_cp<half>(Q, K, V, O, L, batch_size, num_heads, seq_len,
                                             head_dim, scale, causal, comm, rank, world,
                                             reserve_sms, stream));
}

int cuflash_attention_backward_cp_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                       const __nv_bfloat16* V, const __nv_bfloat16* O,
                                       const float* L, const __nv_bfloat16* dO,
                                       __nv_bfloat16* dQ, __nv_bfloat16* dK, __nv_bfloat16* dV,
                                       int batch_size, int num_heads, int seq_len, int head_dim,
                                       float scale, bool causal, ncclComm_t comm, int rank,
                                       int world, int reserve_sms, cudaStream_t stream) {
    return static_cast<int>(backward_cp<__nv_bfloat16>(
        Q, K, V, O, L, dO, dQ, dK, dV, batch_size, num_heads, seq_len, head_dim, scale, causal,
        comm, rank, world, reserve_sms, stream));
}

int cuflash_attention_backward_cp_f16(const half* Q, const half* K, const half* V, const half* O,
                                      const float* L, const half* dO, half* dQ, half* dK,
                                      half* dV, int batch_size, int num_heads, int seq_len,
                                      int head_dim, float scale, bool causal, ncclComm_t comm,
                                      int rank, int world, int reserve_sms, cudaStream_t stream) {
    return static_cast<int>(backward_cp<half>(Q, K, V, O, L, dO, dQ, dK, dV, batch_size,
                                              num_heads, seq_len, head_dim, scale, causal, comm,
                                              rank, world, reserve_sms, stream));
}

int cuflash_cp_ring_schedule(int rank, int world, int step, bool causal, int* kv_owner,
                             int* num_pairs, int* q_slot, int* kv_slot, int* q_chunk,
                             int* kv_chunk, int* fwd_launch) {
    if (!kv_owner || !num_pairs || !q_slot || !kv_slot || !q_chunk || !kv_chunk || !fwd_launch)
        return static_cast<int>(FlashAttentionError::NULL_POINTER);
    if (world <= 0 || rank < 0 || rank >= world || step < 0 || step >= world)
        return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    const StepPlan p = plan_step(rank, world, step, causal);
    *kv_owner = p.owner;
    *num_pairs = p.n;
    for (int i = 0; i < p.n; ++i) {
        q_slot[i] = p.q_slot[i];
        kv_slot[i] = p.kv_slot[i];
        q_chunk[i] = p.q_chunk[i];
        kv_chunk[i] = p.kv_chunk[i];
        fwd_launch[i] = p.launch[i];
    }
    return static_cast<int>(FlashAttentionError::SUCCESS);
}

int cuflash_cp_nccl_unique_id(void* unique_id, int nbytes) {
    if (unique_id == nullptr) return static_cast<int>(FlashAttentionError::NULL_POINTER);
    if (nbytes < static_cast<int>(sizeof(ncclUniqueId)))
        return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess)
        return static_cast<int>(FlashAttentionError::CUDA_ERROR);
    std::memcpy(unique_id, &id, sizeof(id));
    return static_cast<int>(FlashAttentionError::SUCCESS);
}

int cuflash_cp_nccl_comm_init_config(ncclComm_t* comm, int world, const void* unique_id,
                                     int rank, int max_ctas) {
    if (comm == nullptr || unique_id == nullptr)
        return static_cast<int>(FlashAttentionError::NULL_POINTER);
    if (world <= 0 || rank < 0 || rank >= world || max_ctas < 0)
        return static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 1;  // the ring entry points require a blocking communicator
    if (max_ctas > 0) {
        config.minCTAs = 1;
        config.maxCTAs = max_ctas;
    }
    return static_cast<int>(ncclCommInitRankConfig(comm, world, id, rank, &config) == ncclSuccess
                                ? FlashAttentionError::SUCCESS
                                : FlashAttentionError::CUDA_ERROR);
}

int cuflash_cp_nccl_comm_init(ncclComm_t* comm, int world, const void* unique_id, int rank) {
    return cuflash_cp_nccl_comm_init_config(comm, world, unique_id, rank, 0);
}

int cuflash_cp_nccl_comm_destroy(ncclComm_t comm) {
    if (comm == nullptr) return static_cast<int>(FlashAttentionError::NULL_POINTER);
    cuflash_cp::peer_release(comm);
    return static_cast<int>(ncclCommDestroy(comm) == ncclSuccess
                                ? FlashAttentionError::SUCCESS
                                : FlashAttentionError::CUDA_ERROR);
}

int cuflash_cp_set_transport(int transport) {
    return cuflash_cp::set_transport(transport) == 0
               ? static_cast<int>(FlashAttentionError::SUCCESS)
               : static_cast<int>(FlashAttentionError::INVALID_DIMENSION);
}

int cuflash_cp_transport_status(void) { return cuflash_cp::status_read_and_clear(); }

}  // extern "C"
