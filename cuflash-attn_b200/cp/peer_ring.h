// Copy-engine transport of the context-parallel attention (internal to
// libcuflash_attn_cp.so).
//
// Every rank of a communicator exports one device allocation through CUDA
// IPC and opens every other rank's:
//   E        its K and V (both zigzag slots), copied in at the start of a
//            call; the ranks that need them pull them with one copy-engine
//            copy each (through NVSwitch every pair of GPUs has a full link,
//            so each K/V chunk crosses NVLink once per reader, no ring hops)
//   P[2]     this rank's pull slots (another rank's E lands here)
//   S[2]     (backward) this rank's dK/dV of a step, before it is pushed
//   R[w]     (backward) the fp32 dK/dV that rank w computed for this rank's
//            chunks, pushed by w with a copy-engine copy; summed once at the
//            end of the call
// Every buffer a copy between GPUs touches is in this cudaMalloc allocation
// (stream-ordered pool memory would need its own peer-access grants).
// and an int64 flag array, written with system-scope release stores (by this
// rank or by a peer over NVLink):
//   [0]           calls whose export of E finished (this rank)
//   [1]           unused
//   [2 + w]       calls whose contribution from rank w arrived in R[w] (by w)
//   [2 + W + o]   number of the last backward call after which owner o had
//                 summed this rank's R slot on o (by o)
//   [2 + 2W + w]  calls in which rank w finished pulling this rank's E (by w)
// Flags only grow, so a wait is "flag >= target".  Waits run in a one-thread
// kernel with a time limit; a wait that runs out sets the transport status
// (cuflash_cp_transport_status) and lets the stream go on.
//
// NCCL is used only for the collective set-up (allgather of the IPC handles)
// and for a small all-reduce at the start of every call, which checks that
// all ranks use the same transport and the same context.

#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <cstddef>

#include "cuflash/flash_attention.h"

namespace cuflash_cp {

constexpr int kTransportPeer = 0;  // copy engine over CUDA IPC (default)
constexpr int kTransportNccl = 1;  // NCCL send/recv ring

struct PeerCtx {
    ncclComm_t comm = nullptr;
    int dev = -1;
    int rank = 0;
    int world = 0;
    long long id = 0;         // the same on every rank of the context
    size_t e_cap = 0;         // bytes of E (and of one P slot)
    size_t r_cap = 0;         // bytes of one S or R slot
    char* mem = nullptr;      // [E][P_0 P_1][S_0 S_1][R_0 .. R_{W-1}] (R_rank unused)
    long long* flags = nullptr;
    char* peer_mem[256] = {};
    long long* peer_flags[256] = {};
    long long calls = 0;      // calls completed with this context (the same on all ranks)
    long long last_bwd = 0;   // number of the last backward call (0: none yet)
    // recorded on the caller's stream after a call's last read of the pull
    // slots and part buffers; the next call's comm stream waits for it
    // (whatever stream that call is given)
    cudaEvent_t last_use = nullptr;

    static size_t bytes(size_t e_cap, size_t r_cap, int world) {
        return 3 * e_cap + (2 + static_cast<size_t>(world)) * r_cap;
    }
    char* e(int r) const { return r == rank ? mem : peer_mem[r]; }
    char* pull_slot(int x) const { return mem + (1 + x) * e_cap; }
    float* part(int x) const { return reinterpret_cast<float*>(mem + 3 * e_cap + x * r_cap); }
    // rank `from`'s R slot on rank `on`
    char* r_slot(int on, int from) const {
        return e(on) + 3 * e_cap + (2 + static_cast<size_t>(from)) * r_cap;
    }
    long long* fl(int r) const { return r == rank ? flags : peer_flags[r]; }
};

// The transport every call uses (process-wide; all ranks must agree).
int transport();
int set_transport(int mode);

// Collective over `comm`: all ranks call it at the start of a ring call with
// the byte counts they need.  Checks that every rank uses the same transport
// (DIMENSION_MISMATCH otherwise) and, for the copy-engine transport, finds or
// (re)builds the context; *ctx is nullptr when the call must use NCCL (the
// transport is NCCL, or the IPC set-up failed on some rank).  Synchronises `cs`.
cuflash::FlashAttentionError peer_acquire(ncclComm_t comm, int rank, int world, size_t e_bytes,
                                          size_t r_bytes, cudaStream_t cs, PeerCtx** ctx);

// Drops this process's context of `comm` (after a device synchronisation).
void peer_release(ncclComm_t comm);

// Stream operations.  wait_geq waits until *flag >= target (a peer's or this
// rank's flag); wait_all_geq until flags[i] >= target for every i < n except
// `skip`; signal stores `value` into *flag.  Each is one one-thread kernel.
bool wait_geq(const long long* flag, long long target, cudaStream_t st);
bool wait_all_geq(const long long* flags, int n, int skip, long long target, cudaStream_t st);
bool signal(long long* flag, long long value, cudaStream_t st);
// Signals value into flag_of(peer)[index] for every peer but `self` (one kernel).
bool signal_peers(const PeerCtx& ctx, int index, long long value, cudaStream_t st);

// out = convert(own + sum of R[w], w != rank) for `n` fp32 values (the dK/dV
// of this rank's chunks, all contributions added).
template <typename T>
bool sum_contributions(const PeerCtx& ctx, const float* own, T* out_k, T* out_v, long long elems,
                       cudaStream_t st);

// Test switch (CUFLASH_CP_TEST_SKIP_EXPORT_SIGNAL=1, read once): this rank
// copies its export but never signals it, so the other ranks' waits for it
// run out; used to test the bounded waits without a fault.
bool test_skip_export_signal();

// With CUFLASH_CP_DEBUG=1 (read once), prints `what` and the last CUDA error
// to stderr; returns false so that it can end a failing chain of checks.
bool debug_fail(const char* what);

// Read-and-clear of the status a timed-out wait set.
int status_read_and_clear();
bool status_set();

}  // namespace cuflash_cp
