// Copy-engine transport of the context-parallel attention: contexts (IPC
// exports and mappings per communicator), the flag kernels and the final sum
// of the dK/dV contributions.  The protocol is described in peer_ring.h.

#include "peer_ring.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <random>
#include <vector>

namespace cuflash_cp {

using cuflash::FlashAttentionError;

namespace {

constexpr int kMaxRanks = 256;

// ------------------------------------------------------------------ options

std::once_flag g_opt_once;
std::atomic<int> g_transport{kTransportPeer};
unsigned long long g_wait_limit_ns = 60ull * 1000000000ull;
bool g_skip_export_signal = false;  // test switch: never signal this rank's export
bool g_debug = false;

void read_env() {
    std::call_once(g_opt_once, [] {
        const char* t = std::getenv("CUFLASH_CP_TRANSPORT");
        if (t != nullptr && std::strcmp(t, "nccl") == 0) g_transport.store(kTransportNccl);
        const char* w = std::getenv("CUFLASH_CP_WAIT_LIMIT_MS");
        if (w != nullptr) {
            const long long ms = std::atoll(w);
            if (ms > 0) g_wait_limit_ns = static_cast<unsigned long long>(ms) * 1000000ull;
        }
        const char* k = std::getenv("CUFLASH_CP_TEST_SKIP_EXPORT_SIGNAL");
        g_skip_export_signal = k != nullptr && std::atoi(k) == 1;
        const char* d = std::getenv("CUFLASH_CP_DEBUG");
        g_debug = d != nullptr && std::atoi(d) == 1;
    });
}

// ------------------------------------------------------------------- status

int* g_status_host = nullptr;  // host-mapped, one word for the process
int* g_status_dev = nullptr;
std::mutex g_status_mu;

int* status_dev() {
    std::lock_guard<std::mutex> lock(g_status_mu);
    if (g_status_host == nullptr) {
        int* h = nullptr;
        if (cudaHostAlloc(reinterpret_cast<void**>(&h), sizeof(int),
                          cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess)
            return nullptr;
        *h = 0;
        int* d = nullptr;
        if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&d), h, 0) != cudaSuccess) {
            cudaFreeHost(h);
            return nullptr;
        }
        g_status_host = h;
        g_status_dev = d;
    }
    return g_status_dev;
}

// ------------------------------------------------------------------ kernels

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ long long ld_acquire_sys(const long long* p) {
    long long v;
    asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(long long* p, long long v) {
    asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Waits until flags[i] >= target for i < n, i != skip; gives up after
// limit_ns in total, records the failure in *status and returns.
__global__ void wait_kernel(const long long* flags, int n, int skip, long long target,
                            int* status, unsigned long long limit_ns) {
    const unsigned long long t0 = gtimer();
    for (int i = 0; i < n; ++i) {
        if (i == skip) continue;
        while (ld_acquire_sys(flags + i) < target) {
            if (gtimer() - t0 > limit_ns) {
                *reinterpret_cast<volatile int*>(status) = 1;
                __threadfence_system();
                return;
            }
            __nanosleep(256);
        }
    }
}

__global__ void signal_kernel(long long* flag, long long value) {
    __threadfence_system();
    st_release_sys(flag, value);
}

struct PeerFlagPtrs {
    long long* p[kMaxRanks];
};

__global__ void signal_peers_kernel(PeerFlagPtrs ptrs, int world, int self, int index,
                                    long long value) {
    __threadfence_system();
    for (int r = 0; r < world; ++r)
        if (r != self) st_release_sys(ptrs.p[r] + index, value);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<half>(float a, float b) {
    const half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// out = own + sum over w != self of R[w], rounded to T; the 2*elems values
// are dK (first elems) then dV.
template <typename T>
__global__ void __launch_bounds__(256)
    sum_convert_kernel(const float* __restrict__ own, const char* __restrict__ rbase,
                       size_t rstride, int world, int self, T* __restrict__ out_k,
                       T* __restrict__ out_v, long long elems) {
    const long long n4 = 2 * elems / 4;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += stride) {
        float4 a = reinterpret_cast<const float4*>(own)[i];
        for (int w = 0; w < world; ++w) {
            if (w == self) continue;
            const float4 b =
                reinterpret_cast<const float4*>(rbase + static_cast<size_t>(w) * rstride)[i];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        const long long e = 4 * i;
        T* out = e < elems ? out_k + e : out_v + (e - elems);
        uint2 o;
        o.x = pack2<T>(a.x, a.y);
        o.y = pack2<T>(a.z, a.w);
        *reinterpret_cast<uint2*>(out) = o;
    }
}

// ----------------------------------------------------------------- contexts

std::mutex g_ctx_mu;
std::vector<PeerCtx*> g_ctxs;

PeerCtx* find_ctx(ncclComm_t comm, int dev) {
    for (PeerCtx* c : g_ctxs)
        if (c->comm == comm && c->dev == dev) return c;
    return nullptr;
}

void destroy_ctx(PeerCtx* c) {
    if (c == nullptr) return;
    cudaDeviceSynchronize();
    for (int r = 0; r < c->world && r < kMaxRanks; ++r) {
        if (c->peer_mem[r] != nullptr) cudaIpcCloseMemHandle(c->peer_mem[r]);
        if (c->peer_flags[r] != nullptr) cudaIpcCloseMemHandle(c->peer_flags[r]);
    }
    if (c->mem != nullptr) cudaFree(c->mem);
    if (c->flags != nullptr) cudaFree(c->flags);
    if (c->last_use != nullptr) cudaEventDestroy(c->last_use);
    delete c;
}

void drop_ctx(ncclComm_t comm, int dev) {
    for (size_t i = 0; i < g_ctxs.size(); ++i)
        if (g_ctxs[i]->comm == comm && g_ctxs[i]->dev == dev) {
            destroy_ctx(g_ctxs[i]);
            g_ctxs.erase(g_ctxs.begin() + static_cast<long>(i));
            return;
        }
}

// Per-device scratch for the small collectives: 64 KB of device memory (the
// allgather of IPC handles needs 128 bytes per rank) and a pinned host copy.
struct Scratch {
    char* dev = nullptr;
    char* host = nullptr;
};
Scratch g_scratch[64];

bool scratch(int dev, Scratch** out) {
    if (dev < 0 || dev >= 64) return false;
    Scratch& s = g_scratch[dev];
    if (s.dev == nullptr) {
        if (cudaMalloc(reinterpret_cast<void**>(&s.dev), 65536) != cudaSuccess) return false;
        if (cudaMallocHost(reinterpret_cast<void**>(&s.host), 65536) != cudaSuccess) {
            cudaFree(s.dev);
            s.dev = nullptr;
            return false;
        }
    }
    *out = &s;
    return true;
}

// In-place max all-reduce of n int64 values through the scratch buffers.
bool allreduce_max(long long* v, int n, ncclComm_t comm, Scratch* s, cudaStream_t cs) {
    std::memcpy(s->host, v, n * sizeof(long long));
    if (cudaMemcpyAsync(s->dev, s->host, n * sizeof(long long), cudaMemcpyHostToDevice, cs) !=
        cudaSuccess)
        return false;
    if (ncclAllReduce(s->dev, s->dev, n, ncclInt64, ncclMax, comm, cs) != ncclSuccess) return false;
    if (cudaMemcpyAsync(s->host, s->dev, n * sizeof(long long), cudaMemcpyDeviceToHost, cs) !=
        cudaSuccess)
        return false;
    if (cudaStreamSynchronize(cs) != cudaSuccess) return false;
    std::memcpy(v, s->host, n * sizeof(long long));
    return true;
}

// Collective build of a context; returns it with id -1 (and no memory) when
// any rank failed, so that every rank falls back to NCCL alike.
PeerCtx* build_ctx(ncclComm_t comm, int dev, int rank, int world, size_t e_cap, size_t r_cap,
                   Scratch* s, cudaStream_t cs) {
    PeerCtx* c = new PeerCtx();
    c->comm = comm;
    c->dev = dev;
    c->rank = rank;
    c->world = world;
    c->e_cap = e_cap;
    c->r_cap = r_cap;
    const size_t nflags = 2 + 3 * static_cast<size_t>(world);
    bool ok = cudaMalloc(reinterpret_cast<void**>(&c->mem), PeerCtx::bytes(e_cap, r_cap, world)) ==
              cudaSuccess;
    ok = ok && cudaMalloc(reinterpret_cast<void**>(&c->flags), nflags * sizeof(long long)) ==
                   cudaSuccess;
    ok = ok && cudaMemset(c->flags, 0, nflags * sizeof(long long)) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&c->last_use, cudaEventDisableTiming) == cudaSuccess;
    cudaIpcMemHandle_t hm{}, hf{};
    ok = ok && cudaIpcGetMemHandle(&hm, c->mem) == cudaSuccess &&
         cudaIpcGetMemHandle(&hf, c->flags) == cudaSuccess;
    if (!ok) {
        debug_fail("context allocation / cudaIpcGetMemHandle");
        cudaGetLastError();
    }
    // allgather of the handles: 128 bytes per rank (zeros where this rank failed)
    char* mine = s->host + static_cast<size_t>(rank) * 128;
    std::memset(mine, 0, 128);
    if (ok) {
        std::memcpy(mine, &hm, sizeof(hm));
        std::memcpy(mine + 64, &hf, sizeof(hf));
    }
    bool coll = cudaMemcpyAsync(s->dev + static_cast<size_t>(rank) * 128, mine, 128,
                                cudaMemcpyHostToDevice, cs) == cudaSuccess;
    coll = coll && ncclAllGather(s->dev + static_cast<size_t>(rank) * 128, s->dev, 128, ncclUint8,
                                 comm, cs) == ncclSuccess;
    coll = coll && cudaMemcpyAsync(s->host, s->dev, static_cast<size_t>(world) * 128,
                                   cudaMemcpyDeviceToHost, cs) == cudaSuccess;
    coll = coll && cudaStreamSynchronize(cs) == cudaSuccess;
    ok = ok && coll;
    for (int r = 0; ok && r < world; ++r) {
        if (r == rank) continue;
        cudaIpcMemHandle_t pm, pf;
        std::memcpy(&pm, s->host + static_cast<size_t>(r) * 128, sizeof(pm));
        std::memcpy(&pf, s->host + static_cast<size_t>(r) * 128 + 64, sizeof(pf));
        void* a = nullptr;
        void* b = nullptr;
        ok = cudaIpcOpenMemHandle(&a, pm, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        if (ok) c->peer_mem[r] = static_cast<char*>(a);
        ok = ok && cudaIpcOpenMemHandle(&b, pf, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        if (ok) c->peer_flags[r] = static_cast<long long*>(b);
        if (!ok) {
            debug_fail("cudaIpcOpenMemHandle");
            cudaGetLastError();
        }
    }
    // agree on success and on the id (rank 0's)
    long long id0 = 0;
    if (rank == 0) {
        std::random_device rd;
        id0 = (static_cast<long long>(rd()) << 31 ^ static_cast<long long>(rd()) ^
               std::chrono::steady_clock::now().time_since_epoch().count()) &
              0x3fffffffffffffffLL;
        if (id0 <= 0) id0 = 1;
    }
    long long v[2] = {id0, ok ? 0 : 1};
    const bool agreed = coll && allreduce_max(v, 2, comm, s, cs);
    if (!agreed || v[1] != 0) {
        // some rank failed: keep a marker context so that every rank uses NCCL
        PeerCtx* m = new PeerCtx();
        m->comm = comm;
        m->dev = dev;
        m->rank = rank;
        m->world = world;
        m->e_cap = e_cap;
        m->r_cap = r_cap;
        m->id = -1;
        destroy_ctx(c);
        return m;
    }
    c->id = v[0];
    return c;
}

}  // namespace

bool debug_fail(const char* what) {
    read_env();
    if (g_debug) {
        int dev = -1;
        cudaGetDevice(&dev);
        std::fprintf(stderr, "cuflash_cp (device %d): %s failed: %s\n", dev, what,
                     cudaGetErrorString(cudaPeekAtLastError()));
    }
    return false;
}

bool test_skip_export_signal() {
    read_env();
    return g_skip_export_signal;
}

int transport() {
    read_env();
    return g_transport.load();
}

int set_transport(int mode) {
    read_env();
    if (mode != kTransportPeer && mode != kTransportNccl) return -1;
    g_transport.store(mode);
    return 0;
}

FlashAttentionError peer_acquire(ncclComm_t comm, int rank, int world, size_t e_bytes,
                                 size_t r_bytes, cudaStream_t cs, PeerCtx** out) {
    *out = nullptr;
    read_env();
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || world > kMaxRanks)
        return FlashAttentionError::CUDA_ERROR;
    if (status_dev() == nullptr) return FlashAttentionError::CUDA_ERROR;
    std::lock_guard<std::mutex> lock(g_ctx_mu);
    Scratch* s = nullptr;
    if (!scratch(dev, &s)) return FlashAttentionError::CUDA_ERROR;
    const int mode = transport();
    PeerCtx* c = find_ctx(comm, dev);
    const bool fits = c != nullptr && c->rank == rank && c->world == world && c->e_cap >= e_bytes &&
                      c->r_cap >= r_bytes;
    const long long id = c != nullptr ? c->id : 0;
    // max over ranks of: id, -id (so min id), the byte counts, the transport
    // and minus it, whether this rank's context is missing or too small, and
    // whether a wait of this rank gave up (sticky until read)
    const bool failed = g_status_host != nullptr && *reinterpret_cast<volatile int*>(g_status_host);
    long long all[8] = {id,   -id,   static_cast<long long>(e_bytes), static_cast<long long>(r_bytes),
                        mode, -mode, fits ? 0 : 1,                    failed ? 1 : 0};
    if (!allreduce_max(all, 8, comm, s, cs)) {
        debug_fail("per-call all-reduce");
        return FlashAttentionError::CUDA_ERROR;
    }
    if (all[4] != -all[5]) return FlashAttentionError::DIMENSION_MISMATCH;  // transports differ
    if (all[7] != 0) {  // on every rank alike
        debug_fail("a wait for another rank gave up earlier (sticky status)");
        return FlashAttentionError::CUDA_ERROR;
    }
    if (mode == kTransportNccl) return FlashAttentionError::SUCCESS;
    const bool same = all[0] == -all[1] && all[0] != 0;
    if (!same || all[6] != 0) {
        // (re)build on every rank, large enough for every rank's request.
        // Peers may still be writing into this rank's old flags (the end of a
        // backward signals them on the caller's stream): every rank drains
        // its device, then a barrier, before any rank frees its old context.
        long long barrier[1] = {0};
        if (cudaDeviceSynchronize() != cudaSuccess || !allreduce_max(barrier, 1, comm, s, cs)) {
            debug_fail("context rebuild barrier");
            return FlashAttentionError::CUDA_ERROR;
        }
        if (c != nullptr) drop_ctx(comm, dev);
        const size_t e_cap = static_cast<size_t>(all[2]);
        const size_t r_cap = static_cast<size_t>(all[3]);
        c = build_ctx(comm, dev, rank, world, e_cap, r_cap, s, cs);
        g_ctxs.push_back(c);
    }
    if (c->id < 0) return FlashAttentionError::SUCCESS;  // IPC unavailable: NCCL
    *out = c;
    return FlashAttentionError::SUCCESS;
}

void peer_release(ncclComm_t comm) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return;
    std::lock_guard<std::mutex> lock(g_ctx_mu);
    drop_ctx(comm, dev);
}

bool wait_geq(const long long* flag, long long target, cudaStream_t st) {
    return wait_all_geq(flag, 1, -1, target, st);
}

bool wait_all_geq(const long long* flags, int n, int skip, long long target, cudaStream_t st) {
    if (target <= 0) return true;  // flags start at 0
    int* sd = status_dev();
    if (sd == nullptr) return false;
    wait_kernel<<<1, 1, 0, st>>>(flags, n, skip, target, sd, g_wait_limit_ns);
    return cudaGetLastError() == cudaSuccess;
}

bool signal(long long* flag, long long value, cudaStream_t st) {
    signal_kernel<<<1, 1, 0, st>>>(flag, value);
    return cudaGetLastError() == cudaSuccess;
}

bool signal_peers(const PeerCtx& ctx, int index, long long value, cudaStream_t st) {
    PeerFlagPtrs p{};
    for (int r = 0; r < ctx.world; ++r) p.p[r] = ctx.fl(r);
    signal_peers_kernel<<<1, 1, 0, st>>>(p, ctx.world, ctx.rank, index, value);
    return cudaGetLastError() == cudaSuccess;
}

template <typename T>
bool sum_contributions(const PeerCtx& ctx, const float* own, T* out_k, T* out_v, long long elems,
                       cudaStream_t st) {
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long n4 = 2 * elems / 4;
    long long blocks = (n4 + 255) / 256;
    if (blocks > 8LL * sms) blocks = 8LL * sms;
    if (blocks < 1) blocks = 1;
    sum_convert_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        own, ctx.r_slot(ctx.rank, 0), ctx.r_cap, ctx.world, ctx.rank, out_k, out_v, elems);
    return cudaGetLastError() == cudaSuccess;
}

template bool sum_contributions<__nv_bfloat16>(const PeerCtx&, const float*, __nv_bfloat16*,
                                               __nv_bfloat16*, long long, cudaStream_t);
template bool sum_contributions<half>(const PeerCtx&, const float*, half*, half*, long long,
                                      cudaStream_t);

int status_read_and_clear() {
    std::lock_guard<std::mutex> lock(g_status_mu);
    if (g_status_host == nullptr) return 0;
    const int v = *reinterpret_cast<volatile int*>(g_status_host);
    if (v != 0) *reinterpret_cast<volatile int*>(g_status_host) = 0;
    return v;
}

bool status_set() {
    std::lock_guard<std::mutex> lock(g_status_mu);
    return g_status_host != nullptr && *reinterpret_cast<volatile int*>(g_status_host) != 0;
}

}  // namespace cuflash_cp
