// Host-side helpers shared by the launchers: tensor-map encoding through the
// driver entry point (no link-time dependency on libcuda), a per-device
// cache of kernel shared-memory attributes and of the SM count.

#include <cudaTypedefs.h>

#include <atomic>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

}  // namespace

bool encode_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                    uint64_t inner, uint64_t rows, uint64_t outer, uint32_t box_inner,
                    uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
    cuuint64_t dims[3] = {inner, rows, outer};
    cuuint64_t strides[2] = {inner * static_cast<uint64_t>(elem_bytes),
                             inner * rows * static_cast<uint64_t>(elem_bytes)};
    cuuint32_t box[3] = {box_inner, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool encode_tmap_3d_strided(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                            const uint64_t dims[3], const uint64_t stride_bytes[2],
                            const uint32_t box[3], CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
    cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    cuuint64_t st[2] = {stride_bytes[0], stride_bytes[1]};
    cuuint32_t bx[3] = {box[0], box[1], box[2]};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dtype, 3, const_cast<void*>(base), d, st, bx, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool ensure_smem_attr(const void* kernel, int bytes) {
    // (device, kernel, bytes) already configured; a plain table keeps the
    // library from exporting standard-container template instances.
    struct Entry {
        int dev;
        int bytes;
        const void* kernel;
    };
    constexpr int kCap = 512;
    static std::mutex mu;
    static Entry done[kCap];
    static int n_done = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n_done; ++i)
        if (done[i].dev == dev && done[i].kernel == kernel && done[i].bytes >= bytes) return true;
    int optin = 0;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
        cudaSuccess)
        return false;
    if (bytes > optin) return false;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
        cudaSuccess)
        return false;
    if (n_done < kCap) done[n_done++] = Entry{dev, bytes, kernel};
    return true;
}

// CTAs per launch of the persistent kernels: waves x SM count (capped by the
// work).  One wave is the fastest when the kernel has the GPU to itself;
// more waves let the block scheduler rebalance when other kernels (NCCL
// transfers) hold SMs at launch time, at the price of more per-CTA setup.
// CUFLASH_RESERVE_SMS=n keeps n SMs out of every persistent launch, for
// callers that overlap collectives (a data-parallel gradient all-reduce)
// with attention kernels: NCCL's kernels need SMs the persistent CTAs would
// otherwise hold until the launch ends.
int persistent_grid(long long units, int waves) {
    const int sms = current_sm_count();
    int reserve = env_int("CUFLASH_RESERVE_SMS", 0);
    if (reserve >= sms) reserve = sms - 1;
    const long long cap = static_cast<long long>(sms - reserve) * (waves > 0 ? waves : 1);
    return static_cast<int>(units < cap ? units : cap);
}

namespace {

// Process-wide options.  Each starts from its environment variable, read
// once on first use (so no launch calls getenv, which is not safe against a
// concurrent setenv in another thread), and can be changed at any time
// through cuflash_set_option.  -1 = not set (the call site's default).
struct Option {
    const char* name;
    std::atomic<int> value;
};
Option g_options[] = {
    {"CUFLASH_RESERVE_SMS", {-1}},       // SMs left out of every persistent launch
    {"CUFLASH_FWD_WAVES", {-1}},         // persistent forward grid, in waves of SMs
    {"CUFLASH_BWD_WAVES", {-1}},         // persistent backward grid
    {"CUFLASH_CP_WAVES", {-1}},          // context-parallel forward step grid
    {"CUFLASH_DECODE_GQA_TC", {-1}},     // 0 selects the SIMT grouped-query decode
    {"CUFLASH_FAULT_WORKSPACE_OOM", {-1}},  // 1 fails every workspace request (tests)
    // tests of the bounded waits (fp16/bf16 forward only): wait limit in ms
    // (unset: 4 s), and 1 = CTA 0 leaves out its first K load
    {"CUFLASH_TEST_WAIT_LIMIT_MS", {-1}},
    {"CUFLASH_TEST_SKIP_K_LOAD", {-1}},
};
constexpr int kNumOptions = sizeof(g_options) / sizeof(g_options[0]);

Option* find_option(const char* name) {
    static std::once_flag once;
    std::call_once(once, [] {
        for (Option& o : g_options) {
            const char* v = getenv(o.name);
            if (v == nullptr || *v == '\0') continue;
            const int n = atoi(v);
            if (n >= 0 && n <= 100000) o.value.store(n);
        }
    });
    for (int i = 0; i < kNumOptions; ++i)
        if (std::strcmp(g_options[i].name, name) == 0) return &g_options[i];
    return nullptr;
}

}  // namespace

int env_int(const char* name, int dflt) {
    Option* o = find_option(name);
    const int v = o != nullptr ? o->value.load(std::memory_order_relaxed) : -1;
    return v >= 0 ? v : dflt;
}

bool set_option(const char* name, int value) {
    Option* o = find_option(name);
    if (o == nullptr) return false;
    o->value.store(value < 0 ? -1 : value);
    return true;
}

int current_sm_count() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

FlashAttentionError workspace_alloc(void** ptr, size_t bytes, cudaStream_t stream) {
    *ptr = nullptr;
    if (env_int("CUFLASH_FAULT_WORKSPACE_OOM", 0) != 0) return FlashAttentionError::OUT_OF_MEMORY;
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
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
    cudaError_t err = cudaMallocFromPoolAsync(ptr, bytes, pool, stream);
    if (err != cudaSuccess) {
        cudaGetLastError();
        *ptr = nullptr;
        return err == cudaErrorMemoryAllocation ? FlashAttentionError::OUT_OF_MEMORY
                                                : FlashAttentionError::CUDA_ERROR;
    }
    return FlashAttentionError::SUCCESS;
}

cudaStream_t side_stream(int i) {
    constexpr int kMaxDev = 64;
    static std::mutex mu;
    static cudaStream_t streams[kMaxDev][kNumSideStreams] = {};
    int dev = 0;
    if (i < 0 || i >= kNumSideStreams || cudaGetDevice(&dev) != cudaSuccess || dev < 0 ||
        dev >= kMaxDev)
        return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (streams[dev][i] == nullptr) {
        cudaStream_t st = nullptr;
        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
        streams[dev][i] = st;
    }
    return streams[dev][i];
}

void workspace_free(void* ptr, cudaStream_t stream) {
    if (ptr != nullptr) cudaFreeAsync(ptr, stream);
}

namespace {

constexpr int kMaxStatusDevices = 64;

// The host-mapped status words, one per device (pinned, mapped into every
// device's address space), and their device addresses, the sources of the
// copies that bind each kernel family's StatusWord::host on that device.
struct HostStatus {
    int word[kMaxStatusDevices];
    int* dev_word[kMaxStatusDevices];
};
std::atomic<HostStatus*> g_host_status{nullptr};

HostStatus* host_status_block() {
    static std::mutex mu;
    HostStatus* b = g_host_status.load(std::memory_order_acquire);
    if (b != nullptr) return b;
    std::lock_guard<std::mutex> lock(mu);
    b = g_host_status.load(std::memory_order_relaxed);
    if (b != nullptr) return b;
    void* p = nullptr;
    if (cudaHostAlloc(&p, sizeof(HostStatus), cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    b = static_cast<HostStatus*>(p);
    for (int i = 0; i < kMaxStatusDevices; ++i) {
        b->word[i] = 0;
        void* d = nullptr;
        if (cudaHostGetDevicePointer(&d, &b->word[i], 0) != cudaSuccess) {
            cudaGetLastError();
            cudaFreeHost(p);
            return nullptr;
        }
        b->dev_word[i] = static_cast<int*>(d);
    }
    g_host_status.store(b, std::memory_order_release);
    return b;
}

}  // namespace

int host_status() {
    HostStatus* b = g_host_status.load(std::memory_order_acquire);
    if (b == nullptr) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxStatusDevices) return 0;
    return *reinterpret_cast<volatile int*>(&b->word[dev]);
}

bool bind_status_word(const void* symbol, cudaStream_t stream) {
    struct Entry {
        const void* symbol;
        int dev;
    };
    constexpr int kCap = 8 * 64;
    static std::mutex mu;
    static Entry bound[kCap];
    static std::atomic<int> n_bound{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxStatusDevices) return false;
    const int n = n_bound.load(std::memory_order_acquire);
    for (int i = 0; i < n; ++i)
        if (bound[i].symbol == symbol && bound[i].dev == dev) return true;
    std::lock_guard<std::mutex> lock(mu);
    const int m = n_bound.load(std::memory_order_relaxed);
    for (int i = n; i < m; ++i)
        if (bound[i].symbol == symbol && bound[i].dev == dev) return true;
    if (m >= kCap) return false;
    // not while the stream is being captured: the binding is a one-time copy,
    // not part of the caller's work (the next uncaptured launch binds)
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone)
        return false;
    HostStatus* b = host_status_block();
    if (b == nullptr) return false;
    if (cudaMemcpyToSymbolAsync(symbol, &b->dev_word[dev], sizeof(int*),
                                offsetof(sm100::StatusWord, host), cudaMemcpyHostToDevice,
                                stream) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    bound[m] = Entry{symbol, dev};
    n_bound.store(m + 1, std::memory_order_release);
    return true;
}

namespace {

// Event pairs recorded around the backward main kernel (profiling hook):
// slot k holds the k-th launch after cuflash_profile_main_kernels(n).
struct KernelProfile {
    std::mutex mu;
    cudaEvent_t* ev = nullptr;  // [2 * cap]
    int cap = 0;
    int next = 0;
    int dev = -1;
};
KernelProfile g_profile;

void profile_free_locked() {
    for (int i = 0; i < 2 * g_profile.cap; ++i)
        if (g_profile.ev[i] != nullptr) cudaEventDestroy(g_profile.ev[i]);
    delete[] g_profile.ev;
    g_profile.ev = nullptr;
    g_profile.cap = g_profile.next = 0;
    g_profile.dev = -1;
}

}  // namespace

int profile_main_kernels(int n) {
    std::lock_guard<std::mutex> lock(g_profile.mu);
    profile_free_locked();
    if (n <= 0) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    g_profile.ev = new cudaEvent_t[2 * n]();
    for (int i = 0; i < 2 * n; ++i)
        if (cudaEventCreate(&g_profile.ev[i]) != cudaSuccess) {
            profile_free_locked();
            return -1;
        }
    g_profile.cap = n;
    g_profile.dev = dev;
    return 0;
}

void profile_record(bool after, cudaStream_t stream) {
    std::lock_guard<std::mutex> lock(g_profile.mu);
    if (g_profile.cap == 0 || g_profile.next >= g_profile.cap) return;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != g_profile.dev) return;
    cudaEventRecord(g_profile.ev[2 * g_profile.next + (after ? 1 : 0)], stream);
    if (after) ++g_profile.next;
}

int profile_read_ms(float* ms, int max_n) {
    std::lock_guard<std::mutex> lock(g_profile.mu);
    const int n = g_profile.next < max_n ? g_profile.next : max_n;
    for (int k = 0; k < n; ++k) {
        if (cudaEventSynchronize(g_profile.ev[2 * k + 1]) != cudaSuccess ||
            cudaEventElapsedTime(&ms[k], g_profile.ev[2 * k], g_profile.ev[2 * k + 1]) !=
                cudaSuccess)
            return -1;
    }
    return n;
}

int read_and_clear_device_status() {
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    const int a = fwd_sm100_status();
    const int b = bwd_sm100_status();
    const int c = f32_sm100_status();
    const int d = dec_sm100_status();
    const int e = bwd_f32_sm100_status();
    if (a < 0 || b < 0 || c < 0 || d < 0 || e < 0) return -1;
    const int h = host_status();
    int dev = 0;
    HostStatus* blk = g_host_status.load(std::memory_order_acquire);
    if (blk != nullptr && cudaGetDevice(&dev) == cudaSuccess && dev >= 0 &&
        dev < kMaxStatusDevices)
        *reinterpret_cast<volatile int*>(&blk->word[dev]) = 0;
    for (const int v : {a, b, c, d, e, h})
        if (v != 0) return v;
    return 0;
}

}  // namespace detail
}  // namespace cuflash
