#pragma once

// Thin inline-PTX layer for the sm_100a features the kernels use:
// mbarriers (with bounded waits), TMA tensor loads, tcgen05 MMA / TMEM
// management and the shared-memory / instruction descriptors that tcgen05.mma
// consumes.  Encodings follow the PTX ISA description of tcgen05 matrix
// descriptors and instruction descriptors (bit positions are listed next to
// each field).  Nothing here issues a multicast load.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "tmem_access.cuh"

namespace cuflash {
namespace sm100 {

// Bounded waits: a wait that does not complete within this many nanoseconds
// of %globaltimer is abandoned; the kernel records an error code and tears
// down instead of spinning forever.
constexpr unsigned long long kWaitTimeoutNs = 4000000000ull;  // 4 s

// Status codes recorded by kernels in their device status word.
constexpr int kStatusOk = 0;
constexpr int kStatusWaitTimeout = 1;
constexpr int kStatusMisaligned = 2;

// Where the kernels of one family record a failure: `code` in device memory
// (read by every kernel of the family at entry, so work queued behind a
// failed launch is skipped) and, once the host has bound it, `host`, a
// host-mapped pinned word shared by all families that the host entry points
// read without synchronising (so the next call reports the failure).
struct StatusWord {
    int code;
    int pad;
    int* host;
};

__device__ __forceinline__ void record_status(StatusWord* st, int code) {
    atomicExch(&st->code, code);
    int* h = *reinterpret_cast<int* volatile*>(&st->host);
    if (h != nullptr) {
        *reinterpret_cast<volatile int*>(h) = code;
        __threadfence_system();
    }
}

// CTA-uniform entry check: true (for every thread) if an earlier kernel of
// the family recorded a failure; one barrier, before any other work.
__device__ __forceinline__ bool cta_skip(const StatusWord* st) {
    const int mine =
        threadIdx.x == 0 ? *reinterpret_cast<const volatile int*>(&st->code) : 0;
    return __syncthreads_or(mine != 0) != 0;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------ schedules

// Persistent kernels hand out work units round-robin: unit u = r * G + c
// goes to CTA c (G = gridDim.x) in round r.  When the units are items
// listed by decreasing cost, this returns the list position unit u takes if
// the rounds alternate direction ("snake"): the CTA that drew the heaviest
// item of one round draws the lightest of the next, which balances the CTAs'
// totals where few rounds leave no room for averaging.  The last, partial
// round covers exactly the remaining positions.
__device__ __forceinline__ int snake_position(int u, int num_units) {
    const int G = static_cast<int>(gridDim.x);
    const int r = u / G;
    const int c = u - r * G;
    const int rem = min(G, num_units - r * G);
    return r * G + ((r & 1) ? rem - 1 - c : c);
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false if
// the CTA-wide abort flag is (or becomes) set or the wait times out after
// limit_ns; in the latter case the flag is set and `status` records
// kStatusWaitTimeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          StatusWord* status,
                                          unsigned long long limit_ns = kWaitTimeoutNs) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(addr, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > limit_ns) {
            *abort_flag = 1;
            record_status(status, kStatusWaitTimeout);
            return false;
        }
    }
}

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled TMA load (no multicast) completing on `bar` with tx bytes.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// ---------------------------------------------------------------- tcgen05

// Allocates `ncols` TMEM columns (power of two >= 32); whole warp executes.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives on `bar` once every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (fp16/bf16 in, fp32 acc).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc), kind::f16.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::tf32 (fp32 storage, tf32 math).
__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc), kind::tf32.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// ------------------------------------------------------------ descriptors

// Swizzle modes of the tcgen05 shared-memory matrix descriptor (bits 61-63).
constexpr uint32_t kLayoutSw128 = 2;
constexpr uint32_t kLayoutSw64 = 4;
constexpr uint32_t kLayoutSw32 = 6;

// Shared-memory matrix descriptor:
//   bits  0-13 start address >> 4
//   bits 16-29 leading-dimension byte offset >> 4
//   bits 32-45 stride-dimension byte offset >> 4
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 49-51 base offset (0: swizzle atoms are 1024-byte aligned)
//   bit  52    LBO mode (0)
//   bits 61-63 swizzle mode
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                                   uint32_t layout) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(layout & 0x7u) << 61;
    return d;
}

// Instruction descriptor for kind::f16 / kind::tf32 with fp32 accumulation:
//   bits  4-5  D format (1 = f32)
//   bits  7-9  A format (0 = f16, 1 = bf16, 2 = tf32)
//   bits 10-12 B format
//   bit  15    A major (0 = K-major, 1 = MN-major)
//   bit  16    B major
//   bits 17-22 N >> 3
//   bits 24-28 M >> 4
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_format, int M, int N, bool a_mn,
                                                  bool b_mn) {
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((a_mn ? 1u : 0u) << 15) |
           ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

constexpr uint32_t kFmtF16 = 0;
constexpr uint32_t kFmtBF16 = 1;
constexpr uint32_t kFmtTF32 = 2;

// --------------------------------------------------------------- math

// Per-warpgroup register re-allocation (every warp of the warpgroup executes
// the same instruction).  inc must request more than the current count and
// dec less; the increases of all warpgroups must fit in what the launch
// granted the block (threads x registers per thread at launch).
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Packed fp32 pair arithmetic (two lanes of work per instruction).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// 2^x for a pair of values on the FMA pipe (relieves the MUFU unit, which
// evaluates one exponential per lane every 8 cycles per SM sub-partition).
// Range reduction x = n + f with n = round(x) (the 1.5*2^23 addition rounds
// to nearest), f in [-1/2, 1/2]; 2^f by a degree-3 polynomial fitted here by
// iteratively reweighted least squares on Chebyshev nodes (max relative
// error 7.6e-5, below the 2^-9 / 2^-11 rounding of bf16 / fp16 P); 2^n is
// added to the exponent field.  Inputs are clamped to >= -125 so the
// exponent never underflows the field (results there are ~1e-38, i.e. zero
// for every consumer).
__device__ __forceinline__ float2 exp2_poly2(float x0, float x1) {
    const uint64_t xv = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
    const uint64_t kMagic = f2_pack(12582912.f, 12582912.f);  // 1.5 * 2^23
    const uint64_t kNegMagic = f2_pack(-12582912.f, -12582912.f);
    const uint64_t kMinusOne = f2_pack(-1.f, -1.f);
    const uint64_t t = f2_add(xv, kMagic);
    const uint64_t n = f2_add(t, kNegMagic);
    const uint64_t f = f2_fma(n, kMinusOne, xv);
    uint64_t q = f2_fma(f, f2_pack(0.05518639460f, 0.05518639460f),
                        f2_pack(0.24261234700f, 0.24261234700f));
    q = f2_fma(q, f, f2_pack(0.69325828552f, 0.69325828552f));
    q = f2_fma(q, f, f2_pack(0.99992793798f, 0.99992793798f));
    const float2 qf = f2_unpack(q);
    const float2 tf = f2_unpack(t);
    return make_float2(__int_as_float(__float_as_int(qf.x) + (__float_as_int(tf.x) << 23)),
                       __int_as_float(__float_as_int(qf.y) + (__float_as_int(tf.y) << 23)));
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ------------------------------------------------------------- 3xTF32
// A kind::tf32 MMA reads the upper 19 bits of each fp32 operand word, so a
// raw fp32 tile is its own "hi" part and lo = x - hi is exact in fp32; the
// product a*b is carried as hi(a)hi(b) + hi(a)lo(b) + lo(a)hi(b).

__device__ __forceinline__ float tf32_lo(float x) {
    return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// 4x4 block `blk` of an [R][C] fp32 tile (R, C multiples of 32) -> (row
// block i, column block j), for transposes between 128-byte swizzled tiles.
// Eight consecutive threads walk one diagonal of an 8x8 super-block, so the
// eight 16-byte chunks of a shared-memory phase fall in eight different
// chunk columns of the swizzle, for the reads of the [R][C] tile and for the
// writes of its [C][R] transpose alike (no bank conflicts).
template <int R>
__device__ __forceinline__ void diag_block(int blk, int& i, int& j) {
    const int k = blk & 7;
    const int g = blk >> 3;
    const int st = g >> 3, s = g & 7;
    i = (st % (R / 32)) * 8 + k;
    j = (st / (R / 32)) * 8 + ((k + s) & 7);
}

// fp32 K-major operand stored as 128-byte swizzled column blocks of 32
// elements (cb_bytes apart); descriptor of k-step kk (8 elements = 32 bytes).
__device__ __forceinline__ uint64_t f32_kdesc(uint32_t base, int kk, int cb_bytes) {
    const uint32_t byte = static_cast<uint32_t>(kk) * 32u;
    return make_smem_desc(base + (byte >> 7) * cb_bytes + (byte & 127u), 16, 1024, kLayoutSw128);
}

}  // namespace sm100
}  // namespace cuflash
