// Backward attention for fp16/bf16 on sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the reference's three backward kernels
//   compute_D_kernel                        backward_typed.cu:13-34
//   flash_attention_backward_dq_kernel      backward_typed.cu:37-143
//   flash_attention_backward_dkdv_kernel    backward_typed.cu:146-288
// with the same math (P = exp(scale q.k - L), dP = dO V^T,
// D_i = rowsum(dO_i * O_i), dS = P (dP - D), dV = P^T dO,
// dK = scale dS^T Q, dQ = scale dS K) but one pass over the score matrix:
// S and dP are computed once per (kv block, q block) pair instead of twice.
//
// Kernel 1 (preprocess): D_i and L_i*log2(e) into a padded workspace
// (+inf / 0 in the padding rows so padded queries get P = 0), and zeroes the
// fp32 dQ accumulator.
// Kernel 2 (main): one CTA per (128-row K/V block j, batch*head); K_j and V_j
// stay in shared memory while the CTA walks the query blocks i (all of them,
// or i >= j when causal):
//   warp 0      TMA producer: Q_i, dO_i (tiled, swizzled) and the 128 values
//               of L and D for block i (1-D bulk copies), 2-stage ring.
//   warp 1      tcgen05.mma issuer:
//                 S^T  = K_j Q_i^T    -> TMEM [0,128)
//                 dP^T = V_j dO_i^T   -> TMEM [128,256)
//                 dV  += P^T dO_i     (A = P^T from TMEM)   -> TMEM [256,256+D)
//                 dK  += dS^T Q_i     (A = dS^T from TMEM)  -> TMEM [384,384+D)
//                 dQ_i = dS K_j (or dQ_i^T = K_j^T dS^T)    -> TMEM [128,256)
//               in the order dV (as soon as P^T is stored), S^T_{i+1} (head
//               dim 128; otherwise after dQ_i), dK, dQ_i, then (once the drain
//               warps have read dQ_i) dP^T_{i+1}, so the next block's P phase
//               overlaps dK and dQ_i.
//   warps 4-11  two warpgroups, one thread per K/V row (TMEM lane) each,
//               splitting the 128 query columns in halves, in two phases:
//               P^T from S^T (stored back into TMEM as fp16/bf16, kept in
//               fp32 registers), which releases the dV product, then dS^T
//               from dP^T and P (into TMEM, and into shared memory for the dQ
//               product), overlapping dV; at the end one warpgroup stores
//               dV, the other dK.
//   warps 12-15 drain dQ_i from TMEM into the fp32 accumulator: with
//               head_dim 128 dQ is computed transposed and drained with
//               coalesced red.global.add.f32, otherwise through swizzled
//               shared-memory boxes and TMA reduce-add.
// Kernel 3 (convert): dQ = scale * dQ_acc in the output dtype.
//
// CTAs of one (batch, head) are adjacent in launch order, so the dQ
// accumulator tiles they reduce into stay resident in L2.

#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {

__device__ sm100::StatusWord g_bwd_status;

constexpr float kLog2eB = 1.4426950408889634f;
// With kBwdExp2EmuEvery = k > 0, one pair of exponentials in k is computed on
// the FMA pipe (exp2_poly2, relative error below 1e-4, far under the 16-bit
// rounding that P and dS receive) instead of the MUFU unit, which the
// pipelined softmax below saturates.  Measured on B200: k = 4 takes config 3
// from 4.11 to 3.89 ms (k = 2: 3.99, k = 8: 3.97).  Re-measured on the
// current kernel (main kernel, two alternating runs each): k = 4 3.03-3.06
// ms, off 2.99-3.03, k = 8 3.02-3.04, k = 2 3.08-3.14; MUFU no longer
// binds, and k = 4 stays.
#ifndef CUFLASH_BWD_EXP2_EMU_EVERY
#define CUFLASH_BWD_EXP2_EMU_EVERY 4
#endif
constexpr int kBwdExp2EmuEvery = CUFLASH_BWD_EXP2_EMU_EVERY;
// How dQ_i leaves TMEM for the fp32 accumulator:
//   0  dQ_i^T (TMEM lane = head_dim element), one red.global.add.f32 per
//      element from registers (head_dim 128 only: M = head_dim);
//   1  dQ_i row-major (TMEM lane = query), staged through swizzled
//      shared-memory boxes and added by the TMA unit;
//   2  dQ_i row-major, red.global.add.v4.f32 from registers (four
//      consecutive elements of a row per instruction).
#ifndef CUFLASH_BWD_DQ_MODE_128
#define CUFLASH_BWD_DQ_MODE_128 0
#endif
#ifndef CUFLASH_BWD_DQ_MODE_SMALL
#define CUFLASH_BWD_DQ_MODE_SMALL 1
#endif

template <int D>
struct BwdGeom {
    static constexpr int kRows = 128;
    static constexpr int kRowBytes = D * 2;
    static constexpr int kSwz = kRowBytes >= 128 ? 128 : kRowBytes;
    static constexpr int kCbElems = kSwz / 2;
    static constexpr int kNumCb = D / kCbElems;
    static constexpr int kCbBytes = kRows * kSwz;
    static constexpr int kTileBytes = kRows * kRowBytes;
    static constexpr uint32_t kLayout = kSwz == 128 ? sm100::kLayoutSw128 : sm100::kLayoutSw64;
    static constexpr int kStages = 2;
    static constexpr int kDsBytes = 128 * 256;  // 128 kv rows x 128 q (16-bit), SW128
    static constexpr int kOffK = 0;
    static constexpr int kOffV = kTileBytes;
    static constexpr int kOffDs = 2 * kTileBytes;
    static constexpr int kOffStage = kOffDs + kDsBytes;
    static constexpr int kStageBytes = 2 * kTileBytes + 1024;  // Q, dO, L (512 B), D (512 B)
    static constexpr int kOffBar = kOffStage + kStages * kStageBytes;
    static constexpr int kNumBars = 1 + 2 * kStages + 8;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16;
    static_assert(kStageBytes % 1024 == 0, "stage must keep 1024-byte alignment");
};

struct BwdParams {
    float* dq_acc;
    void* dK;
    void* dV;
    const float* l2p;  // -L * log2(e), padded to n_blk_q*128 per query head with -inf
    const float* dvp;  // -rowsum(dO*O), padded with 0
    int Nq;            // query length
    int Nk;            // key length
    int n_blk_q;
    int n_blk_k;
    long long q_off;   // global position of query 0 (keys start at 0); causal: key k visible
                       // to query q iff k <= q_off + q
    int hq;            // query heads per batch entry
    int group;         // query heads per K/V head
    int npairs;        // (n_blk_k + 1) / 2
    int paired;        // 1: a unit is a (heavy, light) pair of kv blocks; 0: one kv block
    int order;         // unpaired: 0 = head-major, 1 = by decreasing cost, snake rounds
    int num_units;     // B*Hkv * npairs, or B*Hkv * n_blk_k when not paired
    int causal;
    float scale_log2;
    float scale;
    // Context-parallel step (kernels instantiated with kCp): query tensors
    // hold query slots and K/V tensors K/V slots, [slot][B*H][chunk][D] each,
    // so query head q_slot * bh_slot + bh and K/V head kv_slot * bh_slot + bh.
    // The step's (query slot, K/V slot) pairs are grouped by K/V slot into
    // segments; an item is one 128-row block of one segment's K/V slot and
    // walks the visible query blocks of every pair of the segment.  dK / dV
    // of the step are added into fp32 accumulators [kv slot][B*H][chunk][D].
    float* dk_acc;
    float* dv_acc;
    int bh_slot;            // B*H
    int nkseg;              // segments (distinct K/V slots among the pairs)
    int seg_units;          // units per segment
    int kseg_slot[4];       // K/V slot of segment s
    int kseg_first[4];      // its pairs: [kseg_first, kseg_first + kseg_count)
    int kseg_count[4];
    int pair_q_slot[4];     // query slot of pair k (pairs sorted by segment)
    long long pair_rel[4];  // query offset - K/V offset of pair k (global positions)
};

// One work item = one 128-row K/V block j of one (b,h).  Unit u of the
// persistent schedule holds two items of the same (b,h): kv blocks j = k and
// j = n_blk-1-k.  Under a causal mask block j visits n_blk-j query blocks, so
// every unit costs n_blk+1 blocks and a round-robin of units over the CTAs is
// balanced; both items read the same Q, dO and dQ rows, which stay in L2.
// Non-causal problems, and problems with fewer units than SMs, use one item
// per unit instead.
struct BwdItem {
    int j;
    int bh;   // K/V head: batch * Hkv + kv head (context-parallel: kv_slot * bh_slot + bh)
    int seg;  // context-parallel segment
    int bhl;  // context-parallel: bh within the slot
};

// The query walk of an item: for each of the group's query heads, the query
// blocks i0..n_blk_q-1 that see any key of block j (all of them unless causal).
// Context-parallel items walk, pair after pair of their segment, the visible
// query blocks of each pair's query slot.
struct BwdWalk {
    int i0;  // first visible query block
    int ni;  // blocks per query head
    int n;   // group * ni (context-parallel: total over the segment's pairs)
};

// First query block with rel + 128 i + 127 >= 128 j (the first that sees any
// key of block j when query 0 sits at global position rel and key 0 at 0).
__device__ __forceinline__ int bwd_first_block(const BwdParams& p, int j, long long rel) {
    if (!p.causal) return 0;
    const long long num = 128LL * j - rel - 127;
    const long long i0 = num <= 0 ? 0 : (num + 127) / 128;
    return static_cast<int>(i0 < p.n_blk_q ? i0 : p.n_blk_q);
}

template <bool kCp>
__device__ __forceinline__ BwdWalk bwd_walk(const BwdParams& p, const BwdItem& itm) {
    BwdWalk w;
    if constexpr (kCp) {
        w.i0 = 0;
        w.ni = 0;
        w.n = 0;
        const int f = p.kseg_first[itm.seg], c = p.kseg_count[itm.seg];
        for (int k = 0; k < c; ++k) w.n += p.n_blk_q - bwd_first_block(p, itm.j, p.pair_rel[f + k]);
    } else {
        w.i0 = bwd_first_block(p, itm.j, p.q_off);
        w.ni = p.n_blk_q - w.i0;
        w.n = p.group * w.ni;
    }
    return w;
}

template <bool kCp>
__device__ __forceinline__ bool bwd_item(const BwdParams& p, int u, int w, BwdItem& it) {
    int v = u, base = 0;
    it.seg = 0;
    if constexpr (kCp) {
        it.seg = u / p.seg_units;
        v = u - it.seg * p.seg_units;
        base = p.kseg_slot[it.seg] * p.bh_slot;
    }
    if (!p.paired) {
        if (w == 1) return false;
        if (!kCp && p.order) {
            // all heads' kv blocks by decreasing cost (ascending j), snake rounds
            const int pos = sm100::snake_position(u, p.num_units);
            const int nbh = p.num_units / p.n_blk_k;
            it.j = pos / nbh;
            it.bhl = pos - it.j * nbh;
        } else {
            it.bhl = v / p.n_blk_k;
            it.j = v - it.bhl * p.n_blk_k;  // ascending j: heaviest first under a causal mask
        }
    } else {
        it.bhl = v / p.npairs;
        const int k = v - it.bhl * p.npairs;
        it.j = w == 0 ? k : p.n_blk_k - 1 - k;
        if (w == 1 && it.j == k) return false;  // middle block of an odd count
    }
    it.bh = base + it.bhl;
    // a context-parallel block that no query of the step sees adds nothing
    if constexpr (kCp) return bwd_walk<true>(p, it).n > 0;
    return true;
}

// Query head, query block and causal offset (global position of the block's
// query 0 minus that of key 0) of walk step `it`.
template <bool kCp>
__device__ __forceinline__ void bwd_step(const BwdParams& p, const BwdItem& itm, const BwdWalk& w,
                                         int it, int& bh_q, int& i, long long& rel) {
    bh_q = 0;
    i = 0;
    rel = 0;
    if constexpr (kCp) {
        const int f = p.kseg_first[itm.seg], c = p.kseg_count[itm.seg];
        int rest = it;
        for (int k = 0; k < c; ++k) {
            const long long r = p.pair_rel[f + k];
            const int i0 = bwd_first_block(p, itm.j, r);
            const int ni = p.n_blk_q - i0;
            if (rest < ni || k == c - 1) {
                i = i0 + rest;
                rel = r;
                bh_q = p.pair_q_slot[f + k] * p.bh_slot + itm.bhl;
                return;
            }
            rest -= ni;
        }
    } else {
        const int gq = w.ni > 0 ? it / w.ni : 0;
        i = w.i0 + (it - gq * w.ni);
        const int hkv = p.hq / p.group;
        bh_q = (itm.bh / hkv) * p.hq + (itm.bh % hkv) * p.group + gq;
        rel = p.q_off;
    }
}

template <int D>
__device__ __forceinline__ uint64_t bkmajor_desc(uint32_t tile_base, int kk) {
    using G = BwdGeom<D>;
    const uint32_t byte = static_cast<uint32_t>(kk) * 32u;
    const uint32_t addr = tile_base + (byte / G::kSwz) * G::kCbBytes + (byte % G::kSwz);
    return sm100::make_smem_desc(addr, 16, 8 * G::kSwz, G::kLayout);
}

template <int D>
__device__ __forceinline__ uint64_t bmnmajor_desc(uint32_t tile_base, int kk) {
    using G = BwdGeom<D>;
    const uint32_t addr = tile_base + static_cast<uint32_t>(kk) * 16u * G::kSwz;
    return sm100::make_smem_desc(addr, G::kCbBytes, 8 * G::kSwz, G::kLayout);
}

// Descriptor of k-step kk = descriptor of k-step 0 + these (start address
// field, 16-byte units; shared addresses stay below 2^18, so no carry).
template <int D>
__host__ __device__ constexpr uint32_t bk_delta(int kk) {
    using G = BwdGeom<D>;
    return ((static_cast<uint32_t>(kk) * 32u / G::kSwz) * G::kCbBytes +
            (static_cast<uint32_t>(kk) * 32u % G::kSwz)) >> 4;
}
template <int D>
__host__ __device__ constexpr uint32_t bmn_delta(int kk) {
    return (static_cast<uint32_t>(kk) * 16u * BwdGeom<D>::kSwz) >> 4;
}
__host__ __device__ constexpr uint32_t ds_delta(int kk) { return static_cast<uint32_t>(kk) * 128u; }

// Keeps a descriptor opaque to the optimiser, so that the per-k-step
// descriptors derived from it are not hoisted out of the loops into live
// registers of the (register-starved) MMA warp.
__device__ __forceinline__ uint64_t opaque(uint64_t d) {
    asm volatile("" : "+l"(d));
    return d;
}

// dS tile: [128 kv rows][128 q], two 64-column SW128 blocks; as the MN-major
// A operand of dQ = dS K (M = q, K = kv), k-step kk covers kv rows 16kk..
__device__ __forceinline__ uint64_t ds_desc(uint32_t ds_base, int kk) {
    return sm100::make_smem_desc(ds_base + static_cast<uint32_t>(kk) * 16u * 128u, 128 * 128, 1024,
                                 sm100::kLayoutSw128);
}

__device__ __forceinline__ bool bwarp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    // Every lane polls the barrier itself: all lanes observe the same phase,
    // timer and abort flag, so the warp stays converged without a shuffle.
    return sm100::mbar_wait(bar, parity, abort_flag, &g_bwd_status);
}

__device__ __forceinline__ void bdrain_wait(uint64_t* bar, uint32_t parity) {
    volatile int never = 0;
    sm100::mbar_wait(bar, parity, &never, &g_bwd_status);
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            sm100::smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(sm100::smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void red_add_f32(float* gptr, float v) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(gptr), "f"(v) : "memory");
}
// Element-wise add of four consecutive floats (16-byte aligned address).
__device__ __forceinline__ void red_add_v4_f32(float* gptr, uint32_t a, uint32_t b, uint32_t c,
                                               uint32_t d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(gptr),
                 "f"(__uint_as_float(a)), "f"(__uint_as_float(b)), "f"(__uint_as_float(c)),
                 "f"(__uint_as_float(d))
                 : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

// Element-wise add of a shared-memory box into global memory through the TMA
// unit (no multicast); completion is tracked with bulk async-groups.
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, uint32_t smem_src, int c0,
                                                  int c1, int c2) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_src), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- preprocess

// D/8 threads per query row, 16-byte loads of O and dO; writes -L*log2(e)
// and -rowsum(dO*O) (the negated forms feed the softmax's fused multiply-adds
// directly) and zeroes the row of the fp32 dQ accumulator.
template <typename T, int D>
__global__ void __launch_bounds__(256)
    bwd_preprocess_kernel(const T* __restrict__ O, const T* __restrict__ dO,
                          const float* __restrict__ L, float* __restrict__ nl2,
                          float* __restrict__ nd, float* __restrict__ dq_acc, int N, int N_pad,
                          long long rows_pad) {
    constexpr int kTpr = D / 8;  // threads per row: 16, 8 or 4 (groups never straddle a warp)
    const long long gt = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long r = gt / kTpr;
    const int part = static_cast<int>(gt - r * kTpr);
    const bool in_range = r < rows_pad;
    const long long bh = in_range ? r / N_pad : 0;
    const int q = in_range ? static_cast<int>(r - bh * N_pad) : 0;
    const bool real = in_range && q < N;
    const long long row = bh * N + q;
    float acc = 0.f;
    if (real) {
        const uint4 o = *reinterpret_cast<const uint4*>(O + row * D + part * 8);
        const uint4 g = *reinterpret_cast<const uint4*>(dO + row * D + part * 8);
        const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
        const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 of = DType<T>::unpack2(ow[e]);
            const float2 gf = DType<T>::unpack2(gw[e]);
            acc = fmaf(of.x, gf.x, acc);
            acc = fmaf(of.y, gf.y, acc);
        }
        float4* z = reinterpret_cast<float4*>(dq_acc + row * D + part * 8);
        z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
        z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int off = kTpr / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (in_range && part == 0) {
        nl2[r] = real ? -L[row] * kLog2eB : -INFINITY;
        nd[r] = -acc;
    }
}

template <typename T>
__global__ void __launch_bounds__(256)
    bwd_convert_dq_kernel(const float* __restrict__ acc, T* __restrict__ dQ, float scale,
                          long long n4) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += stride) {
        const float4 v = reinterpret_cast<const float4*>(acc)[i];
        uint2 o;
        o.x = DType<T>::pack2(v.x * scale, v.y * scale);
        o.y = DType<T>::pack2(v.z * scale, v.w * scale);
        reinterpret_cast<uint2*>(dQ)[i] = o;
    }
}

// The softmax of one (kv block, query block) pair for this thread's kv row r
// (TMEM lane), warpgroup h covering queries [64h, 64h+64), in two phases so
// that the dV product can start before dS exists:
//   bwd_softmax_p   P^T from S^T: p = exp2(scale*log2(e) * s - L*log2(e)),
//                   kept in fp32 registers and stored (16-bit) over S^T;
//   bwd_softmax_ds  dS^T = P^T (dP^T - D) from dP^T and the kept P, stored
//                   (16-bit) over dP^T and into shared memory for dQ.
// sL / sD hold -L*log2(e) and -rowsum(dO*O) of the warpgroup's queries.  Both
// work in 16-query sub-chunks with the next sub-chunk's columns loading while
// one is computed; the 16-bit results of sub-chunk k go to columns [8k, 8k+8)
// of the warpgroup's range, which hold queries already loaded.  kDiag masks
// the keys above the causal diagonal: query q of the block against kv row r
// is hidden iff q < r + delta, delta = 128 (j - i) - q_off.
template <typename T, bool kDiag>
__device__ __forceinline__ void bwd_softmax_p(uint32_t t_s, const float* sL, float c, int h, int r,
                                              int delta, float (&pf)[64]) {
    using namespace sm100;
    const uint64_t c2 = f2_pack(c, c);
    uint32_t sA[16], sB[16];
    tmem_ld_x16_nw(t_s, sA);
    tmem_wait_ld_x16(sA);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t(&sv)[16] = (k & 1) ? sB : sA;
        uint32_t(&sn)[16] = (k & 1) ? sA : sB;
        if (k + 1 < 4) tmem_ld_x16_nw(t_s + 16 * (k + 1), sn);
        uint32_t pp[8];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const float4 lq = reinterpret_cast<const float4*>(sL + 16 * k)[v];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int e = 2 * v + u;                 // pair index in the sub-chunk
                const int q0 = h * 64 + 16 * k + 2 * e;  // query within the block
                const uint64_t nl = u ? f2_pack(lq.z, lq.w) : f2_pack(lq.x, lq.y);
                const float2 xx = f2_unpack(f2_fma(
                    f2_pack(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), c2, nl));
                float p0, p1;
                if (kBwdExp2EmuEvery > 0 &&
                    (e % (kBwdExp2EmuEvery > 0 ? kBwdExp2EmuEvery : 1)) == kBwdExp2EmuEvery - 1) {
                    const float2 ex = exp2_poly2(xx.x, xx.y);  // FMA pipe
                    p0 = ex.x;
                    p1 = ex.y;
                } else {
                    p0 = ex2_approx(xx.x);  // MUFU
                    p1 = ex2_approx(xx.y);
                }
                if (kDiag) {  // query q0 (global q_off + 128 i + q0) vs key 128 j + r
                    if (q0 < r + delta) p0 = 0.f;
                    if (q0 + 1 < r + delta) p1 = 0.f;
                }
                pf[16 * k + 2 * e] = p0;
                pf[16 * k + 2 * e + 1] = p1;
                pp[e] = DType<T>::pack2(p0, p1);
            }
        }
        // P^T overwrites columns this thread has already read
        tmem_st_x8_nw(t_s + 8 * k, pp);
        if (k + 1 < 4) tmem_wait_ld_x16(sn);
    }
}

template <typename T>
__device__ __forceinline__ void bwd_softmax_ds(uint32_t t_dp, uint32_t sDs, const float* sD, int r,
                                               const float (&pf)[64]) {
    using namespace sm100;
    uint32_t dA[16], dB[16];
    tmem_ld_x16_nw(t_dp, dA);
    tmem_wait_ld_x16(dA);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t(&dv)[16] = (k & 1) ? dB : dA;
        uint32_t(&dn)[16] = (k & 1) ? dA : dB;
        if (k + 1 < 4) tmem_ld_x16_nw(t_dp + 16 * (k + 1), dn);
        uint32_t dd[8];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const float4 dq = reinterpret_cast<const float4*>(sD + 16 * k)[v];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int e = 2 * v + u;
                const uint64_t ndv = u ? f2_pack(dq.z, dq.w) : f2_pack(dq.x, dq.y);
                const float2 d = f2_unpack(f2_mul(
                    f2_pack(pf[16 * k + 2 * e], pf[16 * k + 2 * e + 1]),
                    f2_add(f2_pack(__uint_as_float(dv[2 * e]), __uint_as_float(dv[2 * e + 1])), ndv)));
                dd[e] = DType<T>::pack2(d.x, d.y);
            }
        }
        // dS^T overwrites columns this thread has already read
        tmem_st_x8_nw(t_dp + 8 * k, dd);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int chunk = 2 * k + q;
            st_shared_v4(sDs + ((chunk ^ (r & 7)) << 4), dd[4 * q], dd[4 * q + 1], dd[4 * q + 2],
                         dd[4 * q + 3]);
        }
        if (k + 1 < 4) tmem_wait_ld_x16(dn);
    }
}

// ---------------------------------------------------------------- main kernel

constexpr int kBwdThreads = 512;

template <typename T, int D, bool kCp>
__global__ void __launch_bounds__(kBwdThreads, 1)
    fa_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                  const __grid_constant__ CUtensorMap tmdQ, const BwdParams p) {
    using G = BwdGeom<D>;
    using namespace sm100;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // With head_dim 128 dQ is produced transposed (TMEM lane = head_dim
    // element), so a warp's reduction into the accumulator covers 32
    // consecutive floats of one query row: fully coalesced, no staging.
    constexpr int kDqMode = (D == 128) ? CUFLASH_BWD_DQ_MODE_128
                                       : (CUFLASH_BWD_DQ_MODE_SMALL == 0 ? 1 : CUFLASH_BWD_DQ_MODE_SMALL);
    constexpr bool kTransposedDq = (kDqMode == 0);

    if (sm100::cta_skip(&g_bwd_status)) return;
    const uint32_t sbase = smem_u32(smem_raw);
    if ((sbase & 1023u) != 0) {  // swizzled operands need 1024-byte alignment
        if (threadIdx.x == 0) sm100::record_status(&g_bwd_status, sm100::kStatusMisaligned);
        return;
    }
    uint8_t* sptr = smem_raw;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sptr + G::kOffBar);
    uint64_t* bar_kv = bars;  // K_j, V_j of the current item landed
    uint64_t* full = bars + 1;
    uint64_t* empty = full + G::kStages;
    uint64_t* bar_s = empty + G::kStages;  // S^T in TMEM
    uint64_t* bar_dp = bar_s + 1;          // dP^T in TMEM
    uint64_t* bar_p = bar_dp + 1;          // P^T stored (256 arrivals)
    uint64_t* bar_ds = bar_p + 1;          // dS^T stored in TMEM and shared memory (256)
    uint64_t* bar_dq = bar_ds + 1;
    uint64_t* bar_dqfree = bar_dq + 1;
    uint64_t* bar_acc = bar_dqfree + 1;  // all MMAs of the item retired (dV, dK final; K, V free)
    uint64_t* bar_done = bar_acc + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(bar_kv, 1);
        for (int s = 0; s < G::kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        mbar_init(bar_s, 1);
        mbar_init(bar_dp, 1);
        mbar_init(bar_p, 256);
        mbar_init(bar_ds, 256);
        mbar_init(bar_dq, 1);
        mbar_init(bar_dqfree, 128);
        mbar_init(bar_acc, 1);
        mbar_init(bar_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Every role walks the same static list of work items (bwd_item).  The
    // query-block counter g runs across items, so the stage ring and the
    // per-block barrier phases continue from one item to the next; bar_kv and
    // bar_acc complete once per item.
    //
    // TMEM columns: S^T [0,128), dP^T [128,256), dV [256,256+D), dK [384,384+D).
    // Softmax warpgroup h (h = 0, 1) owns query columns [64h, 64h+64): it
    // reads S^T / dP^T columns [64h, 64h+64) and writes P^T / dS^T (16-bit,
    // two per column) into columns [64h, 64h+32) of the same regions, so the
    // two warpgroups never touch each other's columns.  dQ (or dQ^T) is then
    // written by an MMA over the dP^T columns.
    //
    // Registers: launched with 128 per thread (512 x 128 = 65536).
    // warpgroup 0 (producer, MMA, 2 idle) -> 56, the drain -> 152, the two
    // softmax warpgroups -> 152: 128*56 + 128*152 + 256*152 = 65536.
    if (warp < 4) {
        setmaxnreg_dec<56>();
        if (warp == 0 && lane == 0) {
            // ------------------------------------------------ producer
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            prefetch_tmap(&tmdO);
            uint32_t g = 0;        // stage loads issued
            uint32_t items = 0;    // K/V loads issued
            bool ok = true;
            auto load_stage = [&](int bh, int i) {  // bh: query head
                const int s = g % G::kStages;
                if (g >= G::kStages &&
                    !mbar_wait(empty + s, ((g / G::kStages) & 1) ^ 1, abort_flag, &g_bwd_status))
                    return false;
                uint8_t* st = sptr + G::kOffStage + s * G::kStageBytes;
                const size_t lrow = static_cast<size_t>(bh) * p.n_blk_q * 128;
                mbar_arrive_expect_tx(full + s, 2 * G::kTileBytes + 1024);
                for (int cb = 0; cb < G::kNumCb; ++cb) {
                    tma_load_3d(st + cb * G::kCbBytes, &tmQ, full + s, cb * G::kCbElems, i * 128,
                                bh);
                    tma_load_3d(st + G::kTileBytes + cb * G::kCbBytes, &tmdO, full + s,
                                cb * G::kCbElems, i * 128, bh);
                }
                bulk_load(st + 2 * G::kTileBytes, p.l2p + lrow + i * 128, 512, full + s);
                bulk_load(st + 2 * G::kTileBytes + 512, p.dvp + lrow + i * 128, 512, full + s);
                ++g;
                return true;
            };
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                for (int w = 0; ok && w < 2; ++w) {
                    BwdItem itm;
                    if (!bwd_item<kCp>(p, u, w, itm)) continue;
                    const BwdWalk wk = bwd_walk<kCp>(p, itm);
                    const int n_it = wk.n;
                    auto load_step = [&](int it) {
                        int bh_q, i;
                        long long rel;
                        bwd_step<kCp>(p, itm, wk, it, bh_q, i, rel);
                        return load_stage(bh_q, i);
                    };
                    // The item's first stages only need free ring slots, so they go
                    // ahead of K_j, V_j, which wait for the previous item's MMAs
                    // (the first item loads K_j, V_j first).
                    const int pre = items == 0 ? 0 : min(n_it, G::kStages);
                    for (int it = 0; ok && it < pre; ++it) ok = load_step(it);
                    // K_j, V_j: the previous item's MMAs must be done with the buffers
                    if (ok && items > 0)
                        ok = mbar_wait(bar_acc, (items - 1) & 1, abort_flag, &g_bwd_status);
                    if (!ok) break;
                    mbar_arrive_expect_tx(bar_kv, 2 * G::kTileBytes);
                    for (int cb = 0; cb < G::kNumCb; ++cb) {
                        tma_load_3d(sptr + G::kOffK + cb * G::kCbBytes, &tmK, bar_kv,
                                    cb * G::kCbElems, itm.j * 128, itm.bh);
                        tma_load_3d(sptr + G::kOffV + cb * G::kCbBytes, &tmV, bar_kv,
                                    cb * G::kCbElems, itm.j * 128, itm.bh);
                    }
                    ++items;
                    for (int it = pre; ok && it < n_it; ++it) ok = load_step(it);
                }
            }
            // every issued load must land before the CTA can exit
            if (items > 0) bdrain_wait(bar_kv, (items - 1) & 1);
            for (uint32_t q = g > G::kStages ? g - G::kStages : 0; q < g; ++q)
                bdrain_wait(full + q % G::kStages, (q / G::kStages) & 1);
        } else if (warp == 1 && lane == 0) {
            // ------------------------------------------------ MMA issuer
            constexpr uint32_t kFmt = DType<T>::kMmaFmt;
            constexpr uint32_t idesc_ss = make_idesc(kFmt, 128, 128, false, false);
            constexpr uint32_t idesc_acc = make_idesc(kFmt, 128, D, false, true);
            constexpr uint32_t idesc_dq = make_idesc(kFmt, 128, D, true, true);
            constexpr uint32_t idesc_dqt = make_idesc(kFmt, 128, 128, true, true);
            const uint32_t sK = sbase + G::kOffK, sV = sbase + G::kOffV, sDs = sbase + G::kOffDs;
            // TMEM column of k-step kk (16 queries) of a P^T / dS^T operand
            auto acol = [](int kk) { return static_cast<uint32_t>(kk < 4 ? kk * 8 : 64 + (kk - 4) * 8); };
            auto stage_q = [&](int it) {
                return sbase + G::kOffStage + static_cast<uint32_t>(it % G::kStages) * G::kStageBytes;
            };
            // dP^T = V_j dO_i^T -> TMEM [128, 256)
            auto issue_dp = [&](uint32_t sdO) {
                const uint64_t a0 = opaque(bkmajor_desc<D>(sV, 0));
                const uint64_t b0 = opaque(bkmajor_desc<D>(sdO, 0));
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    mma_f16_ss(tmem + 128, a0 + bk_delta<D>(kk), b0 + bk_delta<D>(kk), idesc_ss,
                               kk > 0 ? 1u : 0u);
            };
            // S^T = K_j Q_i^T -> TMEM [0, 128)
            auto issue_s = [&](uint32_t sQ) {
                const uint64_t a0 = opaque(bkmajor_desc<D>(sK, 0));
                const uint64_t b0 = opaque(bkmajor_desc<D>(sQ, 0));
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    mma_f16_ss(tmem, a0 + bk_delta<D>(kk), b0 + bk_delta<D>(kk), idesc_ss,
                               kk > 0 ? 1u : 0u);
            };
            uint32_t g = 0;      // query blocks consumed
            uint32_t items = 0;  // items finished
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                for (int w = 0; ok && w < 2; ++w) {
                    BwdItem itm;
                    if (!bwd_item<kCp>(p, u, w, itm)) continue;
                    const int n_it = bwd_walk<kCp>(p, itm).n;
                    // K_j, V_j and the item's first query block
                    ok = mbar_wait(bar_kv, items & 1, abort_flag, &g_bwd_status) &&
                         mbar_wait(full + g % G::kStages, (g / G::kStages) & 1, abort_flag,
                                   &g_bwd_status);
                    if (!ok) break;
                    tc_fence_after();
                    // S^T columns: the previous item's P^T was read by its last
                    // dV product (issued earlier, so ordered before this one)
                    issue_s(stage_q(g));
                    tc_commit(bar_s);
                    // dP^T columns hold the previous block's dQ until drained
                    if (g > 0 && !mbar_wait(bar_dqfree, (g - 1) & 1, abort_flag, &g_bwd_status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_dp(stage_q(g) + G::kTileBytes);
                    tc_commit(bar_dp);
                    for (int it = 0; ok && it < n_it; ++it, ++g) {
                        const int s = g % G::kStages;
                        const uint32_t sQ = stage_q(g);
                        const uint32_t sdO = sQ + G::kTileBytes;
                        // dV += P^T dO_i as soon as P^T is stored (the softmax warps
                        // compute dS^T meanwhile)
                        if (!mbar_wait(bar_p, g & 1, abort_flag, &g_bwd_status)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        {
                            const uint64_t bo = opaque(bmnmajor_desc<D>(sdO, 0));
#pragma unroll
                            for (int kk = 0; kk < 8; ++kk)
                                mma_f16_ts(tmem + 256, tmem + acol(kk), bo + bmn_delta<D>(kk), idesc_acc,
                                           (it > 0 || kk > 0) ? 1u : 0u);
                        }
                        // head_dim 128: S^T_{i+1} right behind dV (the last reader of
                        // P^T in the S^T columns), so the next block's P phase runs
                        // while the tensor pipe does dK_i and dQ_i (config 3: 3.39 ->
                        // 3.27 ms).  Smaller head dims issue it after dQ_i: their
                        // shorter dK / dQ products leave little to overlap, and
                        // holding dQ_i back delays dP^T_{i+1} (head_dim 64: 2.53 ->
                        // 2.78 ms when issued early).
                        constexpr bool kEarlyS = (D == 128);
                        const bool more = it + 1 < n_it;
                        auto issue_next_s = [&]() {
                            if (!mbar_wait(full + (g + 1) % G::kStages, ((g + 1) / G::kStages) & 1,
                                           abort_flag, &g_bwd_status))
                                return false;
                            tc_fence_after();
                            issue_s(stage_q(g + 1));
                            tc_commit(bar_s);
                            return true;
                        };
                        if (kEarlyS && more) {
                            if (!issue_next_s()) {
                                ok = false;
                                break;
                            }
                        }
                        // dK += dS^T Q_i  (K dimension = 128 query rows)
                        if (!mbar_wait(bar_ds, g & 1, abort_flag, &g_bwd_status)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        {
                            const uint64_t bq = opaque(bmnmajor_desc<D>(sQ, 0));
#pragma unroll
                            for (int kk = 0; kk < 8; ++kk)
                                mma_f16_ts(tmem + 384, tmem + 128 + acol(kk), bq + bmn_delta<D>(kk),
                                           idesc_acc, (it > 0 || kk > 0) ? 1u : 0u);
                        }
                        tc_commit(empty + s);
                        // dQ_i goes into the dP^T columns, whose dS^T the dK product
                        // just read; the drain warps empty them before dP^T_{i+1}.
                        {
                            const uint64_t kt0 = opaque(bmnmajor_desc<D>(sK, 0));
                            const uint64_t ds0 = opaque(ds_desc(sDs, 0));
                            if constexpr (kTransposedDq) {
                                // dQ_i^T = K_j^T dS^T (M = head_dim lanes, N = 128 queries)
#pragma unroll
                                for (int kk = 0; kk < 8; ++kk)
                                    mma_f16_ss(tmem + 128, kt0 + bmn_delta<D>(kk), ds0 + ds_delta(kk),
                                               idesc_dqt, kk > 0 ? 1u : 0u);
                            } else {
                                // dQ_i = dS K_j (M = 128 query lanes, N = head_dim)
#pragma unroll
                                for (int kk = 0; kk < 8; ++kk)
                                    mma_f16_ss(tmem + 128, ds0 + ds_delta(kk), kt0 + bmn_delta<D>(kk),
                                               idesc_dq, kk > 0 ? 1u : 0u);
                            }
                        }
                        tc_commit(bar_dq);
                        if (more) {
                            if (!kEarlyS && !issue_next_s()) {
                                ok = false;
                                break;
                            }
                            // dP^T_{i+1} once the drain warps have read dQ_i
                            if (!mbar_wait(bar_dqfree, g & 1, abort_flag, &g_bwd_status)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            issue_dp(stage_q(g + 1) + G::kTileBytes);
                            tc_commit(bar_dp);
                        }
                    }
                    if (!ok) break;
                    tc_commit(bar_acc);
                    ++items;
                }
            }
            tc_commit(bar_done);
            volatile int never = 0;
            mbar_wait(bar_done, 0, &never, &g_bwd_status);
        }
        __syncwarp();
    } else if (warp < 12) {
        setmaxnreg_inc<152>();
        // ------------------------------------------------ P^T / dS^T, then dK/dV epilogue
        const int h = (warp - 4) >> 2;  // query half
        const int wq = warp & 3;
        const int r = wq * 32 + lane;  // kv row within block j
        const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t t_s = tmem + lane_addr + h * 64;
        const uint32_t t_dp = tmem + lane_addr + 128 + h * 64;
        const uint32_t sDs = sbase + G::kOffDs + h * (128 * 128) + r * 128;
        const float c = p.scale_log2;
        uint32_t g = 0, items = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
            for (int w = 0; ok && w < 2; ++w) {
                BwdItem itm;
                if (!bwd_item<kCp>(p, u, w, itm)) continue;
                const int j = itm.j, bh = itm.bh;  // bh: K/V head (dK, dV rows)
                const BwdWalk wk = bwd_walk<kCp>(p, itm);
                const int n_it = wk.n;
                for (int it = 0; it < n_it; ++it, ++g) {
                    int bh_q, i;
                    long long rel;
                    bwd_step<kCp>(p, itm, wk, it, bh_q, i, rel);
                    const int s = g % G::kStages;
                    // L and D of block i arrived through the async proxy: observe
                    // the stage's own barrier before reading them (it completes
                    // before S is issued, so waiting for it first costs nothing)
                    if (!bwarp_wait(full + s, (g / G::kStages) & 1, abort_flag) ||
                        !bwarp_wait(bar_s, g & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const float* sL =
                        reinterpret_cast<const float*>(sptr + G::kOffStage + s * G::kStageBytes +
                                                       2 * G::kTileBytes) +
                        h * 64;
                    const float* sD = sL + 128;
                    const long long dl = 128LL * (j - i) - rel;
                    float pf[64];  // this row's P for the warpgroup's 64 queries
                    if (p.causal && dl > -127)
                        bwd_softmax_p<T, true>(t_s, sL, c, h, r, static_cast<int>(dl), pf);
                    else
                        bwd_softmax_p<T, false>(t_s, sL, c, h, r, 0, pf);
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(bar_p);
                    // dP^T: issued after S^T, once the previous block's dQ left
                    // its columns; its commit also covers that dQ product, which
                    // read the shared-memory dS this phase overwrites
                    if (!bwarp_wait(bar_dp, g & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    bwd_softmax_ds<T>(t_dp, sDs, sD, r, pf);
                    tmem_wait_st();
                    fence_proxy_async_smem();
                    tc_fence_before();
                    mbar_arrive(bar_ds);
                }
                if (ok) {
                    ok = bwarp_wait(bar_acc, items & 1, abort_flag);
                    tc_fence_after();
                }
                ++items;
                // warpgroup 0 stores dV, warpgroup 1 stores dK (scaled)
                const int kv = j * 128 + r;
                const bool valid = kv < p.Nk;
                const size_t row = (static_cast<size_t>(bh) * p.Nk + kv) * D;
                const float mul = h == 0 ? 1.f : p.scale;
                const uint32_t t_acc = tmem + lane_addr + (h == 0 ? 256 : 384);
                if constexpr (kCp) {
                    // add this step's dV / scale*dK of the row into the fp32 accumulator
                    float* acc = (h == 0 ? p.dv_acc : p.dk_acc) + row;
#pragma unroll
                    for (int cb = 0; cb < D / 32; ++cb) {
                        uint32_t a[32];
                        if (ok) tmem_ld_x32(t_acc + cb * 32, a);
                        if (ok && valid) {
                            float4* dst = reinterpret_cast<float4*>(acc + cb * 32);
                            float4 cur[8];
#pragma unroll
                            for (int q4 = 0; q4 < 8; ++q4) cur[q4] = dst[q4];
#pragma unroll
                            for (int q4 = 0; q4 < 8; ++q4) {
                                cur[q4].x = fmaf(__uint_as_float(a[4 * q4 + 0]), mul, cur[q4].x);
                                cur[q4].y = fmaf(__uint_as_float(a[4 * q4 + 1]), mul, cur[q4].y);
                                cur[q4].z = fmaf(__uint_as_float(a[4 * q4 + 2]), mul, cur[q4].z);
                                cur[q4].w = fmaf(__uint_as_float(a[4 * q4 + 3]), mul, cur[q4].w);
                                dst[q4] = cur[q4];
                            }
                        }
                    }
                    continue;
                }
                T* dst_base = static_cast<T*>(h == 0 ? p.dV : p.dK);
#pragma unroll
                for (int cb = 0; cb < D / 32; ++cb) {
                    uint32_t a[32];
                    if (ok) {
                        tmem_ld_x32(t_acc + cb * 32, a);
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e) a[e] = 0u;
                    }
                    if (valid) {
                        uint4* dst = reinterpret_cast<uint4*>(dst_base + row + cb * 32);
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            uint4 v;
                            v.x = DType<T>::pack2(__uint_as_float(a[8 * q4 + 0]) * mul, __uint_as_float(a[8 * q4 + 1]) * mul);
                            v.y = DType<T>::pack2(__uint_as_float(a[8 * q4 + 2]) * mul, __uint_as_float(a[8 * q4 + 3]) * mul);
                            v.z = DType<T>::pack2(__uint_as_float(a[8 * q4 + 4]) * mul, __uint_as_float(a[8 * q4 + 5]) * mul);
                            v.w = DType<T>::pack2(__uint_as_float(a[8 * q4 + 6]) * mul, __uint_as_float(a[8 * q4 + 7]) * mul);
                            dst[q4] = v;
                        }
                    }
                }
                // The next item's first dS arrival follows these TMEM reads, so
                // its dV / dK products cannot overwrite the accumulators early.
            }
        }
    } else {
        setmaxnreg_inc<152>();
        // ------------------------------------------------ dQ drain
        const int wq = warp & 3;
        const uint32_t t_q = tmem + (static_cast<uint32_t>(wq * 32) << 16) + 128;
        uint32_t g = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
            for (int w = 0; ok && w < 2; ++w) {
                BwdItem itm;
                if (!bwd_item<kCp>(p, u, w, itm)) continue;
                const BwdWalk wk = bwd_walk<kCp>(p, itm);
                const int n_it = wk.n;
                if constexpr (kTransposedDq) {
                    // lane = head_dim element d; TMEM column = query row of block i
                    const int d = wq * 32 + lane;
                    for (int it = 0; it < n_it; ++it, ++g) {
                        int bh, i;  // query head and block
                        long long rel;
                        bwd_step<kCp>(p, itm, wk, it, bh, i, rel);
                        if (!bwarp_wait(bar_dq, g & 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        uint32_t v0[32], v1[32], v2[32], v3[32];
                        tmem_ld2_x32(t_q, v0, t_q + 32, v1);
                        tmem_ld2_x32(t_q + 64, v2, t_q + 96, v3);
                        // TMEM columns are free once loaded: release them before the
                        // reductions so the next dP MMA is not held up
                        tc_fence_before();
                        mbar_arrive(bar_dqfree);
                        float* dst = p.dq_acc + (static_cast<size_t>(bh) * p.Nq + i * 128) * D + d;
                        const int qn = min(128, p.Nq - i * 128);
                        auto flush = [&](const uint32_t(&v)[32], int q0) {
#pragma unroll
                            for (int e = 0; e < 32; ++e)
                                if (q0 + e < qn)
                                    red_add_f32(dst + static_cast<size_t>(q0 + e) * D, __uint_as_float(v[e]));
                        };
                        flush(v0, 0);
                        flush(v1, 32);
                        flush(v2, 64);
                        flush(v3, 96);
                    }
                } else if constexpr (kDqMode == 2) {
                    // lane = query row of block i; TMEM columns = head_dim elements
                    const int qr = wq * 32 + lane;
                    for (int it = 0; it < n_it; ++it, ++g) {
                        int bh, i;  // query head and block
                        long long rel;
                        bwd_step<kCp>(p, itm, wk, it, bh, i, rel);
                        if (!bwarp_wait(bar_dq, g & 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        uint32_t v0[32], v1[32], v2[32], v3[32];
                        if constexpr (D == 32) {
                            tmem_ld_x32(t_q, v0);
                        } else {
                            tmem_ld2_x32(t_q, v0, t_q + 32, v1);
                            if constexpr (D == 128) tmem_ld2_x32(t_q + 64, v2, t_q + 96, v3);
                        }
                        // TMEM columns are free once loaded
                        tc_fence_before();
                        mbar_arrive(bar_dqfree);
                        if (i * 128 + qr < p.Nq) {
                            float* dst = p.dq_acc + (static_cast<size_t>(bh) * p.Nq + i * 128 + qr) * D;
                            auto flush = [&](const uint32_t(&v)[32], int c0) {
#pragma unroll
                                for (int m = 0; m < 8; ++m)
                                    red_add_v4_f32(dst + c0 + 4 * m, v[4 * m], v[4 * m + 1], v[4 * m + 2],
                                                   v[4 * m + 3]);
                            };
                            flush(v0, 0);
                            if constexpr (D >= 64) flush(v1, 32);
                            if constexpr (D == 128) {
                                flush(v2, 64);
                                flush(v3, 96);
                            }
                        }
                    }
                } else {
                    // Each warp owns 32 query rows.  Per 32-column chunk it copies
                    // its 32x32 fp32 block from TMEM into a 128-byte-swizzled
                    // staging box and the TMA unit adds the box into the fp32
                    // accumulator.  Staging lives in the dS buffer, idle from the
                    // completion of dQ_i until the softmax warps write the next
                    // dS, which they do only after the next dP^T, issued once
                    // this drain signals bar_dqfree.
                    const uint32_t stage0 = sbase + G::kOffDs + wq * 8192;
                    for (int it = 0; it < n_it; ++it, ++g) {
                        int bh, i;  // query head and block
                        long long rel;
                        bwd_step<kCp>(p, itm, wk, it, bh, i, rel);
                        if (!bwarp_wait(bar_dq, g & 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
#pragma unroll
                        for (int cb = 0; cb < D / 32; ++cb) {
                            const uint32_t box = stage0 + (cb & 1) * 4096;
                            if (cb >= 2) {
                                if (lane == 0) bulk_wait_group_read<1>();
                                __syncwarp();
                            }
                            uint32_t v[32];
                            tmem_ld_x32(t_q + cb * 32, v);
#pragma unroll
                            for (int k = 0; k < 8; ++k)
                                st_shared_v4(box + lane * 128 + ((k ^ (lane & 7)) << 4), v[4 * k],
                                             v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) {
                                tma_reduce_add_3d(&tmdQ, box, cb * 32, i * 128 + wq * 32, bh);
                                bulk_commit_group();
                            }
                        }
                        // the staging boxes must be read out before dS_{i+1} overwrites them
                        if (lane == 0) bulk_wait_group_read<0>();
                        __syncwarp();
                        tc_fence_before();
                        mbar_arrive(bar_dqfree);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// B*Hq query heads (BH) over Nq queries, B*Hkv = BH/group K/V heads over Nk keys.
template <typename T, int D>
FlashAttentionError bwd_typed(const T* Q, const T* K, const T* V, const T* O, const float* L,
                              const T* dO, T* dQ, T* dK, T* dV, int BH, int Hq, int group, int Nq,
                              int Nk, long long q_off, float scale, bool causal,
                              cudaStream_t stream) {
    using G = BwdGeom<D>;
    const int BHk = BH / group;
    const int n_blk_q = (Nq + 127) / 128;
    const int n_blk_k = (Nk + 127) / 128;
    const long long n_pad = static_cast<long long>(n_blk_q) * 128;
    const size_t acc_elems = static_cast<size_t>(BH) * Nq * D;
    const size_t pad_elems = static_cast<size_t>(BH) * n_pad;
    void* ws = nullptr;
    FlashAttentionError e =
        workspace_alloc(&ws, (acc_elems + 2 * pad_elems) * sizeof(float), stream);
    if (e != FlashAttentionError::SUCCESS) return e;
    float* dq_acc = static_cast<float*>(ws);
    float* l2p = dq_acc + acc_elems;
    float* dvp = l2p + pad_elems;

    auto fail = [&](FlashAttentionError err) {
        workspace_free(ws, stream);
        return err;
    };
    const CUtensorMapSwizzle swz =
        G::kSwz == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUtensorMap mq, mk, mv, mdo, mdq;
    if (!encode_tmap_3d(&mq, Q, DType<T>::kTmaType, 2, D, Nq, BH, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mk, K, DType<T>::kTmaType, 2, D, Nk, BHk, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mv, V, DType<T>::kTmaType, 2, D, Nk, BHk, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mdo, dO, DType<T>::kTmaType, 2, D, Nq, BH, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mdq, dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, Nq, BH, 32, 32,
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return fail(FlashAttentionError::CUDA_ERROR);
    for (const void* ptr : {static_cast<const void*>(O), static_cast<const void*>(dQ),
                            static_cast<const void*>(dK), static_cast<const void*>(dV)})
        if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0)
            return fail(FlashAttentionError::CUDA_ERROR);
    auto kern = fa_bwd_kernel<T, D, false>;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(kern), G::kSmemBytes))
        return fail(FlashAttentionError::CUDA_ERROR);

    const long long rows_pad = static_cast<long long>(BH) * n_pad;
    const long long pre_blocks = (rows_pad * (D / 8) + 255) / 256;
    bwd_preprocess_kernel<T, D><<<static_cast<unsigned>(pre_blocks), 256, 0, stream>>>(
        O, dO, L, l2p, dvp, dq_acc, Nq, static_cast<int>(n_pad), rows_pad);
    if (cudaGetLastError() != cudaSuccess) return fail(FlashAttentionError::CUDA_ERROR);

    BwdParams prm;
    prm.dq_acc = dq_acc;
    prm.dK = dK;
    prm.dV = dV;
    prm.l2p = l2p;
    prm.dvp = dvp;
    prm.Nq = Nq;
    prm.Nk = Nk;
    prm.n_blk_q = n_blk_q;
    prm.n_blk_k = n_blk_k;
    prm.q_off = q_off;
    prm.hq = Hq;
    prm.group = group;
    prm.npairs = (n_blk_k + 1) / 2;
    const int sms = current_sm_count();
    long long units = static_cast<long long>(BHk) * prm.npairs;
    // pairing only balances a causal walk (non-causal items all cost n_blk_q)
    prm.paired = (causal && units >= sms) ? 1 : 0;
    prm.order = 0;
    // Few pairs per SM (a causal problem split over several GPUs): single kv
    // blocks dealt by decreasing cost in snake rounds balance the CTAs better
    // than equal-cost pairs do (512 pairs on 148 SMs: 86 % busy).
    if (prm.paired && units < 5LL * sms && static_cast<long long>(BHk) * n_blk_k > sms) {
        prm.paired = 0;
        prm.order = 1;
    }
    if (!prm.paired) units = static_cast<long long>(BHk) * n_blk_k;
    if (units > 0x7fffffffLL) return fail(FlashAttentionError::CUDA_ERROR);
    prm.num_units = static_cast<int>(units);
    prm.causal = causal ? 1 : 0;
    prm.scale_log2 = scale * kLog2eB;
    prm.scale = scale;
    // persistent: one CTA per SM (the shared-memory footprint allows one)
    const int grid = persistent_grid(units, env_int("CUFLASH_BWD_WAVES", 1));
    bind_status_word(reinterpret_cast<const void*>(&g_bwd_status), stream);
    profile_record(false, stream);
    kern<<<grid, kBwdThreads, G::kSmemBytes, stream>>>(mq, mk, mv, mdo, mdq, prm);
    if (cudaGetLastError() != cudaSuccess) return fail(FlashAttentionError::CUDA_ERROR);
    profile_record(true, stream);

    const long long n4 = static_cast<long long>(acc_elems / 4);
    long long cblocks = (n4 + 255) / 256;
    const long long cap = 32LL * current_sm_count();
    if (cblocks > cap) cblocks = cap;
    bwd_convert_dq_kernel<T><<<static_cast<unsigned>(cblocks), 256, 0, stream>>>(dq_acc, dQ, scale,
                                                                                 n4);
    if (cudaGetLastError() != cudaSuccess) return fail(FlashAttentionError::CUDA_ERROR);
    workspace_free(ws, stream);
    return FlashAttentionError::SUCCESS;
}

template <typename T>
FlashAttentionError bwd_dispatch(const T* Q, const T* K, const T* V, const T* O, const float* L,
                                 const T* dO, T* dQ, T* dK, T* dV, int B, int Hq, int Hkv, int Nq,
                                 int Nk, int D, long long q_off, float scale, bool causal,
                                 cudaStream_t stream) {
    const int BH = B * Hq;
    const int group = Hq / Hkv;
    switch (D) {
        case 32:
            return bwd_typed<T, 32>(Q, K, V, O, L, dO, dQ, dK, dV, BH, Hq, group, Nq, Nk, q_off,
                                    scale, causal, stream);
        case 64:
            return bwd_typed<T, 64>(Q, K, V, O, L, dO, dQ, dK, dV, BH, Hq, group, Nq, Nk, q_off,
                                    scale, causal, stream);
        case 128:
            return bwd_typed<T, 128>(Q, K, V, O, L, dO, dQ, dK, dV, BH, Hq, group, Nq, Nk, q_off,
                                     scale, causal, stream);
        default:
            return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
}

// ------------------------------------------------- context-parallel backward
//
// Workspace of the ring backward, kept across its steps: the fp32 dQ
// accumulator [nq*BH][C][D], then -L*log2(e) and -rowsum(dO*O) per query
// head, each padded to whole 128-row blocks.
struct CpBwdWs {
    float* dq_acc;
    float* l2p;
    float* dvp;
};

inline long long cp_bwd_pad(int C) { return (static_cast<long long>(C) + 127) / 128 * 128; }

inline CpBwdWs cp_bwd_ws(void* ws, long long heads, int C, int D) {
    CpBwdWs w;
    w.dq_acc = static_cast<float*>(ws);
    w.l2p = w.dq_acc + heads * C * D;
    w.dvp = w.l2p + heads * cp_bwd_pad(C);
    return w;
}

template <typename T, int D>
FlashAttentionError bwd_cp_prepare_typed(const T* O, const T* dO, const float* L, void* ws,
                                         long long heads, int C, cudaStream_t stream) {
    const CpBwdWs w = cp_bwd_ws(ws, heads, C, D);
    const long long n_pad = cp_bwd_pad(C);
    const long long rows_pad = heads * n_pad;
    const long long pre_blocks = (rows_pad * (D / 8) + 255) / 256;
    bwd_preprocess_kernel<T, D><<<static_cast<unsigned>(pre_blocks), 256, 0, stream>>>(
        O, dO, L, w.l2p, w.dvp, w.dq_acc, C, static_cast<int>(n_pad), rows_pad);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

template <typename T, int D>
FlashAttentionError bwd_cp_step_typed(const T* Q, const T* dO, const T* K, const T* V, void* ws,
                                      float* dk_acc, float* dv_acc, int nq, int nk, int BH, int C,
                                      float scale, bool causal, int num_pairs, const int* q_slot,
                                      const int* kv_slot, const long long* q_off,
                                      const long long* kv_off, int reserve_sms,
                                      cudaStream_t stream) {
    using G = BwdGeom<D>;
    const long long qheads = static_cast<long long>(nq) * BH;
    const long long kheads = static_cast<long long>(nk) * BH;
    const CpBwdWs w = cp_bwd_ws(ws, qheads, C, D);
    const CUtensorMapSwizzle swz =
        G::kSwz == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUtensorMap mq, mk, mv, mdo, mdq;
    if (!encode_tmap_3d(&mq, Q, DType<T>::kTmaType, 2, D, C, qheads, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mk, K, DType<T>::kTmaType, 2, D, C, kheads, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mv, V, DType<T>::kTmaType, 2, D, C, kheads, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mdo, dO, DType<T>::kTmaType, 2, D, C, qheads, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mdq, w.dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, C, qheads, 32, 32,
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return FlashAttentionError::CUDA_ERROR;
    if ((reinterpret_cast<uintptr_t>(dk_acc) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(dv_acc) & 15u) != 0)
        return FlashAttentionError::CUDA_ERROR;
    auto kern = fa_bwd_kernel<T, D, true>;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(kern), G::kSmemBytes))
        return FlashAttentionError::CUDA_ERROR;

    BwdParams prm{};
    prm.dq_acc = w.dq_acc;
    prm.l2p = w.l2p;
    prm.dvp = w.dvp;
    prm.dk_acc = dk_acc;
    prm.dv_acc = dv_acc;
    prm.Nq = C;
    prm.Nk = C;
    prm.n_blk_q = (C + 127) / 128;
    prm.n_blk_k = prm.n_blk_q;
    prm.q_off = 0;
    prm.hq = 1;
    prm.group = 1;
    prm.npairs = (prm.n_blk_k + 1) / 2;
    prm.causal = causal ? 1 : 0;
    prm.scale_log2 = scale * kLog2eB;
    prm.scale = scale;
    prm.bh_slot = BH;
    // segments: the distinct K/V slots in order of first appearance, each
    // with its pairs in call order
    prm.nkseg = 0;
    int np = 0;
    for (int i = 0; i < num_pairs; ++i) {
        bool seen = false;
        for (int s = 0; s < prm.nkseg; ++s) seen = seen || prm.kseg_slot[s] == kv_slot[i];
        if (seen) continue;
        const int s = prm.nkseg++;
        prm.kseg_slot[s] = kv_slot[i];
        prm.kseg_first[s] = np;
        for (int k = i; k < num_pairs; ++k) {
            if (kv_slot[k] != kv_slot[i]) continue;
            prm.pair_q_slot[np] = q_slot[k];
            prm.pair_rel[np] = q_off[k] - kv_off[k];
            ++np;
        }
        prm.kseg_count[s] = np - prm.kseg_first[s];
    }
    const int sms = current_sm_count();
    long long seg_units = static_cast<long long>(BH) * prm.npairs;
    prm.paired = (causal && seg_units * prm.nkseg >= sms) ? 1 : 0;
    if (!prm.paired) seg_units = static_cast<long long>(BH) * prm.n_blk_k;
    const long long units = seg_units * prm.nkseg;
    if (units > 0x7fffffffLL) return FlashAttentionError::CUDA_ERROR;
    prm.seg_units = static_cast<int>(seg_units);
    prm.num_units = static_cast<int>(units);
    // reserve_sms SMs stay free for the ring's concurrent transfer kernels,
    // as in the forward step.
    int grid = persistent_grid(units, env_int("CUFLASH_BWD_WAVES", 1));
    grid = std::max(1, std::min(grid, sms - reserve_sms));
    bind_status_word(reinterpret_cast<const void*>(&g_bwd_status), stream);
    kern<<<grid, kBwdThreads, G::kSmemBytes, stream>>>(mq, mk, mv, mdo, mdq, prm);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

template <typename T>
FlashAttentionError bwd_cp_finish_typed(const void* ws, T* dQ, long long heads, int C, int D,
                                        float scale, cudaStream_t stream) {
    const float* acc = static_cast<const float*>(ws);
    const long long n4 = heads * C * D / 4;
    long long cblocks = (n4 + 255) / 256;
    const long long cap = 32LL * current_sm_count();
    if (cblocks > cap) cblocks = cap;
    if (cblocks < 1) cblocks = 1;
    bwd_convert_dq_kernel<T><<<static_cast<unsigned>(cblocks), 256, 0, stream>>>(acc, dQ, scale,
                                                                                 n4);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

__global__ void __launch_bounds__(256)
    accumulate_f32_kernel(float* __restrict__ dst, float* __restrict__ src, long long n4,
                          int zero_src) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += stride) {
        float4 a = reinterpret_cast<const float4*>(dst)[i];
        const float4 b = reinterpret_cast<const float4*>(src)[i];
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
        reinterpret_cast<float4*>(dst)[i] = a;
        if (zero_src) reinterpret_cast<float4*>(src)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

}  // namespace

long long bwd_cp_workspace_bytes(int nq, int BH, int C, int D) {
    const long long heads = static_cast<long long>(nq) * BH;
    return (heads * C * D + 2 * heads * cp_bwd_pad(C)) * static_cast<long long>(sizeof(float));
}

template <typename T>
FlashAttentionError launch_bwd_cp_prepare_sm100(const T* O, const T* dO, const float* L, void* ws,
                                                int nq, int BH, int C, int D,
                                                cudaStream_t stream) {
    const long long heads = static_cast<long long>(nq) * BH;
    switch (D) {
        case 32: return bwd_cp_prepare_typed<T, 32>(O, dO, L, ws, heads, C, stream);
        case 64: return bwd_cp_prepare_typed<T, 64>(O, dO, L, ws, heads, C, stream);
        case 128: return bwd_cp_prepare_typed<T, 128>(O, dO, L, ws, heads, C, stream);
        default: return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
}

template <typename T>
FlashAttentionError launch_bwd_cp_step_sm100(const T* Q, const T* dO, const T* K, const T* V,
                                             void* ws, float* dk_acc, float* dv_acc, int nq,
                                             int nk, int BH, int C, int D, float scale,
                                             bool causal, int num_pairs, const int* q_slot,
                                             const int* kv_slot, const long long* q_off,
                                             const long long* kv_off, int reserve_sms,
                                             cudaStream_t stream) {
#define CUFLASH_CP_STEP(DD)                                                                    \
    return bwd_cp_step_typed<T, DD>(Q, dO, K, V, ws, dk_acc, dv_acc, nq, nk, BH, C, scale,    \
                                    causal, num_pairs, q_slot, kv_slot, q_off, kv_off,        \
                                    reserve_sms, stream)
    switch (D) {
        case 32: CUFLASH_CP_STEP(32);
        case 64: CUFLASH_CP_STEP(64);
        case 128: CUFLASH_CP_STEP(128);
        default: return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
#undef CUFLASH_CP_STEP
}

template <typename T>
FlashAttentionError launch_bwd_cp_finish_sm100(const void* ws, T* dQ, int nq, int BH, int C, int D,
                                               float scale, cudaStream_t stream) {
    return bwd_cp_finish_typed<T>(ws, dQ, static_cast<long long>(nq) * BH, C, D, scale, stream);
}

FlashAttentionError launch_accumulate_f32(float* dst, float* src, long long count, bool zero_src,
                                          cudaStream_t stream) {
    const long long n4 = count / 4;
    long long blocks = (n4 + 255) / 256;
    const long long cap = 8LL * current_sm_count();
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    accumulate_f32_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(dst, src, n4,
                                                                             zero_src ? 1 : 0);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

#define CUFLASH_CP_INST(T)                                                                      \
    template FlashAttentionError launch_bwd_cp_prepare_sm100<T>(                                \
        const T*, const T*, const float*, void*, int, int, int, int, cudaStream_t);             \
    template FlashAttentionError launch_bwd_cp_step_sm100<T>(                                   \
        const T*, const T*, const T*, const T*, void*, float*, float*, int, int, int, int, int, \
        float, bool, int, const int*, const int*, const long long*, const long long*, int,      \
        cudaStream_t);                                                                          \
    template FlashAttentionError launch_bwd_cp_finish_sm100<T>(const void*, T*, int, int, int, \
                                                               int, float, cudaStream_t);
CUFLASH_CP_INST(half)
CUFLASH_CP_INST(__nv_bfloat16)
#undef CUFLASH_CP_INST

template <typename T>
FlashAttentionError launch_bwd_sm100(const T* Q, const T* K, const T* V, const T* O,
                                     const float* L, const T* dO, T* dQ, T* dK, T* dV, int B,
                                     int H, int N, int D, float scale, bool causal,
                                     cudaStream_t stream) {
    return bwd_dispatch<T>(Q, K, V, O, L, dO, dQ, dK, dV, B, H, H, N, N, D, 0, scale, causal,
                           stream);
}

template <typename T>
FlashAttentionError launch_bwd_gqa_sm100(const T* Q, const T* K, const T* V, const T* O,
                                         const float* L, const T* dO, T* dQ, T* dK, T* dV, int B,
                                         int Hq, int Hkv, int seq_q, int seq_k, int D, float scale,
                                         bool causal, cudaStream_t stream) {
    // bottom-right causal alignment, as the grouped-query forward
    return bwd_dispatch<T>(Q, K, V, O, L, dO, dQ, dK, dV, B, Hq, Hkv, seq_q, seq_k, D,
                           static_cast<long long>(seq_k) - seq_q, scale, causal, stream);
}

template FlashAttentionError launch_bwd_gqa_sm100<half>(const half*, const half*, const half*,
                                                        const half*, const float*, const half*,
                                                        half*, half*, half*, int, int, int, int,
                                                        int, int, float, bool, cudaStream_t);
template FlashAttentionError launch_bwd_gqa_sm100<__nv_bfloat16>(
    const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
    const float*, const __nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16*, int, int,
    int, int, int, int, float, bool, cudaStream_t);

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
