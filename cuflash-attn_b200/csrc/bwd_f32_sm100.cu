// Backward attention for fp32 inputs on sm_100a tensor cores, 3xTF32.
//
// Replaces the reference's fp32 backward (src/backward/flash_attention_
// backward_typed.cu:13-288: D_i = rowsum(dO_i * O_i), then dQ, dK, dV from P
// recomputed out of the saved logsumexp L) with tcgen05 kind::tf32 MMAs held
// to fp32 accuracy by the three-term split of every product (hi(a)hi(b) +
// hi(a)lo(b) + lo(a)hi(b); the raw fp32 word is the hi operand, lo = a - hi).
//
// Three kernels, one per gradient, each a CTA over a fixed tile of 128 rows
// (TMEM lanes) of one (batch, head) streaming blocks of kBS rows:
//   dV  rows = keys     S^T = K Q^T                     P^T = exp(s S^T - L_q)
//                       dV += P^T dO
//   dK  rows = keys     S^T = K Q^T, dP^T = V dO^T      dS^T = P^T (dP^T - D_q)
//                       dK += s dS^T Q
//   dQ  rows = queries  S = Q K^T, dP = dO V^T           dS = P (dP - D_q)
//                       dQ += s dS K
// Splitting the gradients recomputes S (and dP) per kernel, but keeps every
// accumulator in TMEM for the whole loop and needs no atomics: at head_dim
// 128 the 512 TMEM columns hold the lo parts of the two resident tiles
// (A operands), one fp32 accumulator and the per-block S, dP, dS, dS_lo
// columns, not a second accumulator.
//
// Shared memory: the resident tiles F1 (F2), then three rings of streamed
// tiles, each slot a tile and its lo part:
//   A1  S1 (S^T's B operand: Q for dV/dK, K for dQ)
//   A2  S2 (dP's B operand: dO for dK, V for dQ)
//   T   the accumulation's B operand, transposed in place from its own TMA
//       copy (dO^T for dV, Q^T for dK, K^T for dQ): every tf32 operand is
//       K-major (an MN-major tf32 operand would need the 32-byte-atom swizzle)
// Roles (384 threads):
//   warp 0      TMA producer of F1, F2, A1, A2
//   warp 1      TMEM allocator, MMA issuer
//   warp 2      TMA producer of T
//   warps 4-7   element-wise stage (one thread per resident row) and the
//               epilogue
//   warps 8-11  lo parts of F1/F2 into TMEM, then two splitter groups:
//               warps 8-9 write the lo parts of A1/A2 (element-wise, the
//               swizzled layout is kept), warps 10-11 transpose T and load
//               the per-column scalars -L*log2(e) and D
// The rings are decoupled: a slot of A1 is refilled as soon as its S^T MMAs
// have read it, whatever the transposes or the accumulation are doing.

#include <cmath>

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {

__device__ sm100::StatusWord g_bf32_status;

constexpr float kLog2eB = 1.4426950408889634f;

enum : int { kModeDV = 0, kModeDK = 1, kModeDQ = 2 };

template <int D, int kMode>
struct BF32Geom {
    static constexpr bool kTwo = kMode != kModeDV;  // second product dP (Y)
    static constexpr int kBM = 128;
    static constexpr int kBS = (D == 128) ? 32 : 64;
    static constexpr int kFBytes = kBM * D * 4;
    static constexpr int kFCb = kBM * 128;
    static constexpr int kSBytes = kBS * D * 4;  // streamed tile [kBS][D], or its transpose
    static constexpr int kSCb = kBS * 128;       // column block of [kBS][D] (ring T, raw)
    static constexpr int kACb = 2 * kBS * 128;   // ring A column block: kBS rows, kBS lo rows
    static constexpr int kTCb = D * 128;         // column block of [D][kBS]
    static constexpr int kNumF = kTwo ? 2 : 1;
    static constexpr int kFTotal = kNumF * kFBytes;
    static constexpr int kPair = 2 * kSBytes;  // a ring slot: tile + lo part
    static constexpr int kBudget = 232448 - 2048;
    static constexpr int kRings = kTwo ? 3 : 2;
    static constexpr int kPairsFit = (kBudget - kFTotal) / kPair;
    // one slot per ring, then a second slot for A1, A2, T in that order
    static constexpr int kExtra =
        kPairsFit - kRings < kRings ? kPairsFit - kRings : kRings;
    static constexpr int kStagesA1 = 1 + (kExtra >= 1 ? 1 : 0);
    static constexpr int kStagesA2 = kTwo ? 1 + (kExtra >= 2 ? 1 : 0) : 0;
    static constexpr int kStagesT = 1 + (kExtra >= kRings ? 1 : 0);
    static constexpr int kOffF = 0;
    static constexpr int kOffA1 = kFTotal;
    static constexpr int kOffA2 = kOffA1 + kStagesA1 * kPair;
    static constexpr int kOffT = kOffA2 + kStagesA2 * kPair;
    static constexpr int kOffSc = kOffT + kStagesT * kPair;  // [kStagesT][2][kBS] floats
    static constexpr int kOffBar = kOffSc + kStagesT * 2 * kBS * 4;
    // bar_f, bar_flo, {full, split, empty} x (A1, A2, T slots), bar_x [2],
    // bar_w [2], bar_done
    static constexpr int kNumBars = 2 + 3 * (kStagesA1 + kStagesA2 + kStagesT) + 5;
    static constexpr int kUsed = kOffBar + kNumBars * 8 + 16;
    // at least 116 KB so that one CTA (and its 512 TMEM columns) owns the SM
    static constexpr int kSmemBytes = kUsed > 118784 ? kUsed : 118784;
    static_assert(kExtra >= 0 && kUsed <= 232448, "shared memory budget");
    // TMEM columns.  A product of the resident tile with [S; S_lo] occupies
    // 2 kBS columns: F S^T, then F S_lo^T + F_lo S^T; its value is their
    // sum.  The element-wise stage overwrites the two halves of X with W
    // (P for dV, dS for dK / dQ) and W_lo, the A operands of the accumulation.
    static constexpr int kXBufs = kTwo ? 1 : 2;
    static constexpr int kColF1lo = 0;
    static constexpr int kColF2lo = D;  // dK, dQ
    static constexpr int kColAcc = kNumF * D;
    static constexpr int kColX = kColAcc + D;               // [kXBufs][2 kBS]
    static constexpr int kColY = kColX + kXBufs * 2 * kBS;  // dK, dQ: dP [2 kBS]
    static constexpr int kColEnd = kColY + (kTwo ? 2 * kBS : 0);
    static_assert(kColEnd <= 512, "TMEM budget");
    // 4x4 blocks of the transposed tile per thread of the 64-thread group
    static constexpr int kTBlocks = (kBS / 4) * (D / 4) / 64;
    static_assert(kTBlocks * 64 == (kBS / 4) * (D / 4), "transpose split");
};

struct BF32Params {
    const float* L;
    const float* Dv;
    float* out;
    int N;
    int causal;
    float scale_log2;  // scale * log2(e)
    float out_scale;   // 1 for dV, scale for dK and dQ
};

__device__ __forceinline__ bool bf32_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag) {
    return sm100::mbar_wait(bar, parity, abort_flag, &g_bf32_status);
}

// Barrier of one 64-thread splitter group (id 1: warps 8-9, id 2: 10-11).
template <int kId>
__device__ __forceinline__ void group_sync() {
    asm volatile("bar.sync %0, 64;" ::"n"(kId) : "memory");
}

// Same barrier with an AND vote, so that all threads of a group take the
// same branch after a wait (a named barrier must never miss a participant).
template <int kId>
__device__ __forceinline__ bool group_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, %2, 64, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(r)
        : "r"(v ? 1u : 0u), "n"(kId)
        : "memory");
    return r != 0;
}

// lo parts of a ring A slot: every 128-byte column block holds R rows of the
// tile, then the R rows of its lo part (element-wise: same swizzle phase).
template <int R, int D>
__device__ __forceinline__ void split_lo_stacked(uint8_t* slot, int t) {
    using sm100::tf32_lo;
    float4* s4 = reinterpret_cast<float4*>(slot);
    for (int i = t; i < R * D / 4; i += 64) {
        const int src = (i / (R * 8)) * (R * 16) + i % (R * 8);
        const float4 a = s4[src];
        s4[src + R * 8] = make_float4(tf32_lo(a.x), tf32_lo(a.y), tf32_lo(a.z), tf32_lo(a.w));
    }
}

// lo part of row r of a resident [128][D] tile into TMEM columns col..col+D.
template <int D>
__device__ __forceinline__ void split_rows_to_tmem(const uint8_t* f, uint32_t t_addr, int r) {
    using namespace sm100;
#pragma unroll
    for (int cb = 0; cb < D / 32; ++cb) {
        uint32_t v[32];
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            const float4 x = *reinterpret_cast<const float4*>(f + cb * (128 * 128) + r * 128 +
                                                              ((ch ^ (r & 7)) << 4));
            v[4 * ch] = __float_as_uint(tf32_lo(x.x));
            v[4 * ch + 1] = __float_as_uint(tf32_lo(x.y));
            v[4 * ch + 2] = __float_as_uint(tf32_lo(x.z));
            v[4 * ch + 3] = __float_as_uint(tf32_lo(x.w));
        }
        tmem_st_x32(t_addr + cb * 32, v);
    }
}

template <int D, int kMode>
__global__ void __launch_bounds__(384, 1)
    fa_bwd_f32_kernel(const __grid_constant__ CUtensorMap tmF1,
                      const __grid_constant__ CUtensorMap tmF2,
                      const __grid_constant__ CUtensorMap tmS1,
                      const __grid_constant__ CUtensorMap tmS2, const BF32Params p) {
    using G = BF32Geom<D, kMode>;
    using namespace sm100;
    constexpr int BS = G::kBS;
    constexpr bool kTwo = G::kTwo;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (sm100::cta_skip(&g_bf32_status)) return;
    const uint32_t sbase = smem_u32(smem_raw);
    if ((sbase & 1023u) != 0) {
        if (threadIdx.x == 0) sm100::record_status(&g_bf32_status, sm100::kStatusMisaligned);
        return;
    }
    uint8_t* sptr = smem_raw;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sptr + G::kOffBar);
    uint64_t* bar_f = bars;
    uint64_t* bar_flo = bars + 1;
    uint64_t* fullA1 = bars + 2;
    uint64_t* splitA1 = fullA1 + G::kStagesA1;
    uint64_t* emptyA1 = splitA1 + G::kStagesA1;
    uint64_t* fullA2 = emptyA1 + G::kStagesA1;
    uint64_t* splitA2 = fullA2 + G::kStagesA2;
    uint64_t* emptyA2 = splitA2 + G::kStagesA2;
    uint64_t* fullT = emptyA2 + G::kStagesA2;
    uint64_t* splitT = fullT + G::kStagesT;
    uint64_t* emptyT = splitT + G::kStagesT;
    // dV keeps two blocks in flight (S^T of the next block is issued before
    // the current accumulation), so its X and W barriers are double: a
    // waiter can then never fall two phases behind on one barrier
    uint64_t* bar_x = emptyT + G::kStagesT;  // [2]
    uint64_t* bar_w = bar_x + 2;             // [2]
    uint64_t* bar_done = bar_w + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* sc_all = reinterpret_cast<float*>(sptr + G::kOffSc);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int N = p.N;
    const int nf = (N + G::kBM - 1) / G::kBM;
    const int BHn = static_cast<int>(gridDim.x / nf);
    // heaviest fixed tiles first under the causal mask: low key tiles (dV,
    // dK) see the most query blocks, high query tiles (dQ) the most key blocks
    const int ft = (kMode == kModeDQ) ? nf - 1 - static_cast<int>(blockIdx.x / BHn)
                                      : static_cast<int>(blockIdx.x / BHn);
    const int bh = static_cast<int>(blockIdx.x % BHn);
    const int f0 = ft * G::kBM;
    const int nsb = (N + BS - 1) / BS;
    int jb = 0, n = nsb;
    if (p.causal) {
        if (kMode == kModeDQ) {
            n = min(nsb, (min(f0 + G::kBM, N) - 1) / BS + 1);
        } else {
            jb = f0 / BS;
            n = nsb - jb;
        }
    }

    if (threadIdx.x == 0) {
        mbar_init(bar_f, 1);
        mbar_init(bar_flo, 128);
        for (int s = 0; s < G::kStagesA1; ++s) {
            mbar_init(fullA1 + s, 1);
            mbar_init(splitA1 + s, 64);
            mbar_init(emptyA1 + s, 1);
        }
        for (int s = 0; s < G::kStagesA2; ++s) {
            mbar_init(fullA2 + s, 1);
            mbar_init(splitA2 + s, 64);
            mbar_init(emptyA2 + s, 1);
        }
        for (int s = 0; s < G::kStagesT; ++s) {
            mbar_init(fullT + s, 1);
            mbar_init(splitT + s, 64);
            mbar_init(emptyT + s, 1);
        }
        mbar_init(bar_x, 1);
        mbar_init(bar_x + 1, 1);
        mbar_init(bar_w, 128);
        mbar_init(bar_w + 1, 128);
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

    if (warp == 0) {
        // ------------------------------------------------ TMA producer: F, A1, A2
        if (lane == 0 && n > 0) {
            prefetch_tmap(&tmF1);
            if (kTwo) prefetch_tmap(&tmF2);
            prefetch_tmap(&tmS1);
            if (kTwo) prefetch_tmap(&tmS2);
            mbar_arrive_expect_tx(bar_f, G::kFTotal);
            for (int cb = 0; cb < D / 32; ++cb) {
                tma_load_3d(sptr + G::kOffF + cb * G::kFCb, &tmF1, bar_f, cb * 32, f0, bh);
                if (kTwo)
                    tma_load_3d(sptr + G::kOffF + G::kFBytes + cb * G::kFCb, &tmF2, bar_f,
                                cb * 32, f0, bh);
            }
            int issued1 = 0, issued2 = 0;
            for (int t = 0; t < n; ++t) {
                const int row = (jb + t) * BS;
                const int s1 = t % G::kStagesA1;
                if (t >= G::kStagesA1 &&
                    !bf32_wait(emptyA1 + s1, ((t / G::kStagesA1) & 1) ^ 1, abort_flag))
                    break;
                uint8_t* a1 = sptr + G::kOffA1 + s1 * G::kPair;
                mbar_arrive_expect_tx(fullA1 + s1, G::kSBytes);
                for (int cb = 0; cb < D / 32; ++cb)
                    tma_load_3d(a1 + cb * G::kACb, &tmS1, fullA1 + s1, cb * 32, row, bh);
                ++issued1;
                if constexpr (kTwo) {
                    const int s2 = t % G::kStagesA2;
                    if (t >= G::kStagesA2 &&
                        !bf32_wait(emptyA2 + s2, ((t / G::kStagesA2) & 1) ^ 1, abort_flag))
                        break;
                    uint8_t* a2 = sptr + G::kOffA2 + s2 * G::kPair;
                    mbar_arrive_expect_tx(fullA2 + s2, G::kSBytes);
                    for (int cb = 0; cb < D / 32; ++cb)
                        tma_load_3d(a2 + cb * G::kACb, &tmS2, fullA2 + s2, cb * 32, row, bh);
                    ++issued2;
                }
            }
            // no TMA may be in flight when the CTA exits
            volatile int never = 0;
            mbar_wait(bar_f, 0, &never, &g_bf32_status);
            for (int t = max(0, issued1 - G::kStagesA1); t < issued1; ++t)
                mbar_wait(fullA1 + t % G::kStagesA1, (t / G::kStagesA1) & 1, &never,
                          &g_bf32_status);
            if constexpr (kTwo)
                for (int t = max(0, issued2 - G::kStagesA2); t < issued2; ++t)
                    mbar_wait(fullA2 + t % G::kStagesA2, (t / G::kStagesA2) & 1, &never,
                              &g_bf32_status);
        }
    } else if (warp == 2) {
        // ------------------------------------------------ TMA producer: T
        if (lane == 0 && n > 0) {
            const CUtensorMap* src = kTwo ? &tmS1 : &tmS2;
            prefetch_tmap(src);
            int issued = 0;
            for (int t = 0; t < n; ++t) {
                const int s = t % G::kStagesT;
                if (t >= G::kStagesT &&
                    !bf32_wait(emptyT + s, ((t / G::kStagesT) & 1) ^ 1, abort_flag))
                    break;
                uint8_t* tt = sptr + G::kOffT + s * G::kPair;
                mbar_arrive_expect_tx(fullT + s, G::kSBytes);
                for (int cb = 0; cb < D / 32; ++cb)
                    tma_load_3d(tt + cb * G::kSCb, src, fullT + s, cb * 32, (jb + t) * BS, bh);
                ++issued;
            }
            volatile int never = 0;
            for (int t = max(0, issued - G::kStagesT); t < issued; ++t)
                mbar_wait(fullT + t % G::kStagesT, (t / G::kStagesT) & 1, &never, &g_bf32_status);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_x1 = make_idesc(kFmtTF32, 128, BS, false, false);
            constexpr uint32_t idesc_x2 = make_idesc(kFmtTF32, 128, 2 * BS, false, false);
            constexpr uint32_t idesc_acc = make_idesc(kFmtTF32, 128, D, false, false);
            const uint32_t sF1 = sbase + G::kOffF;
            const uint32_t sF2 = sF1 + G::kFBytes;
            // one 3xTF32 product of a resident tile (A) with a ring A slot:
            // F [S; S_lo]^T in one N = 2 kBS MMA per k-step (a tf32 MMA costs
            // about the same below N = 64 as at N = 64), then F_lo S^T into
            // the second half
            auto product = [&](uint32_t d_t, uint32_t sF, uint32_t f_lo, uint32_t slot) {
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk)
                    mma_tf32_ss(d_t, f32_kdesc(sF, kk, G::kFCb), f32_kdesc(slot, kk, G::kACb),
                                idesc_x2, kk > 0 ? 1u : 0u);
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk)
                    mma_tf32_ts(d_t + BS, f_lo + kk * 8, f32_kdesc(slot, kk, G::kACb), idesc_x1,
                                1u);
            };
            auto ready = [&](uint64_t* full, uint64_t* split, int stages, int t) {
                const int s = t % stages;
                const uint32_t ph = (t / stages) & 1;
                return bf32_wait(full + s, ph, abort_flag) && bf32_wait(split + s, ph, abort_flag);
            };
            // S^T (S) of block t, then (dK, dQ) dP^T (dP); X and Y complete on bar_x
            auto issue_x = [&](int t) -> bool {
                if (!ready(fullA1, splitA1, G::kStagesA1, t)) return false;
                tc_fence_after();
                const int s1 = t % G::kStagesA1;
                product(tmem + G::kColX + (kTwo ? 0 : (t & 1) * 2 * BS), sF1, tmem + G::kColF1lo,
                        sbase + G::kOffA1 + s1 * G::kPair);
                tc_commit(emptyA1 + s1);
                if constexpr (kTwo) {
                    if (!ready(fullA2, splitA2, G::kStagesA2, t)) return false;
                    tc_fence_after();
                    const int s2 = t % G::kStagesA2;
                    product(tmem + G::kColY, sF2, tmem + G::kColF2lo,
                            sbase + G::kOffA2 + s2 * G::kPair);
                    tc_commit(emptyA2 + s2);
                }
                tc_commit(bar_x + (kTwo ? 0 : (t & 1)));
                return true;
            };
            bool ok = n > 0 && bf32_wait(bar_f, 0, abort_flag) && bf32_wait(bar_flo, 0, abort_flag);
            if (ok && !kTwo) ok = issue_x(0);  // dV: S^T(t+1) runs behind the softmax of t
            for (int t = 0; ok && t < n; ++t) {
                if constexpr (kTwo) {
                    if (!issue_x(t)) break;
                } else if (t + 1 < n) {
                    if (!issue_x(t + 1)) break;
                }
                const int sT = t % G::kStagesT;
                const uint32_t wpar = kTwo ? (t & 1) : ((t >> 1) & 1);
                if (!bf32_wait(bar_w + (kTwo ? 0 : (t & 1)), wpar, abort_flag) ||
                    !ready(fullT, splitT, G::kStagesT, t))
                    break;
                tc_fence_after();
                const uint32_t sTh = sbase + G::kOffT + sT * G::kPair;
                const uint32_t sTl = sTh + G::kSBytes;
                const uint32_t a_w = tmem + G::kColX + (kTwo ? 0 : (t & 1) * 2 * BS);
                const uint32_t a_wlo = a_w + BS;
                const uint32_t d_acc = tmem + G::kColAcc;
#pragma unroll
                for (int kk = 0; kk < BS / 8; ++kk)
                    mma_tf32_ts(d_acc, a_w + kk * 8, f32_kdesc(sTh, kk, G::kTCb), idesc_acc,
                                (t > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
                for (int kk = 0; kk < BS / 8; ++kk)
                    mma_tf32_ts(d_acc, a_w + kk * 8, f32_kdesc(sTl, kk, G::kTCb), idesc_acc, 1u);
#pragma unroll
                for (int kk = 0; kk < BS / 8; ++kk)
                    mma_tf32_ts(d_acc, a_wlo + kk * 8, f32_kdesc(sTh, kk, G::kTCb), idesc_acc, 1u);
                tc_commit(emptyT + sT);
            }
            tc_commit(bar_done);
            volatile int never = 0;
            mbar_wait(bar_done, 0, &never, &g_bf32_status);
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------ element-wise / epilogue
        const int wq = warp & 3;
        const int r = wq * 32 + lane;
        const int row = f0 + r;
        const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
        const float c = p.scale_log2;
        const size_t rowbase = static_cast<size_t>(bh) * N;
        float nl2_row = 0.f, dv_row = 0.f;
        if (kMode == kModeDQ && row < N) {
            nl2_row = -p.L[rowbase + row] * kLog2eB;
            dv_row = p.Dv[rowbase + row];
        }
        bool ok = true;
        for (int t = 0; t < n; ++t) {
            const int xb = kTwo ? 0 : (t & 1);
            const uint32_t xpar = kTwo ? (t & 1) : ((t >> 1) & 1);
            const int sT = t % G::kStagesT;
            const bool got = bf32_wait(bar_x + xb, xpar, abort_flag) &&
                             bf32_wait(splitT + sT, (t / G::kStagesT) & 1, abort_flag);
            // warp-uniform, for the .sync.aligned TMEM accesses below
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float* sc = sc_all + sT * 2 * BS;  // [-L log2e][D] per column
            const int col0 = (jb + t) * BS;
            const uint32_t t_x = tmem + lane_addr + G::kColX + xb * 2 * BS;
            const uint32_t t_y = tmem + lane_addr + G::kColY;
#pragma unroll
            for (int ch = 0; ch < BS / 16; ++ch) {
                uint32_t xh[16], xl[16], yh[16], yl[16];
                tmem_ld2_x16_nw(t_x + ch * 16, xh, t_x + BS + ch * 16, xl);
                if constexpr (kTwo) tmem_ld2_x16_nw(t_y + ch * 16, yh, t_y + BS + ch * 16, yl);
                tmem_wait_ld2_x16(xh, xl);
                if constexpr (kTwo) tmem_wait_ld2_x16(yh, yl);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int col = col0 + ch * 16 + i;
                    bool vis = col < N;
                    if (p.causal) vis = vis && (kMode == kModeDQ ? col <= row : col >= row);
                    const float nl2 = (kMode == kModeDQ) ? nl2_row : sc[ch * 16 + i];
                    const float x = __uint_as_float(xh[i]) + __uint_as_float(xl[i]);
                    const float pr = vis ? ex2_approx(fmaf(x, c, nl2)) : 0.f;
                    float w = pr;
                    if constexpr (kTwo) {
                        const float dv = (kMode == kModeDQ) ? dv_row : sc[BS + ch * 16 + i];
                        w = pr * (__uint_as_float(yh[i]) + __uint_as_float(yl[i]) - dv);
                    }
                    xh[i] = __float_as_uint(w);
                    xl[i] = __float_as_uint(tf32_lo(w));
                }
                tmem_st_x16_nw(t_x + ch * 16, xh);
                tmem_st_x16_nw(t_x + BS + ch * 16, xl);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar_w + xb);
        }
        if (ok && n > 0) {
            ok = bf32_wait(bar_done, 0, abort_flag);
            tc_fence_after();
        }
        ok = __all_sync(0xffffffffu, ok) && n > 0;
        float* dst = p.out + (rowbase + row) * D;
#pragma unroll
        for (int cb = 0; cb < D / 32; ++cb) {
            uint32_t o[32];
            if (ok) {  // warp-uniform
                tmem_ld_x32(tmem + lane_addr + G::kColAcc + cb * 32, o);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] = 0u;
            }
            if (row < N) {
                float4* d4 = reinterpret_cast<float4*>(dst + cb * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    d4[i] = make_float4(__uint_as_float(o[4 * i]) * p.out_scale,
                                        __uint_as_float(o[4 * i + 1]) * p.out_scale,
                                        __uint_as_float(o[4 * i + 2]) * p.out_scale,
                                        __uint_as_float(o[4 * i + 3]) * p.out_scale);
            }
        }
    } else if (warp >= 8) {
        // ------------------------------------------------ lo parts / transposes
        const int wq = warp & 3;
        const int r = wq * 32 + lane;
        const bool group_t = warp >= 10;
        const int tg = (threadIdx.x - 256) & 63;  // thread index within the group
        bool ok = n > 0 && bf32_wait(bar_f, 0, abort_flag);
        ok = group_t ? group_all<2>(ok) : group_all<1>(ok);
        if (ok) {
            // lo parts of the resident tiles, rows of this warp's TMEM lanes
            const uint32_t t_lane = tmem + (static_cast<uint32_t>(wq * 32) << 16);
            split_rows_to_tmem<D>(sptr + G::kOffF, t_lane + G::kColF1lo, r);
            if constexpr (kTwo)
                split_rows_to_tmem<D>(sptr + G::kOffF + G::kFBytes, t_lane + G::kColF2lo, r);
            tc_fence_before();
            mbar_arrive(bar_flo);
        }
        if (!group_t) {
            // lo parts of ring A1 (and A2), element-wise in place of the layout
            for (int t = 0; ok && t < n; ++t) {
                const int s1 = t % G::kStagesA1;
                if (!group_all<1>(bf32_wait(fullA1 + s1, (t / G::kStagesA1) & 1, abort_flag)))
                    break;
                split_lo_stacked<BS, D>(sptr + G::kOffA1 + s1 * G::kPair, tg);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(splitA1 + s1);
                if constexpr (kTwo) {
                    const int s2 = t % G::kStagesA2;
                    if (!group_all<1>(
                            bf32_wait(fullA2 + s2, (t / G::kStagesA2) & 1, abort_flag)))
                        break;
                    split_lo_stacked<BS, D>(sptr + G::kOffA2 + s2 * G::kPair, tg);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive(splitA2 + s2);
                }
            }
        } else {
            // ring T: [kBS][D] as loaded -> [D][kBS] in place, and its lo part
            const size_t rowbase = static_cast<size_t>(bh) * N;
            for (int t = 0; ok && t < n; ++t) {
                // the block's per-column scalars, loaded ahead of the wait
                float nl2 = 0.f, dv = 0.f;
                const int col = (jb + t) * BS + tg;
                if (kMode != kModeDQ && tg < BS && col < N) {
                    nl2 = -p.L[rowbase + col] * kLog2eB;
                    if (kTwo) dv = p.Dv[rowbase + col];
                }
                const int s = t % G::kStagesT;
                if (!group_all<2>(bf32_wait(fullT + s, (t / G::kStagesT) & 1, abort_flag))) break;
                uint8_t* tt = sptr + G::kOffT + s * G::kPair;
                float4 rr[G::kTBlocks][4];
#pragma unroll
                for (int b = 0; b < G::kTBlocks; ++b) {
                    int i, j;
                    diag_block<BS>(tg + 64 * b, i, j);
                    const int d0 = 4 * j;
#pragma unroll
                    for (int a = 0; a < 4; ++a) {
                        const int row = 4 * i + a;
                        rr[b][a] = *reinterpret_cast<const float4*>(
                            tt + (d0 >> 5) * G::kSCb + row * 128 +
                            ((((d0 & 31) >> 2) ^ (row & 7)) << 4));
                    }
                }
                group_sync<2>();  // every read of the tile before any write
#pragma unroll
                for (int b = 0; b < G::kTBlocks; ++b) {
                    int i, j;
                    diag_block<BS>(tg + 64 * b, i, j);
                    const int r0 = 4 * i, d0 = 4 * j;
                    const float cols[4][4] = {{rr[b][0].x, rr[b][1].x, rr[b][2].x, rr[b][3].x},
                                              {rr[b][0].y, rr[b][1].y, rr[b][2].y, rr[b][3].y},
                                              {rr[b][0].z, rr[b][1].z, rr[b][2].z, rr[b][3].z},
                                              {rr[b][0].w, rr[b][1].w, rr[b][2].w, rr[b][3].w}};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int d = d0 + c;
                        const int off =
                            (r0 >> 5) * G::kTCb + d * 128 + ((((r0 & 31) >> 2) ^ (d & 7)) << 4);
                        *reinterpret_cast<float4*>(tt + off) =
                            make_float4(cols[c][0], cols[c][1], cols[c][2], cols[c][3]);
                        *reinterpret_cast<float4*>(tt + G::kSBytes + off) =
                            make_float4(tf32_lo(cols[c][0]), tf32_lo(cols[c][1]),
                                        tf32_lo(cols[c][2]), tf32_lo(cols[c][3]));
                    }
                }
                if (tg < BS) {
                    float* sc = sc_all + s * 2 * BS;
                    sc[tg] = nl2;
                    sc[BS + tg] = dv;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(splitT + s);
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

// D_i = rowsum(dO_i * O_i), one warp per row.
template <int D>
__global__ void __launch_bounds__(256)
    bwd_f32_dvec_kernel(const float* __restrict__ O, const float* __restrict__ dO,
                        float* __restrict__ Dv, long long rows) {
    const int lane = threadIdx.x & 31;
    const long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < D / 32; ++e) acc = fmaf(O[r * D + lane + 32 * e], dO[r * D + lane + 32 * e], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) Dv[r] = acc;
}

template <int D, int kMode>
FlashAttentionError launch_mode(const CUtensorMap& f1, const CUtensorMap& f2,
                                const CUtensorMap& s1, const CUtensorMap& s2, const float* L,
                                const float* Dv, float* out, int BH, int N, float scale,
                                bool causal, cudaStream_t stream) {
    using G = BF32Geom<D, kMode>;
    auto kern = fa_bwd_f32_kernel<D, kMode>;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(kern), G::kSmemBytes))
        return FlashAttentionError::CUDA_ERROR;
    BF32Params prm;
    prm.L = L;
    prm.Dv = Dv;
    prm.out = out;
    prm.N = N;
    prm.causal = causal ? 1 : 0;
    prm.scale_log2 = scale * kLog2eB;
    prm.out_scale = kMode == kModeDV ? 1.f : scale;
    const long long nf = (N + G::kBM - 1) / G::kBM;
    bind_status_word(reinterpret_cast<const void*>(&g_bf32_status), stream);
    kern<<<dim3(static_cast<unsigned>(nf * BH)), 384, G::kSmemBytes, stream>>>(f1, f2, s1, s2,
                                                                             prm);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

template <int D>
FlashAttentionError bwd_f32_typed(const float* Q, const float* K, const float* V, const float* O,
                                  const float* L, const float* dO, float* dQ, float* dK, float* dV,
                                  int BH, int N, float scale, bool causal, cudaStream_t stream) {
    constexpr int BS = BF32Geom<D, kModeDV>::kBS;
    const long long rows = static_cast<long long>(BH) * N;
    if (((static_cast<long long>(N) + 127) / 128) * BH > 0x7fffffffLL)
        return FlashAttentionError::INVALID_DIMENSION;
    for (const void* ptr : {static_cast<const void*>(dQ), static_cast<const void*>(dK),
                            static_cast<const void*>(dV)})
        if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return FlashAttentionError::CUDA_ERROR;
    const auto f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
    CUtensorMap q128, k128, v128, do128, qs, ks, vs, dos;
    if (!encode_tmap_3d(&q128, Q, f32, 4, D, N, BH, 32, 128, sw) ||
        !encode_tmap_3d(&k128, K, f32, 4, D, N, BH, 32, 128, sw) ||
        !encode_tmap_3d(&v128, V, f32, 4, D, N, BH, 32, 128, sw) ||
        !encode_tmap_3d(&do128, dO, f32, 4, D, N, BH, 32, 128, sw) ||
        !encode_tmap_3d(&qs, Q, f32, 4, D, N, BH, 32, BS, sw) ||
        !encode_tmap_3d(&ks, K, f32, 4, D, N, BH, 32, BS, sw) ||
        !encode_tmap_3d(&vs, V, f32, 4, D, N, BH, 32, BS, sw) ||
        !encode_tmap_3d(&dos, dO, f32, 4, D, N, BH, 32, BS, sw))
        return FlashAttentionError::CUDA_ERROR;
    void* ws = nullptr;
    FlashAttentionError e =
        workspace_alloc(&ws, static_cast<size_t>(rows) * sizeof(float), stream);
    if (e != FlashAttentionError::SUCCESS) return e;
    float* dvec = static_cast<float*>(ws);
    bwd_f32_dvec_kernel<D><<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, stream>>>(
        O, dO, dvec, rows);
    e = cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                          : FlashAttentionError::CUDA_ERROR;
    // The three gradients are independent: dV and dK run on side streams
    // next to dQ on the caller's stream (a small problem fills the GPU three
    // times over instead of once), joined back before the workspace is freed.
    // Under stream capture everything stays on the caller's stream.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStream_t s_dv = stream, s_dk = stream;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    bool fork = e == FlashAttentionError::SUCCESS &&
                cudaStreamIsCapturing(stream, &cap) == cudaSuccess &&
                cap == cudaStreamCaptureStatusNone;
    if (fork) {
        s_dv = side_stream(0);
        s_dk = side_stream(1);
        fork = s_dv != nullptr && s_dk != nullptr;
        for (int i = 0; fork && i < 3; ++i)
            fork = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) == cudaSuccess;
        fork = fork && cudaEventRecord(ev[0], stream) == cudaSuccess &&
               cudaStreamWaitEvent(s_dv, ev[0], 0) == cudaSuccess &&
               cudaStreamWaitEvent(s_dk, ev[0], 0) == cudaSuccess;
        if (!fork) {
            s_dv = stream;
            s_dk = stream;
        }
    }
    if (e == FlashAttentionError::SUCCESS)
        e = launch_mode<D, kModeDV>(k128, k128, qs, dos, L, dvec, dV, BH, N, scale, causal, s_dv);
    if (e == FlashAttentionError::SUCCESS)
        e = launch_mode<D, kModeDK>(k128, v128, qs, dos, L, dvec, dK, BH, N, scale, causal, s_dk);
    if (e == FlashAttentionError::SUCCESS)
        e = launch_mode<D, kModeDQ>(q128, do128, ks, vs, L, dvec, dQ, BH, N, scale, causal, stream);
    if (fork) {
        // joined whatever happened above, so nothing of this call outlives it
        // on a side stream
        const bool joined = cudaEventRecord(ev[1], s_dv) == cudaSuccess &&
                            cudaEventRecord(ev[2], s_dk) == cudaSuccess &&
                            cudaStreamWaitEvent(stream, ev[1], 0) == cudaSuccess &&
                            cudaStreamWaitEvent(stream, ev[2], 0) == cudaSuccess;
        if (!joined) {
            cudaStreamSynchronize(s_dv);
            cudaStreamSynchronize(s_dk);
            if (e == FlashAttentionError::SUCCESS) e = FlashAttentionError::CUDA_ERROR;
        }
    }
    for (cudaEvent_t x : ev)
        if (x != nullptr) cudaEventDestroy(x);
    workspace_free(ws, stream);
    return e;
}

}  // namespace

FlashAttentionError launch_bwd_f32(const float* Q, const float* K, const float* V,
                                   const float* O, const float* L, const float* dO, float* dQ,
                                   float* dK, float* dV, int B, int H, int N, int D, float scale,
                                   bool causal, cudaStream_t stream) {
    const int BH = B * H;
    switch (D) {
        case 32:
            return bwd_f32_typed<32>(Q, K, V, O, L, dO, dQ, dK, dV, BH, N, scale, causal, stream);
        case 64:
            return bwd_f32_typed<64>(Q, K, V, O, L, dO, dQ, dK, dV, BH, N, scale, causal, stream);
        case 128:
            return bwd_f32_typed<128>(Q, K, V, O, L, dO, dQ, dK, dV, BH, N, scale, causal, stream);
        default:
            return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
}

int bwd_f32_sm100_status() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_bf32_status, sizeof(int)) != cudaSuccess) return -1;
    if (v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_bf32_status, &zero, sizeof(int));
    }
    return v;
}

}  // namespace detail
}  // namespace cuflash
