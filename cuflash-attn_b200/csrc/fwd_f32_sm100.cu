// Forward attention for fp32 inputs on sm_100a tensor cores, 3xTF32.
//
// Replaces the reference's fp32 forward (src/forward/flash_attention_forward_
// typed.cu:16-152, scalar FP32 FMA) with tcgen05 kind::tf32 MMAs held to fp32
// accuracy by the three-term split of each product (the published "3xTF32"
// technique: a*b ~ hi(a)hi(b) + hi(a)lo(b) + lo(a)hi(b) with hi = the tf32
// part the tensor core reads from an fp32 word and lo = a - hi exactly
// representable in fp32; the dropped lo*lo term is ~2^-22 relative).
//
// The tensor core uses the upper 19 bits of each fp32 operand, so "hi" is the
// raw fp32 tile itself; only the lo parts are materialised:
//   S  = Q K^T  = (Q, K) + (Q, K_lo) + (Q_lo, K)
//   O += P V    = (P, V) + (P, V_lo) + (P_lo, V)
// CTA = 128 query rows of one (b,h); 384 threads:
//   warp 0      TMA producer (Q once; K, V blocks of kBN rows, 2-4 stages)
//   warp 1      TMEM allocator, MMA issuer
//   warps 4-7   softmax, one thread per query row (TMEM lane); writes P and
//               P_lo into TMEM (A operands of the PV products)
//   warps 8-11  splitter: Q_lo into TMEM (A operand); per stage K_lo
//               (element-wise over the swizzled buffer, which keeps its
//               layout) and V^T, V^T_lo: V transposed into a K-major tile so
//               that every tf32 operand is K-major (an MN-major tf32 operand
//               would need the 32-byte-atom swizzle)
// S(j+1) is issued before PV(j), so the tensor pipe works on the next block
// while the softmax of the current one runs (S/P double-buffered in TMEM).
// A kind::tf32 MMA costs about the same at N = 32 or 64 as at N = 64, so a
// tile and its lo part are stacked along N: every 128-byte column block of a
// stage holds K's rows then K_lo's rows (and V^T's rows then V^T_lo's), one
// MMA per k-step computes Q [K; K_lo]^T into 2 kBN TMEM columns (Q_lo K^T
// accumulates into the second half, the softmax adds the halves), and at
// head_dim <= 64 likewise P [V^T; V^T_lo]^T into two O halves.

#include <cmath>

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {

__device__ sm100::StatusWord g_f32_status;

constexpr float kLn2F = 0.6931471805599453f;
constexpr float kLog2eF = 1.4426950408889634f;
constexpr float kRescaleF = 8.0f;

template <int D>
struct F32Geom {
    static constexpr int kBM = 128;
    static constexpr int kBN = (D == 128) ? 32 : 64;
    static constexpr int kNumCb = D / 32;           // 128-byte column blocks (32 fp32)
    static constexpr int kQCbBytes = kBM * 128;
    static constexpr int kQBytes = kBM * D * 4;
    static constexpr int kKvCbBytes = kBN * 128;      // V as loaded: kBN rows per block
    static constexpr int kKvBytes = kBN * D * 4;
    static constexpr int kKkCbBytes = 2 * kBN * 128;  // [K; K_lo] column block
    static constexpr int kOffQ = 0;
    static constexpr int kOffStage = kQBytes;
    // [K; K_lo] (2 kKvBytes), then [V^T; V^T_lo] (2 kKvBytes), whose first
    // half receives V as loaded and is transposed in place
    static constexpr int kStageBytes = 4 * kKvBytes;
    static constexpr int kOffVt = 2 * kKvBytes;
    static constexpr int kStagesFit = (232448 - 2048 - kQBytes) / kStageBytes;
    static constexpr int kStagesMain = kStagesFit > 4 ? 4 : kStagesFit;
    static_assert(kStagesMain >= 2, "K/V ring depth");
    // head_dim 128: Q's hi part goes to TMEM next to Q_lo (the S product takes
    // both A operands from TMEM), and Q's shared-memory region, one stage in
    // size, serves as a further stage once the splitter has copied Q out
    static constexpr bool kQInTmem = D == 128;
    static constexpr int kStages = kStagesMain + (kQInTmem ? 1 : 0);
    static_assert(!kQInTmem || kStageBytes == kQBytes, "Q region as a stage");
    static constexpr int kVBlocks = (kBN / 4) * (D / 4) / 128;  // 4x4 blocks per splitter thread
    static_assert(kVBlocks * 128 == (kBN / 4) * (D / 4), "transpose split");
    static constexpr int kVtCbBytes = 2 * D * 128;  // 32 kv of D V^T rows, then D V^T_lo rows
    static constexpr int kOffBar = kOffStage + kStagesMain * kStageBytes;
    static constexpr int kNumBars = 2 + 3 * kStages + 2 + 2 + 1;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16;
    static constexpr bool kStackPV = D <= 64;       // P [V^T; V^T_lo]^T in one MMA
    static constexpr int kOCols = kStackPV ? 2 * D : D;
    // TMEM columns
    static constexpr int kColS = 0;                 // [2][2 kBN]: S halves, then P | P_lo
    static constexpr int kColO = 4 * kBN;           // kOCols (O, or its two halves)
    static constexpr int kColQlo = kColO + kOCols;  // D
    static constexpr int kColQhi = kColQlo + D;     // D (head_dim 128)
    static_assert((kQInTmem ? kColQhi : kColQlo) + D <= 512, "TMEM budget");
    __host__ __device__ static constexpr int stage_off(int s) {
        return s < kStagesMain ? kOffStage + s * kStageBytes : kOffQ;
    }
};

struct F32Params {
    float* O;
    float* L;
    int N;
    int causal;
    float scale_log2;
};

// AND vote over the 128 splitter threads (warps 8-11) on named barrier 1, so
// that they all take the same branch after a wait: the barrier inside the
// splitter loop must never miss a participant.
__device__ __forceinline__ bool splitter_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, 1, 128, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(r)
        : "r"(v ? 1u : 0u)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ bool f32_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    return sm100::mbar_wait(bar, parity, abort_flag, &g_f32_status);
}

template <int D>
__global__ void __launch_bounds__(384, 1)
    fa_fwd_f32_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const F32Params p) {
    using G = F32Geom<D>;
    using namespace sm100;
    constexpr int BN = G::kBN;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (sm100::cta_skip(&g_f32_status)) return;
    const uint32_t sbase = smem_u32(smem_raw);
    if ((sbase & 1023u) != 0) {
        if (threadIdx.x == 0) sm100::record_status(&g_f32_status, sm100::kStatusMisaligned);
        return;
    }
    uint8_t* sptr = smem_raw;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sptr + G::kOffBar);
    uint64_t* bar_q = bars;
    uint64_t* bar_qlo = bars + 1;
    uint64_t* full = bars + 2;
    uint64_t* split = full + G::kStages;
    uint64_t* empty = split + G::kStages;
    uint64_t* bar_s = empty + G::kStages;  // [2]
    uint64_t* bar_p = bar_s + 2;           // P ready (count 128)
    uint64_t* bar_o = bar_p + 1;           // one completion per PV block
    uint64_t* bar_done = bar_o + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nq = (p.N + G::kBM - 1) / G::kBM;
    // one-dimensional grid, query tile major: every (b,h)'s heaviest tile first
    const int BHn = static_cast<int>(gridDim.x / nq);
    const int qt = nq - 1 - static_cast<int>(blockIdx.x / BHn);
    const int bh = static_cast<int>(blockIdx.x % BHn);
    const int q0 = qt * G::kBM;
    const int row_hi = min(q0 + G::kBM, p.N) - 1;
    const int nkv_all = (p.N + BN - 1) / BN;
    const int n = p.causal ? min(nkv_all, row_hi / BN + 1) : nkv_all;

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        mbar_init(bar_qlo, 128);
        for (int s = 0; s < G::kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(split + s, 128);
            mbar_init(empty + s, 1);
        }
        mbar_init(bar_s, 1);
        mbar_init(bar_s + 1, 1);
        mbar_init(bar_p, 128);
        mbar_init(bar_o, 1);
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
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            mbar_arrive_expect_tx(bar_q, G::kQBytes);
            for (int cb = 0; cb < G::kNumCb; ++cb)
                tma_load_3d(sptr + G::kOffQ + cb * G::kQCbBytes, &tmQ, bar_q, cb * 32, q0, bh);
            int issued = 0;
            for (int j = 0; j < n; ++j) {
                const int s = j % G::kStages;
                if (j >= G::kStages &&
                    !mbar_wait(empty + s, ((j / G::kStages) & 1) ^ 1, abort_flag, &g_f32_status))
                    break;
                // the stage in Q's region: only once Q is in TMEM
                if (G::kQInTmem && j == G::kStagesMain &&
                    !mbar_wait(bar_qlo, 0, abort_flag, &g_f32_status))
                    break;
                uint8_t* st = sptr + G::stage_off(s);
                mbar_arrive_expect_tx(full + s, 2 * G::kKvBytes);
                for (int cb = 0; cb < G::kNumCb; ++cb) {
                    tma_load_3d(st + cb * G::kKkCbBytes, &tmK, full + s, cb * 32, j * BN, bh);
                    tma_load_3d(st + G::kOffVt + cb * G::kKvCbBytes, &tmV, full + s, cb * 32,
                                j * BN, bh);
                }
                ++issued;
            }
            volatile int never = 0;
            mbar_wait(bar_q, 0, &never, &g_f32_status);
            for (int j = max(0, issued - G::kStages); j < issued; ++j)
                mbar_wait(full + j % G::kStages, (j / G::kStages) & 1, &never, &g_f32_status);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = make_idesc(kFmtTF32, 128, BN, false, false);
            constexpr uint32_t idesc_s2 = make_idesc(kFmtTF32, 128, 2 * BN, false, false);
            constexpr uint32_t idesc_pv = make_idesc(kFmtTF32, 128, D, false, false);
            constexpr uint32_t idesc_pv2 = make_idesc(kFmtTF32, 128, G::kOCols, false, false);
            const uint32_t sQ = sbase + G::kOffQ;
            auto issue_s = [&](int j) {
                const int s = j % G::kStages;
                const uint32_t sK = sbase + G::stage_off(s);
                const uint32_t d_t = tmem + G::kColS + (j & 1) * 2 * BN;
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk) {
                    if constexpr (G::kQInTmem)
                        mma_tf32_ts(d_t, tmem + G::kColQhi + kk * 8,
                                    f32_kdesc(sK, kk, G::kKkCbBytes), idesc_s2, kk > 0 ? 1u : 0u);
                    else
                        mma_tf32_ss(d_t, f32_kdesc(sQ, kk, G::kQCbBytes),
                                    f32_kdesc(sK, kk, G::kKkCbBytes), idesc_s2, kk > 0 ? 1u : 0u);
                }
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk)
                    mma_tf32_ts(d_t + BN, tmem + G::kColQlo + kk * 8,
                                f32_kdesc(sK, kk, G::kKkCbBytes), idesc_s, 1u);
                tc_commit(bar_s + (j & 1));
            };
            auto stage_ready = [&](int j) {
                const int s = j % G::kStages;
                const uint32_t ph = (j / G::kStages) & 1;
                return mbar_wait(full + s, ph, abort_flag, &g_f32_status) &&
                       mbar_wait(split + s, ph, abort_flag, &g_f32_status);
            };
            bool ok = n > 0 && mbar_wait(bar_q, 0, abort_flag, &g_f32_status) &&
                      mbar_wait(bar_qlo, 0, abort_flag, &g_f32_status) && stage_ready(0);
            if (ok) {
                tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; ok && j < n; ++j) {
                if (j + 1 < n) {
                    if (!stage_ready(j + 1)) break;
                    tc_fence_after();
                    issue_s(j + 1);
                }
                if (!mbar_wait(bar_p, j & 1, abort_flag, &g_f32_status)) break;
                tc_fence_after();
                const int s = j % G::kStages;
                const uint32_t sVt = sbase + G::stage_off(s) + G::kOffVt;
                const uint32_t a_p = tmem + G::kColS + (j & 1) * 2 * BN;
                const uint32_t a_plo = a_p + BN;
                if constexpr (G::kStackPV) {
                    // O | O_lo += P [V^T; V^T_lo]^T, then O_lo += P_lo V^T
#pragma unroll
                    for (int kk = 0; kk < BN / 8; ++kk)
                        mma_tf32_ts(tmem + G::kColO, a_p + kk * 8,
                                    f32_kdesc(sVt, kk, G::kVtCbBytes), idesc_pv2,
                                    (j > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
                    for (int kk = 0; kk < BN / 8; ++kk)
                        mma_tf32_ts(tmem + G::kColO + D, a_plo + kk * 8,
                                    f32_kdesc(sVt, kk, G::kVtCbBytes), idesc_pv, 1u);
                } else {
#pragma unroll
                    for (int kk = 0; kk < BN / 8; ++kk)
                        mma_tf32_ts(tmem + G::kColO, a_p + kk * 8,
                                    f32_kdesc(sVt, kk, G::kVtCbBytes), idesc_pv,
                                    (j > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
                    for (int kk = 0; kk < BN / 8; ++kk)
                        mma_tf32_ts(tmem + G::kColO, a_p + kk * 8,
                                    f32_kdesc(sVt + D * 128, kk, G::kVtCbBytes), idesc_pv, 1u);
#pragma unroll
                    for (int kk = 0; kk < BN / 8; ++kk)
                        mma_tf32_ts(tmem + G::kColO, a_plo + kk * 8,
                                    f32_kdesc(sVt, kk, G::kVtCbBytes), idesc_pv, 1u);
                }
                tc_commit(bar_o);
                tc_commit(empty + s);
            }
            tc_commit(bar_done);
            volatile int never = 0;
            mbar_wait(bar_done, 0, &never, &g_f32_status);
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------ softmax / epilogue
        const int wq = warp & 3;
        const int r = wq * 32 + lane;
        const int row = q0 + r;
        const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
        const float c = p.scale_log2;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < n; ++j) {
            if (!f32_wait(bar_s + (j & 1), (j >> 1) & 1, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t t_s = tmem + lane_addr + G::kColS + (j & 1) * 2 * BN;
            const uint32_t t_plo = t_s + BN;
            uint32_t sr[BN];
            {
                // S = Q K^T + (Q K_lo^T + Q_lo K^T): the two halves of the block
                uint32_t sl[BN];
                if constexpr (BN == 64) {
                    tmem_ld_x64(t_s, sr);
                    tmem_ld_x64(t_plo, sl);
                } else {
                    tmem_ld2_x32(t_s, *reinterpret_cast<uint32_t(*)[32]>(sr), t_plo,
                                 *reinterpret_cast<uint32_t(*)[32]>(sl));
                }
#pragma unroll
                for (int i = 0; i < BN; ++i)
                    sr[i] = __float_as_uint(__uint_as_float(sr[i]) + __uint_as_float(sl[i]));
            }
            const int col0 = j * BN;
            const int vis_end = (p.causal ? min(row, p.N - 1) : p.N - 1) - col0;
            if (vis_end < BN - 1) {
#pragma unroll
                for (int i = 0; i < BN; ++i)
                    if (i > vis_end) sr[i] = __float_as_uint(-INFINITY);
            }
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < BN; ++i) mx = fmaxf(mx, __uint_as_float(sr[i]));
            mx *= c;
            float alpha = 1.f;
            if (j == 0) {
                m_run = mx;
            } else {
                // PV(j-1) must have finished before O is touched (S(j) was
                // issued ahead of it); every PV completion is observed in order
                if (!f32_wait(bar_o, (j - 1) & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const bool need = mx > m_run + kRescaleF;
                if (need) {
                    alpha = ex2_approx(m_run - mx);
                    m_run = mx;
                }
                if (__any_sync(0xffffffffu, need)) {
                    const uint32_t t_o = tmem + lane_addr + G::kColO;
#pragma unroll
                    for (int cb = 0; cb < G::kOCols / 32; ++cb) {
                        uint32_t o[32];
                        tmem_ld_x32(t_o + cb * 32, o);
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st_x32(t_o + cb * 32, o);
                    }
                }
            }
            const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
            float sum = 0.f;
            uint32_t lo[BN];
#pragma unroll
            for (int i = 0; i < BN; ++i) {
                const float pv = ex2_approx(fmaf(__uint_as_float(sr[i]), c, -m_use));
                sum += pv;
                sr[i] = __float_as_uint(pv);
                lo[i] = __float_as_uint(tf32_lo(pv));
            }
            l_run = l_run * alpha + sum;
            if constexpr (BN == 64) {
                uint32_t (&a)[32] = *reinterpret_cast<uint32_t(*)[32]>(sr);
                uint32_t (&b)[32] = *reinterpret_cast<uint32_t(*)[32]>(sr + 32);
                uint32_t (&la)[32] = *reinterpret_cast<uint32_t(*)[32]>(lo);
                uint32_t (&lb)[32] = *reinterpret_cast<uint32_t(*)[32]>(lo + 32);
                tmem_st_x32_nw(t_s, a);
                tmem_st_x32_nw(t_s + 32, b);
                tmem_st_x32_nw(t_plo, la);
                tmem_st_x32_nw(t_plo + 32, lb);
            } else {
                tmem_st_x32_nw(t_s, *reinterpret_cast<uint32_t(*)[32]>(sr));
                tmem_st_x32_nw(t_plo, *reinterpret_cast<uint32_t(*)[32]>(lo));
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar_p);
        }
        if (ok && n > 0) {
            ok = f32_wait(bar_o, (n - 1) & 1, abort_flag);
            tc_fence_after();
        }
        const bool valid = row < p.N;
        const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
        float* dst = p.O + (static_cast<size_t>(bh) * p.N + row) * D;
#pragma unroll
        for (int cb = 0; cb < D / 32; ++cb) {
            uint32_t o[32];
            if (ok && n > 0) {
                tmem_ld_x32(tmem + lane_addr + G::kColO + cb * 32, o);
                if constexpr (G::kStackPV) {
                    uint32_t o2[32];
                    tmem_ld_x32(tmem + lane_addr + G::kColO + D + cb * 32, o2);
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        o[i] = __float_as_uint(__uint_as_float(o[i]) + __uint_as_float(o2[i]));
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] = 0u;
            }
            if (valid) {
                float4* d4 = reinterpret_cast<float4*>(dst + cb * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    d4[i] = make_float4(__uint_as_float(o[4 * i]) * inv_l,
                                        __uint_as_float(o[4 * i + 1]) * inv_l,
                                        __uint_as_float(o[4 * i + 2]) * inv_l,
                                        __uint_as_float(o[4 * i + 3]) * inv_l);
            }
        }
        if (valid)
            p.L[static_cast<size_t>(bh) * p.N + row] =
                l_run > 0.f ? (m_run + log2f(l_run)) * kLn2F : -INFINITY;
    } else if (warp >= 8) {
        // ------------------------------------------------ splitter
        const int t = threadIdx.x - 256;  // 0..127
        const int wq = warp & 3;
        const int r = wq * 32 + lane;
        bool ok = splitter_all(n > 0 && f32_wait(bar_q, 0, abort_flag));
        if (ok) {
            // Q_lo of row r into TMEM (A operand of the (Q_lo, K) product),
            // and at head_dim 128 Q itself (A operand of Q [K; K_lo]^T)
            const uint8_t* sQ = sptr + G::kOffQ;
            const uint32_t t_q = tmem + (static_cast<uint32_t>(wq * 32) << 16) + G::kColQlo;
#pragma unroll
            for (int cb = 0; cb < D / 32; ++cb) {
                uint32_t v[32], h[32];
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    const float4 x = *reinterpret_cast<const float4*>(
                        sQ + cb * G::kQCbBytes + r * 128 + ((ch ^ (r & 7)) << 4));
                    v[4 * ch] = __float_as_uint(tf32_lo(x.x));
                    v[4 * ch + 1] = __float_as_uint(tf32_lo(x.y));
                    v[4 * ch + 2] = __float_as_uint(tf32_lo(x.z));
                    v[4 * ch + 3] = __float_as_uint(tf32_lo(x.w));
                    h[4 * ch] = __float_as_uint(x.x);
                    h[4 * ch + 1] = __float_as_uint(x.y);
                    h[4 * ch + 2] = __float_as_uint(x.z);
                    h[4 * ch + 3] = __float_as_uint(x.w);
                }
                tmem_st_x32(t_q + cb * 32, v);
                if constexpr (G::kQInTmem) tmem_st_x32(t_q + D + cb * 32, h);
            }
            tc_fence_before();
            // head_dim 128: the producer refills Q's region by TMA after this
            // arrival, so the reads above are ordered before those writes
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(bar_qlo);
        }
        for (int j = 0; ok && j < n; ++j) {
            const int s = j % G::kStages;
            if (!splitter_all(f32_wait(full + s, (j / G::kStages) & 1, abort_flag))) break;
            uint8_t* st = sptr + G::stage_off(s);
            // K_lo: element-wise, into the rows below K's in each column block
            // (same swizzle phase, so the layout is preserved)
            float4* k4 = reinterpret_cast<float4*>(st);
            for (int i = t; i < G::kKvBytes / 16; i += 128) {
                const int src = (i / (BN * 8)) * (BN * 16) + i % (BN * 8);
                const float4 a = k4[src];
                k4[src + BN * 8] =
                    make_float4(tf32_lo(a.x), tf32_lo(a.y), tf32_lo(a.z), tf32_lo(a.w));
            }
            // V^T and V^T_lo, in place: V as loaded is [kv][d] (32-float,
            // 128-byte swizzled column blocks of kBN rows) in the first half of
            // the region; V^T is [d][kv], 32-kv column blocks of D V^T rows and
            // D V^T_lo rows.  Every thread reads its 4x4 blocks, then all write.
            uint8_t* vt = st + G::kOffVt;
            float4 rr[G::kVBlocks][4];
#pragma unroll
            for (int b = 0; b < G::kVBlocks; ++b) {
                int bi, bj;
                diag_block<BN>(t + 128 * b, bi, bj);
                const int d0 = bj * 4;
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const int kv = bi * 4 + a;
                    rr[b][a] = *reinterpret_cast<const float4*>(
                        vt + (d0 >> 5) * G::kKvCbBytes + kv * 128 +
                        ((((d0 & 31) >> 2) ^ (kv & 7)) << 4));
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
            for (int b = 0; b < G::kVBlocks; ++b) {
                int bi, bj;
                diag_block<BN>(t + 128 * b, bi, bj);
                const int kv0 = bi * 4, d0 = bj * 4;
                const float cols[4][4] = {{rr[b][0].x, rr[b][1].x, rr[b][2].x, rr[b][3].x},
                                          {rr[b][0].y, rr[b][1].y, rr[b][2].y, rr[b][3].y},
                                          {rr[b][0].z, rr[b][1].z, rr[b][2].z, rr[b][3].z},
                                          {rr[b][0].w, rr[b][1].w, rr[b][2].w, rr[b][3].w}};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int d = d0 + c;
                    const int off = (kv0 >> 5) * G::kVtCbBytes + d * 128 +
                                    ((((kv0 & 31) >> 2) ^ (d & 7)) << 4);
                    *reinterpret_cast<float4*>(vt + off) =
                        make_float4(cols[c][0], cols[c][1], cols[c][2], cols[c][3]);
                    *reinterpret_cast<float4*>(vt + D * 128 + off) =
                        make_float4(tf32_lo(cols[c][0]), tf32_lo(cols[c][1]),
                                    tf32_lo(cols[c][2]), tf32_lo(cols[c][3]));
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(split + s);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <int D>
FlashAttentionError fwd_f32_typed(const float* Q, const float* K, const float* V, float* O,
                                  float* L, int BH, int N, float scale, bool causal,
                                  cudaStream_t stream) {
    using G = F32Geom<D>;
    CUtensorMap mq, mk, mv;
    if (!encode_tmap_3d(&mq, Q, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, N, BH, 32, G::kBM,
                        CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap_3d(&mk, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, N, BH, 32, G::kBN,
                        CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap_3d(&mv, V, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, N, BH, 32, G::kBN,
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return FlashAttentionError::CUDA_ERROR;
    if ((reinterpret_cast<uintptr_t>(O) & 15u) != 0) return FlashAttentionError::CUDA_ERROR;
    auto kern = fa_fwd_f32_kernel<D>;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(kern), G::kSmemBytes))
        return FlashAttentionError::CUDA_ERROR;
    const int nq = (N + G::kBM - 1) / G::kBM;
    if (static_cast<long long>(nq) * BH > 0x7fffffffLL) return FlashAttentionError::INVALID_DIMENSION;
    F32Params prm;
    prm.O = O;
    prm.L = L;
    prm.N = N;
    prm.causal = causal ? 1 : 0;
    prm.scale_log2 = fmaxf(scale * kLog2eF, 1e-30f);
    bind_status_word(reinterpret_cast<const void*>(&g_f32_status), stream);
    kern<<<dim3(static_cast<unsigned>(static_cast<long long>(nq) * BH)), 384, G::kSmemBytes,
           stream>>>(mq, mk, mv, prm);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

}  // namespace

FlashAttentionError launch_fwd_f32(const float* Q, const float* K, const float* V, float* O,
                                   float* L, int B, int H, int N, int D, float scale, bool causal,
                                   cudaStream_t stream) {
    const int BH = B * H;
    switch (D) {
        case 32: return fwd_f32_typed<32>(Q, K, V, O, L, BH, N, scale, causal, stream);
        case 64: return fwd_f32_typed<64>(Q, K, V, O, L, BH, N, scale, causal, stream);
        case 128: return fwd_f32_typed<128>(Q, K, V, O, L, BH, N, scale, causal, stream);
        default: return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
}

int f32_sm100_status() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_f32_status, sizeof(int)) != cudaSuccess) return -1;
    if (v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_f32_status, &zero, sizeof(int));
    }
    return v;
}

}  // namespace detail
}  // namespace cuflash
