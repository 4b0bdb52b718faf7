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
// Roles (384 threads):
//   warp 0      TMA producer: the resident tiles F1 (and F2) once, then per
//               block the streamed tiles S1, S2 into ring A
//   warp 1      TMEM allocator, MMA issuer
//   warps 4-7   element-wise stage (one thread per resident row) and the
//               epilogue
//   warps 8-11  splitter: lo parts of F1/F2 into TMEM; per block the lo
//               parts of S1 (and S2) in place of the ring A layout, and the
//               transposed operand of the accumulation (dO^T for dV, Q^T for
//               dK, K^T for dQ) with its lo part into ring T, plus the
//               per-column scalars -L*log2(e) and D
// Every tf32 operand is K-major (an MN-major tf32 operand would need the
// 32-byte-atom swizzle), hence the transposed copies.

#include <cmath>

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {

__device__ int g_bf32_status;

constexpr float kLog2eB = 1.4426950408889634f;

enum : int { kModeDV = 0, kModeDK = 1, kModeDQ = 2 };

template <int D, int kMode>
struct BF32Geom {
    static constexpr bool kTwo = kMode != kModeDV;  // second product dP (Y)
    static constexpr int kBM = 128;
    static constexpr int kBS = (D == 128) ? 32 : 64;
    static constexpr int kFBytes = kBM * D * 4;
    static constexpr int kFCb = kBM * 128;
    static constexpr int kSBytes = kBS * D * 4;     // streamed tile [kBS][D]
    static constexpr int kSCb = kBS * 128;
    static constexpr int kTBytes = D * kBS * 4;     // transposed tile [D][kBS]
    static constexpr int kTCb = D * 128;
    static constexpr int kNumF = kTwo ? 2 : 1;
    // ring A: S1, S1_lo, S2 (raw for dV), S2_lo (dK, dQ)
    static constexpr int kATiles = kTwo ? 4 : 3;
    static constexpr int kABytes = kATiles * kSBytes;
    static constexpr int kTStageBytes = 2 * kTBytes;  // T, T_lo
    static constexpr int kTileBudget = 232448 - 2048;
    static constexpr int kFTotal = kNumF * kFBytes;
    static constexpr int kStagesA = (kFTotal + 2 * kABytes + kTStageBytes <= kTileBudget) ? 2 : 1;
    static constexpr int kStagesT =
        (kFTotal + kStagesA * kABytes + 2 * kTStageBytes <= kTileBudget) ? 2 : 1;
    static constexpr int kOffF = 0;
    static constexpr int kOffA = kFTotal;
    static constexpr int kOffT = kOffA + kStagesA * kABytes;
    static constexpr int kOffSc = kOffT + kStagesT * kTStageBytes;  // [kStagesT][2][kBS] floats
    static constexpr int kOffBar = kOffSc + kStagesT * 2 * kBS * 4;
    // bar_f, bar_flo, fullA/splitA/emptyA [kStagesA], splitT/emptyT [kStagesT],
    // bar_x [2], bar_w [2], bar_done
    static constexpr int kNumBars = 2 + 3 * kStagesA + 2 * kStagesT + 2 + 2 + 1;
    static constexpr int kUsed = kOffBar + kNumBars * 8 + 16;
    // at least 116 KB so that one CTA (and its 512 TMEM columns) owns the SM
    static constexpr int kSmemBytes = kUsed > 118784 ? kUsed : 118784;
    static_assert(kUsed <= 232448, "shared memory budget");
    // TMEM columns
    static constexpr int kXBufs = kTwo ? 1 : 2;
    static constexpr int kColF1lo = 0;
    static constexpr int kColF2lo = D;  // dK, dQ
    static constexpr int kColAcc = kNumF * D;
    static constexpr int kColX = kColAcc + D;           // [kXBufs][kBS]; dV: P in place
    static constexpr int kColY = kColX + kXBufs * kBS;  // dK, dQ: dP
    static constexpr int kColW = kTwo ? kColY + kBS : kColX;          // dS (dV: P = X)
    static constexpr int kColWlo = kTwo ? kColW + kBS : kColY;        // [kXBufs][kBS]
    static constexpr int kColEnd = kColWlo + kXBufs * kBS;
    static_assert(kColEnd <= 512, "TMEM budget");
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

// Splitter barrier among warps 8-11.
__device__ __forceinline__ void splitter_sync() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Same barrier with an AND vote, so that all splitter threads take the same
// branch after a wait (the named barrier must never miss a participant).
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

// raw [R][D] (128-byte swizzled column blocks of R rows) -> hi, lo [D][R]
// (128-byte swizzled column blocks of D rows): 4x4 blocks through registers.
template <int R, int D>
__device__ __forceinline__ void split_transpose(const uint8_t* raw, uint8_t* thi, uint8_t* tlo,
                                                int t) {
    using sm100::tf32_lo;
    for (int blk = t; blk < (R / 4) * (D / 4); blk += 128) {
        const int r0 = (blk % (R / 4)) * 4;
        const int d0 = (blk / (R / 4)) * 4;
        float4 rr[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int r = r0 + a;
            rr[a] = *reinterpret_cast<const float4*>(raw + (d0 >> 5) * (R * 128) + r * 128 +
                                                     ((((d0 & 31) >> 2) ^ (r & 7)) << 4));
        }
        const float cols[4][4] = {{rr[0].x, rr[1].x, rr[2].x, rr[3].x},
                                  {rr[0].y, rr[1].y, rr[2].y, rr[3].y},
                                  {rr[0].z, rr[1].z, rr[2].z, rr[3].z},
                                  {rr[0].w, rr[1].w, rr[2].w, rr[3].w}};
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int d = d0 + b;
            const int off =
                (r0 >> 5) * (D * 128) + d * 128 + ((((r0 & 31) >> 2) ^ (d & 7)) << 4);
            *reinterpret_cast<float4*>(thi + off) =
                make_float4(cols[b][0], cols[b][1], cols[b][2], cols[b][3]);
            *reinterpret_cast<float4*>(tlo + off) = make_float4(
                tf32_lo(cols[b][0]), tf32_lo(cols[b][1]), tf32_lo(cols[b][2]), tf32_lo(cols[b][3]));
        }
    }
}

// lo parts over a whole swizzled tile (element-wise, so the layout is kept).
__device__ __forceinline__ void split_lo(const uint8_t* hi, uint8_t* lo, int bytes, int t) {
    using sm100::tf32_lo;
    const float4* h4 = reinterpret_cast<const float4*>(hi);
    float4* l4 = reinterpret_cast<float4*>(lo);
    for (int i = t; i < bytes / 16; i += 128) {
        const float4 a = h4[i];
        l4[i] = make_float4(tf32_lo(a.x), tf32_lo(a.y), tf32_lo(a.z), tf32_lo(a.w));
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
    if (*reinterpret_cast<volatile int*>(&g_bf32_status) != 0) return;
    const uint32_t sbase = smem_u32(smem_raw);
    if ((sbase & 1023u) != 0) {
        if (threadIdx.x == 0) atomicExch(&g_bf32_status, 2);
        return;
    }
    uint8_t* sptr = smem_raw;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sptr + G::kOffBar);
    uint64_t* bar_f = bars;
    uint64_t* bar_flo = bars + 1;
    uint64_t* fullA = bars + 2;
    uint64_t* splitA = fullA + G::kStagesA;
    uint64_t* emptyA = splitA + G::kStagesA;
    uint64_t* splitT = emptyA + G::kStagesA;
    uint64_t* emptyT = splitT + G::kStagesT;
    uint64_t* bar_x = emptyT + G::kStagesT;  // [2]
    // dV keeps two blocks in flight (S^T of the next block is issued before
    // the current accumulation), so its X and W barriers are double: a
    // waiter can then never fall two phases behind on one barrier
    uint64_t* bar_w = bar_x + 2;  // [2]
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
        for (int s = 0; s < G::kStagesA; ++s) {
            mbar_init(fullA + s, 1);
            mbar_init(splitA + s, 128);
            mbar_init(emptyA + s, 2);  // the MMA commit and the splitter
        }
        for (int s = 0; s < G::kStagesT; ++s) {
            mbar_init(splitT + s, 128);
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
        // ------------------------------------------------ TMA producer
        if (lane == 0 && n > 0) {
            prefetch_tmap(&tmF1);
            if (kTwo) prefetch_tmap(&tmF2);
            prefetch_tmap(&tmS1);
            prefetch_tmap(&tmS2);
            mbar_arrive_expect_tx(bar_f, G::kFTotal);
            for (int cb = 0; cb < D / 32; ++cb) {
                tma_load_3d(sptr + G::kOffF + cb * G::kFCb, &tmF1, bar_f, cb * 32, f0, bh);
                if (kTwo)
                    tma_load_3d(sptr + G::kOffF + G::kFBytes + cb * G::kFCb, &tmF2, bar_f,
                                cb * 32, f0, bh);
            }
            int issued = 0;
            for (int t = 0; t < n; ++t) {
                const int s = t % G::kStagesA;
                if (t >= G::kStagesA &&
                    !bf32_wait(emptyA + s, ((t / G::kStagesA) & 1) ^ 1, abort_flag))
                    break;
                uint8_t* st = sptr + G::kOffA + s * G::kABytes;
                const int row = (jb + t) * BS;
                mbar_arrive_expect_tx(fullA + s, 2 * G::kSBytes);
                for (int cb = 0; cb < D / 32; ++cb) {
                    tma_load_3d(st + cb * G::kSCb, &tmS1, fullA + s, cb * 32, row, bh);
                    tma_load_3d(st + 2 * G::kSBytes + cb * G::kSCb, &tmS2, fullA + s, cb * 32, row,
                                bh);
                }
                ++issued;
            }
            // no TMA may be in flight when the CTA exits
            volatile int never = 0;
            mbar_wait(bar_f, 0, &never, &g_bf32_status);
            for (int t = max(0, issued - G::kStagesA); t < issued; ++t)
                mbar_wait(fullA + t % G::kStagesA, (t / G::kStagesA) & 1, &never, &g_bf32_status);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_x = make_idesc(kFmtTF32, 128, BS, false, false);
            constexpr uint32_t idesc_acc = make_idesc(kFmtTF32, 128, D, false, false);
            const uint32_t sF1 = sbase + G::kOffF;
            const uint32_t sF2 = sF1 + G::kFBytes;
            // one 3xTF32 product of a resident tile (A) with a streamed tile (B)
            auto product = [&](uint32_t d_t, uint32_t sF, uint32_t f_lo, uint32_t sS,
                               uint32_t sSlo) {
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk)
                    mma_tf32_ss(d_t, f32_kdesc(sF, kk, G::kFCb), f32_kdesc(sS, kk, G::kSCb), idesc_x,
                                kk > 0 ? 1u : 0u);
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk)
                    mma_tf32_ss(d_t, f32_kdesc(sF, kk, G::kFCb), f32_kdesc(sSlo, kk, G::kSCb),
                                idesc_x, 1u);
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk)
                    mma_tf32_ts(d_t, f_lo + kk * 8, f32_kdesc(sS, kk, G::kSCb), idesc_x, 1u);
            };
            auto a_ready = [&](int t) {
                const int s = t % G::kStagesA;
                const uint32_t ph = (t / G::kStagesA) & 1;
                return bf32_wait(fullA + s, ph, abort_flag) && bf32_wait(splitA + s, ph, abort_flag);
            };
            auto issue_x = [&](int t) {
                const int s = t % G::kStagesA;
                const uint32_t sS1 = sbase + G::kOffA + s * G::kABytes;
                product(tmem + G::kColX + (kTwo ? 0 : (t & 1) * BS), sF1, tmem + G::kColF1lo, sS1,
                        sS1 + G::kSBytes);
                if constexpr (kTwo)
                    product(tmem + G::kColY, sF2, tmem + G::kColF2lo, sS1 + 2 * G::kSBytes,
                            sS1 + 3 * G::kSBytes);
                tc_commit(bar_x + (kTwo ? 0 : (t & 1)));
                tc_commit(emptyA + s);
            };
            bool ok = n > 0 && bf32_wait(bar_f, 0, abort_flag) && bf32_wait(bar_flo, 0, abort_flag);
            if (ok && !kTwo) {  // dV: S^T of the next block runs behind the current softmax
                ok = a_ready(0);
                if (ok) {
                    tc_fence_after();
                    issue_x(0);
                }
            }
            for (int t = 0; ok && t < n; ++t) {
                if constexpr (kTwo) {
                    if (!a_ready(t)) break;
                    tc_fence_after();
                    issue_x(t);
                } else if (t + 1 < n) {
                    if (!a_ready(t + 1)) break;
                    tc_fence_after();
                    issue_x(t + 1);
                }
                const int sT = t % G::kStagesT;
                const uint32_t wpar = kTwo ? (t & 1) : ((t >> 1) & 1);
                if (!bf32_wait(bar_w + (kTwo ? 0 : (t & 1)), wpar, abort_flag) ||
                    !bf32_wait(splitT + sT, (t / G::kStagesT) & 1, abort_flag))
                    break;
                tc_fence_after();
                const uint32_t sTh = sbase + G::kOffT + sT * G::kTStageBytes;
                const uint32_t sTl = sTh + G::kTBytes;
                const uint32_t a_w = tmem + G::kColW + (kTwo ? 0 : (t & 1) * BS);
                const uint32_t a_wlo = tmem + G::kColWlo + (kTwo ? 0 : (t & 1) * BS);
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
#pragma unroll
            for (int ch = 0; ch < BS / 32; ++ch) {
                uint32_t xv[32];
                uint32_t yv[32];
                tmem_ld_x32(tmem + lane_addr + G::kColX + xb * BS + ch * 32, xv);
                if constexpr (kTwo) tmem_ld_x32(tmem + lane_addr + G::kColY + ch * 32, yv);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int col = col0 + ch * 32 + i;
                    bool vis = col < N;
                    if (p.causal) vis = vis && (kMode == kModeDQ ? col <= row : col >= row);
                    const float nl2 = (kMode == kModeDQ) ? nl2_row : sc[ch * 32 + i];
                    const float pr = vis ? ex2_approx(fmaf(__uint_as_float(xv[i]), c, nl2)) : 0.f;
                    float w = pr;
                    if constexpr (kTwo) {
                        const float dv = (kMode == kModeDQ) ? dv_row : sc[BS + ch * 32 + i];
                        w = pr * (__uint_as_float(yv[i]) - dv);
                    }
                    xv[i] = __float_as_uint(w);
                    yv[i] = __float_as_uint(tf32_lo(w));
                }
                tmem_st_x32_nw(tmem + lane_addr + G::kColW + xb * BS + ch * 32, xv);
                tmem_st_x32_nw(tmem + lane_addr + G::kColWlo + xb * BS + ch * 32, yv);
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
        // ------------------------------------------------ splitter
        const int t0 = threadIdx.x - 256;  // 0..127
        const int wq = warp & 3;
        const int r = wq * 32 + lane;
        bool ok = splitter_all(n > 0 && bf32_wait(bar_f, 0, abort_flag));
        if (ok) {
            const uint32_t t_lane = tmem + (static_cast<uint32_t>(wq * 32) << 16);
            split_rows_to_tmem<D>(sptr + G::kOffF, t_lane + G::kColF1lo, r);
            if constexpr (kTwo)
                split_rows_to_tmem<D>(sptr + G::kOffF + G::kFBytes, t_lane + G::kColF2lo, r);
            tc_fence_before();
            mbar_arrive(bar_flo);
        }
        const size_t rowbase = static_cast<size_t>(bh) * N;
        for (int t = 0; ok && t < n; ++t) {
            const int s = t % G::kStagesA;
            if (!splitter_all(bf32_wait(fullA + s, (t / G::kStagesA) & 1, abort_flag))) break;
            uint8_t* st = sptr + G::kOffA + s * G::kABytes;
            split_lo(st, st + G::kSBytes, G::kSBytes, t0);
            if constexpr (kTwo) split_lo(st + 2 * G::kSBytes, st + 3 * G::kSBytes, G::kSBytes, t0);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(splitA + s);
            const int sT = t % G::kStagesT;
            if (!splitter_all(t < G::kStagesT ||
                              bf32_wait(emptyT + sT, ((t / G::kStagesT) & 1) ^ 1, abort_flag)))
                break;
            uint8_t* tt = sptr + G::kOffT + sT * G::kTStageBytes;
            // dV: dO^T (the raw S2); dK, dQ: the S1 operand transposed
            split_transpose<BS, D>(kTwo ? st : st + 2 * G::kSBytes, tt, tt + G::kTBytes, t0);
            if (kMode != kModeDQ && t0 < BS) {
                const int col = (jb + t) * BS + t0;
                float* sc = sc_all + sT * 2 * BS;
                sc[t0] = col < N ? -p.L[rowbase + col] * kLog2eB : 0.f;
                sc[BS + t0] = (kTwo && col < N) ? p.Dv[rowbase + col] : 0.f;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(splitT + sT);
            // ring A slot is free once every splitter thread is done reading it
            splitter_sync();
            if (t0 == 0) mbar_arrive(emptyA + s);
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
    if (e == FlashAttentionError::SUCCESS)
        e = launch_mode<D, kModeDV>(k128, k128, qs, dos, L, dvec, dV, BH, N, scale, causal, stream);
    if (e == FlashAttentionError::SUCCESS)
        e = launch_mode<D, kModeDK>(k128, v128, qs, dos, L, dvec, dK, BH, N, scale, causal, stream);
    if (e == FlashAttentionError::SUCCESS)
        e = launch_mode<D, kModeDQ>(q128, do128, ks, vs, L, dvec, dQ, BH, N, scale, causal, stream);
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
