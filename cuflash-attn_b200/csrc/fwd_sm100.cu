// Forward attention for fp16/bf16 on sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the reference's forward kernels
//   src/forward/flash_attention_forward_wmma.cu:30-207   (fp16/bf16, WMMA)
//   src/forward/flash_attention_forward_typed.cu:16-152   (scalar fallback)
// with the same math: O = softmax(scale * Q K^T [+ causal mask]) V and
// L = rowmax + log(rowsum) of the scaled scores (natural log), P rounded to
// the input dtype before the PV product (flash_attention_forward_wmma.cu:152),
// fp32 accumulation, O rounded to nearest on store (type_adapter.cuh:24-32).
//
// CTA = 256 query rows of one (batch, head) = two 128-row tiles.
//   warp 0      TMA producer: Q tiles once, then K/V blocks of 128 rows
//               through a 2-stage ring (full/empty mbarriers).
//   warp 1      TMEM allocator and tcgen05.mma issuer (one thread).
//   warps 4-7   softmax for tile 0, warps 8-11 softmax for tile 1; one
//               thread per query row (= one TMEM lane).
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [384,384+D).
// P (fp16/bf16) is written back into the first 64 columns of S_t and used as
// the TMEM A operand of O_t += P V.  The two tiles ping-pong: while the
// softmax warps work on tile 0, the tensor pipe runs tile 1's MMAs.
//
// Online softmax works in the log2 domain (x = s * scale * log2 e) and only
// rescales O when a row maximum grows by more than 2^8; otherwise the stale
// maximum is kept (exact in real arithmetic, bounded growth of P in fp32).
//
// Causal: kv blocks entirely above the diagonal are skipped, the diagonal
// block is masked element-wise; CTAs are launched heaviest first.

#include <cmath>

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {

__device__ int g_fwd_status;

constexpr float kRescaleThreshold = 8.0f;  // log2 units
// With kExp2EmuEvery = k > 0, one pair of exponentials in k is computed on the
// FMA pipe (exp2_poly2) instead of the MUFU unit.  Measured on B200 at
// config 3 it does not pay (MUFU is not the binding limit), so it is off.
#ifndef CUFLASH_FWD_EXP2_EMU_EVERY
#define CUFLASH_FWD_EXP2_EMU_EVERY 0
#endif
constexpr int kExp2EmuEvery = CUFLASH_FWD_EXP2_EMU_EVERY;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct FwdGeom {
    static constexpr int kRows = 128;
    static constexpr int kRowBytes = D * 2;
    static constexpr int kSwz = kRowBytes >= 128 ? 128 : kRowBytes;  // 128 or 64 bytes
    static constexpr int kCbElems = kSwz / 2;                         // elements per column block
    static constexpr int kNumCb = D / kCbElems;
    static constexpr int kCbBytes = kRows * kSwz;
    static constexpr int kTileBytes = kRows * kRowBytes;
    static constexpr int kStages = 2;
    static constexpr uint32_t kLayout = kSwz == 128 ? sm100::kLayoutSw128 : sm100::kLayoutSw64;
    static constexpr int kOffQ = 0;
    static constexpr int kOffK = 2 * kTileBytes;
    static constexpr int kOffV = kOffK + kStages * kTileBytes;
    static constexpr int kOffBar = kOffV + kStages * kTileBytes;
    static constexpr int kNumBars = 1 + 4 * kStages + 2 + 2 + 2 + 1;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
};

struct FwdParams {
    void* O;
    float* L;
    int seq_q;
    int seq_k;
    int num_ctiles;
    int causal;
    float scale_log2;
    long long q_offset;
    long long k_offset;
};

// K-major operand (rows x D, D contiguous) for k-step kk (16 elements).
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_base, int kk) {
    using G = FwdGeom<D>;
    const uint32_t byte = static_cast<uint32_t>(kk) * 32u;
    const uint32_t addr = tile_base + (byte / G::kSwz) * G::kCbBytes + (byte % G::kSwz);
    return sm100::make_smem_desc(addr, 16, 8 * G::kSwz, G::kLayout);
}

// MN-major operand (kv rows = K dimension, D contiguous = N dimension) for
// k-step kk (16 kv rows).
template <int D>
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile_base, int kk) {
    using G = FwdGeom<D>;
    const uint32_t addr = tile_base + static_cast<uint32_t>(kk) * 16u * G::kSwz;
    return sm100::make_smem_desc(addr, G::kCbBytes, 8 * G::kSwz, G::kLayout);
}

// Warp-uniform bounded wait.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    // Every lane polls the barrier itself: all lanes observe the same phase,
    // timer and abort flag, so the warp stays converged without a shuffle.
    return sm100::mbar_wait(bar, parity, abort_flag, &g_fwd_status);
}

// Wait used by the producer at exit to make sure its TMA writes have landed;
// ignores the abort flag but is still bounded in time.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    volatile int never = 0;
    sm100::mbar_wait(bar, parity, &never, &g_fwd_status);
}

template <typename T, int D, bool kF32Out>
__global__ void __launch_bounds__(384, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
    using G = FwdGeom<D>;
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];

    if (*reinterpret_cast<volatile int*>(&g_fwd_status) != 0) return;

    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
    uint8_t* sptr = smem_raw + (sbase - raw_addr);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sptr + G::kOffBar);
    uint64_t* bar_q = bars;
    uint64_t* full_k = bars + 1;
    uint64_t* empty_k = full_k + G::kStages;
    uint64_t* full_v = empty_k + G::kStages;
    uint64_t* empty_v = full_v + G::kStages;
    uint64_t* bar_s = empty_v + G::kStages;
    uint64_t* bar_p = bar_s + 2;
    uint64_t* bar_o = bar_p + 2;
    uint64_t* bar_done = bar_o + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // (q tile, b*h) grid with q tiles fastest: the CTAs running at the same
    // time share few (b,h), so their K/V blocks are reused from L2.
    const int bh = blockIdx.y;
    const int ct = p.num_ctiles - 1 - static_cast<int>(blockIdx.x);
    const int q_row0 = ct * 256;

    // kv blocks needed by each 128-row tile
    const int nkv_all = (p.seq_k + 127) / 128;
    int n_t[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const int r_lo = q_row0 + t * 128;
        if (r_lo >= p.seq_q) {
            n_t[t] = 0;
        } else if (!p.causal) {
            n_t[t] = nkv_all;
        } else {
            const int r_hi = min(r_lo + 127, p.seq_q - 1);
            const long long lim = p.q_offset + r_hi - p.k_offset;  // largest visible local key
            const long long nb = lim / 128 + 1;
            n_t[t] = lim < 0 ? 0 : (nb < nkv_all ? static_cast<int>(nb) : nkv_all);
        }
    }
    const int n_max = max(n_t[0], n_t[1]);

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        for (int s = 0; s < G::kStages; ++s) {
            mbar_init(full_k + s, 1);
            mbar_init(empty_k + s, 1);
            mbar_init(full_v + s, 1);
            mbar_init(empty_v + s, 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(bar_s + t, 1);
            mbar_init(bar_p + t, 128);
            mbar_init(bar_o + t, 1);
        }
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

    // Registers: launched with 168 per thread (384 x 168 = 64512); warpgroup 0
    // (producer, MMA, 2 idle warps) gives back down to 56 and the two softmax
    // warpgroups take 216 each: 128*56 + 256*216 = 62464 <= 64512.
    if (warp < 4) {
        setmaxnreg_dec<56>();
    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0 && n_max > 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            const int ntiles_loaded = (n_t[0] > 0 ? 1 : 0) + (n_t[1] > 0 ? 1 : 0);
            mbar_arrive_expect_tx(bar_q, ntiles_loaded * G::kTileBytes);
            for (int t = 0; t < 2; ++t) {
                if (n_t[t] == 0) continue;
                for (int cb = 0; cb < G::kNumCb; ++cb)
                    tma_load_3d(sptr + G::kOffQ + t * G::kTileBytes + cb * G::kCbBytes, &tmQ,
                                bar_q, cb * G::kCbElems, q_row0 + t * 128, bh);
            }
            int issued_k = 0, issued_v = 0;
            for (int j = 0; j < n_max; ++j) {
                const int s = j % G::kStages;
                const uint32_t ph = (j / G::kStages) & 1;
                if (j >= G::kStages && !mbar_wait(empty_k + s, ph ^ 1, abort_flag, &g_fwd_status))
                    break;
                mbar_arrive_expect_tx(full_k + s, G::kTileBytes);
                for (int cb = 0; cb < G::kNumCb; ++cb)
                    tma_load_3d(sptr + G::kOffK + s * G::kTileBytes + cb * G::kCbBytes, &tmK,
                                full_k + s, cb * G::kCbElems, j * 128, bh);
                ++issued_k;
                if (j >= G::kStages && !mbar_wait(empty_v + s, ph ^ 1, abort_flag, &g_fwd_status))
                    break;
                mbar_arrive_expect_tx(full_v + s, G::kTileBytes);
                for (int cb = 0; cb < G::kNumCb; ++cb)
                    tma_load_3d(sptr + G::kOffV + s * G::kTileBytes + cb * G::kCbBytes, &tmV,
                                full_v + s, cb * G::kCbElems, j * 128, bh);
                ++issued_v;
            }
            // every issued load must land before the CTA can exit
            drain_wait(bar_q, 0);
            for (int j = max(0, issued_k - G::kStages); j < issued_k; ++j)
                drain_wait(full_k + j % G::kStages, (j / G::kStages) & 1);
            for (int j = max(0, issued_v - G::kStages); j < issued_v; ++j)
                drain_wait(full_v + j % G::kStages, (j / G::kStages) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0 && n_max > 0) {
            constexpr uint32_t idesc_qk = make_idesc(DType<T>::kMmaFmt, 128, 128, false, false);
            constexpr uint32_t idesc_pv = make_idesc(DType<T>::kMmaFmt, 128, D, false, true);
            auto issue_qk = [&](int t, int s) {
                const uint32_t d_tmem = tmem + t * 128;
                const uint32_t a_base = sbase + G::kOffQ + t * G::kTileBytes;
                const uint32_t b_base = sbase + G::kOffK + s * G::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    mma_f16_ss(d_tmem, kmajor_desc<D>(a_base, kk), kmajor_desc<D>(b_base, kk),
                               idesc_qk, kk > 0 ? 1u : 0u);
            };
            auto issue_pv = [&](int t, int s, bool acc) {
                const uint32_t d_tmem = tmem + 256 + t * 128;
                const uint32_t p_tmem = tmem + t * 128;
                const uint32_t v_base = sbase + G::kOffV + s * G::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < 128 / 16; ++kk)
                    mma_f16_ts(d_tmem, p_tmem + kk * 8, mnmajor_desc<D>(v_base, kk), idesc_pv,
                               (acc || kk > 0) ? 1u : 0u);
            };
            bool ok = mbar_wait(bar_q, 0, abort_flag, &g_fwd_status) &&
                      mbar_wait(full_k, 0, abort_flag, &g_fwd_status);
            if (ok) {
                tc_fence_after();
                for (int t = 0; t < 2; ++t) {
                    if (n_t[t] > 0) {
                        issue_qk(t, 0);
                        tc_commit(bar_s + t);
                    }
                }
                tc_commit(empty_k);
            }
            for (int j = 0; ok && j < n_max; ++j) {
                const int s = j % G::kStages;
                const uint32_t ph = (j / G::kStages) & 1;
                if (!mbar_wait(full_v + s, ph, abort_flag, &g_fwd_status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int jn = j + 1;
                const int sn = jn % G::kStages;
                const uint32_t phn = (jn / G::kStages) & 1;
                bool k_next_ready = false;
                for (int t = 0; t < 2 && ok; ++t) {
                    if (j >= n_t[t]) continue;
                    if (!mbar_wait(bar_p + t, j & 1, abort_flag, &g_fwd_status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv(t, s, j > 0);
                    if (j == n_t[t] - 1) tc_commit(bar_o + t);
                    if (jn < n_t[t]) {
                        if (!k_next_ready) {
                            if (!mbar_wait(full_k + sn, phn, abort_flag, &g_fwd_status)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            k_next_ready = true;
                        }
                        issue_qk(t, sn);
                        tc_commit(bar_s + t);
                    }
                }
                if (!ok) break;
                tc_commit(empty_v + s);
                if (k_next_ready) tc_commit(empty_k + sn);
            }
            // all MMAs (and their commits) retire before teardown
            tc_commit(bar_done);
            volatile int never = 0;
            mbar_wait(bar_done, 0, &never, &g_fwd_status);
        }
        __syncwarp();
    }
    } else {
        setmaxnreg_inc<216>();
        // ------------------------------------------------ softmax / epilogue
        const int t = (warp - 4) >> 2;
        const int wq = warp & 3;
        const int r = wq * 32 + lane;
        const int row = q_row0 + t * 128 + r;
        const long long grow = p.q_offset + row;
        const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t s_tmem = tmem + lane_addr + t * 128;
        const uint32_t o_tmem = tmem + lane_addr + 256 + t * 128;
        const int n = n_t[t];
        const float c = p.scale_log2;
        const long long tile_g0 = p.q_offset + q_row0 + t * 128;

        float m_run = -INFINITY;
        float l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < n; ++j) {
            if (!warp_wait(bar_s + t, j & 1, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sr[128];
            tmem_ld_x128(s_tmem, sr);
            const int col0 = j * 128;
            const bool need_mask = (col0 + 128 > p.seq_k) ||
                                   (p.causal && (p.k_offset + col0 + 127 > tile_g0));
            if (need_mask) {
                // largest visible local key column for this row (32-bit safe)
                const long long lim64 = grow - p.k_offset;
                const int lim = p.causal ? static_cast<int>(lim64 < -1 ? -1 : (lim64 > 0x7fffffff ? 0x7fffffff : lim64))
                                         : 0x7fffffff;
                const int vis_end = min(p.seq_k - 1, lim) - col0;  // visible iff i <= vis_end
#pragma unroll
                for (int i = 0; i < 128; ++i)
                    if (i > vis_end) sr[i] = __float_as_uint(-INFINITY);
            }
            // row maximum: 3-input max over four independent chains
            float mx;
            {
                float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
                for (int i = 0; i < 128; i += 8) {
                    m0 = fmax3(m0, __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
                    m1 = fmax3(m1, __uint_as_float(sr[i + 2]), __uint_as_float(sr[i + 3]));
                    m2 = fmax3(m2, __uint_as_float(sr[i + 4]), __uint_as_float(sr[i + 5]));
                    m3 = fmax3(m3, __uint_as_float(sr[i + 6]), __uint_as_float(sr[i + 7]));
                }
                mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)) * c;  // c > 0
            }
            // Decide the new running maximum; O is rescaled after P is stored so
            // that the score registers are dead by then.
            float alpha = 1.f;
            bool need = false;
            if (j == 0) {
                m_run = mx;
            } else {
                need = mx > m_run + kRescaleThreshold;
                if (need) {
                    alpha = ex2_approx(m_run - mx);
                    m_run = mx;
                }
            }
            const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
            const uint64_t c2 = f2_pack(c, c);
            const uint64_t nm2 = f2_pack(-m_use, -m_use);
            uint64_t acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;  // (0.f, 0.f) pairs
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t pk[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int c0 = h * 64 + 2 * i;
                    const float2 x = f2_unpack(
                        f2_fma(f2_pack(__uint_as_float(sr[c0]), __uint_as_float(sr[c0 + 1])), c2, nm2));
                    float p0, p1;
                    if (kExp2EmuEvery > 0 && (i % kExp2EmuEvery) == kExp2EmuEvery - 1) {
                        const float2 e = exp2_poly2(x.x, x.y);  // FMA pipe
                        p0 = e.x;
                        p1 = e.y;
                    } else {
                        p0 = ex2_approx(x.x);  // MUFU
                        p1 = ex2_approx(x.y);
                    }
                    const uint64_t pp = f2_pack(p0, p1);
                    switch (i & 3) {
                        case 0: acc0 = f2_add(acc0, pp); break;
                        case 1: acc1 = f2_add(acc1, pp); break;
                        case 2: acc2 = f2_add(acc2, pp); break;
                        default: acc3 = f2_add(acc3, pp); break;
                    }
                    pk[i] = DType<T>::pack2(p0, p1);
                }
                tmem_st_x32(s_tmem + h * 32, pk);
            }
            float sum;
            {
                const float2 a = f2_unpack(f2_add(f2_add(acc0, acc1), f2_add(acc2, acc3)));
                sum = a.x + a.y;
            }
            l_run = l_run * alpha + sum;
            // PV_{j-1} has completed: S_t(j) was issued after it and its commit
            // covers every earlier tcgen05 operation.
            if (__any_sync(0xffffffffu, need)) {
#pragma unroll
                for (int cb = 0; cb < D / 32; ++cb) {
                    uint32_t o[32];
                    tmem_ld_x32(o_tmem + cb * 32, o);
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st_x32(o_tmem + cb * 32, o);
                }
            }
            tc_fence_before();
            mbar_arrive(bar_p + t);
        }

        // epilogue
        if (n > 0 && ok) {
            ok = warp_wait(bar_o + t, 0, abort_flag);
            tc_fence_after();
        }
        const bool valid_row = row < p.seq_q;
        const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
        const size_t row_elem = (static_cast<size_t>(bh) * p.seq_q + row) * D;
#pragma unroll
        for (int cb = 0; cb < D / 32; ++cb) {
            uint32_t o[32];
            if (n > 0 && ok) {
                tmem_ld_x32(o_tmem + cb * 32, o);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] = 0u;
            }
            if (valid_row) {
                if constexpr (kF32Out) {
                    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.O) + row_elem +
                                                            cb * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv_l,
                                             __uint_as_float(o[4 * i + 1]) * inv_l,
                                             __uint_as_float(o[4 * i + 2]) * inv_l,
                                             __uint_as_float(o[4 * i + 3]) * inv_l);
                } else {
                    uint4* dst =
                        reinterpret_cast<uint4*>(static_cast<T*>(p.O) + row_elem + cb * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint4 v;
                        v.x = DType<T>::pack2(__uint_as_float(o[8 * i + 0]) * inv_l,
                                              __uint_as_float(o[8 * i + 1]) * inv_l);
                        v.y = DType<T>::pack2(__uint_as_float(o[8 * i + 2]) * inv_l,
                                              __uint_as_float(o[8 * i + 3]) * inv_l);
                        v.z = DType<T>::pack2(__uint_as_float(o[8 * i + 4]) * inv_l,
                                              __uint_as_float(o[8 * i + 5]) * inv_l);
                        v.w = DType<T>::pack2(__uint_as_float(o[8 * i + 6]) * inv_l,
                                              __uint_as_float(o[8 * i + 7]) * inv_l);
                        dst[i] = v;
                    }
                }
            }
        }
        if (valid_row) {
            p.L[static_cast<size_t>(bh) * p.seq_q + row] =
                l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <typename T, int D, bool kF32Out>
FlashAttentionError launch_typed(const T* Q, const T* K, const T* V, void* O, float* L, int BH,
                                 int seq_q, int seq_k, float scale, bool causal,
                                 long long q_offset, long long k_offset, cudaStream_t stream) {
    using G = FwdGeom<D>;
    const CUtensorMapSwizzle swz =
        G::kSwz == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUtensorMap mq, mk, mv;
    if (!encode_tmap_3d(&mq, Q, DType<T>::kTmaType, 2, D, seq_q, BH, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mk, K, DType<T>::kTmaType, 2, D, seq_k, BH, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mv, V, DType<T>::kTmaType, 2, D, seq_k, BH, G::kCbElems, 128, swz))
        return FlashAttentionError::CUDA_ERROR;
    auto kern = fa_fwd_kernel<T, D, kF32Out>;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(kern), G::kSmemBytes))
        return FlashAttentionError::CUDA_ERROR;
    FwdParams prm;
    prm.O = O;
    prm.L = L;
    prm.seq_q = seq_q;
    prm.seq_k = seq_k;
    prm.num_ctiles = (seq_q + 255) / 256;
    prm.causal = causal ? 1 : 0;
    // A zero scale is replaced by a tiny positive one so that masked scores
    // (-inf) still map to -inf; the effect on results is below fp32 resolution.
    prm.scale_log2 = fmaxf(scale * kLog2e, 1e-30f);
    prm.q_offset = q_offset;
    prm.k_offset = k_offset;
    if (BH > 65535) return FlashAttentionError::CUDA_ERROR;
    dim3 grid(static_cast<unsigned>(prm.num_ctiles), static_cast<unsigned>(BH));
    kern<<<grid, 384, G::kSmemBytes, stream>>>(mq, mk, mv, prm);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

template <typename T, bool kF32Out>
FlashAttentionError dispatch_d(const T* Q, const T* K, const T* V, void* O, float* L, int BH,
                               int seq_q, int seq_k, int D, float scale, bool causal,
                               long long q_offset, long long k_offset, cudaStream_t stream) {
    switch (D) {
        case 32:
            return launch_typed<T, 32, kF32Out>(Q, K, V, O, L, BH, seq_q, seq_k, scale, causal,
                                                q_offset, k_offset, stream);
        case 64:
            return launch_typed<T, 64, kF32Out>(Q, K, V, O, L, BH, seq_q, seq_k, scale, causal,
                                                q_offset, k_offset, stream);
        case 128:
            return launch_typed<T, 128, kF32Out>(Q, K, V, O, L, BH, seq_q, seq_k, scale, causal,
                                                 q_offset, k_offset, stream);
        default:
            return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
}

}  // namespace

template <typename T>
FlashAttentionError launch_fwd_sm100(const T* Q, const T* K, const T* V, void* O, float* L, int B,
                                     int H, int seq_q, int seq_k, int D, float scale, bool causal,
                                     long long q_offset, long long k_offset, bool out_f32_partial,
                                     cudaStream_t stream) {
    const int BH = B * H;
    if (out_f32_partial)
        return dispatch_d<T, true>(Q, K, V, O, L, BH, seq_q, seq_k, D, scale, causal, q_offset,
                                   k_offset, stream);
    return dispatch_d<T, false>(Q, K, V, O, L, BH, seq_q, seq_k, D, scale, causal, q_offset,
                                k_offset, stream);
}

template FlashAttentionError launch_fwd_sm100<__nv_bfloat16>(const __nv_bfloat16*,
                                                             const __nv_bfloat16*,
                                                             const __nv_bfloat16*, void*, float*,
                                                             int, int, int, int, int, float, bool,
                                                             long long, long long, bool,
                                                             cudaStream_t);
template FlashAttentionError launch_fwd_sm100<half>(const half*, const half*, const half*, void*,
                                                    float*, int, int, int, int, int, float, bool,
                                                    long long, long long, bool, cudaStream_t);

int fwd_sm100_status() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_fwd_status, sizeof(int)) != cudaSuccess) return -1;
    if (v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_fwd_status, &zero, sizeof(int));
    }
    return v;
}

}  // namespace detail
}  // namespace cuflash
