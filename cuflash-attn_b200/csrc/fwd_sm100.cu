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
// Persistent kernel, one CTA per SM.  A work item is 256 query rows of one
// (batch, head) = two 128-row tiles; each CTA walks a static list of items
// (fwd_item) and keeps its barriers, TMEM and K/V ring across them, so the
// next item's Q loads and first S products overlap the current item's last
// softmax block and epilogue.
//   warp 0      TMA producer: Q tiles per item (once the previous item's
//               last QK on that slot retired), K/V blocks of 128 rows
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

#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {

__device__ sm100::StatusWord g_fwd_status;

constexpr float kRescaleThreshold = 8.0f;  // log2 units
// With kExp2EmuEvery = k > 0, one pair of exponentials in k is computed on the
// FMA pipe (exp2_poly2) instead of the MUFU unit.  Measured on B200 at
// config 3 it does not pay (MUFU is not the binding limit), so it is off.
#ifndef CUFLASH_FWD_EXP2_EMU_EVERY
#define CUFLASH_FWD_EXP2_EMU_EVERY 0
#endif
constexpr int kExp2EmuEvery = CUFLASH_FWD_EXP2_EMU_EVERY;
// P is handed to the MMA warp in two halves of 64 keys: the first half of
// O += P V runs on the tensor pipe while the second half's exponentials are
// computed.
#ifndef CUFLASH_FWD_SPLIT_P
#define CUFLASH_FWD_SPLIT_P 1
#endif
constexpr bool kSplitP = CUFLASH_FWD_SPLIT_P != 0;
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
    static constexpr int kNumBars = 2 + 4 * kStages + 2 + 2 + 2 + 2 + 2 + 1;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
};

struct FwdParams {
    void* O;
    float* L;
    int seq_q;
    int seq_k;
    int num_ctiles;  // 256-row query tiles per (b,h)
    int npairs;      // (num_ctiles + 1) / 2
    int paired;      // 1: a unit is a (heavy, light) item pair; 0: one item
    int order;       // unpaired: 0 = (b,h)-major, 1 = by decreasing cost, snake rounds
    int num_units;   // units over all segments
    int causal;
    int merge;       // fp32 output: log-sum-exp merge into O / L in place
    float scale_log2;
    // Segments: one launch can run up to kMaxSegs (query slot, K/V slot)
    // pairs, each over all B*H heads with its own global offsets.  Q / O / L
    // hold the query slots stacked as [slot][B*H] along the outer dimension,
    // K / V the K/V slots the same way.
    int num_segs;
    int seg_units;   // units of one segment
    int hq;          // query heads per batch entry
    int group;       // query heads per K/V head (grouped-query attention; 1 = MHA)
    int q_base[4];   // outer index of the segment's first (b,h) in Q / O / L
    int k_base[4];   // outer index of the segment's first (b,h) in K / V
    long long q_off[4];
    long long k_off[4];
    // Bounded waits give up after wait_ns.  Test hook: with skip_k_load set,
    // CTA 0's producer leaves out its first K load (it still counts it), so
    // the MMA thread's wait for it runs out and the kernel reports
    // kStatusWaitTimeout and tears down.
    unsigned long long wait_ns;
    int skip_k_load;
};
constexpr int kMaxSegs = 4;

// K-major operand (rows x D, D contiguous) for k-step kk (16 elements).
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_base, int kk) {
    using G = FwdGeom<D>;
    const uint32_t byte = static_cast<uint32_t>(kk) * 32u;
    const uint32_t addr = tile_base + (byte / G::kSwz) * G::kCbBytes + (byte % G::kSwz);
    return sm100::make_smem_desc(addr, 16, 8 * G::kSwz, G::kLayout);
}

// Descriptor of k-step kk = descriptor of k-step 0 + this (start address
// field, in 16-byte units; shared addresses stay below 2^18 so no carry).
template <int D>
__host__ __device__ constexpr uint32_t kmajor_delta(int kk) {
    using G = FwdGeom<D>;
    return ((static_cast<uint32_t>(kk) * 32u / G::kSwz) * G::kCbBytes +
            (static_cast<uint32_t>(kk) * 32u % G::kSwz)) >> 4;
}
template <int D>
__host__ __device__ constexpr uint32_t mnmajor_delta(int kk) {
    return (static_cast<uint32_t>(kk) * 16u * FwdGeom<D>::kSwz) >> 4;
}

// MN-major operand (kv rows = K dimension, D contiguous = N dimension) for
// k-step kk (16 kv rows).
template <int D>
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile_base, int kk) {
    using G = FwdGeom<D>;
    const uint32_t addr = tile_base + static_cast<uint32_t>(kk) * 16u * G::kSwz;
    return sm100::make_smem_desc(addr, G::kCbBytes, 8 * G::kSwz, G::kLayout);
}

// One work item = 256 query rows (two 128-row tiles) of one (b,h).  Unit u
// of the persistent schedule holds two items of the same (b,h): q tile pair
// ct = num_ctiles-1-k and ct = k.  Under a causal mask their costs add up to
// about the same for every k, so a static round-robin of units over the CTAs
// is balanced, and the second item re-reads K/V blocks the first one has just
// brought into L2.  Problems with fewer units than SMs use one item per unit
// instead (more CTAs, same per-item work as a non-persistent grid).
struct FwdItem {
    int bh;      // outer index in Q / O / L
    int bhk;     // outer index in K / V
    int q_row0;
    long long q_off;  // global position of query row 0 / key row 0
    long long k_off;
};

__device__ __forceinline__ bool fwd_item(const FwdParams& p, int u, int w, FwdItem& it) {
    int sg = 0;
#pragma unroll
    for (int i = 1; i < kMaxSegs; ++i)
        if (i < p.num_segs && u >= i * p.seg_units) sg = i;
    u -= sg * p.seg_units;
    int bh, ct;
    if (!p.paired) {  // one item per unit, heaviest first within a (b,h)
        if (w == 1) return false;
        if (p.order) {
            // all heads' items by decreasing cost (query tile), snake rounds
            const int pos = sm100::snake_position(u, p.num_units);
            const int nbh = p.seg_units / p.num_ctiles;
            const int rank = pos / nbh;
            bh = pos - rank * nbh;
            ct = p.num_ctiles - 1 - rank;
        } else {
            bh = u / p.num_ctiles;
            ct = p.num_ctiles - 1 - (u - bh * p.num_ctiles);
        }
    } else {
        bh = u / p.npairs;
        const int k = u - bh * p.npairs;
        ct = w == 0 ? p.num_ctiles - 1 - k : k;
        if (w == 1 && ct == p.num_ctiles - 1 - k) return false;  // middle tile of an odd count
    }
    it.bh = p.q_base[sg] + bh;
    // K/V head of query head h = h / group within the same batch entry
    it.bhk = p.k_base[sg] +
             (p.group == 1 ? bh : (bh / p.hq) * (p.hq / p.group) + (bh % p.hq) / p.group);
    it.q_row0 = ct * 256;
    it.q_off = p.q_off[sg];
    it.k_off = p.k_off[sg];
    return true;
}

// kv blocks the 128-row tile starting at query row r_lo visits.
__device__ __forceinline__ int tile_blocks(const FwdParams& p, const FwdItem& it, int r_lo) {
    const int nkv_all = (p.seq_k + 127) / 128;
    if (r_lo >= p.seq_q) return 0;
    if (!p.causal) return nkv_all;
    const int r_hi = min(r_lo + 127, p.seq_q - 1);
    const long long lim = it.q_off + r_hi - it.k_off;  // largest visible local key
    const long long nb = lim / 128 + 1;
    return lim < 0 ? 0 : (nb < nkv_all ? static_cast<int>(nb) : nkv_all);
}

// Warp-uniform bounded wait.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned long long limit_ns) {
    // Every lane polls the barrier itself: all lanes observe the same phase,
    // timer and abort flag, so the warp stays converged without a shuffle.
    return sm100::mbar_wait(bar, parity, abort_flag, &g_fwd_status, limit_ns);
}

// Wait used by the producer at exit to make sure its TMA writes have landed;
// ignores the abort flag but is still bounded in time.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity,
                                           unsigned long long limit_ns) {
    volatile int never = 0;
    sm100::mbar_wait(bar, parity, &never, &g_fwd_status, limit_ns);
}

template <typename T, int D, bool kF32Out>
__global__ void __launch_bounds__(384, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
    using G = FwdGeom<D>;
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];

    if (sm100::cta_skip(&g_fwd_status)) return;

    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
    uint8_t* sptr = smem_raw + (sbase - raw_addr);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sptr + G::kOffBar);
    uint64_t* bar_q = bars;  // [2] Q tile t landed
    uint64_t* full_k = bar_q + 2;
    uint64_t* empty_k = full_k + G::kStages;
    uint64_t* full_v = empty_k + G::kStages;
    uint64_t* empty_v = full_v + G::kStages;
    uint64_t* bar_s = empty_v + G::kStages;  // [2] S_t in TMEM
    uint64_t* bar_p = bar_s + 2;             // [2] P_t stored (128 arrivals)
    uint64_t* bar_o = bar_p + 2;             // [2] O_t final for the item
    uint64_t* bar_qfree = bar_o + 2;         // [2] last QK of the item's tile t retired
    uint64_t* bar_p2 = bar_qfree + 2;        // [2] second half of P_t stored (split mode)
    uint64_t* bar_done = bar_p2 + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::kStages; ++s) {
            mbar_init(full_k + s, 1);
            mbar_init(empty_k + s, 1);
            mbar_init(full_v + s, 1);
            mbar_init(empty_v + s, 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(bar_q + t, 1);
            mbar_init(bar_s + t, 1);
            mbar_init(bar_p + t, 128);
            mbar_init(bar_p2 + t, 128);
            mbar_init(bar_o + t, 1);
            mbar_init(bar_qfree + t, 1);
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
    // (producer, MMA, 2 idle warps) gives back down to 72 and the two softmax
    // warpgroups take 216 each: 128*72 + 256*216 = 64512 <= 64512.
    if (warp < 4) {
        setmaxnreg_dec<72>();
    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            uint32_t q_cnt[2] = {0u, 0u};  // Q loads per tile slot
            uint32_t issued_k = 0, issued_v = 0;  // K/V blocks through the ring
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                for (int w = 0; ok && w < 2; ++w) {
                    FwdItem it;
                    if (!fwd_item(p, u, w, it)) continue;
                    const int nt[2] = {tile_blocks(p, it, it.q_row0),
                                       tile_blocks(p, it, it.q_row0 + 128)};
                    const int n_max = max(nt[0], nt[1]);
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        if (nt[t] == 0 || !ok) continue;
                        // the slot is free once the previous item's last QK on it retired
                        if (q_cnt[t] > 0 && !mbar_wait(bar_qfree + t, (q_cnt[t] - 1) & 1,
                                                       abort_flag, &g_fwd_status, p.wait_ns)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(bar_q + t, G::kTileBytes);
                        for (int cb = 0; cb < G::kNumCb; ++cb)
                            tma_load_3d(sptr + G::kOffQ + t * G::kTileBytes + cb * G::kCbBytes,
                                        &tmQ, bar_q + t, cb * G::kCbElems, it.q_row0 + t * 128,
                                        it.bh);
                        ++q_cnt[t];
                    }
                    for (int j = 0; ok && j < n_max; ++j) {
                        const uint32_t g = issued_v;
                        const int s = g % G::kStages;
                        const uint32_t ph = (g / G::kStages) & 1;
                        if (g >= G::kStages &&
                            !mbar_wait(empty_k + s, ph ^ 1, abort_flag, &g_fwd_status, p.wait_ns)) {
                            ok = false;
                            break;
                        }
                        if (!(p.skip_k_load && blockIdx.x == 0 && issued_k == 0)) {
                            mbar_arrive_expect_tx(full_k + s, G::kTileBytes);
                            for (int cb = 0; cb < G::kNumCb; ++cb)
                                tma_load_3d(sptr + G::kOffK + s * G::kTileBytes + cb * G::kCbBytes,
                                            &tmK, full_k + s, cb * G::kCbElems, j * 128, it.bhk);
                        }
                        ++issued_k;
                        if (g >= G::kStages &&
                            !mbar_wait(empty_v + s, ph ^ 1, abort_flag, &g_fwd_status, p.wait_ns)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(full_v + s, G::kTileBytes);
                        for (int cb = 0; cb < G::kNumCb; ++cb)
                            tma_load_3d(sptr + G::kOffV + s * G::kTileBytes + cb * G::kCbBytes,
                                        &tmV, full_v + s, cb * G::kCbElems, j * 128, it.bhk);
                        ++issued_v;
                    }
                }
            }
            // every issued load must land before the CTA can exit
#pragma unroll
            for (int t = 0; t < 2; ++t)
                if (q_cnt[t] > 0) drain_wait(bar_q + t, (q_cnt[t] - 1) & 1, p.wait_ns);
            for (uint32_t g = issued_k > G::kStages ? issued_k - G::kStages : 0; g < issued_k; ++g)
                drain_wait(full_k + g % G::kStages, (g / G::kStages) & 1, p.wait_ns);
            for (uint32_t g = issued_v > G::kStages ? issued_v - G::kStages : 0; g < issued_v; ++g)
                drain_wait(full_v + g % G::kStages, (g / G::kStages) & 1, p.wait_ns);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_qk = make_idesc(DType<T>::kMmaFmt, 128, 128, false, false);
            constexpr uint32_t idesc_pv = make_idesc(DType<T>::kMmaFmt, 128, D, false, true);
            auto issue_qk = [&](int t, int s) {
                const uint32_t d_tmem = tmem + t * 128;
                const uint32_t a_base = sbase + G::kOffQ + t * G::kTileBytes;
                const uint32_t b_base = sbase + G::kOffK + s * G::kTileBytes;
                uint64_t a0 = kmajor_desc<D>(a_base, 0);
                uint64_t b0 = kmajor_desc<D>(b_base, 0);
                // opaque to the optimiser: keeps the 2 x D/16 descriptors from
                // being hoisted out of the item loop into live registers
                asm volatile("" : "+l"(a0), "+l"(b0));
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    mma_f16_ss(d_tmem, a0 + kmajor_delta<D>(kk), b0 + kmajor_delta<D>(kk),
                               idesc_qk, kk > 0 ? 1u : 0u);
            };
            // O_t += P_t V over key k-steps [kk0, kk1)
            auto issue_pv = [&](int t, int s, bool acc, int kk0, int kk1) {
                const uint32_t d_tmem = tmem + 256 + t * 128;
                const uint32_t p_tmem = tmem + t * 128;
                uint64_t v0 = mnmajor_desc<D>(sbase + G::kOffV + s * G::kTileBytes, 0);
                asm volatile("" : "+l"(v0));
#pragma unroll
                for (int kk = 0; kk < 128 / 16; ++kk)
                    if (kk >= kk0 && kk < kk1)
                        mma_f16_ts(d_tmem, p_tmem + kk * 8, v0 + mnmajor_delta<D>(kk), idesc_pv,
                                   (acc || kk > 0) ? 1u : 0u);
            };
            uint32_t q_cnt[2] = {0u, 0u};  // bar_q phases consumed
            uint32_t p_cnt[2] = {0u, 0u};  // bar_p phases consumed
            uint32_t kv_g = 0;             // first ring slot of the current item
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                for (int w = 0; ok && w < 2; ++w) {
                    FwdItem it;
                    if (!fwd_item(p, u, w, it)) continue;
                    const int nt[2] = {tile_blocks(p, it, it.q_row0),
                                       tile_blocks(p, it, it.q_row0 + 128)};
                    const int n_max = max(nt[0], nt[1]);
                    if (n_max == 0) continue;
                    // The item's first S tiles.  In-order issue keeps them
                    // behind the previous item's last PV products, which
                    // still read P from the same TMEM columns.
                    {
                        const int s0 = kv_g % G::kStages;
                        const uint32_t ph0 = (kv_g / G::kStages) & 1;
#pragma unroll
                        for (int t = 0; t < 2; ++t)
                            if (nt[t] > 0 && ok)
                                ok = mbar_wait(bar_q + t, q_cnt[t] & 1, abort_flag, &g_fwd_status, p.wait_ns);
                        ok = ok && mbar_wait(full_k + s0, ph0, abort_flag, &g_fwd_status, p.wait_ns);
                        if (!ok) break;
                        tc_fence_after();
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            if (nt[t] == 0) continue;
                            issue_qk(t, s0);
                            tc_commit(bar_s + t);
                            if (nt[t] == 1) tc_commit(bar_qfree + t);
                            ++q_cnt[t];
                        }
                        tc_commit(empty_k + s0);
                    }
                    for (int j = 0; ok && j < n_max; ++j) {
                        const uint32_t g = kv_g + j;
                        const int s = g % G::kStages;
                        const uint32_t ph = (g / G::kStages) & 1;
                        if (!mbar_wait(full_v + s, ph, abort_flag, &g_fwd_status, p.wait_ns)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t gn = g + 1;
                        const int sn = gn % G::kStages;
                        const uint32_t phn = (gn / G::kStages) & 1;
                        bool k_next_ready = false;
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            if (j >= nt[t] || !ok) continue;
                            if (!mbar_wait(bar_p + t, p_cnt[t] & 1, abort_flag, &g_fwd_status, p.wait_ns)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            if (kSplitP) {
                                issue_pv(t, s, j > 0, 0, 4);
                                if (!mbar_wait(bar_p2 + t, p_cnt[t] & 1, abort_flag,
                                               &g_fwd_status, p.wait_ns)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                                issue_pv(t, s, j > 0, 4, 8);
                            } else {
                                issue_pv(t, s, j > 0, 0, 8);
                            }
                            ++p_cnt[t];
                            if (j == nt[t] - 1) tc_commit(bar_o + t);
                            if (j + 1 < nt[t]) {
                                if (!k_next_ready) {
                                    if (!mbar_wait(full_k + sn, phn, abort_flag, &g_fwd_status, p.wait_ns)) {
                                        ok = false;
                                        break;
                                    }
                                    tc_fence_after();
                                    k_next_ready = true;
                                }
                                issue_qk(t, sn);
                                tc_commit(bar_s + t);
                                if (j + 2 == nt[t]) tc_commit(bar_qfree + t);
                            }
                        }
                        if (!ok) break;
                        tc_commit(empty_v + s);
                        if (k_next_ready) tc_commit(empty_k + sn);
                    }
                    kv_g += n_max;
                }
            }
            // all MMAs (and their commits) retire before teardown
            tc_commit(bar_done);
            volatile int never = 0;
            mbar_wait(bar_done, 0, &never, &g_fwd_status, p.wait_ns);
        }
        __syncwarp();
    }
    } else {
        setmaxnreg_inc<216>();
        // ------------------------------------------------ softmax / epilogue
        const int t = (warp - 4) >> 2;
        const int wq = warp & 3;
        const int r = wq * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t s_tmem = tmem + lane_addr + t * 128;
        const uint32_t o_tmem = tmem + lane_addr + 256 + t * 128;
        const float c = p.scale_log2;
        uint32_t s_cnt = 0, o_cnt = 0;  // bar_s / bar_o phases consumed
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
            for (int w = 0; ok && w < 2; ++w) {
                FwdItem it;
                if (!fwd_item(p, u, w, it)) continue;
                const int row = it.q_row0 + t * 128 + r;
                const long long grow = it.q_off + row;
                const int n = tile_blocks(p, it, it.q_row0 + t * 128);
                const long long tile_g0 = it.q_off + it.q_row0 + t * 128;

                float m_run = -INFINITY;
                float l_run = 0.f;
                for (int j = 0; j < n; ++j) {
                    if (!warp_wait(bar_s + t, s_cnt & 1, abort_flag, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    ++s_cnt;
                    tc_fence_after();
                    uint32_t sr[128];
                    tmem_ld_x128(s_tmem, sr);
                    const int col0 = j * 128;
                    const bool need_mask = (col0 + 128 > p.seq_k) ||
                                           (p.causal && (it.k_off + col0 + 127 > tile_g0));
                    if (need_mask) {
                        // largest visible local key column for this row (32-bit safe)
                        const long long lim64 = grow - it.k_off;
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
                    // Decide the new running maximum.  O is rescaled before the first
                    // P half is handed over (split mode) or after P is stored, when the
                    // score registers are dead.
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
                    // PV_{j-1} has completed: S_t(j) was issued after it and its commit
                    // covers every earlier tcgen05 operation.
                    auto rescale_o = [&]() {
                        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
                            for (int cb = 0; cb < D / 16; ++cb) {
                                uint32_t o[16];
                                tmem_ld_x16(o_tmem + cb * 16, o);
#pragma unroll
                                for (int i = 0; i < 16; ++i)
                                    o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                                tmem_st_x16(o_tmem + cb * 16, o);
                            }
                        }
                    };
                    if (kSplitP) rescale_o();
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
                            if (kExp2EmuEvery > 0 &&
                                (i % (kExp2EmuEvery > 0 ? kExp2EmuEvery : 1)) == kExp2EmuEvery - 1) {
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
                        if (kSplitP) {
                            tc_fence_before();
                            mbar_arrive((h == 0 ? bar_p : bar_p2) + t);
                        }
                    }
                    float sum;
                    {
                        const float2 a = f2_unpack(f2_add(f2_add(acc0, acc1), f2_add(acc2, acc3)));
                        sum = a.x + a.y;
                    }
                    l_run = l_run * alpha + sum;
                    if (!kSplitP) {
                        rescale_o();
                        tc_fence_before();
                        mbar_arrive(bar_p + t);
                    }
                }

                // epilogue
                if (n > 0 && ok) {
                    ok = warp_wait(bar_o + t, o_cnt & 1, abort_flag, p.wait_ns);
                    ++o_cnt;
                    tc_fence_after();
                }
                const bool valid_row = row < p.seq_q;
                const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
                const size_t row_elem = (static_cast<size_t>(it.bh) * p.seq_q + row) * D;
                const size_t l_idx = static_cast<size_t>(it.bh) * p.seq_q + row;
                const float lse_part = l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
                // Merge mode: (O, L) already hold a normalised result for these
                // rows; fold this one in with the log-sum-exp weights (same
                // algebra as cuflash_lse_merge_f32): wa * O + wb * O_part.
                float wa = 0.f, wb = inv_l, lse_out = lse_part;
                if (kF32Out && p.merge && valid_row) {
                    const float la = p.L[l_idx];
                    const float M = fmaxf(la, lse_part);
                    wa = 0.f;
                    wb = 0.f;
                    lse_out = -INFINITY;
                    if (M != -INFINITY) {
                        const float ea = __expf(la - M), eb = __expf(lse_part - M);
                        const float tot = ea + eb;
                        wa = ea / tot;
                        wb = eb / tot * inv_l;
                        lse_out = M + logf(tot);
                    }
                }
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
                            for (int i = 0; i < 8; ++i) {
                                float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
                                if (wa != 0.f) a = dst[i];  // wa == 0: O may hold anything
                                dst[i] = make_float4(fmaf(wa, a.x, __uint_as_float(o[4 * i]) * wb),
                                                     fmaf(wa, a.y, __uint_as_float(o[4 * i + 1]) * wb),
                                                     fmaf(wa, a.z, __uint_as_float(o[4 * i + 2]) * wb),
                                                     fmaf(wa, a.w, __uint_as_float(o[4 * i + 3]) * wb));
                            }
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
                if (valid_row) p.L[l_idx] = lse_out;
                // The next item's first P store (and its bar_p arrival) follows
                // these TMEM reads of O_t, so its PV product cannot overwrite
                // O_t early.
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

// Query/K-V slot layout and segment list of one launch (see FwdParams).
struct FwdSegs {
    int nq_slots = 1;  // Q / O / L hold nq_slots x B*H outer rows
    int nk_slots = 1;  // K / V hold nk_slots x B*H outer rows
    int num_segs = 1;
    int q_slot[kMaxSegs] = {0, 0, 0, 0};
    int k_slot[kMaxSegs] = {0, 0, 0, 0};
    long long q_off[kMaxSegs] = {0, 0, 0, 0};
    long long k_off[kMaxSegs] = {0, 0, 0, 0};
    bool merge = false;
    int reserve_sms = 0;  // SMs a ring-step launch leaves free (merge only)
    int hq = 1;     // query heads per batch entry (BH = batch * hq)
    int group = 1;  // query heads per K/V head
};

template <typename T, int D, bool kF32Out>
FlashAttentionError launch_typed(const T* Q, const T* K, const T* V, void* O, float* L, int BH,
                                 int seq_q, int seq_k, float scale, bool causal,
                                 const FwdSegs& sg, cudaStream_t stream) {
    using G = FwdGeom<D>;
    const CUtensorMapSwizzle swz =
        G::kSwz == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUtensorMap mq, mk, mv;
    const uint64_t q_outer = static_cast<uint64_t>(sg.nq_slots) * BH;
    const uint64_t k_outer = static_cast<uint64_t>(sg.nk_slots) * (BH / sg.group);
    if (!encode_tmap_3d(&mq, Q, DType<T>::kTmaType, 2, D, seq_q, q_outer, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mk, K, DType<T>::kTmaType, 2, D, seq_k, k_outer, G::kCbElems, 128, swz) ||
        !encode_tmap_3d(&mv, V, DType<T>::kTmaType, 2, D, seq_k, k_outer, G::kCbElems, 128, swz))
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
    prm.merge = sg.merge ? 1 : 0;
    // A zero scale is replaced by a tiny positive one so that masked scores
    // (-inf) still map to -inf; the effect on results is below fp32 resolution.
    prm.scale_log2 = fmaxf(scale * kLog2e, 1e-30f);
    prm.num_segs = sg.num_segs;
    prm.hq = sg.hq;
    prm.group = sg.group;
    for (int i = 0; i < kMaxSegs; ++i) {
        prm.q_base[i] = sg.q_slot[i] * BH;
        prm.k_base[i] = sg.k_slot[i] * (BH / sg.group);
        prm.q_off[i] = sg.q_off[i];
        prm.k_off[i] = sg.k_off[i];
    }
    prm.npairs = (prm.num_ctiles + 1) / 2;
    const int limit_ms = env_int("CUFLASH_TEST_WAIT_LIMIT_MS", 0);
    prm.wait_ns = limit_ms > 0 ? static_cast<unsigned long long>(limit_ms) * 1000000ull
                               : sm100::kWaitTimeoutNs;
    prm.skip_k_load = env_int("CUFLASH_TEST_SKIP_K_LOAD", 0) != 0 ? 1 : 0;
    const int sms = current_sm_count();
    long long seg_units = static_cast<long long>(BH) * prm.npairs;
    prm.paired = seg_units * sg.num_segs >= sms ? 1 : 0;
    prm.order = 0;
    // Few units per SM (a causal problem split over several GPUs): equal-cost
    // pairs quantise badly (256 pairs on 148 SMs: 86 % busy), while single
    // items dealt by decreasing cost in snake rounds balance to within a few
    // per cent.  With many units the pairing is already balanced and keeps a
    // head's K/V hot in L2 across its two items.
    if (causal && !sg.merge && prm.paired && seg_units < 5LL * sms &&
        static_cast<long long>(BH) * prm.num_ctiles > sms) {
        prm.paired = 0;
        prm.order = 1;
    }
    if (!prm.paired) seg_units = static_cast<long long>(BH) * prm.num_ctiles;
    const long long units = seg_units * sg.num_segs;
    if (units > 0x7fffffffLL) return FlashAttentionError::CUDA_ERROR;
    prm.seg_units = static_cast<int>(seg_units);
    prm.num_units = static_cast<int>(units);
    // persistent: one CTA per SM (the shared-memory footprint allows one)
    // per wave; multi-segment (ring step) launches overlap NCCL transfers
    int grid = persistent_grid(units, sg.merge ? env_int("CUFLASH_CP_WAVES", 1)
                                               : env_int("CUFLASH_FWD_WAVES", 1));
    // A ring step runs while NCCL moves the next step's K/V; a CTA of this
    // kernel fills an SM (registers and shared memory), so SMs left free let
    // the transfer kernels run concurrently instead of after this launch.
    // Measured on 8 B200s (config 5): 16 free SMs 17.0 ms per step, 8: 21.3,
    // none: 20.4 (the transfer then waits for the launch to end).
    if (sg.merge) grid = std::max(1, std::min(grid, sms - sg.reserve_sms));
    if (grid <= 0) return FlashAttentionError::SUCCESS;
    bind_status_word(reinterpret_cast<const void*>(&g_fwd_status), stream);
    kern<<<grid, 384, G::kSmemBytes, stream>>>(mq, mk, mv, prm);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

template <typename T, bool kF32Out>
FlashAttentionError dispatch_d(const T* Q, const T* K, const T* V, void* O, float* L, int BH,
                               int seq_q, int seq_k, int D, float scale, bool causal,
                               const FwdSegs& sg, cudaStream_t stream) {
    switch (D) {
        case 32:
            return launch_typed<T, 32, kF32Out>(Q, K, V, O, L, BH, seq_q, seq_k, scale, causal, sg,
                                                stream);
        case 64:
            return launch_typed<T, 64, kF32Out>(Q, K, V, O, L, BH, seq_q, seq_k, scale, causal, sg,
                                                stream);
        case 128:
            return launch_typed<T, 128, kF32Out>(Q, K, V, O, L, BH, seq_q, seq_k, scale, causal, sg,
                                                 stream);
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
    FwdSegs sg;
    sg.q_off[0] = q_offset;
    sg.k_off[0] = k_offset;
    if (out_f32_partial)
        return dispatch_d<T, true>(Q, K, V, O, L, BH, seq_q, seq_k, D, scale, causal, sg, stream);
    return dispatch_d<T, false>(Q, K, V, O, L, BH, seq_q, seq_k, D, scale, causal, sg, stream);
}

template <typename T>
FlashAttentionError launch_fwd_gqa_sm100(const T* Q, const T* K, const T* V, T* O, float* L, int B,
                                         int Hq, int Hkv, int seq_q, int seq_k, int D, float scale,
                                         bool causal, cudaStream_t stream) {
    FwdSegs sg;
    sg.hq = Hq;
    sg.group = Hq / Hkv;
    // bottom-right causal alignment: query i sits at global position
    // seq_k - seq_q + i, keys at 0..seq_k-1
    sg.q_off[0] = static_cast<long long>(seq_k) - seq_q;
    return dispatch_d<T, false>(Q, K, V, O, L, B * Hq, seq_q, seq_k, D, scale, causal, sg, stream);
}

template FlashAttentionError launch_fwd_gqa_sm100<__nv_bfloat16>(
    const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, __nv_bfloat16*, float*, int,
    int, int, int, int, int, float, bool, cudaStream_t);
template FlashAttentionError launch_fwd_gqa_sm100<half>(const half*, const half*, const half*,
                                                        half*, float*, int, int, int, int, int,
                                                        int, float, bool, cudaStream_t);

template <typename T>
FlashAttentionError launch_fwd_cp_step_sm100(const T* Q, const T* K, const T* V, float* O_acc,
                                             float* L_acc, int nq, int nk, int B, int H, int C,
                                             int D, float scale, bool causal, int num_pairs,
                                             const int* q_slot, const int* k_slot,
                                             const long long* q_off, const long long* k_off,
                                             int reserve_sms, cudaStream_t stream) {
    if (num_pairs < 1 || num_pairs > kMaxSegs) return FlashAttentionError::INVALID_DIMENSION;
    FwdSegs sg;
    sg.nq_slots = nq;
    sg.nk_slots = nk;
    sg.num_segs = num_pairs;
    sg.merge = true;
    sg.reserve_sms = reserve_sms;
    for (int i = 0; i < num_pairs; ++i) {
        sg.q_slot[i] = q_slot[i];
        sg.k_slot[i] = k_slot[i];
        sg.q_off[i] = q_off[i];
        sg.k_off[i] = k_off[i];
    }
    return dispatch_d<T, true>(Q, K, V, O_acc, L_acc, B * H, C, C, D, scale, causal, sg, stream);
}

template FlashAttentionError launch_fwd_cp_step_sm100<__nv_bfloat16>(
    const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, float*, float*, int, int,
    int, int, int, int, float, bool, int, const int*, const int*, const long long*,
    const long long*, int, cudaStream_t);
template FlashAttentionError launch_fwd_cp_step_sm100<half>(
    const half*, const half*, const half*, float*, float*, int, int, int, int, int, int, float,
    bool, int, const int*, const int*, const long long*, const long long*, int, cudaStream_t);

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
