// Split-KV decode, log-sum-exp merge and fp32 -> fp16/bf16 conversion.
//
// Decode has no reference counterpart (the reference lists "FlashDecoding /
// Split-KV" as future work, ROADMAP.md:22-26).  It computes, for one query
// token per (batch, head), o = softmax(scale * q K^T) V over a KV cache of
// kv_len rows.  M = 1, so this is a bandwidth problem, not a tensor-core one:
// every K and V byte is read exactly once with 128-bit non-allocating loads.
//
// Thread layout: each lane owns 8 consecutive head_dim elements (16 bytes),
// D/8 lanes cover one K/V row, a warp covers 32/(D/8) rows per load
// instruction.  q.k is reduced across the row's lanes with xor shuffles, the
// PV product needs no cross-lane traffic (a lane accumulates its own 8
// output elements).  Each row group keeps its own online-softmax state
// (m, l, acc); the groups are merged through shared memory at the end of
// the split, and the splits are merged by the log-sum-exp combine kernel.
//
// The merge algebra is the reference's OnlineSoftmaxState merge
// (src/kernels/impl/online_softmax.cuh:16-59) in the log2 domain.

#include <algorithm>
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace cuflash {
namespace detail {

namespace {

constexpr float kLn2f = 0.6931471805599453f;
constexpr float kLog2ef = 1.4426950408889634f;
constexpr int kDecodeThreads = 256;
constexpr int kDecodeWarps = kDecodeThreads / 32;
constexpr int kDecodeUnroll = 8;

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
    float2 a = DType<T>::unpack2(v.x), b = DType<T>::unpack2(v.y), c = DType<T>::unpack2(v.z),
           d = DType<T>::unpack2(v.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

// grid (B*H, num_splits); one CTA streams rows [split*chunk, min(kv_len, (split+1)*chunk)).
// kDirect: num_splits == 1, write the final O (dtype) and L; else write the
// normalised split partial (fp32) and its log-sum-exp.
// The explicit minimum of one block per SM changes ptxas' register target:
// measured on sm_100a, it compiles this kernel into 127 registers instead of
// 143-149 (no spills), so two CTAs fit on an SM, and config 4 goes from 5.35
// to 7.2 TB/s.
template <typename T, int D, bool kDirect>
__global__ void __launch_bounds__(kDecodeThreads, 1)
    decode_split_kernel(const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V,
                        T* __restrict__ O, float* __restrict__ L, float* __restrict__ O_part,
                        float* __restrict__ L_part, int kv_len, int chunk, float scale_log2) {
    constexpr int LPR = D / 8;     // lanes per row
    constexpr int RPW = 32 / LPR;  // rows per warp per load
    constexpr int G = kDecodeWarps * RPW;  // row groups per CTA
    constexpr int STEP = kDecodeWarps * RPW;

    __shared__ float s_m[G];
    __shared__ float s_l[G];
    __shared__ float s_acc[G][D];

    const int split = blockIdx.y;
    const int num_splits = gridDim.y;
    const long long bh = blockIdx.x;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR;
    const int li = lane % LPR;
    const int grp = warp * RPW + sub;

    float q[8];
    {
        const uint4 qv = *reinterpret_cast<const uint4*>(Q + bh * D + li * 8);
        unpack8<T>(qv, q);
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] *= scale_log2;
    }

    const int r_begin = split * chunk;
    const int r_end = min(kv_len, r_begin + chunk);
    const T* Kb = K + bh * static_cast<long long>(kv_len) * D + li * 8;
    const T* Vb = V + bh * static_cast<long long>(kv_len) * D + li * 8;

    float m = -INFINITY, l = 0.f;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;

    // The loop bound is warp-uniform so that every lane reaches the shuffles.
    for (int rb = r_begin + warp * RPW; rb < r_end; rb += STEP * kDecodeUnroll) {
        uint4 kv[kDecodeUnroll], vv[kDecodeUnroll];
#pragma unroll
        for (int u = 0; u < kDecodeUnroll; ++u) {
            const int row = rb + sub + u * STEP;
            if (row < r_end) {
                kv[u] = ld_stream(Kb + static_cast<long long>(row) * D);
                vv[u] = ld_stream(Vb + static_cast<long long>(row) * D);
            } else {
                kv[u] = make_uint4(0, 0, 0, 0);
                vv[u] = make_uint4(0, 0, 0, 0);
            }
        }
        float s[kDecodeUnroll];
#pragma unroll
        for (int u = 0; u < kDecodeUnroll; ++u) {
            float kf[8];
            unpack8<T>(kv[u], kf);
            float dot = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) dot = fmaf(q[e], kf[e], dot);
#pragma unroll
            for (int off = LPR / 2; off > 0; off >>= 1)
                dot += __shfl_xor_sync(0xffffffffu, dot, off);
            s[u] = (rb + sub + u * STEP < r_end) ? dot : -INFINITY;
        }
        float mx = s[0];
#pragma unroll
        for (int u = 1; u < kDecodeUnroll; ++u) mx = fmaxf(mx, s[u]);
        const float m_new = fmaxf(m, mx);
        if (m_new != -INFINITY) {
            const float alpha = sm100::ex2_approx(m - m_new);
            l *= alpha;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] *= alpha;
#pragma unroll
            for (int u = 0; u < kDecodeUnroll; ++u) {
                const float pr = sm100::ex2_approx(s[u] - m_new);
                l += pr;
                float vf[8];
                unpack8<T>(vv[u], vf);
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] = fmaf(pr, vf[e], acc[e]);
            }
            m = m_new;
        }
    }

    if (li == 0) {
        s_m[grp] = m;
        s_l[grp] = l;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) s_acc[grp][li * 8 + e] = acc[e];
    __syncthreads();

    if (threadIdx.x < D) {
        const int d = threadIdx.x;
        float M = -INFINITY;
        for (int g = 0; g < G; ++g) M = fmaxf(M, s_m[g]);
        float lt = 0.f, o = 0.f;
        if (M != -INFINITY) {
            for (int g = 0; g < G; ++g) {
                const float w = sm100::ex2_approx(s_m[g] - M);
                lt = fmaf(w, s_l[g], lt);
                o = fmaf(w, s_acc[g][d], o);
            }
        }
        const float outv = lt > 0.f ? o / lt : 0.f;
        const float lse = lt > 0.f ? (M + log2f(lt)) * kLn2f : -INFINITY;
        if constexpr (kDirect) {
            O[bh * D + d] = DType<T>::from_float(outv);
            if (d == 0) L[bh] = lse;
        } else {
            O_part[(bh * num_splits + split) * D + d] = outv;
            if (d == 0) L_part[bh * num_splits + split] = lse;
        }
    }
}

// ---------------------------------------------------------------------------
// Grouped-query and paged decode.  A CTA serves TILE query heads that share
// one K/V head, so every K/V row is read once for all of them (the point of
// grouped-query attention in decode: the cache traffic shrinks by the group
// size).  The K/V cache is either contiguous [B, Hkv, kv_len, D] or paged:
// [num_pages, page_size, Hkv, D] with a block table [B, max_pages] of page
// indices and per-sequence lengths seq_lens[B] (the layout of paged KV-cache
// serving engines).  Page indices are clamped to [0, num_pages) so a bad
// table entry reads the wrong page instead of faulting.
// ---------------------------------------------------------------------------
template <typename T>
struct DecodeKv {
    const T* K;
    const T* V;
    const int* block_table;  // paged: [B, max_pages]
    const int* seq_lens;     // paged: [B]
    int kv_len;              // contiguous: rows per K/V head
    int hkv;
    int page_shift;          // log2(page_size)
    int max_pages;
    int num_pages;
};

template <typename T, int D, int TILE, bool kPaged, bool kDirect>
__global__ void __launch_bounds__(kDecodeThreads, 1)
    decode_group_kernel(const T* __restrict__ Q, const DecodeKv<T> kvp, T* __restrict__ O,
                        float* __restrict__ L, float* __restrict__ O_part,
                        float* __restrict__ L_part, int hq, int group, int chunk,
                        float scale_log2) {
    constexpr int LPR = D / 8;     // lanes per row
    constexpr int RPW = 32 / LPR;  // rows per warp per load
    constexpr int G = kDecodeWarps * RPW;
    constexpr int STEP = G;
    constexpr int U = (8 / TILE) > 2 ? (8 / TILE) : 2;  // rows in flight per lane group
    extern __shared__ float dsm[];
    float* s_m = dsm;                  // [G][TILE]
    float* s_l = s_m + G * TILE;       // [G][TILE]
    float* s_acc = s_l + G * TILE;     // [G][TILE][D]

    const int split = blockIdx.y;
    const int num_splits = gridDim.y;
    const int tiles = group / TILE;
    const int bhk = blockIdx.x / tiles;
    const int tq = blockIdx.x - bhk * tiles;
    const int b = bhk / kvp.hkv;
    const int hk = bhk - b * kvp.hkv;
    const long long bhq0 = static_cast<long long>(b) * hq + hk * group + tq * TILE;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR;
    const int li = lane % LPR;
    const int grp = warp * RPW + sub;

    float q[TILE][8];
#pragma unroll
    for (int t = 0; t < TILE; ++t) {
        const uint4 qv = *reinterpret_cast<const uint4*>(Q + (bhq0 + t) * D + li * 8);
        unpack8<T>(qv, q[t]);
#pragma unroll
        for (int e = 0; e < 8; ++e) q[t][e] *= scale_log2;
    }

    // a paged length is clamped to what the block table can address
    const int len = kPaged ? min(max(kvp.seq_lens[b], 0), kvp.max_pages << kvp.page_shift)
                           : kvp.kv_len;
    const int r_begin = split * chunk;
    const int r_end = min(len, r_begin + chunk);
    auto row_off = [&](int row) -> long long {  // element offset of (row, hk, li*8)
        if constexpr (kPaged) {
            int page = kvp.block_table[static_cast<long long>(b) * kvp.max_pages +
                                       (row >> kvp.page_shift)];
            page = min(max(page, 0), kvp.num_pages - 1);
            const long long slot = (static_cast<long long>(page) << kvp.page_shift) +
                                   (row & ((1 << kvp.page_shift) - 1));
            return (slot * kvp.hkv + hk) * D + li * 8;
        } else {
            return (static_cast<long long>(bhk) * kvp.kv_len + row) * D + li * 8;
        }
    };

    float m[TILE], l[TILE], acc[TILE][8];
#pragma unroll
    for (int t = 0; t < TILE; ++t) {
        m[t] = -INFINITY;
        l[t] = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[t][e] = 0.f;
    }

    // The loop bound is warp-uniform so that every lane reaches the shuffles.
    for (int rb = r_begin + warp * RPW; rb < r_end; rb += STEP * U) {
        uint4 kv[U], vv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int row = rb + sub + u * STEP;
            if (row < r_end) {
                const long long off = row_off(row);
                kv[u] = ld_stream(kvp.K + off);
                vv[u] = ld_stream(kvp.V + off);
            } else {
                kv[u] = make_uint4(0, 0, 0, 0);
                vv[u] = make_uint4(0, 0, 0, 0);
            }
        }
        float sc[U][TILE];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float kf[8];
            unpack8<T>(kv[u], kf);
            const bool live = rb + sub + u * STEP < r_end;
#pragma unroll
            for (int t = 0; t < TILE; ++t) {
                float dot = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) dot = fmaf(q[t][e], kf[e], dot);
#pragma unroll
                for (int off = LPR / 2; off > 0; off >>= 1)
                    dot += __shfl_xor_sync(0xffffffffu, dot, off);
                sc[u][t] = live ? dot : -INFINITY;
            }
        }
#pragma unroll
        for (int t = 0; t < TILE; ++t) {
            float mx = sc[0][t];
#pragma unroll
            for (int u = 1; u < U; ++u) mx = fmaxf(mx, sc[u][t]);
            const float m_new = fmaxf(m[t], mx);
            if (m_new != -INFINITY) {
                const float alpha = sm100::ex2_approx(m[t] - m_new);
                l[t] *= alpha;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[t][e] *= alpha;
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const float pr = sm100::ex2_approx(sc[u][t] - m_new);
                    l[t] += pr;
                    float vf[8];
                    unpack8<T>(vv[u], vf);
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[t][e] = fmaf(pr, vf[e], acc[t][e]);
                }
                m[t] = m_new;
            }
        }
    }

#pragma unroll
    for (int t = 0; t < TILE; ++t) {
        if (li == 0) {
            s_m[grp * TILE + t] = m[t];
            s_l[grp * TILE + t] = l[t];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) s_acc[(grp * TILE + t) * D + li * 8 + e] = acc[t][e];
    }
    __syncthreads();

    for (int idx = threadIdx.x; idx < TILE * D; idx += kDecodeThreads) {
        const int t = idx / D;
        const int d = idx - t * D;
        float M = -INFINITY;
        for (int g = 0; g < G; ++g) M = fmaxf(M, s_m[g * TILE + t]);
        float lt = 0.f, o = 0.f;
        if (M != -INFINITY) {
            for (int g = 0; g < G; ++g) {
                const float w = sm100::ex2_approx(s_m[g * TILE + t] - M);
                lt = fmaf(w, s_l[g * TILE + t], lt);
                o = fmaf(w, s_acc[(g * TILE + t) * D + d], o);
            }
        }
        const float outv = lt > 0.f ? o / lt : 0.f;
        const float lse = lt > 0.f ? (M + log2f(lt)) * kLn2f : -INFINITY;
        const long long bhq = bhq0 + t;
        if constexpr (kDirect) {
            O[bhq * D + d] = DType<T>::from_float(outv);
            if (d == 0) L[bhq] = lse;
        } else {
            O_part[(bhq * num_splits + split) * D + d] = outv;
            if (d == 0) L_part[bhq * num_splits + split] = lse;
        }
    }
}

// grid (B*H); merges num_splits normalised partials by their log-sum-exp.
template <typename T, int D>
__global__ void __launch_bounds__(128)
    decode_combine_kernel(const float* __restrict__ O_part, const float* __restrict__ L_part,
                          T* __restrict__ O, float* __restrict__ L, int num_splits) {
    const long long bh = blockIdx.x;
    const float* lp = L_part + bh * num_splits;
    float M = -INFINITY;
    for (int s = 0; s < num_splits; ++s) M = fmaxf(M, lp[s]);
    float tot = 0.f;
    if (M != -INFINITY)
        for (int s = 0; s < num_splits; ++s) tot += __expf(lp[s] - M);
    const float lse = tot > 0.f ? M + logf(tot) : -INFINITY;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float o = 0.f;
        if (tot > 0.f)
            for (int s = 0; s < num_splits; ++s)
                o = fmaf(__expf(lp[s] - lse), O_part[(bh * num_splits + s) * D + d], o);
        O[bh * D + d] = DType<T>::from_float(o);
    }
    if (threadIdx.x == 0) L[bh] = lse;
}

// One warp per row: O_acc/L_acc <- merge(O_acc/L_acc, O_part/L_part).
__global__ void __launch_bounds__(256)
    lse_merge_kernel(float* __restrict__ O_acc, float* __restrict__ L_acc,
                     const float* __restrict__ O_part, const float* __restrict__ L_part,
                     long long rows, int D) {
    const int lane = threadIdx.x & 31;
    const long long warp_global = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
    for (long long r = warp_global; r < rows; r += nwarps) {
        const float la = L_acc[r];
        const float lb = L_part[r];
        const float M = fmaxf(la, lb);
        float wa = 0.f, wb = 0.f, lse = -INFINITY;
        if (M != -INFINITY) {
            const float ea = __expf(la - M), eb = __expf(lb - M);
            const float tot = ea + eb;
            wa = ea / tot;
            wb = eb / tot;
            lse = M + logf(tot);
        }
        float* oa = O_acc + r * D;
        const float* ob = O_part + r * D;
        for (int d = lane; d < D; d += 32) {
            const float a = (wa != 0.f) ? oa[d] : 0.f;
            const float b = (wb != 0.f) ? ob[d] : 0.f;
            oa[d] = wa * a + wb * b;
        }
        __syncwarp();
        if (lane == 0) L_acc[r] = lse;
    }
}

template <typename T>
__global__ void convert_kernel(const float* __restrict__ src, T* __restrict__ dst, long long n) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride)
        dst[i] = DType<T>::from_float(src[i]);
}

int auto_splits(long long bh, int kv_len) {
    const long long target = 4LL * current_sm_count();  // a few CTAs per SM
    long long s = (target + bh - 1) / bh;
    const long long max_by_len = (kv_len + 511) / 512;  // keep >= 512 rows per split
    if (s > max_by_len) s = max_by_len;
    if (s < 1) s = 1;
    if (s > 64) s = 64;
    return static_cast<int>(s);
}

template <typename T, int D>
FlashAttentionError decode_typed(const T* Q, const T* K, const T* V, T* O, float* L, int BH,
                                 int kv_len, float scale, int num_splits, cudaStream_t stream) {
    for (const void* p : {static_cast<const void*>(Q), static_cast<const void*>(K),
                          static_cast<const void*>(V), static_cast<const void*>(O)})
        if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return FlashAttentionError::CUDA_ERROR;
    int S = num_splits == 0 ? auto_splits(BH, kv_len) : num_splits;
    if (S > kv_len) S = kv_len;
    const int chunk = (kv_len + S - 1) / S;
    S = (kv_len + chunk - 1) / chunk;  // no empty splits
    const float sl2 = scale * kLog2ef;
    if (S == 1) {
        decode_split_kernel<T, D, true><<<dim3(BH, 1), kDecodeThreads, 0, stream>>>(
            Q, K, V, O, L, nullptr, nullptr, kv_len, chunk, sl2);
        return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                                 : FlashAttentionError::CUDA_ERROR;
    }
    const size_t part_elems = static_cast<size_t>(BH) * S * D;
    const size_t bytes = (part_elems + static_cast<size_t>(BH) * S) * sizeof(float);
    void* wsv = nullptr;
    FlashAttentionError werr = workspace_alloc(&wsv, bytes, stream);
    if (werr != FlashAttentionError::SUCCESS) return werr;
    float* ws = static_cast<float*>(wsv);
    float* o_part = ws;
    float* l_part = ws + part_elems;
    decode_split_kernel<T, D, false><<<dim3(BH, S), kDecodeThreads, 0, stream>>>(
        Q, K, V, nullptr, nullptr, o_part, l_part, kv_len, chunk, sl2);
    cudaError_t e1 = cudaGetLastError();
    decode_combine_kernel<T, D><<<BH, 128, 0, stream>>>(o_part, l_part, O, L, S);
    cudaError_t e2 = cudaGetLastError();
    workspace_free(ws, stream);
    return (e1 == cudaSuccess && e2 == cudaSuccess) ? FlashAttentionError::SUCCESS
                                                    : FlashAttentionError::CUDA_ERROR;
}

template <typename T, int D, int TILE, bool kPaged>
FlashAttentionError decode_group_typed(const T* Q, const DecodeKv<T>& kvp, T* O, float* L, int B,
                                       int hq, int max_len, float scale, int num_splits,
                                       cudaStream_t stream) {
    constexpr int G = kDecodeWarps * (32 / (D / 8));
    const size_t smem = static_cast<size_t>(G) * TILE * (D + 2) * sizeof(float);
    const int group = hq / kvp.hkv;
    const int ctas_y = B * kvp.hkv * (group / TILE);
    const int BHq = B * hq;
    int S = num_splits == 0 ? auto_splits(ctas_y, max_len) : num_splits;
    if (S > max_len) S = max_len;
    if (S < 1) S = 1;
    const int chunk = (max_len + S - 1) / S;
    S = (max_len + chunk - 1) / chunk;
    const float sl2 = scale * kLog2ef;
    if (S == 1) {
        auto k = decode_group_kernel<T, D, TILE, kPaged, true>;
        if (!ensure_smem_attr(reinterpret_cast<const void*>(k), static_cast<int>(smem)))
            return FlashAttentionError::CUDA_ERROR;
        k<<<dim3(ctas_y, 1), kDecodeThreads, smem, stream>>>(Q, kvp, O, L, nullptr, nullptr, hq,
                                                              group, chunk, sl2);
        return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                                 : FlashAttentionError::CUDA_ERROR;
    }
    const size_t part_elems = static_cast<size_t>(BHq) * S * D;
    const size_t bytes = (part_elems + static_cast<size_t>(BHq) * S) * sizeof(float);
    void* wsv = nullptr;
    FlashAttentionError werr = workspace_alloc(&wsv, bytes, stream);
    if (werr != FlashAttentionError::SUCCESS) return werr;
    float* o_part = static_cast<float*>(wsv);
    float* l_part = o_part + part_elems;
    auto k = decode_group_kernel<T, D, TILE, kPaged, false>;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(k), static_cast<int>(smem))) {
        workspace_free(wsv, stream);
        return FlashAttentionError::CUDA_ERROR;
    }
    k<<<dim3(ctas_y, S), kDecodeThreads, smem, stream>>>(Q, kvp, nullptr, nullptr, o_part, l_part,
                                                          hq, group, chunk, sl2);
    cudaError_t e1 = cudaGetLastError();
    decode_combine_kernel<T, D><<<BHq, 128, 0, stream>>>(o_part, l_part, O, L, S);
    cudaError_t e2 = cudaGetLastError();
    workspace_free(wsv, stream);
    return (e1 == cudaSuccess && e2 == cudaSuccess) ? FlashAttentionError::SUCCESS
                                                    : FlashAttentionError::CUDA_ERROR;
}

// ---------------------------------------------------------------------------
// Grouped-query decode on the tensor cores (head_dim 64 and 128).  The SIMT kernel
// above reduces every (cache row, query head) dot product across 16 lanes
// with shuffles, and that chain, not the cache bytes, sets its speed.  Here a
// CTA serves up to 16 query heads of one K/V head over a range of cache rows,
// 128 rows at a time:
//   S^T = K Q^T    tcgen05 M = 128 cache rows, N = 16 heads, K = head_dim
//                  (A = the K block, B = the padded query tile; both K-major);
//   softmax        one thread per cache row: per-head block maxima by warp
//                  shuffles and a 4-warp exchange, running maxima raised only
//                  when they grow by more than 2^8 (then O^T is rescaled),
//                  P^T (16-bit) written to shared memory;
//   O^T += V^T P^T M = head_dim, N = 16 heads, K = 128 cache rows (A = the V
//                  block read MN-major, B = P^T K-major).
// K/V blocks arrive by TMA through a ring of 3 stages (head_dim 128; head_dim
// 64: 2 stages, two CTAs per SM) (contiguous cache: one box
// per 64 columns; paged cache: one box per page and 64 columns, pages of 8 or
// more rows).  MMA order S0, S1, O0, S2, O1, ...: S_j is issued right behind
// O_{j-2}, so the completion of S_j (which the softmax waits for) also means
// O_{j-2} has read the P^T buffer the softmax is about to overwrite.  TMEM:
// S^T double-buffered in columns [0,32), O^T in [32,48).  At head_dim 64 the
// V block keeps its 128-element width with the upper half zero, so O^T stays
// an M = 128 product (at N = 16 it costs what an M = 64 one does) and its
// rows 64-127, never read, stay zero.
// ---------------------------------------------------------------------------
__device__ sm100::StatusWord g_dec_status;

constexpr int kTcHeads = 16;
constexpr int kTcRows = 128;
constexpr int kTcThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 softmax / epilogue

template <int D>
struct TcGeom {
    // head_dim 64: two CTAs per SM (a 128-row block is half the bytes for the
    // same MMA / softmax chain), so two stages each; head_dim 128: one CTA,
    // three stages
    static constexpr int kCtasPerSm = D == 64 ? 2 : 1;
    static constexpr int kStages = D == 64 ? 2 : 3;
    static constexpr int kKcb = D / 64;                   // 64-element column blocks of K, Q
    static constexpr int kKvCbBytes = kTcRows * 128;      // 128 rows x 64 elements
    static constexpr int kKTileBytes = kKcb * kKvCbBytes;  // one K block
    static constexpr int kVTileBytes = 2 * kKvCbBytes;     // one V block, 128 wide (see above)
    static constexpr int kStageBytes = kKTileBytes + kVTileBytes;
    static constexpr int kLoadBytes = 2 * kKTileBytes;     // TMA bytes per stage (K, V)
    static constexpr int kQCbBytes = kTcHeads * 128;
    static constexpr int kQBytes = kKcb * kQCbBytes;
    static constexpr int kPCbBytes = kTcHeads * 128;      // 16 heads x 64 cache rows (16-bit)
    static constexpr int kPBytes = 2 * kPCbBytes;
    static constexpr int kOffQ = kStages * kStageBytes;
    static constexpr int kOffP = kOffQ + kQBytes;
    static constexpr int kOffRed = kOffP + 2 * kPBytes;
    static constexpr int kRedFloats = 4 * kTcHeads;
    static constexpr int kOffBar = kOffRed + 3 * kRedFloats * 4;
    static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2 + 1 + 1;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
    static_assert(kOffQ % 1024 == 0 && kOffP % 1024 == 0, "swizzled tiles need 1024-byte alignment");
};

struct TcParams {
    void* O;
    float* L;
    float* O_part;
    float* L_part;
    const int* block_table;
    const int* seq_lens;
    int kv_len;
    int hkv;
    int hq;
    int group;
    int head_tiles;
    int chunk;  // rows per split, a multiple of 128
    int page_shift;
    int max_pages;
    int num_pages;
    float scale_log2;
};

// K-major operand of 64-element (128-byte) swizzled rows, `cb_bytes` per
// 64-column block: descriptor of k-step kk (16 elements).
__device__ __forceinline__ uint64_t tc_kmajor(uint32_t base, uint32_t cb_bytes, int kk) {
    const uint32_t byte = static_cast<uint32_t>(kk) * 32u;
    return sm100::make_smem_desc(base + (byte >> 7) * cb_bytes + (byte & 127u), 16, 1024,
                                 sm100::kLayoutSw128);
}
// MN-major operand (K dimension = rows of 128 bytes): k-step kk covers 16 rows.
__device__ __forceinline__ uint64_t tc_mnmajor(uint32_t base, uint32_t cb_bytes, int kk) {
    return sm100::make_smem_desc(base + static_cast<uint32_t>(kk) * 16u * 128u, cb_bytes, 1024,
                                 sm100::kLayoutSw128);
}

__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem_dec() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void softmax_group_sync() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

template <typename T, int D, bool kPaged, bool kDirect>
__global__ void __launch_bounds__(kTcThreads, TcGeom<D>::kCtasPerSm)
    decode_gqa_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const TcParams p) {
    using G = TcGeom<D>;
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    if (sm100::cta_skip(&g_dec_status)) return;
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t* sptr = smem_raw + (sbase - raw);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sptr + G::kOffBar);
    uint64_t* bar_q = bars;
    uint64_t* full = bar_q + 1;
    uint64_t* empty = full + G::kStages;
    uint64_t* bar_s = empty + G::kStages;  // [2] S^T_j in TMEM
    uint64_t* bar_sfree = bar_s + 2;      // [2] S^T_j read by the softmax (128 arrivals)
    uint64_t* bar_p = bar_sfree + 2;      // [2] P^T_j in shared memory (128 arrivals)
    uint64_t* bar_ofin = bar_p + 2;       // one completion per O^T product
    uint64_t* bar_done = bar_ofin + 1;    // every MMA retired
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* red = reinterpret_cast<float*>(sptr + G::kOffRed);  // 3 x [4 warps][16 heads]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int split = blockIdx.y;
    const int tile = blockIdx.x % p.head_tiles;
    const int bhk = blockIdx.x / p.head_tiles;
    const int b = bhk / p.hkv;
    const int hk = bhk - b * p.hkv;
    const int g0 = tile * kTcHeads;
    const int nh = min(kTcHeads, p.group - g0);
    const long long bhq0 = static_cast<long long>(b) * p.hq + static_cast<long long>(hk) * p.group + g0;
    // a paged length is clamped to what the block table can address
    const int len = kPaged ? min(max(p.seq_lens[b], 0), p.max_pages << p.page_shift) : p.kv_len;
    const int r_begin = split * p.chunk;
    const int r_end = min(len, r_begin + p.chunk);
    const int nb = r_end > r_begin ? (r_end - r_begin + kTcRows - 1) / kTcRows : 0;

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        for (int s = 0; s < G::kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(bar_s + t, 1);
            mbar_init(bar_sfree + t, 128);
            mbar_init(bar_p + t, 128);
        }
        mbar_init(bar_ofin, 1);
        mbar_init(bar_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 64);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        // Lane 0 owns the ring (waits, expected bytes); on a paged cache each
        // lane q < boxes-per-block also loads its page's index and issues that
        // page's boxes, so small pages do not serialise dozens of copies on
        // one thread (16-row pages: 32 boxes per 128-row block).
        if (nb > 0) {
            if (lane == 0) {
                prefetch_tmap(&tmQ);
                prefetch_tmap(&tmK);
                prefetch_tmap(&tmV);
                // query rows bhq0 .. bhq0+15; rows of the next group or past the
                // tensor end fill heads this CTA does not report
                mbar_arrive_expect_tx(bar_q, G::kQBytes);
                for (int cb = 0; cb < G::kKcb; ++cb)
                    tma_load_3d(sptr + G::kOffQ + cb * G::kQCbBytes, &tmQ, bar_q, cb * 64,
                                static_cast<int>(bhq0), 0);
            }
            int issued = 0;
            const int ps = 1 << p.page_shift;
            const int per = ps < kTcRows ? ps : kTcRows;  // rows per TMA box (paged)
            const int npb = kTcRows / per;                // boxes per block (paged, <= 16)
            for (int j = 0; j < nb; ++j) {
                const int s = j % G::kStages;
                const int r0 = r_begin + j * kTcRows;
                // paged: this lane's page index, loaded before the ring wait so
                // that its latency overlaps it
                int page = 0;
                if (kPaged && lane < npb) {
                    const int pi = min((r0 + lane * per) >> p.page_shift, p.max_pages - 1);
                    page = p.block_table[static_cast<long long>(b) * p.max_pages + pi];
                }
                bool go = true;
                if (lane == 0) {
                    go = j < G::kStages ||
                         mbar_wait(empty + s, ((j / G::kStages) - 1) & 1, abort_flag, &g_dec_status);
                    if (go) mbar_arrive_expect_tx(full + s, G::kLoadBytes);
                }
                // every lane sees lane 0's decision; its expect_tx precedes
                // every lane's copies
                if (!__shfl_sync(0xffffffffu, go, 0)) break;
                __syncwarp();
                ++issued;
                uint8_t* st = sptr + s * G::kStageBytes;
                if constexpr (!kPaged) {
                    if (lane == 0) {
                        for (int cb = 0; cb < G::kKcb; ++cb) {
                            tma_load_3d(st + cb * G::kKvCbBytes, &tmK, full + s, cb * 64, r0, bhk);
                            tma_load_3d(st + G::kKTileBytes + cb * G::kKvCbBytes, &tmV, full + s,
                                        cb * 64, r0, bhk);
                        }
                    }
                } else if (lane < npb) {
                    const int rr = lane * per;
                    const int pg = min(max(page, 0), p.num_pages - 1);
                    const int slot = (pg << p.page_shift) + ((r0 + rr) & (ps - 1));
                    for (int cb = 0; cb < G::kKcb; ++cb) {
                        tma_load_3d(st + cb * G::kKvCbBytes + rr * 128, &tmK, full + s, cb * 64,
                                    hk, slot);
                        tma_load_3d(st + G::kKTileBytes + cb * G::kKvCbBytes + rr * 128, &tmV,
                                    full + s, cb * 64, hk, slot);
                    }
                }
            }
            // every issued copy lands before the CTA can exit, also after an abort
            if (lane == 0) {
                volatile int never = 0;
                mbar_wait(bar_q, 0, &never, &g_dec_status);
                for (int j = issued > G::kStages ? issued - G::kStages : 0; j < issued; ++j)
                    mbar_wait(full + j % G::kStages, (j / G::kStages) & 1, &never, &g_dec_status);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0 && nb > 0) {
            constexpr uint32_t kFmt = DType<T>::kMmaFmt;
            constexpr uint32_t idesc_s = make_idesc(kFmt, 128, kTcHeads, false, false);
            constexpr uint32_t idesc_o = make_idesc(kFmt, 128, kTcHeads, true, false);
            const uint32_t sQ = sbase + G::kOffQ;
            bool ok = mbar_wait(bar_q, 0, abort_flag, &g_dec_status);
            auto issue_s = [&](int j) {
                const int s = j % G::kStages;
                if (!mbar_wait(full + s, (j / G::kStages) & 1, abort_flag, &g_dec_status)) return false;
                if (j >= 2 &&
                    !mbar_wait(bar_sfree + (j & 1), ((j >> 1) - 1) & 1, abort_flag, &g_dec_status))
                    return false;
                tc_fence_after();
                const uint32_t sK = sbase + s * G::kStageBytes;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    mma_f16_ss(tmem + (j & 1) * kTcHeads, tc_kmajor(sK, G::kKvCbBytes, kk),
                               tc_kmajor(sQ, G::kQCbBytes, kk), idesc_s, kk > 0 ? 1u : 0u);
                tc_commit(bar_s + (j & 1));
                return true;
            };
            auto issue_o = [&](int j) {
                if (!mbar_wait(bar_p + (j & 1), (j >> 1) & 1, abort_flag, &g_dec_status)) return false;
                tc_fence_after();
                const uint32_t sV = sbase + (j % G::kStages) * G::kStageBytes + G::kKTileBytes;
                const uint32_t sP = sbase + G::kOffP + (j & 1) * G::kPBytes;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_f16_ss(tmem + 2 * kTcHeads, tc_mnmajor(sV, G::kKvCbBytes, kk),
                               tc_kmajor(sP, G::kPCbBytes, kk), idesc_o,
                               (j > 0 || kk > 0) ? 1u : 0u);
                tc_commit(empty + (j % G::kStages));
                tc_commit(bar_ofin);
                return true;
            };
            ok = ok && issue_s(0);
            if (nb > 1) ok = ok && issue_s(1);
            for (int j = 0; ok && j < nb; ++j) {
                ok = issue_o(j);
                if (ok && j + 2 < nb) ok = issue_s(j + 2);
            }
            tc_commit(bar_done);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ softmax and epilogue
        const int q4 = warp & 3;     // TMEM lane quarter of this warp
        const int wsm = warp - 2;    // index in the cross-warp exchange
        const int r = q4 * 32 + lane;  // cache row of the block (S^T) / head_dim element (O^T)
        const uint32_t lane_addr = static_cast<uint32_t>(q4 * 32) << 16;
        const float c = p.scale_log2;
        float m_run[kTcHeads], l_part[kTcHeads];
#pragma unroll
        for (int g = 0; g < kTcHeads; ++g) {
            m_run[g] = -INFINITY;
            l_part[g] = 0.f;
        }
        if constexpr (D < 128) {
            // the V blocks' upper 64 columns: zero once, never loaded (made
            // visible to the tensor core by the proxy fence before the first
            // P^T hand-off)
            const int t = threadIdx.x - 64;
            for (int s = 0; s < G::kStages; ++s) {
                const uint32_t hi = sbase + s * G::kStageBytes + G::kKTileBytes + G::kKvCbBytes;
                for (int i = t; i < G::kKvCbBytes / 16; i += 128)
                    asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(hi + i * 16),
                                 "r"(0u)
                                 : "memory");
            }
        }
        // Every softmax thread runs all nb iterations and both group barriers
        // per iteration whatever happens; after a failed (timed-out or
        // aborted) wait, `ok` turns false warp-uniformly and the warp skips
        // its TMEM and barrier traffic, so no thread is left in bar.sync.
        bool ok = true;
        for (int j = 0; j < nb; ++j) {
            if (ok) ok = mbar_wait(bar_s + (j & 1), (j >> 1) & 1, abort_flag, &g_dec_status);
            ok = __all_sync(0xffffffffu, ok);
            uint32_t sv[16];
            if (ok) {
                tc_fence_after();
                tmem_ld_x16(tmem + lane_addr + (j & 1) * kTcHeads, sv);
                tc_fence_before();
                mbar_arrive(bar_sfree + (j & 1));
            } else {
#pragma unroll
                for (int g = 0; g < kTcHeads; ++g) sv[g] = 0u;
            }
            const bool live = r_begin + j * kTcRows + r < r_end;
            float x[kTcHeads];
#pragma unroll
            for (int g = 0; g < kTcHeads; ++g) x[g] = live ? __uint_as_float(sv[g]) * c : -INFINITY;
            // per-head block maxima: warp shuffles, then the four warps
            float* rm = red + (j & 1) * G::kRedFloats;
#pragma unroll
            for (int g = 0; g < kTcHeads; ++g) {
                float v = x[g];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
                if (lane == 0) rm[wsm * kTcHeads + g] = v;
            }
            softmax_group_sync();
            bool resc = false;
            float alpha[kTcHeads];
#pragma unroll
            for (int g = 0; g < kTcHeads; ++g) {
                const float bm = fmaxf(fmaxf(rm[g], rm[kTcHeads + g]),
                                       fmaxf(rm[2 * kTcHeads + g], rm[3 * kTcHeads + g]));
                float mn = m_run[g];
                if (mn == -INFINITY || bm > mn + 8.f) mn = fmaxf(mn, bm);
                alpha[g] = (m_run[g] == -INFINITY || mn == m_run[g]) ? 1.f : ex2_approx(m_run[g] - mn);
                resc = resc || alpha[g] != 1.f;
                m_run[g] = mn;
            }
            if (resc && ok) {  // resc is uniform: every thread saw the same maxima
                // O^T_{j-1} must be complete (j >= 1 here: the first block never rescales)
                ok = mbar_wait(bar_ofin, (j - 1) & 1, abort_flag, &g_dec_status);
                ok = __all_sync(0xffffffffu, ok);
            }
            if (resc && ok) {
                tc_fence_after();
                uint32_t ov[16];
                tmem_ld_x16(tmem + lane_addr + 2 * kTcHeads, ov);
#pragma unroll
                for (int g = 0; g < kTcHeads; ++g) {
                    ov[g] = __float_as_uint(__uint_as_float(ov[g]) * alpha[g]);
                    l_part[g] *= alpha[g];
                }
                tmem_st_x16(tmem + lane_addr + 2 * kTcHeads, ov);
                tc_fence_before();
            }
            // P^T (head g, cache row r) into buffer j & 1, 128-byte swizzled K-major
            const uint32_t pb = sbase + G::kOffP + (j & 1) * G::kPBytes + (r >> 6) * G::kPCbBytes;
            const int kr = r & 63;
#pragma unroll
            for (int g = 0; g < kTcHeads; ++g) {
                const float pv = m_run[g] == -INFINITY ? 0.f : ex2_approx(x[g] - m_run[g]);
                l_part[g] += pv;
                const uint32_t addr = pb + g * 128 + ((((kr >> 3) ^ (g & 7))) << 4) + (kr & 7) * 2;
                const T h = DType<T>::from_float(pv);
                st_shared_u16(addr, *reinterpret_cast<const uint16_t*>(&h));
            }
            if constexpr (kPaged) {
                // rows past the sequence end hold whatever the cache page has;
                // zero their V so that P = 0 cannot meet a non-finite value
                if (!live) {
                    const uint32_t vrow = sbase + (j % G::kStages) * G::kStageBytes + G::kKTileBytes +
                                          r * 128;
#pragma unroll
                    for (int cb = 0; cb < 2; ++cb)
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(
                                             vrow + cb * G::kKvCbBytes + q * 16),
                                         "r"(0u)
                                         : "memory");
                }
            }
            if (ok) {
                fence_proxy_async_smem_dec();
                mbar_arrive(bar_p + (j & 1));
            }
        }
        // ---- epilogue: normalise, write the split's result
        if (ok && nb > 0) {
            ok = mbar_wait(bar_done, 0, abort_flag, &g_dec_status);
            tc_fence_after();
        }
        ok = __all_sync(0xffffffffu, ok);
        float* rs = red + 2 * G::kRedFloats;
#pragma unroll
        for (int g = 0; g < kTcHeads; ++g) {
            float v = l_part[g];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) rs[wsm * kTcHeads + g] = v;
        }
        softmax_group_sync();
        uint32_t ov[16];
        if (ok && nb > 0) {
            tmem_ld_x16(tmem + lane_addr + 2 * kTcHeads, ov);
        } else {
#pragma unroll
            for (int g = 0; g < kTcHeads; ++g) ov[g] = 0u;
        }
        const int d = r;
#pragma unroll
        for (int g = 0; g < kTcHeads; ++g) {
            if (g >= nh || d >= D) continue;
            const float lt = rs[g] + rs[kTcHeads + g] + rs[2 * kTcHeads + g] + rs[3 * kTcHeads + g];
            const float outv = lt > 0.f ? __uint_as_float(ov[g]) / lt : 0.f;
            const float lse = lt > 0.f ? (m_run[g] + log2f(lt)) * kLn2f : -INFINITY;
            const long long bhq = bhq0 + g;
            if constexpr (kDirect) {
                static_cast<T*>(p.O)[bhq * D + d] = DType<T>::from_float(outv);
                if (d == 0) p.L[bhq] = lse;
            } else {
                p.O_part[(bhq * gridDim.y + split) * D + d] = outv;
                if (d == 0) p.L_part[bhq * gridDim.y + split] = lse;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 64);
    }
}

// Tensor-core grouped-query decode for head_dim 64 and 128 (see the kernel above).
template <typename T, int D, bool kPaged>
FlashAttentionError decode_gqa_tc(const T* Q, const DecodeKv<T>& kvp, T* O, float* L, int B,
                                  int hq, int max_len, float scale, int num_splits,
                                  cudaStream_t stream) {
    using G = TcGeom<D>;
    const int group = hq / kvp.hkv;
    const int tiles = (group + kTcHeads - 1) / kTcHeads;
    const long long units = static_cast<long long>(B) * kvp.hkv * tiles;
    if (units > 0x7fffffffLL) return FlashAttentionError::INVALID_DIMENSION;
    const int blocks_total = (max_len + kTcRows - 1) / kTcRows;
    int S = num_splits;
    if (S == 0) {
        // One wave of CTAs (one per SM, each streaming its rows): measured on
        // B200 over B 8-64, Nkv 4k-32k, groups 2-16, the best split count is
        // about SMs / units (units 16 / 32 / 64 / >= 128 -> 8 / 4 / 2 / 1);
        // at least two blocks per split.
        S = static_cast<int>(
            std::max<long long>(1, static_cast<long long>(G::kCtasPerSm) * current_sm_count() / units));
        S = std::min(S, std::max(1, blocks_total / 2));
    }
    S = std::max(1, std::min(S, std::min(64, std::max(1, blocks_total))));
    const int chunk = ((blocks_total + S - 1) / S) * kTcRows;
    S = (max_len + chunk - 1) / chunk;
    if (S < 1) S = 1;

    const CUtensorMapDataType dt = DType<T>::kTmaType;
    CUtensorMap mq, mk, mv;
    if (!encode_tmap_3d(&mq, Q, dt, 2, D, static_cast<uint64_t>(B) * hq, 1, 64, kTcHeads,
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return FlashAttentionError::CUDA_ERROR;
    if (!kPaged) {
        if (!encode_tmap_3d(&mk, kvp.K, dt, 2, D, kvp.kv_len, static_cast<uint64_t>(B) * kvp.hkv,
                            64, kTcRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !encode_tmap_3d(&mv, kvp.V, dt, 2, D, kvp.kv_len, static_cast<uint64_t>(B) * kvp.hkv,
                            64, kTcRows, CU_TENSOR_MAP_SWIZZLE_128B))
            return FlashAttentionError::CUDA_ERROR;
    } else {
        const int ps = 1 << kvp.page_shift;
        const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(kvp.hkv),
                                  static_cast<uint64_t>(kvp.num_pages) << kvp.page_shift};
        const uint64_t strides[2] = {static_cast<uint64_t>(D) * 2,
                                     static_cast<uint64_t>(kvp.hkv) * D * 2};
        const uint32_t box[3] = {64, 1, static_cast<uint32_t>(ps < kTcRows ? ps : kTcRows)};
        if (!encode_tmap_3d_strided(&mk, kvp.K, dt, dims, strides, box,
                                    CU_TENSOR_MAP_SWIZZLE_128B) ||
            !encode_tmap_3d_strided(&mv, kvp.V, dt, dims, strides, box,
                                    CU_TENSOR_MAP_SWIZZLE_128B))
            return FlashAttentionError::CUDA_ERROR;
    }
    TcParams prm{};
    prm.block_table = kvp.block_table;
    prm.seq_lens = kvp.seq_lens;
    prm.kv_len = kvp.kv_len;
    prm.hkv = kvp.hkv;
    prm.hq = hq;
    prm.group = group;
    prm.head_tiles = tiles;
    prm.chunk = chunk;
    prm.page_shift = kvp.page_shift;
    prm.max_pages = kvp.max_pages;
    prm.num_pages = kvp.num_pages;
    prm.scale_log2 = scale * kLog2ef;
    const dim3 grid(static_cast<unsigned>(units), S);
    if (S == 1) {
        auto k = decode_gqa_tc_kernel<T, D, kPaged, true>;
        if (!ensure_smem_attr(reinterpret_cast<const void*>(k), G::kSmemBytes))
            return FlashAttentionError::CUDA_ERROR;
        prm.O = O;
        prm.L = L;
        bind_status_word(reinterpret_cast<const void*>(&g_dec_status), stream);
        k<<<grid, kTcThreads, G::kSmemBytes, stream>>>(mq, mk, mv, prm);
        return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                                 : FlashAttentionError::CUDA_ERROR;
    }
    const int BHq = B * hq;
    const size_t part_elems = static_cast<size_t>(BHq) * S * D;
    const size_t bytes = (part_elems + static_cast<size_t>(BHq) * S) * sizeof(float);
    void* wsv = nullptr;
    FlashAttentionError werr = workspace_alloc(&wsv, bytes, stream);
    if (werr != FlashAttentionError::SUCCESS) return werr;
    prm.O_part = static_cast<float*>(wsv);
    prm.L_part = prm.O_part + part_elems;
    auto k = decode_gqa_tc_kernel<T, D, kPaged, false>;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(k), G::kSmemBytes)) {
        workspace_free(wsv, stream);
        return FlashAttentionError::CUDA_ERROR;
    }
    bind_status_word(reinterpret_cast<const void*>(&g_dec_status), stream);
    k<<<grid, kTcThreads, G::kSmemBytes, stream>>>(mq, mk, mv, prm);
    cudaError_t e1 = cudaGetLastError();
    decode_combine_kernel<T, D><<<BHq, 128, 0, stream>>>(prm.O_part, prm.L_part, O, L, S);
    cudaError_t e2 = cudaGetLastError();
    workspace_free(wsv, stream);
    return (e1 == cudaSuccess && e2 == cudaSuccess) ? FlashAttentionError::SUCCESS
                                                    : FlashAttentionError::CUDA_ERROR;
}

template <typename T, int D, bool kPaged>
FlashAttentionError decode_group_tile(const T* Q, const DecodeKv<T>& kvp, T* O, float* L, int B,
                                      int hq, int max_len, float scale, int num_splits,
                                      cudaStream_t stream) {
    // Query heads per CTA: at most 4 on a contiguous cache and 2 on a paged
    // one.  Larger tiles read each cache row once for more heads but hold more
    // registers (8 heads: 216 per thread, one CTA per SM) and have too few
    // bytes in flight; measured on B200 at B64 Hq32 Nkv16384 D128 (group 4 /
    // 8): contiguous 1.31 / 1.26 ms with 4 heads per CTA against 1.31 / 1.96
    // with 8; paged 1.67 / 1.62 ms with 2 against 2.91 / 2.76 with 4.
    const int group = hq / kvp.hkv;
    if constexpr (D == 128 || D == 64) {
        // tensor-core kernel from two heads per K/V head up (pages of 8+ rows)
        if (group >= 2 && (!kPaged || kvp.page_shift >= 3) && env_int("CUFLASH_DECODE_GQA_TC", 1) != 0)
            return decode_gqa_tc<T, D, kPaged>(Q, kvp, O, L, B, hq, max_len, scale, num_splits,
                                               stream);
    }
    if (group % 4 == 0 && !kPaged)
        return decode_group_typed<T, D, 4, kPaged>(Q, kvp, O, L, B, hq, max_len, scale,
                                                   num_splits, stream);
    if (group % 2 == 0)
        return decode_group_typed<T, D, 2, kPaged>(Q, kvp, O, L, B, hq, max_len, scale,
                                                   num_splits, stream);
    return decode_group_typed<T, D, 1, kPaged>(Q, kvp, O, L, B, hq, max_len, scale, num_splits,
                                               stream);
}

}  // namespace

template <typename T>
FlashAttentionError launch_decode(const T* Q, const T* K, const T* V, T* O, float* L, int B, int H,
                                  int kv_len, int D, float scale, int num_splits,
                                  cudaStream_t stream) {
    const int BH = B * H;
    switch (D) {
        case 32:
            return decode_typed<T, 32>(Q, K, V, O, L, BH, kv_len, scale, num_splits, stream);
        case 64:
            return decode_typed<T, 64>(Q, K, V, O, L, BH, kv_len, scale, num_splits, stream);
        case 128:
            return decode_typed<T, 128>(Q, K, V, O, L, BH, kv_len, scale, num_splits, stream);
        default:
            return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
}

template FlashAttentionError launch_decode<half>(const half*, const half*, const half*, half*,
                                                 float*, int, int, int, int, float, int,
                                                 cudaStream_t);
template FlashAttentionError launch_decode<__nv_bfloat16>(const __nv_bfloat16*,
                                                          const __nv_bfloat16*,
                                                          const __nv_bfloat16*, __nv_bfloat16*,
                                                          float*, int, int, int, int, float, int,
                                                          cudaStream_t);

template <typename T>
FlashAttentionError launch_decode_gqa(const T* Q, const T* K, const T* V, T* O, float* L, int B,
                                      int Hq, int Hkv, int kv_len, int D, float scale,
                                      int num_splits, const int* block_table,
                                      const int* seq_lens, int page_size, int max_pages,
                                      int num_pages, cudaStream_t stream) {
    for (const void* p : {static_cast<const void*>(Q), static_cast<const void*>(K),
                          static_cast<const void*>(V), static_cast<const void*>(O)})
        if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return FlashAttentionError::CUDA_ERROR;
    DecodeKv<T> kvp;
    kvp.K = K;
    kvp.V = V;
    kvp.block_table = block_table;
    kvp.seq_lens = seq_lens;
    kvp.kv_len = kv_len;
    kvp.hkv = Hkv;
    kvp.page_shift = 0;
    while (page_size > 0 && (1 << kvp.page_shift) < page_size) ++kvp.page_shift;
    kvp.max_pages = max_pages;
    kvp.num_pages = num_pages;
    const bool paged = block_table != nullptr;
    const int max_len = paged ? max_pages * page_size : kv_len;
#define CUFLASH_DECODE_GQA(DD)                                                                    \
    return paged ? decode_group_tile<T, DD, true>(Q, kvp, O, L, B, Hq, max_len, scale,           \
                                                  num_splits, stream)                            \
                 : decode_group_tile<T, DD, false>(Q, kvp, O, L, B, Hq, max_len, scale,          \
                                                   num_splits, stream)
    switch (D) {
        case 32: CUFLASH_DECODE_GQA(32);
        case 64: CUFLASH_DECODE_GQA(64);
        case 128: CUFLASH_DECODE_GQA(128);
        default: return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
#undef CUFLASH_DECODE_GQA
}

int dec_sm100_status() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_dec_status, sizeof(int)) != cudaSuccess) return -1;
    if (v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_dec_status, &zero, sizeof(int));
    }
    return v;
}

template FlashAttentionError launch_decode_gqa<half>(const half*, const half*, const half*, half*,
                                                     float*, int, int, int, int, int, float, int,
                                                     const int*, const int*, int, int, int,
                                                     cudaStream_t);
template FlashAttentionError launch_decode_gqa<__nv_bfloat16>(
    const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, __nv_bfloat16*, float*,
    int, int, int, int, int, float, int, const int*, const int*, int, int, int, cudaStream_t);

FlashAttentionError launch_lse_merge(float* O_acc, float* L_acc, const float* O_part,
                                     const float* L_part, long long rows, int D,
                                     cudaStream_t stream) {
    long long blocks = (rows * 32 + 255) / 256;
    const long long cap = 16LL * current_sm_count();
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    lse_merge_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(O_acc, L_acc, O_part,
                                                                         L_part, rows, D);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

template <typename T>
FlashAttentionError launch_convert_f32(const float* src, T* dst, long long count,
                                       cudaStream_t stream) {
    long long blocks = (count + 255) / 256;
    const long long cap = 32LL * current_sm_count();
    if (blocks > cap) blocks = cap;
    convert_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, dst, count);
    return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                             : FlashAttentionError::CUDA_ERROR;
}

template FlashAttentionError launch_convert_f32<half>(const float*, half*, long long,
                                                      cudaStream_t);
template FlashAttentionError launch_convert_f32<__nv_bfloat16>(const float*, __nv_bfloat16*,
                                                               long long, cudaStream_t);


// ---------------------------------------------------------------------------
// Split-KV decode without any allocation.
//
// Some callers cannot let a library allocate device memory: serving engines
// that claim nearly all of HBM at start-up for their KV-cache pages and hand
// memory out only through their own allocator (a stray cudaMalloc either
// fails or fragments that reservation), and latency-critical decode loops that
// keep allocation calls, whose cost is unpredictable, off the per-token path.
// For them the split partials live in this fixed buffer instead of the
// stream-ordered workspace.
//
// kNoAllocScratchFloats fp32 values (8 MiB) are reserved on every GPU that
// loads the library and stay reserved until the process exits.  The buffer
// is shared by all calls and keeps whatever the last call left in it; each
// call overwrites every partial it reads, so nothing needs clearing first.
// Two calls whose kernels overlap on the GPU (different streams, or
// different host threads) race on the buffer and must be serialised by the
// caller.
// ---------------------------------------------------------------------------
constexpr long long kNoAllocScratchFloats = 2LL * 1024 * 1024;  // 8 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

namespace {

// Device address of g_noalloc_scratch on the current device.  In host code
// the symbol is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
FlashAttentionError noalloc_scratch_ptr(float** out) {
    static std::mutex mu;
    static float* cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return FlashAttentionError::CUDA_ERROR;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == nullptr) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) {
            cudaGetLastError();
            return FlashAttentionError::CUDA_ERROR;
        }
        cache[dev] = static_cast<float*>(ptr);
    }
    *out = cache[dev];
    return FlashAttentionError::SUCCESS;
}

template <int D>
FlashAttentionError decode_noalloc_typed(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                         const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                         int BH, int kv_len, float scale, int num_splits,
                                         cudaStream_t stream) {
    using T = __nv_bfloat16;
    for (const void* p : {static_cast<const void*>(Q), static_cast<const void*>(K),
                          static_cast<const void*>(V), static_cast<const void*>(O)})
        if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return FlashAttentionError::CUDA_ERROR;
    const long long per_split = static_cast<long long>(BH) * (D + 1);  // partial O + its LSE
    int S;
    if (num_splits == 0) {
        S = auto_splits(BH, kv_len);
        const long long fit = kNoAllocScratchFloats / per_split;  // auto mode stays within it
        if (S > fit) S = static_cast<int>(fit < 1 ? 1 : fit);
    } else {
        S = num_splits;
    }
    if (S > kv_len) S = kv_len;
    const int chunk = (kv_len + S - 1) / S;
    S = (kv_len + chunk - 1) / chunk;
    const float sl2 = scale * kLog2ef;
    if (S == 1) {
        decode_split_kernel<T, D, true><<<dim3(BH, 1), kDecodeThreads, 0, stream>>>(
            Q, K, V, O, L, nullptr, nullptr, kv_len, chunk, sl2);
        return cudaGetLastError() == cudaSuccess ? FlashAttentionError::SUCCESS
                                                 : FlashAttentionError::CUDA_ERROR;
    }
    if (per_split * S > kNoAllocScratchFloats) return FlashAttentionError::OUT_OF_MEMORY;
    float* scratch = nullptr;
    FlashAttentionError e = noalloc_scratch_ptr(&scratch);
    if (e != FlashAttentionError::SUCCESS) return e;
    float* o_part = scratch;
    float* l_part = scratch + static_cast<size_t>(BH) * S * D;
    decode_split_kernel<T, D, false><<<dim3(BH, S), kDecodeThreads, 0, stream>>>(
        Q, K, V, nullptr, nullptr, o_part, l_part, kv_len, chunk, sl2);
    cudaError_t e1 = cudaGetLastError();
    decode_combine_kernel<T, D><<<BH, 128, 0, stream>>>(o_part, l_part, O, L, S);
    cudaError_t e2 = cudaGetLastError();
    return (e1 == cudaSuccess && e2 == cudaSuccess) ? FlashAttentionError::SUCCESS
                                                    : FlashAttentionError::CUDA_ERROR;
}

}  // namespace

FlashAttentionError launch_decode_bf16_noalloc(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                               const __nv_bfloat16* V, __nv_bfloat16* O, float* L,
                                               int B, int H, int kv_len, int D, float scale,
                                               int num_splits, cudaStream_t stream) {
    const int BH = B * H;
    switch (D) {
        case 32:
            return decode_noalloc_typed<32>(Q, K, V, O, L, BH, kv_len, scale, num_splits, stream);
        case 64:
            return decode_noalloc_typed<64>(Q, K, V, O, L, BH, kv_len, scale, num_splits, stream);
        case 128:
            return decode_noalloc_typed<128>(Q, K, V, O, L, BH, kv_len, scale, num_splits, stream);
        default:
            return FlashAttentionError::UNSUPPORTED_HEAD_DIM;
    }
}

}  // namespace detail
}  // namespace cuflash
