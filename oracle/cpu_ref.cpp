// TEST INFRASTRUCTURE ONLY — the CPU oracle for parity tests and the CPU
// baseline leg of bench.py.  Nothing in the library calls this code.
//
// Restates the reference's CPU attention (AICL-Lab/cuflash-attn v0.5.0):
//   * reference_attention_forward   tests/unit/test_forward.cu:21-69
//   * reference_logsumexp           tests/unit/test_forward.cu:83-118
//   * reference_attention_backward  tests/unit/test_backward.cu:21-127
// in two precisions:
//   * *_f32: the reference's arithmetic (fp32 values, fp32 accumulation in
//     the same loop order, std::exp / std::log on floats) — this is the
//     "reference CPU path" that bench.py times;
//   * *_f64: the same formulas in double precision — the ground truth the
//     GPU results are held to.
// plus the reference tests' input generators (std::mt19937 with
// std::uniform_real_distribution<float>, filled interleaved per index as in
// test_forward.cu:133-139 / test_backward.cu:148-157) and the
// BASELINE.json generators (one mt19937 per tensor, normal or uniform).
//
// Work is split over (batch, head) units; every entry point takes an
// explicit unit range and a thread count so callers can time a bounded
// sample of a large problem on a stated number of host cores.
//
// Parity pins for this file: tests/test_oracle.py (known-answer identities
// taken from the reference's tests and the committed golden vectors that the
// reference's own CUDA library produced; see tests/golden/).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

namespace {

template <typename F>
void parallel_units(long long u0, long long u1, int nthreads, F&& fn) {
    if (nthreads <= 1 || u1 - u0 <= 1) {
        for (long long u = u0; u < u1; ++u) fn(u);
        return;
    }
    const long long n = u1 - u0;
    const int nt = static_cast<int>(std::min<long long>(nthreads, n));
    std::vector<std::thread> th;
    th.reserve(nt);
    for (int t = 0; t < nt; ++t) {
        th.emplace_back([&, t] {
            for (long long u = u0 + t; u < u1; u += nt) fn(u);
        });
    }
    for (auto& x : th) x.join();
}

// ---- fp32, as the reference: one (b,h) unit, rows [0, N) --------------------

// test_forward.cu:21-69 (O) fused with test_forward.cu:83-118 (L).  The O loop
// keeps the reference's order: scores with -inf mask, running max over all
// j, exp(s - max) summed in j order, divide, then O[d] = sum_j p_j V[j][d].
void fwd_unit_f32(const float* Q, const float* K, const float* V, float* O, float* L, int N, int D,
                  float scale, bool causal) {
    std::vector<float> scores(N);
    for (int i = 0; i < N; ++i) {
        float max_score = -INFINITY;
        for (int j = 0; j < N; ++j) {
            if (causal && j > i) {
                scores[j] = -INFINITY;
            } else {
                float dot = 0.0f;
                for (int d = 0; d < D; ++d) dot += Q[(size_t)i * D + d] * K[(size_t)j * D + d];
                scores[j] = dot * scale;
            }
            max_score = std::max(max_score, scores[j]);
        }
        // logsumexp as test_forward.cu:103-114: separate sum over visible j
        if (L) {
            float sum_l = 0.0f;
            for (int j = 0; j < N; ++j) {
                if (causal && j > i) continue;
                sum_l += std::exp(scores[j] - max_score);
            }
            L[i] = max_score + std::log(sum_l);
        }
        if (O) {
            float sum_exp = 0.0f;
            for (int j = 0; j < N; ++j) {
                scores[j] = std::exp(scores[j] - max_score);
                sum_exp += scores[j];
            }
            for (int j = 0; j < N; ++j) scores[j] /= sum_exp;
            for (int d = 0; d < D; ++d) {
                float sum = 0.0f;
                for (int j = 0; j < N; ++j) sum += scores[j] * V[(size_t)j * D + d];
                O[(size_t)i * D + d] = sum;
            }
        }
    }
}

// test_backward.cu:21-127 for one unit: P, dV = P^T dO, dP = dO V^T,
// D_i = sum_j P_ij dP_ij, dS = P (dP - D) (0 where masked), dQ = dS K scale,
// dK = dS^T Q scale.
void bwd_unit_f32(const float* Q, const float* K, const float* V, const float* dO, float* dQ,
                  float* dK, float* dV, int N, int D, float scale, bool causal) {
    std::vector<float> P((size_t)N * N), dP((size_t)N * N), scores(N);
    for (int i = 0; i < N; ++i) {
        float max_score = -INFINITY;
        for (int j = 0; j < N; ++j) {
            if (causal && j > i) {
                scores[j] = -INFINITY;
            } else {
                float dot = 0.0f;
                for (int d = 0; d < D; ++d) dot += Q[(size_t)i * D + d] * K[(size_t)j * D + d];
                scores[j] = dot * scale;
            }
            max_score = std::max(max_score, scores[j]);
        }
        float sum_exp = 0.0f;
        for (int j = 0; j < N; ++j) {
            scores[j] = std::exp(scores[j] - max_score);
            sum_exp += scores[j];
        }
        for (int j = 0; j < N; ++j) P[(size_t)i * N + j] = scores[j] / sum_exp;
    }
    for (int j = 0; j < N; ++j)
        for (int d = 0; d < D; ++d) {
            float sum = 0.0f;
            for (int i = 0; i < N; ++i) sum += P[(size_t)i * N + j] * dO[(size_t)i * D + d];
            dV[(size_t)j * D + d] = sum;
        }
    for (int i = 0; i < N; ++i)
        for (int j = 0; j < N; ++j) {
            float sum = 0.0f;
            for (int d = 0; d < D; ++d) sum += dO[(size_t)i * D + d] * V[(size_t)j * D + d];
            dP[(size_t)i * N + j] = sum;
        }
    // dS overwrites dP in place
    for (int i = 0; i < N; ++i) {
        float Di = 0.0f;
        for (int j = 0; j < N; ++j) Di += P[(size_t)i * N + j] * dP[(size_t)i * N + j];
        for (int j = 0; j < N; ++j) {
            float& x = dP[(size_t)i * N + j];
            x = (causal && j > i) ? 0.0f : P[(size_t)i * N + j] * (x - Di);
        }
    }
    for (int i = 0; i < N; ++i)
        for (int d = 0; d < D; ++d) {
            float sum = 0.0f;
            for (int j = 0; j < N; ++j) sum += dP[(size_t)i * N + j] * K[(size_t)j * D + d];
            dQ[(size_t)i * D + d] = sum * scale;
        }
    for (int j = 0; j < N; ++j)
        for (int d = 0; d < D; ++d) {
            float sum = 0.0f;
            for (int i = 0; i < N; ++i) sum += dP[(size_t)i * N + j] * Q[(size_t)i * D + d];
            dK[(size_t)j * D + d] = sum * scale;
        }
}

// ---- fp64 ground truth -------------------------------------------------------

// Generalised to separate query/key lengths and global offsets (used for the
// partial / context-parallel entry points): key gk is masked for query gq iff
// causal && gk > gq.  A row with no visible key gets O = 0, L = -inf.
void fwd_unit_f64(const float* Q, const float* K, const float* V, double* O, double* L, int Nq,
                  int Nk, int D, double scale, bool causal, long long q_off, long long k_off) {
    std::vector<double> s(Nk);
    for (int i = 0; i < Nq; ++i) {
        double mx = -INFINITY;
        for (int j = 0; j < Nk; ++j) {
            if (causal && k_off + j > q_off + i) {
                s[j] = -INFINITY;
                continue;
            }
            double dot = 0.0;
            for (int d = 0; d < D; ++d) dot += (double)Q[(size_t)i * D + d] * K[(size_t)j * D + d];
            s[j] = dot * scale;
            mx = std::max(mx, s[j]);
        }
        if (mx == -INFINITY) {
            if (O) for (int d = 0; d < D; ++d) O[(size_t)i * D + d] = 0.0;
            if (L) L[i] = -INFINITY;
            continue;
        }
        double sum = 0.0;
        for (int j = 0; j < Nk; ++j) {
            s[j] = (s[j] == -INFINITY) ? 0.0 : std::exp(s[j] - mx);
            sum += s[j];
        }
        if (L) L[i] = mx + std::log(sum);
        if (O) {
            for (int d = 0; d < D; ++d) O[(size_t)i * D + d] = 0.0;
            for (int j = 0; j < Nk; ++j) {
                const double pj = s[j] / sum;
                if (pj == 0.0) continue;
                for (int d = 0; d < D; ++d) O[(size_t)i * D + d] += pj * V[(size_t)j * D + d];
            }
        }
    }
}

// fp64 backward of one unit, O(N^2) memory free: D_i from P and dP (as the
// reference oracle does), recomputing the softmax row by row.
// General fp64 backward: queries [Nq, D] at global positions q_off.., keys
// [Nk, D] at k_off..; with causal, key j is visible to query i iff
// k_off + j <= q_off + i.  Rows that see no key contribute nothing.
void bwd_unit_gen_f64(const float* Q, const float* K, const float* V, const float* dO, double* dQ,
                      double* dK, double* dV, int Nq, int Nk, int D, double scale, bool causal,
                      long long q_off, long long k_off) {
    std::vector<double> p(Nk), dp(Nk);
    std::fill(dQ, dQ + (size_t)Nq * D, 0.0);
    std::fill(dK, dK + (size_t)Nk * D, 0.0);
    std::fill(dV, dV + (size_t)Nk * D, 0.0);
    for (int i = 0; i < Nq; ++i) {
        long long lim = causal ? q_off + i - k_off + 1 : Nk;  // visible keys: j < lim
        const int jend = static_cast<int>(lim < 0 ? 0 : (lim > Nk ? Nk : lim));
        if (jend == 0) continue;
        double mx = -INFINITY;
        for (int j = 0; j < jend; ++j) {
            double dot = 0.0;
            for (int d = 0; d < D; ++d) dot += (double)Q[(size_t)i * D + d] * K[(size_t)j * D + d];
            p[j] = dot * scale;
            mx = std::max(mx, p[j]);
        }
        double sum = 0.0;
        for (int j = 0; j < jend; ++j) {
            p[j] = std::exp(p[j] - mx);
            sum += p[j];
        }
        double Di = 0.0;
        for (int j = 0; j < jend; ++j) {
            p[j] /= sum;
            double g = 0.0;
            for (int d = 0; d < D; ++d) g += (double)dO[(size_t)i * D + d] * V[(size_t)j * D + d];
            dp[j] = g;
            Di += p[j] * g;
        }
        for (int j = 0; j < jend; ++j) {
            const double ds = p[j] * (dp[j] - Di);
            for (int d = 0; d < D; ++d) {
                dQ[(size_t)i * D + d] += ds * K[(size_t)j * D + d] * scale;
                dK[(size_t)j * D + d] += ds * Q[(size_t)i * D + d] * scale;
                dV[(size_t)j * D + d] += p[j] * dO[(size_t)i * D + d];
            }
        }
    }
}

void bwd_unit_f64(const float* Q, const float* K, const float* V, const float* dO, double* dQ,
                  double* dK, double* dV, int N, int D, double scale, bool causal) {
    std::vector<double> p(N), dp(N);
    std::fill(dQ, dQ + (size_t)N * D, 0.0);
    std::fill(dK, dK + (size_t)N * D, 0.0);
    std::fill(dV, dV + (size_t)N * D, 0.0);
    for (int i = 0; i < N; ++i) {
        const int jend = causal ? i + 1 : N;
        double mx = -INFINITY;
        for (int j = 0; j < jend; ++j) {
            double dot = 0.0;
            for (int d = 0; d < D; ++d) dot += (double)Q[(size_t)i * D + d] * K[(size_t)j * D + d];
            p[j] = dot * scale;
            mx = std::max(mx, p[j]);
        }
        double sum = 0.0;
        for (int j = 0; j < jend; ++j) {
            p[j] = std::exp(p[j] - mx);
            sum += p[j];
        }
        double Di = 0.0;
        for (int j = 0; j < jend; ++j) {
            p[j] /= sum;
            double g = 0.0;
            for (int d = 0; d < D; ++d) g += (double)dO[(size_t)i * D + d] * V[(size_t)j * D + d];
            dp[j] = g;
            Di += p[j] * g;
        }
        for (int j = 0; j < jend; ++j) {
            const double ds = p[j] * (dp[j] - Di);
            for (int d = 0; d < D; ++d) {
                dQ[(size_t)i * D + d] += ds * K[(size_t)j * D + d] * scale;
                dK[(size_t)j * D + d] += ds * Q[(size_t)i * D + d] * scale;
                dV[(size_t)j * D + d] += p[j] * dO[(size_t)i * D + d];
            }
        }
    }
}

// One training step (forward + backward) of the reference CPU path restricted
// to a sample of query rows of one unit, for timing: for each sampled row i
// the forward row of test_forward.cu:21-69 (scores with -inf mask, max,
// exp, sum, normalise, P V) and the backward row of test_backward.cu:21-127
// (P row, dV_j += P_ij dO_i, dP_ij = dO_i.V_j, D_i = sum_j P_ij dP_ij,
// dS_ij, dQ_i = scale sum_j dS_ij K_j, dK_j += scale dS_ij Q_i).  Summed over
// all rows this is exactly the reference's arithmetic; a sample costs the
// same per row.  Returns the number of visible (i, j) pairs processed.
long long step_rows_f32(const float* Q, const float* K, const float* V, const float* dO, float* O,
                        float* L, float* dQ, float* dK, float* dV, int N, int D, float scale,
                        bool causal, int row_begin, int row_step) {
    std::vector<float> s(N), dp(N);
    long long pairs = 0;
    for (int i = row_begin; i < N; i += row_step) {
        float mx = -INFINITY;
        for (int j = 0; j < N; ++j) {
            if (causal && j > i) {
                s[j] = -INFINITY;
            } else {
                float dot = 0.0f;
                for (int d = 0; d < D; ++d) dot += Q[(size_t)i * D + d] * K[(size_t)j * D + d];
                s[j] = dot * scale;
                ++pairs;
            }
            mx = std::max(mx, s[j]);
        }
        float sum = 0.0f;
        for (int j = 0; j < N; ++j) {
            s[j] = std::exp(s[j] - mx);
            sum += s[j];
        }
        for (int j = 0; j < N; ++j) s[j] /= sum;
        L[i] = mx + std::log(sum);
        for (int d = 0; d < D; ++d) {
            float acc = 0.0f;
            for (int j = 0; j < N; ++j) acc += s[j] * V[(size_t)j * D + d];
            O[(size_t)i * D + d] = acc;
        }
        float Di = 0.0f;
        for (int j = 0; j < N; ++j) {
            float g = 0.0f;
            for (int d = 0; d < D; ++d) g += dO[(size_t)i * D + d] * V[(size_t)j * D + d];
            dp[j] = g;
            Di += s[j] * g;
            for (int d = 0; d < D; ++d) dV[(size_t)j * D + d] += s[j] * dO[(size_t)i * D + d];
        }
        for (int j = 0; j < N; ++j) dp[j] = (causal && j > i) ? 0.0f : s[j] * (dp[j] - Di);
        for (int d = 0; d < D; ++d) {
            float acc = 0.0f;
            for (int j = 0; j < N; ++j) acc += dp[j] * K[(size_t)j * D + d];
            dQ[(size_t)i * D + d] = acc * scale;
        }
        for (int j = 0; j < N; ++j)
            for (int d = 0; d < D; ++d) dK[(size_t)j * D + d] += dp[j] * Q[(size_t)i * D + d] * scale;
    }
    return pairs;
}

}  // namespace

extern "C" {

// ---- generators ----------------------------------------------------------------

// The reference tests' pattern: one mt19937(seed), uniform_real_distribution
// <float>(lo, hi), tensors filled interleaved per index (a[i], b[i], c[i],
// d[i]); pass d = nullptr for three tensors.
void oracle_fill_interleaved_uniform(float* a, float* b, float* c, float* d, long long n,
                                     unsigned seed, float lo, float hi) {
    std::mt19937 gen(seed);
    std::uniform_real_distribution<float> dist(lo, hi);
    for (long long i = 0; i < n; ++i) {
        a[i] = dist(gen);
        b[i] = dist(gen);
        c[i] = dist(gen);
        if (d) d[i] = dist(gen);
    }
}

// One mt19937(seed) per tensor, filled in linear order.
void oracle_fill_uniform(float* dst, long long n, unsigned seed, float lo, float hi) {
    std::mt19937 gen(seed);
    std::uniform_real_distribution<float> dist(lo, hi);
    for (long long i = 0; i < n; ++i) dst[i] = dist(gen);
}

void oracle_fill_normal(float* dst, long long n, unsigned seed, float mean, float stddev) {
    std::mt19937 gen(seed);
    std::normal_distribution<float> dist(mean, stddev);
    for (long long i = 0; i < n; ++i) dst[i] = dist(gen);
}

// ---- fp32 reference path ---------------------------------------------------------

// Units [u0, u1) of a [units, N, D] problem; O and/or L may be null.
void oracle_forward_f32(const float* Q, const float* K, const float* V, float* O, float* L,
                        long long u0, long long u1, int N, int D, float scale, int causal,
                        int nthreads) {
    const size_t T = (size_t)N * D;
    parallel_units(u0, u1, nthreads, [&](long long u) {
        fwd_unit_f32(Q + u * T, K + u * T, V + u * T, O ? O + u * T : nullptr,
                     L ? L + u * (size_t)N : nullptr, N, D, scale, causal != 0);
    });
}

void oracle_backward_f32(const float* Q, const float* K, const float* V, const float* dO,
                         float* dQ, float* dK, float* dV, long long u0, long long u1, int N, int D,
                         float scale, int causal, int nthreads) {
    const size_t T = (size_t)N * D;
    parallel_units(u0, u1, nthreads, [&](long long u) {
        bwd_unit_f32(Q + u * T, K + u * T, V + u * T, dO + u * T, dQ + u * T, dK + u * T,
                     dV + u * T, N, D, scale, causal != 0);
    });
}

// ---- fp64 ground truth -------------------------------------------------------------

// General forward: Q [units, Nq, D], K/V [units, Nk, D], global offsets for
// the causal mask.  O [units, Nq, D], L [units, Nq] (either may be null).
void oracle_forward_f64(const float* Q, const float* K, const float* V, double* O, double* L,
                        long long u0, long long u1, int Nq, int Nk, int D, double scale,
                        int causal, long long q_off, long long k_off, int nthreads) {
    const size_t Tq = (size_t)Nq * D, Tk = (size_t)Nk * D;
    parallel_units(u0, u1, nthreads, [&](long long u) {
        fwd_unit_f64(Q + u * Tq, K + u * Tk, V + u * Tk, O ? O + u * Tq : nullptr,
                     L ? L + u * (size_t)Nq : nullptr, Nq, Nk, D, scale, causal != 0, q_off,
                     k_off);
    });
}

void oracle_backward_f64(const float* Q, const float* K, const float* V, const float* dO,
                         double* dQ, double* dK, double* dV, long long u0, long long u1, int N,
                         int D, double scale, int causal, int nthreads) {
    const size_t T = (size_t)N * D;
    parallel_units(u0, u1, nthreads, [&](long long u) {
        bwd_unit_f64(Q + u * T, K + u * T, V + u * T, dO + u * T, dQ + u * T, dK + u * T,
                     dV + u * T, N, D, scale, causal != 0);
    });
}

void oracle_backward_gen_f64(const float* Q, const float* K, const float* V, const float* dO,
                             double* dQ, double* dK, double* dV, long long u0, long long u1,
                             int Nq, int Nk, int D, double scale, int causal, long long q_off,
                             long long k_off, int nthreads) {
    const size_t Tq = (size_t)Nq * D, Tk = (size_t)Nk * D;
    parallel_units(u0, u1, nthreads, [&](long long u) {
        bwd_unit_gen_f64(Q + u * Tq, K + u * Tk, V + u * Tk, dO + u * Tq, dQ + u * Tq, dK + u * Tk,
                         dV + u * Tk, Nq, Nk, D, scale, causal != 0, q_off, k_off);
    });
}

// Timed CPU baseline: a forward+backward step of the reference CPU path on
// units [u0, u1) (one unit per thread), rows row_begin, row_begin+row_step, ...
// of each unit.  dK/dV must be zeroed by the caller.  Returns visible pairs.
long long oracle_train_step_rows_f32(const float* Q, const float* K, const float* V,
                                     const float* dO, float* O, float* L, float* dQ, float* dK,
                                     float* dV, long long u0, long long u1, int N, int D,
                                     float scale, int causal, int row_begin, int row_step,
                                     int nthreads) {
    const size_t T = (size_t)N * D;
    std::vector<long long> pairs(u1 - u0, 0);
    parallel_units(u0, u1, nthreads, [&](long long u) {
        pairs[u - u0] = step_rows_f32(Q + u * T, K + u * T, V + u * T, dO + u * T, O + u * T,
                                      L + u * (size_t)N, dQ + u * T, dK + u * T, dV + u * T, N, D,
                                      scale, causal != 0, row_begin, row_step);
    });
    long long tot = 0;
    for (long long x : pairs) tot += x;
    return tot;
}

// fp64 forward of selected query rows only (for problems too large for the
// full O(N^2) oracle): Q, K, V [U, N, D]; rows[r] is both the row index and
// the query's global position (keys at 0..N-1), so each sampled row is
// fwd_unit_f64 with one query; O [U, nrows, D], L [U, nrows] for the units
// u0 <= u < u1 (indexed from u0).  Work items are (unit, row) pairs.
void oracle_forward_rows_f64(const float* Q, const float* K, const float* V, double* O, double* L,
                             long long u0, long long u1, const long long* rows, int nrows, int N,
                             int D, double scale, int causal, int nthreads) {
    const size_t T = (size_t)N * D;
    parallel_units(0, (u1 - u0) * nrows, nthreads, [&](long long w) {
        const long long u = u0 + w / nrows;
        const int r = static_cast<int>(w % nrows);
        fwd_unit_f64(Q + u * T + (size_t)rows[r] * D, K + u * T, V + u * T, O + (size_t)w * D,
                     L + w, 1, N, D, scale, causal != 0, rows[r], 0);
    });
}

int oracle_abi_version(void) { return 1; }

}  // extern "C"
