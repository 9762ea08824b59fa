// SPDX-License-Identifier: Apache-2.0
//
// Scheme II INT8 planner (host). Makes the decisions of the reference's planner so that Info and the
// moduli set are the same for the same input:
//   precision policy   choose_precision_policy / oz2_measure_stats / estimate_product_norm
//                      (src/backend/ozaki2/auto_precision.hpp:24-108, common/norm_estimate.hpp:20-73)
//   moduli and width   ozaki2_choose_moduli for the INT8 route (src/backend/ozaki2/moduli.hpp:180-769):
//                      table with the INT8 cap K*floor(m/2)^2 <= 2^31-1, coprime extension below 151,
//                      b from the window, tail trimming and reselection, accumulation check
//   passes, digits     oz2_choose_passes, oz2_recon1_log2, ND = 3/4/5 (plan.hpp:245-306)
//   CRT constants      y_i, fl32(1/m_i), 2^(20j) mod m_i (moduli.hpp:615-703)
// The statistics run on all host threads. Every sum keeps the reference's order: per-row and
// per-column quantities are computed in parallel, their totals sequentially, so the results are bit
// for bit those of the single-threaded reference (x86 80-bit long double where the reference uses it;
// this file is compiled without floating-point contraction).
#include <sched.h>

#include <algorithm>
#include <bit>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <numeric>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "oztt_cuda.h"
#include "planner.hpp"

static_assert(LDBL_MANT_DIG == 64, "the planner needs the x86 80-bit long double (as the reference host code)");

namespace oztt {
namespace {

constexpr int kMaxS = 24;
constexpr int kDigitBits = 20;
constexpr int kMaxDigit = 5;
constexpr int kTargetBits = 53;
constexpr int kDefaultB = 54;
constexpr int kAccBits = 31;
constexpr double kWinEps = 1e-9;
constexpr double kTailTol = 0.25;
constexpr double kRecon1EpsLog2 = -70.0;
constexpr double kRecon1Thr = -(kTargetBits + 2.0);
constexpr uint32_t kDefSInt8 = 16;
constexpr int kTable[] = {255, 254, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217,
                          211, 199, 197, 193, 191, 181, 179, 173, 167, 163, 157, 151};
constexpr int kTableMin = 151;

bool fits_int32(uint32_t K, int m) {
    const unsigned __int128 r = (unsigned)(m / 2);
    return (unsigned __int128)K * r * r <= (((unsigned __int128)1 << kAccBits) - 1);
}
long residue_cap(uint32_t K) {  // largest r with K*r^2 <= 2^31-1
    const unsigned __int128 lim = ((unsigned __int128)1 << kAccBits) - 1;
    long r = (long)std::floor(std::sqrt((double)lim / (double)K));
    while (r > 0 && (unsigned __int128)K * r * r > lim) --r;
    while ((unsigned __int128)K * (r + 1) * (r + 1) <= lim) ++r;
    return r;
}
long inverse_mod(long a, long mod) {
    long t = 0, nt = 1, r = mod, nr = a % mod;
    while (nr) {
        const long q = r / nr;
        long x = t - q * nt;
        t = nt;
        nt = x;
        x = r - q * nr;
        r = nr;
        nr = x;
    }
    return t < 0 ? t + mod : t;
}
bool coprime_to_all(int v, const std::vector<int>& set) {
    for (int x : set)
        if (std::gcd(x, v) != 1) return false;
    return true;
}

}  // namespace

ModuliChoice choose_moduli_int8(uint32_t K, int num_moduli, int b_cap) {
    ModuliChoice o;
    const double log2K = std::log2((double)K);
    const int m_cap = (int)std::min<long>(255, 2 * residue_cap(K) + 1);
    double logM = 0.0;
    for (int v : kTable) {
        if ((int)o.m.size() >= num_moduli) break;
        if (v > m_cap) continue;
        o.m.push_back(v);
        logM += std::log2((double)v);
    }
    const int want = std::min(num_moduli, kMaxS);
    for (int v = std::min(m_cap, kTableMin - 1); v >= 3 && (int)o.m.size() < want; --v)
        if (coprime_to_all(v, o.m)) {
            o.m.push_back(v);
            logM += std::log2((double)v);
        }
    o.m_cap = m_cap;
    o.ncand = (int)o.m.size();
    const int b_win = (int)std::floor((logM - 1.0 - log2K - kWinEps) / 2.0);
    o.b = std::min(std::min(b_win, kMaxDigit * kDigitBits), b_cap);
    const double need = 2.0 * o.b + 1.0 + log2K + kWinEps;
    // Surplus moduli only widen the window; drop them from the end.
    while (o.m.size() > 2) {
        const double last = std::log2((double)o.m.back());
        if (logM - last < need) break;
        o.m.pop_back();
        logM -= last;
    }
    // Replace the last two by one modulus or a coprime pair closer to the window: fewer moduli first,
    // then an excess within 1/4 bit, then the smaller excess.
    if (o.m.size() >= 2 && logM > need) {
        const std::vector<int> head(o.m.begin(), o.m.end() - 2);
        double base = 0.0;
        for (int x : head) base += std::log2((double)x);
        double best = logM;
        int best_p = o.m[o.m.size() - 2], best_q = o.m.back(), best_count = 2;
        const auto excess_flag = [&](double l) { return (l - need) > kTailTol ? 1 : 0; };
        const auto better = [&](int count, double l) {
            if (count != best_count) return count < best_count;
            if (excess_flag(l) != excess_flag(best)) return excess_flag(l) < excess_flag(best);
            return l < best;
        };
        bool even_head = false;
        for (int x : head) even_head = even_head || (x % 2 == 0);
        const int step = even_head ? 2 : 1;
        for (int p = 3; p <= m_cap; p += step) {
            if (!coprime_to_all(p, head)) continue;
            const double lp = base + std::log2((double)p);
            if (lp >= need && better(1, lp)) {
                best = lp;
                best_p = p;
                best_q = 0;
                best_count = 1;
            }
            for (int q = p + step; q <= m_cap; q += step) {
                if (std::gcd(p, q) != 1 || !coprime_to_all(q, head)) continue;
                const double lq = lp + std::log2((double)q);
                if (lq >= need && better(2, lq)) {
                    best = lq;
                    best_p = p;
                    best_q = q;
                    best_count = 2;
                }
            }
        }
        o.m = head;
        o.m.push_back(best_p);
        if (best_q) o.m.push_back(best_q);
        logM = best;
    }
    const int s = (int)o.m.size();
    o.ok = logM >= need && s > 0 && s <= kMaxS && s <= num_moduli && o.b > 0;
    for (int i = 0; i < s; ++i)
        for (int j = i + 1; j < s; ++j)
            if (std::gcd(o.m[i], o.m[j]) != 1) o.ok = false;
    for (int v : o.m)
        if (!fits_int32(K, v)) {
            o.ok = false;
            o.acc_ok = false;
            if (o.acc_fail_m == 0) o.acc_fail_m = v;
        }
    o.logM = logM;
    return o;
}

unsigned host_threads() {
    static const unsigned n = [] {
        cpu_set_t set;
        CPU_ZERO(&set);
        if (sched_getaffinity(0, sizeof set, &set) == 0) {
            const int c = CPU_COUNT(&set);
            if (c > 0) return (unsigned)c;
        }
        return std::max(1u, std::thread::hardware_concurrency());
    }();
    return n;
}

void value_maxima(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint64_t* row_max,
                  uint64_t* col_max) {
    // magnitude patterns as signed 64-bit integers (the sign bit cleared, so they order like the unsigned
    // patterns): maxima that the compiler vectorises (this file is built for x86-64-v3)
    constexpr int64_t kMag = 0x7FFFFFFFFFFFFFFFll;
    parallel_ranges(m, [&](uint64_t r0, uint64_t r1) {
        for (uint64_t i = r0; i < r1; ++i) {
            const double* p = a + i * k;
            int64_t mx = 0;
            for (uint64_t j = 0; j < k; ++j) mx = std::max(mx, std::bit_cast<int64_t>(p[j]) & kMag);
            row_max[i] = (uint64_t)mx;
        }
    });
    parallel_ranges(n, [&](uint64_t c0, uint64_t c1) {
        std::vector<int64_t> mx(c1 - c0, 0);
        for (uint64_t i = 0; i < k; ++i) {
            const double* p = b + i * n + c0;
            for (uint64_t j = 0; j < c1 - c0; ++j) mx[j] = std::max(mx[j], std::bit_cast<int64_t>(p[j]) & kMag);
        }
        for (uint64_t j = c0; j < c1; ++j) col_max[j] = (uint64_t)mx[j - c0];
    });
}

double pow2_normalizer(const double* v, uint64_t rows, uint64_t cols, uint64_t ld) {
    std::vector<double> row_max(rows, 0.0);
    parallel_ranges(rows, [&](uint64_t b, uint64_t e) {
        for (uint64_t i = b; i < e; ++i) {
            double mx = 0;
            const double* p = v + i * ld;
            for (uint64_t j = 0; j < cols; ++j) mx = std::max(mx, std::fabs(p[j]));
            row_max[i] = mx;
        }
    });
    double mx = 0;
    for (double x : row_max) mx = std::max(mx, x);
    if (!(mx > 0) || !std::isfinite(mx)) return 1.0;
    int e;
    std::frexp(mx, &e);
    e = std::min(std::max(e, -1000), 1000);
    return std::ldexp(1.0, e);
}

double product_norm_estimate(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                             double rgA, double rgB) {
    // Hutchinson estimate of ||C||_F^2 with 8 Gaussian vectors of the padded length N from
    // mt19937(12345); the largest sample is dropped and the mean divided by 1 + 2 sqrt(2/8).
    // Padding rows and columns contribute exact zeros, so only the real block is traversed.
    const uint32_t L = 8;
    std::mt19937 rng(12345);
    std::normal_distribution<double> normal(0.0, 1.0);
    std::vector<double> g(N), y(k, 0.0), s(m);
    double cs2 = 0, cmax = 0;
    for (uint32_t l = 0; l < L; ++l) {
        for (uint32_t j = 0; j < N; ++j) g[j] = normal(rng);
        parallel_ranges(k, [&](uint64_t r0, uint64_t r1) {
            for (uint64_t r = r0; r < r1; ++r) {
                long double acc = 0;
                const double* p = b + r * n;
                for (uint64_t j = 0; j < n; ++j) acc += (long double)(p[j] * rgB) * g[j];
                y[r] = (double)acc;
            }
        });
        parallel_ranges(m, [&](uint64_t r0, uint64_t r1) {
            for (uint64_t i = r0; i < r1; ++i) {
                long double acc = 0;
                const double* p = a + i * k;
                for (uint64_t c = 0; c < k; ++c) acc += (long double)(p[c] * rgA) * y[c];
                s[i] = (double)acc;
            }
        });
        double q = 0;
        for (uint64_t i = 0; i < m; ++i) q += s[i] * s[i];
        cs2 += q;
        cmax = std::max(cmax, q);
    }
    return (cs2 - cmax) / (L - 1) / (1.0 + 2.0 * std::sqrt(2.0 / (double)L));
}

PolicyStats measure_policy_stats(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                                 uint32_t K) {
    PolicyStats st;
    const double rgA = 1.0 / pow2_normalizer(a, m, k, k), rgB = 1.0 / pow2_normalizer(b, k, n, n);
    // Rows of A: tau^2 of the power-of-two scale and the sum of squares, summed in row order.
    {
        std::vector<double> tau2(m), s2(m);
        parallel_ranges(m, [&](uint64_t r0, uint64_t r1) {
            for (uint64_t r = r0; r < r1; ++r) {
                double mx = 0, sq = 0;
                for (uint64_t c = 0; c < k; ++c) {
                    const double v = a[r * k + c] * rgA;
                    mx = std::max(mx, std::fabs(v));
                    sq += v * v;
                }
                double t2 = 0;
                if (mx > 0) {
                    const double t = std::exp2(std::ceil(std::log2(mx)));
                    t2 = t * t;
                }
                tau2[r] = t2;
                s2[r] = sq;
            }
        });
        for (uint64_t r = 0; r < m; ++r) {
            if (tau2[r] > 0) st.TA += tau2[r];
            st.nA += s2[r];
        }
    }
    // Columns of B: the same per column, accumulated down the rows.
    {
        std::vector<double> mx(n, 0.0), s2(n, 0.0);
        parallel_ranges(n, [&](uint64_t c0, uint64_t c1) {
            for (uint64_t r = 0; r < k; ++r) {
                const double* p = b + r * n;
                for (uint64_t c = c0; c < c1; ++c) {
                    const double v = p[c] * rgB;
                    mx[c] = std::max(mx[c], std::fabs(v));
                    s2[c] += v * v;
                }
            }
        });
        for (uint64_t c = 0; c < n; ++c) {
            if (mx[c] > 0) {
                const double t = std::exp2(std::ceil(std::log2(mx[c])));
                st.TB += t * t;
            }
            st.nB += s2[c];
        }
    }
    st.nC = product_norm_estimate(a, b, m, n, k, N, rgA, rgB);
    st.measured = true;
    return st;
}

int policy_width_cap(const PolicyStats& st) {
    const double k2 =
        std::min(std::sqrt((st.TA * st.nB + st.TB * st.nA) / std::max(12.0 * st.nC, 1e-300)), 1e18);
    return std::min(kMaxDigit * kDigitBits, kTargetBits + (int)std::ceil(std::log2(std::max(k2, 1.0))));
}

bool plan_ii_int8_never_fails(uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli) {
    if (m == 0 || n == 0 || k == 0 || max_moduli > (uint32_t)kMaxS) return false;
    // the outcome depends on the padded K and the limit only (choose_moduli_int8)
    static std::mutex mu;
    static std::map<std::pair<uint64_t, uint32_t>, bool> known;
    const std::pair<uint64_t, uint32_t> key{(k + 31) / 32 * 32, max_moduli};
    {
        std::lock_guard<std::mutex> lock(mu);
        const auto it = known.find(key);
        if (it != known.end()) return it->second;
    }
    bool ok = true;
    for (int b = kTargetBits; ok && b <= kMaxDigit * kDigitBits; ++b) {
        // statistics whose k2 is exactly 2^(b - 53): the width cap b
        PolicyStats st;
        st.measured = true;
        st.TA = 12.0 * std::ldexp(1.0, 2 * (b - kTargetBits));
        st.nB = 1.0;
        st.nC = 1.0;
        oztt_ii_plan p;
        std::string err;
        ok = plan_ii_int8_with([&](uint32_t, uint32_t) { return st; }, m, n, k, max_moduli, OZTT_RECON_AUTO, 0, p,
                               err) == OZTT_OK;
    }
    std::lock_guard<std::mutex> lock(mu);
    known[key] = ok;
    return ok;
}

double one_pass_error_log2(const std::vector<int>& mods, int b, const PolicyStats& st) {
    if (!st.measured || !(st.nC > 0) || !(st.TA > 0) || !(st.TB > 0)) return -INFINITY;
    double l2m = 0;
    for (int v : mods) l2m += std::log2((double)v);
    return kRecon1EpsLog2 + l2m - 2.0 * b + 0.5 * (std::log2(st.TA) + std::log2(st.TB) - std::log2(st.nC));
}

// Why the moduli fall short, and what the caller can change (the causes distinguished by
// oz2_short_cause, src/backend/ozaki2/plan.hpp:120-150).
static std::string shortfall_cause(const ModuliChoice& mo, uint32_t S_req, uint32_t K, int b_cap, int target) {
    std::string s;
    if (mo.m_cap < 255)
        s = "For this K the INT8 moduli are limited to " + std::to_string(mo.m_cap) +
            " or less, because the GEMM output bound K*floor(m/2)^2 must not exceed 2^31-1. ";
    const uint32_t want = std::min<uint32_t>(S_req, kMaxS);
    if ((uint32_t)mo.ncand < want)
        return s + "Every candidate modulus is in use (" + std::to_string(mo.ncand) +
               "), so a larger Options::max_moduli does not help; use a smaller K or a different format.";
    if (want >= (uint32_t)kMaxS)
        return s + "The maximum of 24 moduli is not enough; use a smaller K or a different format.";
    ModuliChoice t;
    for (uint32_t n = S_req + 1; n <= (uint32_t)kMaxS; ++n) {
        t = choose_moduli_int8(K, (int)n, b_cap);
        if (t.ok && t.b >= target)
            return s + "The limit of " + std::to_string(S_req) + " moduli is too small; set Options::max_moduli to " +
                   std::to_string(n) + " or more.";
    }
    return s + "The limit of " + std::to_string(S_req) + " moduli is too small, and the maximum of 24 moduli still gives only " +
           std::to_string(t.ok ? t.b : 0) + " bits; use a smaller K or a different format.";
}

void fill_crt_constants(const std::vector<int>& mods, oztt_ii_plan& p) {
    const int S = (int)mods.size();
    p.S = S;
    for (int i = 0; i < S; ++i) {
        const long mi = mods[i];
        long prod = 1;
        for (int j = 0; j < S; ++j)
            if (j != i) prod = (prod * (mods[j] % mi)) % mi;
        p.moduli[i] = mods[i];
        p.yi[i] = (int32_t)inverse_mod(prod, mi);
        // fl32(fl64(1/m)): for the moduli here this is the correctly rounded binary32 reciprocal.
        p.rinv[i] = (float)(1.0 / (double)mods[i]);
        for (int j = 0; j < 4; ++j) {
            long r = 1 % mi;
            for (int e = 0; e < kDigitBits * (j + 1); ++e) r = (r * 2) % mi;
            p.c[j][i] = (float)r;
        }
    }
}

int plan_ii_int8(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli,
                 int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan& p, std::string& err) {
    return plan_ii_int8_with(
        [&](uint32_t N, uint32_t K) { return measure_policy_stats(a, b, m, n, k, N, K); }, m, n, k, max_moduli,
        reconstruction, fixed_bits, p, err);
}

int plan_ii_int8_with(const std::function<PolicyStats(uint32_t, uint32_t)>& stats, uint64_t m, uint64_t n, uint64_t k,
                      uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan& p,
                      std::string& err) {
    std::memset(&p, 0, sizeof(p));
    if (m == 0 || n == 0 || k == 0) {
        err = "matrix dimensions are zero";
        return OZTT_EINVAL;
    }
    if (max_moduli > (uint32_t)kMaxS) {
        err = "max_moduli exceeds the supported bound of 24";
        return OZTT_EINVAL;
    }
    if (reconstruction < 0 || reconstruction > 2) {
        err = "unknown reconstruction mode";
        return OZTT_EINVAL;
    }
    const auto pad = [](uint64_t v, uint64_t q) { return (v + q - 1) / q * q; };
    p.M = (uint32_t)pad(m, 64);
    p.N = (uint32_t)pad(n, 64);
    p.K = (uint32_t)pad(k, 32);
    const bool b_fixed = fixed_bits > 0;
    PolicyStats st;
    int b_cap = kDefaultB;
    if (b_fixed) {
        b_cap = fixed_bits;
    } else {
        st = stats(p.N, p.K);
        b_cap = policy_width_cap(st);
    }
    const uint32_t S_req = max_moduli ? max_moduli : (b_fixed ? kDefSInt8 : (uint32_t)kMaxS);
    if (b_fixed && reconstruction == OZTT_RECON_AUTO) st = stats(p.N, p.K);
    const ModuliChoice mo = choose_moduli_int8(p.K, (int)S_req, b_cap);
    p.b_cap = b_cap;
    p.S_req = (int32_t)S_req;
    p.TA = st.TA;
    p.TB = st.TB;
    p.nA = st.nA;
    p.nB = st.nB;
    p.nC = st.nC;
    if (!mo.ok) {
        if (!mo.acc_ok)
            err = "Ozaki II: the padded inner dimension K=" + std::to_string(p.K) +
                  " is too large for this format: the GEMM output bound K*floor(m/2)^2 of modulus " +
                  std::to_string(mo.acc_fail_m) +
                  " exceeds the sign-magnitude int32 range 2^31-1. Use a smaller K or a different format; "
                  "Options::max_moduli does not change this limit.";
        else
            err = "Ozaki II: the available moduli do not cover the CRT window for the padded inner dimension K=" +
                  std::to_string(p.K) + ". " + shortfall_cause(mo, S_req, p.K, b_cap, b_fixed ? 1 : kTargetBits);
        return OZTT_ERUNTIME;
    }
    if (!b_fixed && mo.b < kTargetBits) {
        err = "Ozaki II: for the padded inner dimension K=" + std::to_string(p.K) + " the " +
              std::to_string(mo.m.size()) + " selected moduli cover a width of only " + std::to_string(mo.b) +
              " bits, below the 53 bits of FP64-equivalent accuracy. " +
              shortfall_cause(mo, S_req, p.K, b_cap, kTargetBits);
        return OZTT_ERUNTIME;
    }
    p.b = mo.b;
    p.recon1_log2 = one_pass_error_log2(mo.m, mo.b, st);
    p.two_pass = reconstruction != OZTT_RECON_AUTO ? (reconstruction == OZTT_RECON_TWO)
                                                   : !(p.recon1_log2 <= kRecon1Thr);
    p.nd = mo.b > 4 * kDigitBits ? 5 : (mo.b > 3 * kDigitBits ? 4 : 3);
    p.shift = mo.b - (p.nd - 1) * kDigitBits;
    fill_crt_constants(mo.m, p);
    return OZTT_OK;
}

// The width cap grows with nA and falls with nC, the one-pass error estimate falls with nC; both are
// evaluated at the corners of the bounds, each a relative 1e-12 beyond them, so that the few roundings of
// the decision formulas cannot tip a case the bounds call decided.
int plan_ii_int8_certified(const PolicyBounds& bounds, uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli,
                           int32_t reconstruction, oztt_ii_plan& p, std::string& err, bool& decided) {
    decided = false;
    if (!bounds.usable) return OZTT_OK;
    PolicyStats low = bounds.lo, high = bounds.hi;  // k2 at its least and at its greatest
    low.nC = bounds.hi.nC * (1 + 1e-12);
    low.nA = bounds.lo.nA * (1 - 1e-12);
    low.nB = bounds.lo.nB * (1 - 1e-12);
    high.nC = bounds.lo.nC * (1 - 1e-12);
    high.nA = bounds.hi.nA * (1 + 1e-12);
    high.nB = bounds.hi.nB * (1 + 1e-12);
    for (const PolicyStats* q : {&low, &high})
        if (!(q->nC > 0) || !(q->nA >= 0) || !(q->nB >= 0) || !std::isfinite(q->nC) || !std::isfinite(q->nA) ||
            !std::isfinite(q->nB))
            return OZTT_OK;
    const int b_cap = policy_width_cap(low);
    if (policy_width_cap(high) != b_cap) return OZTT_OK;
    // plan at the middle of the bounds: its width cap is the decided one
    PolicyStats mid = bounds.lo;
    mid.nA = 0.5 * (bounds.lo.nA + bounds.hi.nA);
    mid.nB = 0.5 * (bounds.lo.nB + bounds.hi.nB);
    mid.nC = 0.5 * (bounds.lo.nC + bounds.hi.nC);
    mid.measured = true;
    const int rc = plan_ii_int8_with([&](uint32_t, uint32_t) { return mid; }, m, n, k, max_moduli, reconstruction, 0,
                                     p, err);
    if (rc != OZTT_OK || p.b_cap != b_cap) return rc;
    if (reconstruction == OZTT_RECON_AUTO) {
        std::vector<int> mods(p.moduli, p.moduli + p.S);
        const double r_lo = one_pass_error_log2(mods, p.b, high), r_hi = one_pass_error_log2(mods, p.b, low);
        // the estimate falls as nC grows: r_lo at the largest nC, r_hi at the smallest
        const bool two_lo = !(r_lo + 1e-9 <= kRecon1Thr), two_hi = !(r_hi - 1e-9 <= kRecon1Thr);
        if (two_lo != two_hi || two_lo != (p.two_pass != 0)) return OZTT_OK;
    }
    decided = true;
    return OZTT_OK;
}

}  // namespace oztt

extern "C" int oztt_ii_int8_plan(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                                 uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan* plan,
                                 char* err, size_t errlen) {
    std::string msg;
    int rc;
    try {
        if (!plan || !a || !b) {
            msg = "null argument";
            rc = OZTT_EINVAL;
        } else {
            rc = oztt::plan_ii_int8(a, b, m, n, k, max_moduli, reconstruction, fixed_bits, *plan, msg);
        }
    } catch (const std::bad_alloc&) {
        msg = "host memory exhausted";
        rc = OZTT_ENOMEM;
    } catch (const std::exception& e) {
        msg = e.what();
        rc = OZTT_ERUNTIME;
    }
    if (err && errlen) {
        std::strncpy(err, msg.c_str(), errlen - 1);
        err[errlen - 1] = 0;
    }
    return rc;
}
