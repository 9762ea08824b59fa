// SPDX-License-Identifier: Apache-2.0
//
// Scheme I planner (host), INT8 and FP8 formats. Decides what the reference decides before its device
// pipeline runs:
//   slices p       as requested, or selected from the input (oz_fp64_p and its helpers,
//                  src/backend/ozaki1/auto_precision.hpp:65-526): the smallest p in a doubling +
//                  bisection search for which two models of the truncation error stay below 2^-53
//                  relative: (1) a sum of squares with independent signs over all elements, against
//                  the Hutchinson estimate of ||C||_F^2, and (2) a simulation of the device result on
//                  32 + 32 sampled rows and columns (largest norms plus a seeded uniform draw)
//   feasibility    plan_issue / issue_feasible (src/backend/ozaki1/plan.hpp:141-226, format.hpp:98-190):
//                  a K block length that keeps the accumulation exact for the chosen issue (INT8: the
//                  concatenated issue with one K block only, K (L+1) 127^2 <= 2^31 - 1), and the FP32
//                  exponent budget of the Horner evaluation
// The format constants (ozaki1/param.hpp:47-50, format.hpp:32-97): INT8 radix 254, digits +-127,
// Int32 partial sums, row/column maxima rounded up to BF16; FP8 radix 32, digits +-16, FP32 partial
// sums (24 exact bits), maxima truncated to BF16; both normalize to 2^-1. Every floating-point sum keeps
// the reference's order (independent quantities run in parallel, sums over them run sequentially or in
// the reference's fixed chunks), so p is the reference's for the same input. Compiled without
// floating-point contraction.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <exception>
#include <functional>
#include <random>
#include <string>
#include <vector>

#include "oztt_cuda.h"
#include "planner.hpp"

namespace oztt {
namespace {

constexpr uint32_t kSampleTop = 32, kSampleUniform = 32;
constexpr uint32_t kSeedRows = 20261021u, kSeedCols = 20261022u;
constexpr uint32_t kTileWidth = 32;

// |mx| -> BF16 (rounded up for ceil_mode 1, truncated for 0), then e = ceil(log2) of it
// (scale_bits.h:33-63); in_range is false for 0 and for the values the device flags (above BF16, below
// 2^-126, Inf/NaN).
int device_exponent(double mx, uint32_t ceil_mode, bool& in_range) {
    uint64_t u;
    std::memcpy(&u, &mx, 8);
    const uint32_t h = (uint32_t)(u >> 32) & 0x7FFFFFFFu, l = (uint32_t)u;
    const int32_t E = (int32_t)((h >> 20) & 0x7FFu);
    uint32_t v;
    if (E == 0x7FF)
        v = 0xFFC0u;
    else if (E - 896 <= 0)
        v = (h | l) ? 0xFF80u : 0u;
    else if (E - 896 >= 255)
        v = 0x7F80u;
    else {
        v = ((uint32_t)(E - 896) << 7) | ((h >> 13) & 0x7Fu);
        if (ceil_mode == 1 && ((h & 0x1FFFu) || l)) v += 1u;
    }
    const uint32_t be = (v >> 7) & 0xFFu, bm = v & 0x7Fu;
    in_range = v != 0 && be != 0xFFu;
    if (be == 0u || be == 0xFFu) return 0;
    return (int)be - 127 + (bm ? 1 : 0);
}

// Error-free sum s + e = a + b.
inline void two_sum(double a, double b, double& s, double& e) {
    s = a + b;
    const double bb = s - a;
    e = (a - (s - bb)) + (b - bb);
}

// The balanced radix expansion of one element, advanced by the device slicer's rule: u = radix t,
// d = clamp(round-half-even(fl32(u_hi)), +-dmax), t = u - d, with t held as two doubles.
struct Expansion {
    double th = 0.0, tl = 0.0;
    double radix = 254.0, dmax = 127.0;
    double step() {
        const double ph = radix * th, pe = std::fma(radix, th, -ph);
        double uh, ul;
        two_sum(ph, pe + radix * tl, uh, ul);
        const double d = std::min(dmax, std::max(-dmax, std::nearbyint((double)(float)uh)));
        two_sum(uh - d, ul, th, tl);
        return d;
    }
    double value() const { return th + tl; }
};

struct Dims {
    uint64_t m, n, k;  // the real block
    uint32_t M, N, K;  // padded planning dimensions
    int pmax;
    I1Format f;
    Expansion expansion() const {
        Expansion t;
        t.radix = f.radix;
        t.dmax = f.dmax;
        return t;
    }
};

using Normalization = I1Normalization;

// The exponent and scaled divisor of a row (column) from its largest magnitude.
void row_scale(double mx, double rg, const Dims& d, int& e_out, double& s_out) {
    bool ok = false;
    const int e = device_exponent(mx, d.f.ceil_mode, ok);
    if (mx > 0 && ok) {
        e_out = e;
        s_out = std::ldexp(rg, e - d.f.nshift);
    }
}

Normalization normalize(const double* a, const double* b, const Dims& d) {
    Normalization nm;
    nm.rgA = 1.0 / pow2_normalizer(a, d.m, d.k, d.k);
    nm.rgB = 1.0 / pow2_normalizer(b, d.k, d.n, d.n);
    nm.eA.assign(d.m, 0);
    nm.sA.assign(d.m, 0.0);
    nm.nrA.assign(d.m, 0.0);
    nm.eB.assign(d.n, 0);
    nm.sB.assign(d.n, 0.0);
    nm.nrB.assign(d.n, 0.0);
    parallel_ranges(d.m, [&](uint64_t r0, uint64_t r1) {
        for (uint64_t i = r0; i < r1; ++i) {
            double mx = 0, nr = 0;
            for (uint64_t c = 0; c < d.k; ++c) {
                const double v = a[i * d.k + c];
                mx = std::max(mx, std::fabs(v));
                nr += (v * nm.rgA) * (v * nm.rgA);
            }
            row_scale(mx, nm.rgA, d, nm.eA[i], nm.sA[i]);
            nm.nrA[i] = nr;
        }
    });
    std::vector<double> mx(d.n, 0.0);
    parallel_ranges(d.n, [&](uint64_t c0, uint64_t c1) {
        for (uint64_t r = 0; r < d.k; ++r) {
            const double* p = b + r * d.n;
            for (uint64_t c = c0; c < c1; ++c) {
                mx[c] = std::max(mx[c], std::fabs(p[c]));
                nm.nrB[c] += (p[c] * nm.rgB) * (p[c] * nm.rgB);
            }
        }
        for (uint64_t c = c0; c < c1; ++c) {
            row_scale(mx[c], nm.rgB, d, nm.eB[c], nm.sB[c]);
        }
    });
    return nm;
}

// Model (1): err2[q] = expected ||E||_F^2 for q slices with independent signs (q = 2..pmax), scaled
// units of the normalization. First the per-k terms (independent_terms; the device computes the same
// arrays, plan1_dev.cu), then their combination (combine_terms).
I1Terms independent_terms(const double* a, const double* b, const Dims& d, const Normalization& nm) {
    const int pmax = d.pmax;
    const size_t P1 = (size_t)pmax + 1, K = d.k;
    // Per k: slice contributions S[i][k], residual contributions R[q][k], column norms N[k].
    I1Terms terms;
    terms.SA.assign(P1 * K, 0.0);
    terms.RA.assign(P1 * K, 0.0);
    terms.SB.assign(P1 * K, 0.0);
    terms.RB.assign(P1 * K, 0.0);
    terms.NA.assign(K, 0.0);
    terms.NB.assign(K, 0.0);
    std::vector<double>&SA = terms.SA, &RA = terms.RA, &SB = terms.SB, &RB = terms.RB, &NA = terms.NA, &NB = terms.NB;
    // Expands up to four elements of different k side by side (their chains are independent, so they
    // overlap in the pipeline); each element adds its slice and residual terms to its own column k, in
    // the order of its own steps, and stops once its residual is exactly zero.
    constexpr int LANES = 4;
    auto cut = [&](const double (&x)[LANES], const double (&s)[LANES], const size_t (&col)[LANES], double* S,
                   double* R) {
        Expansion t[LANES];
        bool active[LANES];
        int live = 0;
        for (int l = 0; l < LANES; ++l) {
            t[l] = d.expansion();
            t[l].th = x[l];
            active[l] = s[l] > 0;
            live += active[l];
        }
        double w = 1.0;
        for (int i = 0; i < pmax && live; ++i) {
            w /= d.f.radix;
            for (int l = 0; l < LANES; ++l) {
                if (!active[l]) continue;
                const double dg = t[l].step();
                S[(size_t)i * K + col[l]] += (s[l] * dg * w) * (s[l] * dg * w);
                const double r = s[l] * t[l].value() * w;
                R[(size_t)(i + 1) * K + col[l]] += r * r;
                if (t[l].th == 0) {
                    active[l] = false;
                    --live;
                }
            }
        }
    };
    // Collects the elements to expand of one row (A) or one k (B) in groups of LANES.
    struct Batch {
        double x[LANES] = {}, s[LANES] = {};
        size_t col[LANES] = {};
        int n = 0;
    };
    auto flush = [&](Batch& bt, double* S, double* R) {
        for (int l = bt.n; l < LANES; ++l) bt.s[l] = 0.0;
        cut(bt.x, bt.s, bt.col, S, R);
        bt.n = 0;
    };
    auto push = [&](Batch& bt, double x, double sc, size_t c, double* S, double* R) {
        bt.x[bt.n] = x;
        bt.s[bt.n] = sc;
        bt.col[bt.n] = c;
        if (++bt.n == LANES) flush(bt, S, R);
    };
    // Per k, the rows of A and the columns of B are visited in ascending order (the reference's order of
    // the sums); for A the loops are interchanged so that each thread walks its k range of a row
    // contiguously, which leaves the order of every per-k sum unchanged.
    // The lanes of a batch always belong to different k (distinct accumulators): for A the elements of
    // one row, for B the elements of one column at LANES consecutive k. Every per-k sum still receives
    // its terms row by row (A) or column by column (B), as in the reference's sequential loops.
    parallel_ranges(K, [&](uint64_t k0, uint64_t k1) {
        Batch bt;
        for (uint64_t i = 0; i < d.m; ++i) {
            const double* row = a + i * d.k;
            const bool counted = nm.sA[i] > 0;
            for (uint64_t c = k0; c < k1; ++c) {
                const double v = row[c];
                NA[c] += (v * nm.rgA) * (v * nm.rgA);
                if (v != 0 && counted)
                    push(bt, std::ldexp(v, d.f.nshift - nm.eA[i]), nm.sA[i], c, SA.data(), RA.data());
            }
            if (bt.n) flush(bt, SA.data(), RA.data());
        }
        for (uint64_t c0 = k0; c0 < k1; c0 += LANES) {
            const int nl = (int)std::min<uint64_t>(LANES, k1 - c0);
            double nb[LANES] = {};
            for (uint64_t j = 0; j < d.n; ++j) {
                const bool counted = nm.sB[j] > 0;
                for (int l = 0; l < nl; ++l) {
                    const double v = b[(c0 + l) * d.n + j];
                    nb[l] += (v * nm.rgB) * (v * nm.rgB);
                    if (v != 0 && counted)
                        push(bt, std::ldexp(v, d.f.nshift - nm.eB[j]), nm.sB[j], c0 + l, SB.data(), RB.data());
                }
                if (bt.n) flush(bt, SB.data(), RB.data());
            }
            for (int l = 0; l < nl; ++l) NB[c0 + l] = nb[l];
        }
    });
    return terms;
}

std::vector<double> combine_terms(const I1Terms& terms, const Dims& d) {
    const int pmax = d.pmax;
    const size_t P1 = (size_t)pmax + 1, K = d.k;
    const std::vector<double>&SA = terms.SA, &RA = terms.RA, &SB = terms.SB, &RB = terms.RB, &NA = terms.NA,
                             &NB = terms.NB;
    // G[i][j] = sum_k SA_i[k] SB_j[k]: the pairs the device drops.
    std::vector<double> G((size_t)pmax * pmax, 0.0);
    parallel_ranges((uint64_t)pmax * pmax, [&](uint64_t t0, uint64_t t1) {
        for (uint64_t t = t0; t < t1; ++t) {
            const size_t i = t / pmax, j = t % pmax;
            double g = 0;
            for (size_t c = 0; c < K; ++c) g += SA[i * K + c] * SB[j * K + c];
            G[t] = g;
        }
    });
    std::vector<double> err2(P1, 0.0);
    for (int q = 2; q <= pmax; ++q) {
        double e2 = 0;
        for (int i = 0; i < q; ++i)
            for (int j = std::max(0, q - i); j < q; ++j) e2 += G[(size_t)i * pmax + j];
        for (size_t c = 0; c < K; ++c) e2 += RA[(size_t)q * K + c] * NB[c] + NA[c] * RB[(size_t)q * K + c];
        err2[q] = e2;
    }
    return err2;
}

// Model (2)'s last step for one q: E = the per-pair sums of the dropped terms (chunk partial sums
// part[ch][s][u], combined in chunk order), and the simulated rounding of C - E against C.
double model2_finish(const double* part, uint32_t nch, const std::vector<uint32_t>& rows,
                     const std::vector<uint32_t>& cols, const std::vector<double>& wr, const std::vector<double>& wc,
                     const std::vector<double>& Ch, const std::vector<double>& Cl, const Normalization& nm,
                     double norm2) {
    const size_t na = rows.size(), nb = cols.size();
    double e2 = 0;
    for (size_t s = 0; s < na; ++s)
        for (size_t u = 0; u < nb; ++u) {
            double E = 0;
            for (uint32_t ch = 0; ch < nch; ++ch) E += part[((size_t)ch * na + s) * nb + u];
            // The device's 64-bit assembly window can move a value by about 2^-60 relative before
            // its rounding: within 2^-59 of a rounding midpoint the side farther from C is taken.
            const size_t su = s * nb + u;
            double h, r;
            two_sum(Ch[su], Cl[su] - nm.sA[rows[s]] * nm.sB[cols[u]] * E, h, r);
            double out = h;
            if (h != 0) {
                const double h2 = std::nextafter(h, r >= 0 ? INFINITY : -INFINITY);
                const double gap = 0.5 * std::fabs(h2 - h) - std::fabs(r);
                if (gap <= std::ldexp(1.0, std::ilogb(h) - 59)) {
                    const double d1 = (h - Ch[su]) - Cl[su], d2 = (h2 - Ch[su]) - Cl[su];
                    if (std::fabs(d2) > std::fabs(d1)) out = h2;
                }
            }
            const double dv = (out - Ch[su]) - Cl[su];
            e2 += wr[s] * wc[u] * dv * dv;
        }
    return norm2 > 0 ? e2 / norm2 : (e2 > 0 ? INFINITY : 0.0);
}

// Model (2): the sampled rows and columns with their products in double-double.
struct Sample {
    const Dims* d = nullptr;
    const Normalization* nm = nullptr;
    std::vector<uint32_t> rows, cols;
    std::vector<double> wr, wc;
    std::vector<double> X, Y;    // normalized values, [sample][real k]
    std::vector<double> Ch, Cl;  // C of the sampled pairs (scaled), two words
    double norm2 = 0;

    // ||fl(C - E) - C||_F^2 / ||C||_F^2 estimated from the sample for q slices. k runs in 64 fixed
    // chunks of the padded K, each summed alone and the chunks combined in order.
    double err2(int q) const {
        const size_t na = rows.size(), nb = cols.size();
        if (na == 0 || nb == 0) return 0.0;
        const uint64_t K = d->K, kreal = d->k;
        constexpr uint32_t NCH = kI1Chunks;
        std::vector<double> part((size_t)NCH * na * nb, 0.0);
        parallel_ranges(NCH, [&](uint64_t c0, uint64_t c1) {
            std::vector<double> D(na * q), RX(na), RY(nb * (q + 1)), Yk(nb);
            for (uint64_t ch = c0; ch < c1; ++ch) {
                const uint64_t k0 = K * ch / NCH, k1 = std::min<uint64_t>(K * (ch + 1) / NCH, kreal);
                double* acc = &part[(size_t)ch * na * nb];
                for (uint64_t c = k0; c < k1; ++c) {
                    for (size_t s = 0; s < na; ++s) {
                        Expansion t = d->expansion();
                        t.th = X[s * kreal + c];
                        double w = 1.0;
                        for (int i = 0; i < q; ++i) {
                            const double dg = t.step();
                            w /= d->f.radix;
                            D[s * q + i] = dg * w;
                        }
                        RX[s] = t.value() * w;
                    }
                    for (size_t s = 0; s < nb; ++s) {
                        Expansion t = d->expansion();
                        t.th = Yk[s] = Y[s * kreal + c];
                        double w = 1.0;
                        for (int r = 1; r <= q; ++r) {
                            (void)t.step();
                            w /= d->f.radix;
                            RY[s * (q + 1) + r] = t.value() * w;
                        }
                    }
                    for (size_t s = 0; s < na; ++s)
                        for (size_t u = 0; u < nb; ++u) {
                            double e = RX[s] * Yk[u];
                            for (int i = 0; i < q; ++i) e += D[s * q + i] * RY[u * (q + 1) + (q - i)];
                            acc[s * nb + u] += e;
                        }
                }
            }
        });
        return model2_finish(part.data(), NCH, rows, cols, wr, wc, Ch, Cl, *nm, norm2);
    }
};

// The sample: per operand the 32 rows (columns) of largest norm with weight 1 (ties to the lower
// index), then 32 drawn uniformly from the rest by a seeded mt19937 partial shuffle with weight
// (rest)/(drawn). Zero and out-of-range rows and columns are left out.
void pick(const std::vector<double>& nr, const std::vector<double>& s, uint32_t seed, std::vector<uint32_t>& idx,
          std::vector<double>& wt) {
    std::vector<uint32_t> ord;
    for (uint32_t i = 0; i < (uint32_t)s.size(); ++i)
        if (s[i] > 0) ord.push_back(i);
    const size_t nt = std::min<size_t>(kSampleTop, ord.size());
    // The order the shuffle sees is the one std::partial_sort leaves behind the first nt.
    std::partial_sort(ord.begin(), ord.begin() + nt, ord.end(),
                      [&](uint32_t x, uint32_t y) { return nr[x] > nr[y] || (nr[x] == nr[y] && x < y); });
    for (size_t i = 0; i < nt; ++i) {
        idx.push_back(ord[i]);
        wt.push_back(1.0);
    }
    std::vector<uint32_t> rest(ord.begin() + nt, ord.end());
    const size_t nu = std::min<size_t>(kSampleUniform, rest.size());
    std::mt19937 rng(seed);
    for (size_t i = 0; i < nu; ++i) {
        std::swap(rest[i], rest[i + rng() % (rest.size() - i)]);
        idx.push_back(rest[i]);
        wt.push_back((double)rest.size() / (double)nu);
    }
}

Sample sample(const double* a, const double* b, const Dims& d, const Normalization& nm, double nC) {
    Sample sm;
    sm.d = &d;
    sm.nm = &nm;
    pick(nm.nrA, nm.sA, kSeedRows, sm.rows, sm.wr);
    pick(nm.nrB, nm.sB, kSeedCols, sm.cols, sm.wc);
    const size_t na = sm.rows.size(), nb = sm.cols.size(), K = d.k;
    sm.X.assign(na * K, 0.0);
    sm.Y.assign(nb * K, 0.0);
    for (size_t s = 0; s < na; ++s)
        for (size_t c = 0; c < K; ++c)
            sm.X[s * K + c] = std::ldexp(a[(size_t)sm.rows[s] * d.k + c], d.f.nshift - nm.eA[sm.rows[s]]);
    for (size_t s = 0; s < nb; ++s)
        for (size_t c = 0; c < K; ++c)
            sm.Y[s * K + c] = std::ldexp(b[c * d.n + sm.cols[s]], d.f.nshift - nm.eB[sm.cols[s]]);
    // C of the sampled pairs by a compensated dot product (TwoProduct with an FMA, TwoSum).
    sm.Ch.assign(na * nb, 0.0);
    sm.Cl.assign(na * nb, 0.0);
    parallel_ranges(na * nb, [&](uint64_t t0, uint64_t t1) {
        for (uint64_t t = t0; t < t1; ++t) {
            const size_t s = t / nb, u = t % nb;
            double hi = 0, lo = 0;
            for (size_t c = 0; c < K; ++c) {
                const double x = a[(size_t)sm.rows[s] * d.k + c] * nm.rgA, y = b[c * d.n + sm.cols[u]] * nm.rgB;
                const double pr = x * y, pe = std::fma(x, y, -pr);
                double v, ve;
                two_sum(hi, pr, v, ve);
                hi = v;
                lo += pe + ve;
            }
            two_sum(hi, lo, sm.Ch[t], sm.Cl[t]);
        }
    });
    // Denominator: the larger of the weighted sample's ||C||_F^2 and the Hutchinson estimate.
    double ns = 0;
    for (size_t s = 0; s < na; ++s)
        for (size_t u = 0; u < nb; ++u) ns += sm.wr[s] * sm.wc[u] * sm.Ch[s * nb + u] * sm.Ch[s * nb + u];
    sm.norm2 = std::max(nC, ns);
    return sm;
}

// Starts at the smallest q that model (1) accepts; if model (2) rejects it, doubles the step upward
// until a q passes both, then bisects. pmax when the target is not reached.
int search(const std::vector<double>& r1, const std::function<double(int)>& model2, int pmax, double tgt) {
    std::vector<double> cache((size_t)pmax + 1, -1.0);
    auto f = [&](int q) {
        if (cache[q] < 0) cache[q] = model2(q);
        return std::max(r1[q], cache[q]);
    };
    int q0 = pmax;
    for (int q = 2; q <= pmax; ++q)
        if (r1[q] <= tgt) {
            q0 = q;
            break;
        }
    if (f(q0) <= tgt) return q0;
    int lo = q0, hi = -1;
    for (int step = 1; lo < pmax; step *= 2) {
        const int q = std::min(pmax, lo + step);
        if (f(q) <= tgt) {
            hi = q;
            break;
        }
        lo = q;
    }
    if (hi < 0) return pmax;
    while (hi - lo > 1) {
        const int mid = (lo + hi) / 2;
        if (f(mid) <= tgt)
            hi = mid;
        else
            lo = mid;
    }
    return hi;
}

// K block length (ozaki_block_k, ozaki1/format.hpp:134-156) for L+1 slice pairs per accumulation: K
// when no blocking is needed, else the largest multiple of 32 dividing K within the budget, 0 if none.
uint32_t block_k(uint32_t K, int L, const I1Format& f) {
    const uint64_t d2 = (uint64_t)f.dmax * (uint64_t)f.dmax;
    uint32_t pb = 0;
    while ((1ull << pb) < d2) ++pb;
    if (f.acc_bits < pb + 1) return 0;
    uint64_t keff_max = 1ull << (f.acc_bits - pb);
    if (f.int32_partial) keff_max = std::min<uint64_t>(keff_max, (uint64_t)INT32_MAX / d2);
    const uint64_t kc_max = keff_max / (uint64_t)(L + 1);
    if (kc_max >= (uint64_t)K) return K;
    uint32_t best = 0;
    for (uint32_t c = kTileWidth; c <= kc_max; c += kTileWidth)
        if (K % c == 0) best = c;
    return best;
}

// The slice count from model (1)'s terms, nC and model (2) (model2(q): its error for q slices).
int select_with(const I1Terms& terms, const Dims& d, double nC, const std::function<double(int)>& model2) {
    const std::vector<double> err2 = combine_terms(terms, d);
    const double tgt = std::ldexp(1.0, -106);
    std::vector<double> r1((size_t)d.pmax + 1, INFINITY);
    for (int q = 2; q <= d.pmax; ++q) r1[q] = nC > 0 ? err2[q] / nC : (err2[q] > 0 ? INFINITY : 0.0);
    return search(r1, model2, d.pmax, tgt);
}

// The slice count from the normalization, the per-k terms of model (1) and nC, however measured.
int select_from(const double* a, const double* b, const Dims& d, const Normalization& nm, const I1Terms& terms,
                double nC) {
    const Sample sm = sample(a, b, d, nm, nC);
    return select_with(terms, d, nC, [&](int q) { return sm.err2(q); });
}

Dims make_dims(uint64_t m, uint64_t n, uint64_t k, uint32_t M, uint32_t N, uint32_t K, const I1Format& f) {
    Dims d{m, n, k, M, N, K, 0, f};
    d.pmax = i1_pmax(f);
    return d;
}

}  // namespace

int i1_pmax(const I1Format& f) { return (int)std::ceil(160.0 / std::log2(f.radix)) + 1; }

I1Normalization i1_normalization(double rgA, double rgB, const uint64_t* row_max, const uint64_t* col_max,
                                 const double* nrA, const double* nrB, uint64_t m, uint64_t n, const I1Format& f) {
    const Dims d = make_dims(m, n, 1, 64, 64, 32, f);
    Normalization nm;
    nm.rgA = rgA;
    nm.rgB = rgB;
    nm.eA.assign(m, 0);
    nm.sA.assign(m, 0.0);
    nm.eB.assign(n, 0);
    nm.sB.assign(n, 0.0);
    nm.nrA.assign(nrA, nrA + m);
    nm.nrB.assign(nrB, nrB + n);
    const auto value = [](uint64_t u) {
        double x;
        std::memcpy(&x, &u, 8);
        return x;
    };
    for (uint64_t i = 0; i < m; ++i) row_scale(value(row_max[i]), rgA, d, nm.eA[i], nm.sA[i]);
    for (uint64_t j = 0; j < n; ++j) row_scale(value(col_max[j]), rgB, d, nm.eB[j], nm.sB[j]);
    return nm;
}

I1SamplePick i1_pick(const I1Normalization& nm) {
    I1SamplePick sp;
    pick(nm.nrA, nm.sA, kSeedRows, sp.rows, sp.wr);
    pick(nm.nrB, nm.sB, kSeedCols, sp.cols, sp.wc);
    return sp;
}

double i1_sample_norm2(const I1SamplePick& sp, const std::vector<double>& Ch, double nC) {
    const size_t na = sp.rows.size(), nb = sp.cols.size();
    double ns = 0;
    for (size_t s = 0; s < na; ++s)
        for (size_t u = 0; u < nb; ++u) ns += sp.wr[s] * sp.wc[u] * Ch[s * nb + u] * Ch[s * nb + u];
    return std::max(nC, ns);
}

double i1_model2_finish(const double* part, uint32_t nch, const I1SamplePick& sp, const std::vector<double>& Ch,
                        const std::vector<double>& Cl, const I1Normalization& nm, double norm2) {
    if (sp.rows.empty() || sp.cols.empty()) return 0.0;
    return model2_finish(part, nch, sp.rows, sp.cols, sp.wr, sp.wc, Ch, Cl, nm, norm2);
}

int i1_select_with(const I1Terms& terms, uint64_t m, uint64_t n, uint64_t k, uint32_t M, uint32_t N, uint32_t K,
                   const I1Format& f, double nC, const std::function<double(int)>& model2) {
    return select_with(terms, make_dims(m, n, k, M, N, K, f), nC, model2);
}

std::vector<double> i1_model1_errors(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                                     const I1Format& f, const I1Terms* terms, const I1Normalization* nm_in) {
    const Dims d = make_dims(m, n, k, 64, 64, 32, f);
    if (terms) return combine_terms(*terms, d);
    const Normalization nm = nm_in ? *nm_in : normalize(a, b, d);
    return combine_terms(independent_terms(a, b, d, nm), d);
}

int select_slices(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t M, uint32_t N,
                  uint32_t K, const I1Format& f) {
    const Dims d = make_dims(m, n, k, M, N, K, f);
    const Normalization nm = normalize(a, b, d);
    const I1Terms terms = independent_terms(a, b, d, nm);
    const double nC = product_norm_estimate(a, b, m, n, k, N, nm.rgA, nm.rgB);
    return select_from(a, b, d, nm, terms, nC);
}

int select_slices_int8(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t M, uint32_t N,
                       uint32_t K) {
    return select_slices(a, b, m, n, k, M, N, K, kI1Int8);
}

int plan_i(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t slices, const I1Format& f,
           oztt_i_plan& p, std::string& err) {
    return plan_i_with([&](uint32_t M, uint32_t N, uint32_t K) { return select_slices(a, b, m, n, k, M, N, K, f); },
                       m, n, k, slices, f, p, err);
}

int plan_i_with(const std::function<int(uint32_t, uint32_t, uint32_t)>& select, uint64_t m, uint64_t n, uint64_t k,
                uint32_t slices, const I1Format& f, oztt_i_plan& p, std::string& err) {
    auto pad = [](uint64_t v, uint64_t q) { return (v + q - 1) / q * q; };
    std::memset(&p, 0, sizeof p);
    if (!m || !n || !k) {
        err = "matrix dimensions are zero";
        return OZTT_EINVAL;
    }
    if (slices > 256) {
        err = "slices must be zero (automatic) or at most 256";
        return OZTT_EINVAL;
    }
    if (pad(m, 64) > UINT32_MAX || pad(n, 64) > UINT32_MAX || pad(k, 32) > UINT32_MAX) {
        err = "matrix dimensions exceed the 32-bit planning range";
        return OZTT_EINVAL;
    }
    p.M = (uint32_t)pad(m, 64);
    p.N = (uint32_t)pad(n, 64);
    p.K = (uint32_t)pad(k, 32);
    p.auto_p = slices == 0;
    p.format = f.format;
    p.radix = (int32_t)f.radix;
    p.dmax = (int32_t)f.dmax;
    p.p = slices ? (int32_t)slices : select(p.M, p.N, p.K);
    const int L = p.p - 1;
    char msg[512];
    // The issue the reference plans (plan_issue, ozaki1/plan.hpp:141-226): the pair loop or the pairwise
    // issue when the formats' FP32 partial products can be folded into Int32 (not INT8), else the
    // concatenated issue; each must have a K block length.
    const uint32_t kc_cat = block_k(p.K, L, f), kc_pw = block_k(p.K, 0, f);
    const uint64_t keff = (uint64_t)(L + 1) * p.K, d2 = (uint64_t)f.dmax * (uint64_t)f.dmax;
    const bool defer_ok = d2 != 0 && keff <= (uint64_t)INT32_MAX / d2;
    const bool fuse_ok = !f.int32_partial && defer_ok;
    const uint32_t ndiag = (uint32_t)p.p;
    const uint64_t n_cat = kc_cat ? (uint64_t)ndiag * (p.K / kc_cat) : UINT64_MAX;
    const uint64_t n_pw = kc_pw ? (uint64_t)ndiag * (ndiag + 1) / 2 * (p.K / kc_pw) : 0;
    const bool pairloop = fuse_ok && kc_pw && p.K / kc_pw == 1;
    const bool pairwise = !pairloop && fuse_ok && kc_pw && n_pw < n_cat;
    const uint32_t kc = (pairloop || pairwise) ? kc_pw : kc_cat;
    if (kc == 0) {
        std::snprintf(msg, sizeof msg,
                      "Ozaki scheme I: the partial products for k=%u with %d slices cannot be accumulated without "
                      "error in this format (no K block length satisfies the exactness condition). Use fewer "
                      "slices (Options::slices) or a smaller k.",
                      p.K, p.p);
        err = msg;
        return OZTT_ERUNTIME;
    }
    const uint32_t nkb = p.K / kc;
    if (f.int32_partial && nkb > 1) {
        std::snprintf(msg, sizeof msg,
                      "Ozaki scheme I with Format::INT8 does not support K blocking, but k=%u with %d slices needs "
                      "%u K blocks of %u columns. Use a smaller k, fewer slices (Options::slices) or another format.",
                      p.K, p.p, nkb, kc);
        err = msg;
        return OZTT_ERUNTIME;
    }
    if (!(std::log2((double)p.K) + (double)(L + 1) * std::log2(f.radix) + 12.0 < 128.0)) {
        std::snprintf(msg, sizeof msg,
                      "Ozaki scheme I: the reconstruction would overflow FP32 for k=%u with %d slices (radix %d): "
                      "log2(k) + slices*log2(radix) + 12 must be below 128. Use fewer slices (Options::slices) or "
                      "a smaller k.",
                      p.K, p.p, p.radix);
        err = msg;
        return OZTT_ERUNTIME;
    }
    return OZTT_OK;
}

int plan_i_int8(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t slices,
                oztt_i_plan& p, std::string& err) {
    return plan_i(a, b, m, n, k, slices, kI1Int8, p, err);
}

}  // namespace oztt

namespace {
int plan_i_c(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t slices,
             const oztt::I1Format& f, oztt_i_plan* plan, char* err, size_t errlen) {
    std::string msg;
    int rc;
    try {
        if (!plan || (slices == 0 && (!a || !b))) {
            msg = "null argument";
            rc = OZTT_EINVAL;
        } else {
            rc = oztt::plan_i(a, b, m, n, k, slices, f, *plan, msg);
        }
    } catch (const std::bad_alloc&) {
        msg = "out of host memory while planning";
        rc = OZTT_ENOMEM;
    } catch (const std::exception& e) {
        msg = e.what();
        rc = OZTT_ERUNTIME;
    }
    if (err && errlen) {
        std::snprintf(err, errlen, "%s", rc == OZTT_OK ? "" : msg.c_str());
    }
    return rc;
}
}  // namespace

extern "C" int oztt_i_int8_plan(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                                uint32_t slices, oztt_i_plan* plan, char* err, size_t errlen) {
    return plan_i_c(a, b, m, n, k, slices, oztt::kI1Int8, plan, err, errlen);
}

extern "C" int oztt_i_format_plan(int32_t format, const double* a, const double* b, uint64_t m, uint64_t n,
                                  uint64_t k, uint32_t slices, oztt_i_plan* plan, char* err, size_t errlen) {
    const oztt::I1Format* f = oztt::i1_format(format);
    if (!f) {
        if (err && errlen) std::snprintf(err, errlen, "%s", "format is unknown or was not built");
        return OZTT_EINVAL;
    }
    return plan_i_c(a, b, m, n, k, slices, *f, plan, err, errlen);
}
