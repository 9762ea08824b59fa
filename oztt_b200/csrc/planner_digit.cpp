// SPDX-License-Identifier: Apache-2.0
//
// Scheme II planner for the FP8 (e4m3) digit format (host). The residues modulo moduli up to 2401 do
// not fit one e4m3 value, so each residue is split into two or three small digits and the product of
// two residues is assembled from products of digit planes; this file makes the reference's decisions
// for that path (src/backend/ozaki2/split.hpp, moduli.hpp, plan.hpp, route OZ2_ROUTE_FP8):
//   splitting     per modulus: square moduli q^2 by rounding to nearest (SQ, 3 products), squares of odd
//                 q <= 49 with the sparse e4m3 digits {|x| <= 16} + {even x, |x| <= 32} (SQS), other
//                 moduli up to 513 by radix-16 Karatsuba (KAR, 3 products), larger ones with two digits
//                 of radix ~sqrt(m) (WIDE, 4 products) (split.hpp:160-330)
//   concatenation digit products of equal weight added along K into one GEMM output while g*K*d_l*d_h
//                 plus the modulus stays within 2^24 (oz2_product_groups, oz2_maxg_for)
//   selection     the FP8 table (sparse squares while K*32^2 + 2401 <= 2^24, else the dense table with
//                 cap 1089), width from the window, tail trim and reselection by (products, excess,
//                 outputs and planes), accumulation and composition conditions (moduli.hpp:180-710)
// The precision policy and the pass decision are the INT8 path's (planner.cpp).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

#include "oztt_cuda.h"
#include "planner.hpp"

namespace oztt {
namespace digit {

constexpr int kModCap = 2401, kDmax = 16, kSparse = 32;
constexpr uint32_t kDefS = 14;
constexpr int kMaxS = 24, kDigitBits = 20, kMaxDigit = 5, kTargetBits = 53, kDefaultB = 54;
constexpr double kWinEps = 1e-9, kTailTol = 0.25;
constexpr long kComposeSplit = 1L << 12;
constexpr int kTableF8[] = {1089, 1024, 961, 841, 625, 529, 511, 509, 503, 499,
                            491,  487,  481, 479, 467, 463, 461, 457, 449, 443};
constexpr int kTableF8S[] = {2401, 2209, 1849, 1681, 1521, 1369, 1024, 961, 841, 625, 529, 361,
                             289,  121,  509,  503,  499,  491,  487,  479, 467, 463, 461, 457};

// |r| bound of the slicer's last ModRound (m/2 plus its rounding allowance, at most floor(m/2)+1).
long resid_bound(int m) {
    long c0 = 1 % m;
    for (int i = 0; i < kDigitBits; ++i) c0 = (c0 * 2) % m;
    const long c1 = (c0 * c0) % m, c2 = (c1 * c0) % m;
    const double u = std::ldexp(1.0, -23) * (1.0 + std::ldexp(1.0, -23));
    const double d0 = 524288.0 + 65536.0 + 1.0;
    const double s3 = d0 + (double)(m / 2) * (double)(c0 + c1);
    const double s4 = m / 2.0 + 2.0 + (double)(m / 2) * (double)c2;
    return std::min<long>((long)std::floor(m / 2.0 + std::max(s3, s4) * u), m / 2 + 1);
}
int isqrt(int m) {
    int r = (int)std::sqrt((double)m);
    while ((long)(r + 1) * (r + 1) <= m) ++r;
    while ((long)r * r > m) --r;
    return r;
}
int square_root_of(int m) {
    const int r = isqrt(m);
    return (long)r * r == m ? r : 0;
}
// Digits by rounding to nearest with radix q: bound max(round((m/2)/q), q/2).
int bound_rnd(int m, int q) {
    const int rs = m / 2;
    return std::max((rs + q / 2) / q, q / 2);
}
// Radix-16 Karatsuba digits (rounded up): bound max(ceil((m/2)/16), 15).
int bound_kar(int m) { return std::max((m / 2 + 15) / 16, 15); }
// The q near sqrt(m) that minimises the rounding bound.
int radix_rnd(int m) {
    const int r = isqrt(m);
    int best = r + 1, bb = bound_rnd(m, r + 1);
    for (int q = r; q <= r + 3; ++q) {
        const int v = bound_rnd(m, q);
        if (v < bb) {
            bb = v;
            best = q;
        }
    }
    return best;
}
// e4m3 represents the integer v exactly (at most 4 significant bits).
bool e4m3_integer(long v) {
    if (v < 0) v = -v;
    if (v == 0) return true;
    int e = 0;
    for (long x = v; x; x >>= 1) ++e;
    return e <= 4 || (v % (1L << (e - 4))) == 0;
}
// The sparse digit set {x exact in e4m3, |x| <= smax} holds a complete residue system modulo q.
bool sparse_covers(int q, int smax) {
    if (q <= 0 || smax <= 0 || q > 2 * smax + 1) return false;
    std::vector<char> hit(q, 0);
    int n = 0;
    for (int x = -smax; x <= smax; ++x)
        if (e4m3_integer(x)) {
            const int r = ((x % q) + q) % q;
            if (!hit[r]) {
                hit[r] = 1;
                ++n;
            }
        }
    return n == q;
}
// Sparse split of r modulo q^2 (q odd): rounding to nearest, then odd digits of magnitude >= 17 moved
// by q into the even sparse digits.
void sqs_split(long r, int q, long& l, long& h) {
    long h0 = (2 * r + (r >= 0 ? q : -q)) / (2 * q);
    long t = r - (long)q * h0;
    const long st = t > 0 ? 1 : (t < 0 ? -1 : 0);
    if ((t & 1) && (t >= 17 || t <= -17)) {
        t -= st * q;
        h0 += st;
    }
    const long sh = h0 > 0 ? 1 : (h0 < 0 ? -1 : 0);
    if ((h0 & 1) && (h0 >= 17 || h0 <= -17)) h0 -= sh * q;
    l = t;
    h = h0;
}
void sqs_bounds(int q, int& dl, int& dh) {
    const long m = (long)q * q, R = m / 2 + 1;
    dl = dh = 0;
    for (long r = -R; r <= R; ++r) {
        long l, h;
        sqs_split(r, q, l, h);
        dl = std::max<int>(dl, (int)std::labs(l));
        dh = std::max<int>(dh, (int)std::labs(h));
    }
}

// Splitting method of m with dense digit bound dmax = 16 and sparse bound smax (0: dense only).
int split_mode(int m, int smax) {
    if (const int q = square_root_of(m)) {
        if (smax && bound_rnd(m, q) > kDmax && (q & 1) && sparse_covers(q, smax)) return OZTT_SPLIT_SQS;
        return OZTT_SPLIT_SQ;
    }
    if (bound_kar(m) <= kDmax) return OZTT_SPLIT_KAR;
    return OZTT_SPLIT_WIDE;
}
int radix_of(int m) {
    const int mode = split_mode(m, 0);
    if (mode == OZTT_SPLIT_SQ) return square_root_of(m);
    return mode == OZTT_SPLIT_KAR ? 16 : radix_rnd(m);
}
int dense_bound(int m) {
    const int mode = split_mode(m, 0);
    if (mode == OZTT_SPLIT_KAR) return bound_kar(m);
    return bound_rnd(m, radix_of(m));
}
bool usable(int m, int smax) {
    if (split_mode(m, smax) == OZTT_SPLIT_SQS) return true;
    return dense_bound(m) <= kDmax;
}
int planes_of(int m) { return split_mode(m, 0) == OZTT_SPLIT_KAR ? 3 : 2; }
// Bound on |digit| of plane `plane` (0 low, 1 high, 2 sum) of m.
int plane_bound(int m, int plane, int smax) {
    if (!smax) return kDmax;
    if (split_mode(m, smax) == OZTT_SPLIT_SQS) {
        int dl, dh;
        sqs_bounds(square_root_of(m), dl, dh);
        return plane == 0 ? dl : dh;
    }
    return dense_bound(m);
}

struct Term {
    int a, b;
    long coeff;  // in [0, m)
};
// Digit products of m and their composition coefficients (before concatenation).
std::vector<Term> product_terms(int m) {
    auto rm = [&](long v) {
        const long r = v % m;
        return r < 0 ? r + m : r;
    };
    const int mode = split_mode(m, 0), q = radix_of(m);
    if (mode == OZTT_SPLIT_KAR) {  // B^2 HH + B (SS - HH - LL) + LL with B = 16: (1-B) LL, (B^2-B) HH, B SS
        const long B = q;
        return {{0, 0, rm(1 - B)}, {1, 1, rm(B * B - B)}, {2, 2, rm(B)}};
    }
    std::vector<Term> t = {{0, 0, rm(1)}, {1, 0, rm(q)}, {0, 1, rm(q)}};
    if (mode == OZTT_SPLIT_WIDE) t.push_back({1, 1, rm((long)q * q)});
    return t;
}
struct Group {
    int a0, b0, g;  // planes a0..a0+g-1 of A against positions b0..b0+g-1 of the reversed B stack
    long coeff;
};
// Products of equal weight (a + b) in runs of at most maxg consecutive A planes.
std::vector<Group> product_groups(int m, int maxg) {
    const std::vector<Term> t = product_terms(m);
    const int np = planes_of(m);
    std::vector<Group> out;
    for (int key = 0; key <= 2 * (np - 1); ++key) {
        std::vector<int> as;
        long c = 0;
        for (const Term& x : t)
            if (x.a + x.b == key) {
                as.push_back(x.a);
                c = x.coeff;
            }
        std::sort(as.begin(), as.end());
        for (size_t i = 0; i < as.size();) {
            int g = 1;
            while (i + g < as.size() && g < maxg && as[i + g] == as[i] + g) ++g;
            out.push_back({as[i], np - 1 - (key - as[i]), g, c});
            i += g;
        }
    }
    return out;
}
double group_bound(int m, const Group& g, double K, int smax) {
    const int np = planes_of(m);
    double s = 0;
    for (int t = 0; t < g.g; ++t) s += K * plane_bound(m, g.a0 + t, smax) * plane_bound(m, np - 1 - (g.b0 + t), smax);
    return s;
}
int maxg_for(int m, uint32_t K, int cap, int smax) {
    const double pb = (double)plane_bound(m, 0, smax) * plane_bound(m, std::min(1, planes_of(m) - 1), smax);
    return std::max(1, (int)std::floor((std::ldexp(1.0, 24) - cap) / ((double)K * pb)));
}

struct Choice {
    bool ok = false, acc_ok = true, fold_first = false;
    int b = 0, m_cap = 0, ncand = 0;
    std::vector<int> m, maxg;
    std::string acc_why;  // first failed accumulation condition ("digit" or "compose")
    int acc_m = 0, acc_d = 0;
    double acc_val = 0;
};

Choice choose(uint32_t K, int num_moduli, int b_cap) {
    int mod_cap = kModCap, smax = kSparse;
    const double wlog2 = std::log2((double)K);
    if ((double)K * smax * smax + mod_cap > std::ldexp(1.0, 24)) {  // dense digits for large K
        smax = 0;
        mod_cap = std::min(mod_cap, (2 * kDmax + 1) * (2 * kDmax + 1));
    }
    Choice o;
    o.m_cap = mod_cap;
    double logM = 0;
    const int* table = smax ? kTableF8S : kTableF8;
    const int tn = smax ? (int)std::size(kTableF8S) : (int)std::size(kTableF8);
    for (int t = 0; t < tn && (int)o.m.size() < num_moduli; ++t) {
        const int mm = table[t];
        if (mm > mod_cap || !usable(mm, smax)) continue;
        o.m.push_back(mm);
        logM += std::log2((double)mm);
    }
    o.ncand = (int)o.m.size();
    const double room = logM - 1.0 - wlog2 - kWinEps;
    o.b = std::min(std::min((int)std::floor(room / 2.0), kMaxDigit * kDigitBits), b_cap);
    const double need = 2.0 * o.b + 1.0 + wlog2 + kWinEps;
    // trim: drop moduli from the end while the window stays covered
    while (o.m.size() > 2) {
        const double l2 = std::log2((double)o.m.back());
        if (logM - l2 < need) break;
        o.m.pop_back();
        logM -= l2;
    }
    // reselect the last two
    if (o.m.size() >= 2 && logM > need) {
        std::vector<int> head(o.m.begin(), o.m.end() - 2);
        double base = 0;
        for (int x : head) base += std::log2((double)x);
        auto cop_head = [&](int mm) {
            for (int x : head)
                if (std::gcd(mm, x) != 1) return false;
            return true;
        };
        std::vector<char> use_c(mod_cap + 1, 0);
        std::vector<int> np_c(mod_cap + 1, 0), lay_c(mod_cap + 1, 0);
        for (int mm = 3; mm <= mod_cap; ++mm)
            if (usable(mm, smax)) {
                use_c[mm] = 1;
                np_c[mm] = (int)product_terms(mm).size();
                lay_c[mm] = 1000 * (int)product_groups(mm, maxg_for(mm, K, mod_cap, smax)).size() + planes_of(mm);
            }
        auto ok_c = [&](int mm) { return mm >= 3 && mm <= mod_cap && use_c[mm]; };
        auto over = [&](double l) { return (l - need) > kTailTol ? 1 : 0; };
        double best = logM;
        int bp = o.m[o.m.size() - 2], bq = o.m.back();
        int bcost = np_c[bp] + np_c[bq], blay = lay_c[bp] + lay_c[bq];
        auto better = [&](int c, int lay, double l) {
            if (c != bcost) return c < bcost;
            if (over(l) != over(best)) return over(l) < over(best);
            return lay < blay || (lay == blay && l < best);
        };
        bool head_even = false;
        for (int x : head) head_even = head_even || (x % 2 == 0);
        const int step = head_even ? 2 : 1;
        for (int p2 = 3; p2 <= mod_cap; p2 += step) {
            if (!ok_c(p2) || !cop_head(p2)) continue;
            const double lp = base + std::log2((double)p2);
            if (lp >= need && better(np_c[p2], lay_c[p2], lp)) {
                best = lp;
                bp = p2;
                bq = 0;
                bcost = np_c[p2];
                blay = lay_c[p2];
            }
            for (int q = p2 + step; q <= mod_cap; q += step) {
                if (!ok_c(q) || std::gcd(p2, q) != 1 || !cop_head(q)) continue;
                const double lq = lp + std::log2((double)q);
                const int c = np_c[p2] + np_c[q], lay = lay_c[p2] + lay_c[q];
                if (lq >= need && better(c, lay, lq)) {
                    best = lq;
                    bp = p2;
                    bq = q;
                    bcost = c;
                    blay = lay;
                }
            }
        }
        o.m = head;
        o.m.push_back(bp);
        if (bq) o.m.push_back(bq);
        logM = best;
    }
    const int S = (int)o.m.size();
    o.ok = logM >= need && S > 0 && S <= kMaxS && S <= num_moduli && o.b > 0;
    for (int i = 0; i < S; ++i)
        for (int j = i + 1; j < S; ++j)
            if (std::gcd(o.m[i], o.m[j]) != 1) o.ok = false;
    auto fail = [&](const char* why, int mm, int d, double v) {
        if (o.acc_why.empty()) {
            o.acc_why = why;
            o.acc_m = mm;
            o.acc_d = d;
            o.acc_val = v;
        }
        o.ok = o.acc_ok = false;
    };
    // exact FP32 accumulation of the digit products (per-plane bounds on the sparse path)
    int deff = kDmax;
    if (smax) {
        deff = 0;
        for (int mm : o.m)
            for (int pl = 0; pl < planes_of(mm); ++pl) deff = std::max(deff, plane_bound(mm, pl, smax));
    }
    if ((double)K * deff * deff > std::ldexp(1.0, 24)) fail("digit", 0, deff, (double)K * deff * deff);
    // concatenation and composition
    int mmax = 0;
    for (int mm : o.m) mmax = std::max(mmax, mm);
    o.maxg.assign(S, 1);
    for (int i = 0; i < S; ++i) o.maxg[i] = maxg_for(o.m[i], K, mmax, smax);
    auto maxg_all = [&] {
        int g = 1;
        for (int x : o.maxg) g = std::max(g, x);
        return g;
    };
    auto compose_sum = [&](int i, bool fold) {
        const int mm = o.m[i];
        double sum = 0;
        for (const Group& g : product_groups(mm, o.maxg[i])) {
            const double hi = (double)((g.coeff * kComposeSplit) % mm);
            sum += fold ? std::fabs((double)g.coeff) * ((double)mm / 2.0 + 2.0)
                        : std::floor(group_bound(mm, g, (double)K, smax) / (double)kComposeSplit + 0.5) *
                                  std::fabs(hi) +
                              (double)(kComposeSplit / 2) * std::fabs((double)g.coeff);
        }
        return sum;
    };
    for (int attempt = 0; attempt < 2; ++attempt) {
        bool can_fold = true;
        for (int i = 0; i < S; ++i) {
            double gmax = 0;
            for (const Group& g : product_groups(o.m[i], o.maxg[i]))
                gmax = std::max(gmax, group_bound(o.m[i], g, (double)K, smax));
            if (gmax + o.m[i] > std::ldexp(1.0, 24) || compose_sum(i, true) >= std::ldexp(1.0, 22)) can_fold = false;
        }
        if (maxg_all() > 1 && !can_fold) {
            o.maxg.assign(S, 1);
            continue;
        }
        o.fold_first = can_fold;
        if (!can_fold)
            for (int i = 0; i < S; ++i)
                if (const double cs = compose_sum(i, false); cs >= std::ldexp(1.0, 22)) fail("compose", o.m[i], 0, cs);
        break;
    }
    return o;
}

std::string short_cause(const Choice& mo, uint32_t S_req, uint32_t K, int b_cap, int target) {
    const uint32_t want = std::min<uint32_t>(S_req, kMaxS);
    if ((uint32_t)mo.ncand < want)
        return "Every candidate modulus is in use (" + std::to_string(mo.ncand) +
               "), so a larger Options::max_moduli does not help; use a smaller K or a different format.";
    if (want >= (uint32_t)kMaxS) return "The maximum of 24 moduli is not enough; use a smaller K or a different format.";
    Choice t;
    for (uint32_t n = S_req + 1; n <= (uint32_t)kMaxS; ++n) {
        t = choose(K, (int)n, b_cap);
        if (t.ok && t.b >= target)
            return "The limit of " + std::to_string(S_req) + " moduli is too small; set Options::max_moduli to " +
                   std::to_string(n) + " or more.";
    }
    return "The limit of " + std::to_string(S_req) + " moduli is too small, and the maximum of 24 moduli still gives only " +
           std::to_string(t.ok ? t.b : 0) + " bits; use a smaller K or a different format.";
}

}  // namespace digit

int plan_fp8_with(const std::function<PolicyStats(uint32_t, uint32_t)>& stats, uint64_t m, uint64_t n, uint64_t k,
                  uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_fp8_plan& p,
                  std::string& err) {
    using namespace digit;
    std::memset(&p, 0, sizeof p);
    oztt_ii_plan& base = p.base;
    if (!m || !n || !k) {
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
    auto pad = [](uint64_t v, uint64_t q) { return (v + q - 1) / q * q; };
    base.M = (uint32_t)pad(m, 64);
    base.N = (uint32_t)pad(n, 64);
    base.K = (uint32_t)pad(k, 32);
    const bool b_fixed = fixed_bits > 0;
    PolicyStats st;
    int b_cap = kDefaultB;
    if (b_fixed)
        b_cap = fixed_bits;
    else {
        st = stats(base.N, base.K);
        b_cap = policy_width_cap(st);
    }
    const uint32_t S_req = max_moduli ? max_moduli : (b_fixed ? kDefS : (uint32_t)kMaxS);
    if (b_fixed && reconstruction == OZTT_RECON_AUTO) st = stats(base.N, base.K);
    const Choice mo = choose(base.K, (int)S_req, b_cap);
    base.b_cap = b_cap;
    base.S_req = (int32_t)S_req;
    base.TA = st.TA;
    base.TB = st.TB;
    base.nA = st.nA;
    base.nB = st.nB;
    base.nC = st.nC;
    if (!mo.ok) {
        if (!mo.acc_ok) {
            std::string cause = "an exactness condition of the accumulation does not hold";
            char buf[400];
            if (mo.acc_why == "digit") {
                std::snprintf(buf, sizeof buf,
                              "the digit-product bound K*d^2 = %.0f (digit bound d=%d) exceeds 2^24, the limit of "
                              "exact FP32 accumulation",
                              mo.acc_val, mo.acc_d);
                cause = buf;
            } else if (mo.acc_why == "compose") {
                std::snprintf(buf, sizeof buf,
                              "the digit products of modulus %d cannot be composed exactly (the bound %.0f of the "
                              "composition sum reaches 2^22)",
                              mo.acc_m, mo.acc_val);
                cause = buf;
            }
            err = "Ozaki II: the padded inner dimension K=" + std::to_string(base.K) +
                  " is too large for this format: " + cause +
                  ". Use a smaller K or a different format; Options::max_moduli does not change this limit.";
        } else {
            err = "Ozaki II: the available moduli do not cover the CRT window for the padded inner dimension K=" +
                  std::to_string(base.K) + ". " + short_cause(mo, S_req, base.K, b_cap, b_fixed ? 1 : kTargetBits);
        }
        return OZTT_ERUNTIME;
    }
    if (!b_fixed && mo.b < kTargetBits) {
        err = "Ozaki II: for the padded inner dimension K=" + std::to_string(base.K) + " the " +
              std::to_string(mo.m.size()) + " selected moduli cover a width of only " + std::to_string(mo.b) +
              " bits, below the 53 bits of FP64-equivalent accuracy. " +
              short_cause(mo, S_req, base.K, b_cap, kTargetBits);
        return OZTT_ERUNTIME;
    }
    base.b = mo.b;
    base.recon1_log2 = one_pass_error_log2(mo.m, mo.b, st);
    base.two_pass =
        reconstruction != OZTT_RECON_AUTO ? (reconstruction == OZTT_RECON_TWO) : !(base.recon1_log2 <= -55.0);
    base.nd = mo.b > 4 * kDigitBits ? 5 : (mo.b > 3 * kDigitBits ? 4 : 3);
    base.shift = mo.b - (base.nd - 1) * kDigitBits;
    fill_crt_constants(mo.m, base);
    // layout: digit planes, GEMM outputs (jobs) and composition coefficients
    const int smax = ((double)base.K * kSparse * kSparse + kModCap > std::ldexp(1.0, 24)) ? 0 : kSparse;
    p.fold_first = mo.fold_first ? 1 : 0;
    int plane = 0, out = 0;
    for (int i = 0; i < (int)mo.m.size(); ++i) {
        const int mm = mo.m[i];
        p.q[i] = radix_of(mm);
        p.mode[i] = split_mode(mm, smax);
        p.poff[i] = plane;
        p.npl[i] = planes_of(mm);
        p.oout[i] = out;
        p.nprod += (int32_t)product_terms(mm).size();
        for (const Group& g : product_groups(mm, mo.maxg[i])) {
            if (out >= OZTT_MAXOUT) {
                err = "internal error: too many GEMM outputs";
                return OZTT_ERUNTIME;
            }
            p.out_a[out] = plane + g.a0;
            p.out_b[out] = plane + (p.npl[i] - 1 - g.b0);
            p.out_g[out] = g.g;
            p.out_mod[out] = i;
            p.coeff[out] = (int32_t)g.coeff;
            ++out;
        }
        plane += p.npl[i];
    }
    p.oout[mo.m.size()] = out;
    p.nplane = plane;
    p.nout = out;
    return OZTT_OK;
}

int plan_fp8(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli,
             int32_t reconstruction, int32_t fixed_bits, oztt_fp8_plan& p, std::string& err) {
    return plan_fp8_with([&](uint32_t N, uint32_t K) { return measure_policy_stats(a, b, m, n, k, N, K); }, m, n, k,
                         max_moduli, reconstruction, fixed_bits, p, err);
}

}  // namespace oztt

extern "C" int oztt_ii_fp8_plan(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                                uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_fp8_plan* plan,
                             char* err, size_t errlen) {
    std::string msg;
    int rc;
    try {
        if (!plan || (fixed_bits <= 0 && (!a || !b))) {
            msg = "null argument";
            rc = OZTT_EINVAL;
        } else {
            rc = oztt::plan_fp8(a, b, m, n, k, max_moduli, reconstruction, fixed_bits, *plan, msg);
        }
    } catch (const std::bad_alloc&) {
        msg = "out of host memory while planning";
        rc = OZTT_ENOMEM;
    } catch (const std::exception& e) {
        msg = e.what();
        rc = OZTT_ERUNTIME;
    }
    if (err && errlen) std::snprintf(err, errlen, "%s", rc == OZTT_OK ? "" : msg.c_str());
    return rc;
}
