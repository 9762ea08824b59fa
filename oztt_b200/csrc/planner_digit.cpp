// SPDX-License-Identifier: Apache-2.0
//
// Scheme II planner for the digit formats (host): FP8 (e4m3), BF16, FP16 and TF32. The residues modulo
// moduli up to 4096 do not fit one low-precision value, so each residue is split into one to three small
// digits and the product of two residues is assembled from products of digit planes; this file makes the
// reference's decisions for those paths (src/backend/ozaki2/split.hpp, moduli.hpp, awe.hpp, plan.hpp):
//   routes        FP8: digits <= 16, the sparse e4m3 digits up to 32 for squares of odd q <= 49, moduli up
//                 to 2401, table selection; TF32: digits <= 32, moduli up to 4096, table selection; BF16 and
//                 FP16: digits <= 32, one-digit moduli (the residue itself, |r| <= 32), the moduli set of
//                 the stage-time model search (split.hpp:46-137)
//   splitting     per modulus (split.hpp:160-560): one digit (ONE), squares q^2 by rounding to nearest (SQ,
//                 3 products), sparse squares (SQS), radix-16 Karatsuba up to 513 (KAR, 3 products), two
//                 digits of radix ~sqrt(m) (WIDE, 4 products)
//   concatenation digit products of equal weight added along K into one GEMM output while g*K*d_l*d_h
//                 plus the modulus stays within 2^24 (oz2_product_groups, oz2_maxg_for)
//   selection     the route's table, width from the window, tail trim and reselection by (products, excess,
//                 outputs and planes); for BF16/FP16 the set minimising the fitted stage-time model under
//                 the window (awe.hpp: classes of equal cost, pruned enumeration of count vectors, coprime
//                 assignment, the same cutoffs); accumulation and composition conditions (moduli.hpp:180-770)
// The precision policy and the pass decision are the INT8 path's (planner.cpp).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <mutex>
#include <numeric>
#include <string>
#include <vector>

#include "oztt_cuda.h"
#include "planner.hpp"

namespace oztt {
namespace digit {

constexpr int kMaxS = 24, kDigitBits = 20, kMaxDigit = 5, kTargetBits = 53, kDefaultB = 54;
constexpr double kWinEps = 1e-9, kTailTol = 0.25;
constexpr long kComposeSplit = 1L << 12;
constexpr double kTwo24 = 16777216.0, kTwo22 = 4194304.0;

// A format's path (Oz2Route, split.hpp:46-137): modulus cap, digit bound, default limit on the moduli
// with a fixed width, sparse digit bound (FP8), row of the stage-time model (0: table selection),
// one-digit moduli, and the bytes of one 32x32 tile of its digit planes (the model's DRAM estimate).
struct Route {
    int format, mod_cap, dmax;
    uint32_t def_s;
    int smax, awe;
    bool one;
    double slice_tile;
};
constexpr Route kRoutes[] = {
    {OZTT_FMT_FP8, 2401, 16, 14u, 32, 0, false, 1024.0},
    {OZTT_FMT_TF32, 4096, 32, 11u, 0, 0, false, 4096.0},
    {OZTT_FMT_BF16, 4096, 32, 24u, 0, 3, true, 2048.0},
    {OZTT_FMT_FP16, 4096, 32, 24u, 0, 4, true, 2048.0},
};
const Route* route_of(int32_t format) {
    for (const Route& r : kRoutes)
        if (r.format == format) return &r;
    return nullptr;
}

// Candidate tables (moduli.hpp:184-205): FP8 dense (from 33^2), FP8 sparse squares, digit bound 32
// (squares of pairwise coprime q <= 64).
constexpr int kTableF8[] = {1089, 1024, 961, 841, 625, 529, 511, 509, 503, 499,
                            491,  487,  481, 479, 467, 463, 461, 457, 449, 443};
constexpr int kTableF8S[] = {2401, 2209, 1849, 1681, 1521, 1369, 1024, 961, 841, 625, 529, 361,
                             289,  121,  509,  503,  499,  491,  487,  479, 467, 463, 461, 457};
constexpr int kTableB8[] = {4096, 3969, 3721, 3481, 3025, 2809, 2209, 1849, 1681, 1369, 961, 841, 529, 361, 289, 169};

// The path during one selection: digit bound, one-digit moduli, and the sparse bound and modulus cap
// after FP8's fallback to dense digits for large K.
struct Path {
    uint32_t K;
    int mod_cap, dmax, smax;
    bool one;
};

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

// Splitting method of m on a path with digit bound dmax (>= 16 here), one-digit moduli `one`, and the
// sparse bound smax (0: dense only; the methods that count products and planes pass 0).
int split_mode(int m, const Path& p, int smax) {
    if (p.one && p.dmax && resid_bound(m) <= p.dmax) return OZTT_SPLIT_ONE;
    if (const int q = square_root_of(m)) {
        if (smax && p.dmax && bound_rnd(m, q) > p.dmax && (q & 1) && sparse_covers(q, smax)) return OZTT_SPLIT_SQS;
        return OZTT_SPLIT_SQ;
    }
    if (bound_kar(m) <= std::min(16, p.dmax)) return OZTT_SPLIT_KAR;
    return OZTT_SPLIT_WIDE;
}
int radix_of(int m, const Path& p) {
    const int mode = split_mode(m, p, 0);
    if (mode == OZTT_SPLIT_ONE) return 1;
    if (mode == OZTT_SPLIT_SQ) return square_root_of(m);
    return mode == OZTT_SPLIT_KAR ? 16 : radix_rnd(m);
}
int dense_bound(int m, const Path& p) {
    const int mode = split_mode(m, p, 0);
    if (mode == OZTT_SPLIT_ONE) return (int)resid_bound(m);
    if (mode == OZTT_SPLIT_KAR) return bound_kar(m);
    return bound_rnd(m, radix_of(m, p));
}
bool usable(int m, const Path& p, int smax) {
    if (split_mode(m, p, smax) == OZTT_SPLIT_SQS) return true;
    return dense_bound(m, p) <= p.dmax;
}
int planes_of(int m, const Path& p) {
    const int mode = split_mode(m, p, 0);
    if (mode == OZTT_SPLIT_ONE) return 1;
    return mode == OZTT_SPLIT_KAR ? 3 : 2;
}
// Bound on |digit| of plane `plane` (0 low, 1 high, 2 sum) of m (oz2_plane_bound, split.hpp:470-500).
int plane_bound(int m, int plane, const Path& p, int smax) {
    if (p.one && !smax) {
        const int mode = split_mode(m, p, 0), R = (int)resid_bound(m);
        if (mode == OZTT_SPLIT_ONE) return R;
        if (mode == OZTT_SPLIT_KAR) {
            const int h = (R + 15) / 16;
            return plane == 0 ? 15 : (plane == 1 ? h : std::max(h, 15));
        }
        const int q = radix_of(m, p);
        return plane == 0 ? q / 2 : (R + q / 2) / q;
    }
    if (!smax) return p.dmax;
    if (split_mode(m, p, smax) == OZTT_SPLIT_SQS) {
        int dl, dh;
        sqs_bounds(square_root_of(m), dl, dh);
        return plane == 0 ? dl : dh;
    }
    return dense_bound(m, p);
}

struct Term {
    int a, b;
    long coeff;  // in [0, m)
};
// Digit products of m and their composition coefficients (before concatenation).
std::vector<Term> product_terms(int m, const Path& p) {
    auto rm = [&](long v) {
        const long r = v % m;
        return r < 0 ? r + m : r;
    };
    const int mode = split_mode(m, p, 0), q = radix_of(m, p);
    if (mode == OZTT_SPLIT_ONE) return {{0, 0, rm(1)}};
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
std::vector<Group> product_groups(int m, const Path& p, int maxg) {
    const std::vector<Term> t = product_terms(m, p);
    const int np = planes_of(m, p);
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
double group_bound(int m, const Group& g, double K, const Path& p, int smax) {
    const int np = planes_of(m, p);
    double s = 0;
    for (int t = 0; t < g.g; ++t)
        s += K * plane_bound(m, g.a0 + t, p, smax) * plane_bound(m, np - 1 - (g.b0 + t), p, smax);
    return s;
}
int maxg_for(int m, uint32_t K, int cap, const Path& p, int smax) {
    const double pb =
        (double)plane_bound(m, 0, p, smax) * plane_bound(m, std::min(1, planes_of(m, p) - 1), p, smax);
    return std::max(1, (int)std::floor((kTwo24 - cap) / ((double)K * pb)));
}

// ---- stage-time model search (awe.hpp) ----------------------------------------------------------
// Fitted coefficients of the reference's model rows for BF16 and FP16 at K = 3520, 7040, 14080 (columns
// K, gp, go, co, cs, sop, spl, R0, ra, rb; awe_coef.inc rows 3 and 4). The model's decisions depend on
// these values, so they are the reference's data.
struct AweCoef {
    double K, gp, go, co, cs, sop, spl, R0, ra, rb;
};
constexpr AweCoef kAweBF16[3] = {
    {3520, 0.18, 0.32, 0.22216, 0.019318, 0.035712, 0.007885, 17.05, 0.48028, 1.1507},
    {7040, 1.6623, 0.86117, 0.89522, 0.048653, 0.14382, 0.032161, 68.35, 1.363, 4.6101},
    {14080, 18.496, 1.2997, 3.7014, 2.5704, 0.57273, 0.12705, 278.85, 63.651, 15.155},
};
constexpr AweCoef kAweFP16[3] = {
    {3520, 0.1811, 0.32017, 0.22564, 0.019621, 0.035752, 0.56545, 17.17, 0.48366, 1.1588},
    {7040, 1.6436, 0.86032, 0.91946, 0.049971, 0.14307, 2.2615, 68.45, 1.365, 4.6168},
    {14080, 18.324, 1.3003, 3.6652, 2.5453, 0.57267, 9.0297, 275.92, 62.982, 14.996},
};
constexpr double kAweOneRecon = 0.062, kAweDramFree = 31.0e9, kDramMargin = 512.0 * 1048576.0;
constexpr size_t kAweVecMax = 200000;
constexpr long kAweNodeMax = 400000, kAweNodeBudget = 10000000;
constexpr double kAweOverNeedBits = 16.0, kAweUbSlack = 1.05;

// Coefficients at K: power-law interpolation in log2 K between the two nearest fitted rows.
AweCoef awe_coef(int awe, uint32_t K) {
    const AweCoef* t = awe == 3 ? kAweBF16 : kAweFP16;
    const double x = std::log2((double)K);
    const int i = x > std::log2(t[1].K) ? 1 : 0;
    const double x0 = std::log2(t[i].K), x1 = std::log2(t[i + 1].K), f = (x - x0) / (x1 - x0);
    auto ip = [&](double a, double b) {
        if (a > 0 && b > 0) return std::exp(std::log(a) + f * (std::log(b) - std::log(a)));
        return a + f * (b - a);
    };
    const AweCoef &a = t[i], &b = t[i + 1];
    return {(double)K, ip(a.gp, b.gp), ip(a.go, b.go), ip(a.co, b.co), ip(a.cs, b.cs),
            ip(a.sop, b.sop), ip(a.spl, b.spl), ip(a.R0, b.R0), ip(a.ra, b.ra), ip(a.rb, b.rb)};
}
double awe_recon(const AweCoef& c, int S) { return std::max(c.R0, c.ra + c.rb * S); }
// Slicer operations of making the digits of m, beyond the 19 up to the residue.
int awe_ops(int m, const Path& p, int smax) {
    const int mode = split_mode(m, p, smax);
    if (mode == OZTT_SPLIT_ONE) return 0;
    if (mode == OZTT_SPLIT_KAR) return 12;
    if (mode == OZTT_SPLIT_SQS) return 13;
    return 6;
}
// Planes of the composition stage for the largest output count mx of a composed modulus.
double compose_planes(bool composes, uint32_t mx) {
    if (!composes) return 0;
    const uint32_t max_nout = std::max<uint32_t>(mx, 3u);
    const uint32_t chunk = max_nout > 12 ? 5u : max_nout;
    return chunk < max_nout ? chunk + (max_nout + chunk - 1) / chunk : max_nout;
}

struct AweCand {
    int m;
    double bits;
};
struct AweClass {
    int nprod, nout, npl, ops;
    bool one;
    double cost;
    std::vector<AweCand> v;
    std::vector<double> est;
};

// Usable moduli sorted into classes of equal cost, each with its greedy coprime bit estimate; classes
// ordered by cost per bit of their largest member (ties by cost).
std::vector<AweClass> awe_classes(uint32_t K, const AweCoef& C, const Path& p, int smax) {
    std::vector<AweClass> ks;
    const int mod_cap = p.mod_cap;
    for (int m = mod_cap; m >= 2; --m) {
        if (!usable(m, p, smax)) continue;
        const int mg = maxg_for(m, K, mod_cap, p, smax);
        const int pl = planes_of(m, p);
        const int np = (int)product_terms(m, p).size();
        const std::vector<Group> gr = product_groups(m, p, mg);
        const int no = (int)gr.size(), op = awe_ops(m, p, smax);
        const bool one = split_mode(m, p, smax) == OZTT_SPLIT_ONE;
        double csum = 0, gmax = 0;
        for (const Group& g : gr) {
            csum += std::fabs((double)g.coeff);
            gmax = std::max(gmax, group_bound(m, g, (double)K, p, smax));
        }
        if (gr.empty() || gmax + mod_cap > kTwo24 || csum * (m / 2.0 + 2.0) >= kTwo22) continue;
        AweClass* k = nullptr;
        for (AweClass& x : ks)
            if (x.nprod == np && x.nout == no && x.npl == pl && x.ops == op && x.one == one) {
                k = &x;
                break;
            }
        if (!k) {
            const double cost = one ? C.gp * np + C.go * no + C.sop * (19 + op) + C.spl * pl + kAweOneRecon * C.rb
                                    : C.gp * np + (C.go + C.co) * no + C.cs + C.sop * (19 + op) + C.spl * pl;
            ks.push_back({np, no, pl, op, one, cost, {}, {}});
            k = &ks.back();
        }
        k->v.push_back({m, std::log2((double)m)});
    }
    for (AweClass& k : ks) {
        std::vector<int> got;
        k.est.assign(1, 0.0);
        for (const AweCand& c : k.v) {
            bool ok = true;
            for (int g : got)
                if (std::gcd(g, c.m) != 1) {
                    ok = false;
                    break;
                }
            if (ok) {
                got.push_back(c.m);
                k.est.push_back(k.est.back() + c.bits);
            }
        }
    }
    std::sort(ks.begin(), ks.end(), [](const AweClass& a, const AweClass& b) {
        const double ra = a.cost / a.v[0].bits, rb = b.cost / b.v[0].bits;
        return ra != rb ? ra < rb : a.cost < b.cost;
    });
    return ks;
}

struct AweSearch {
    const std::vector<AweClass>& ks;
    const AweCoef& C;
    double need, tol;
    int max_moduli;
    std::vector<double> minrate;
    double P, out, F;
    // S moduli with npl digit planes fit the model's free DRAM without output bands.
    bool dram_ok(int S, int npl, int mxo) const {
        const double Q = (compose_planes(mxo > 0, (uint32_t)mxo) + S) * out;
        return npl * P + (Q > F ? Q - F : 0.0) + kDramMargin <= kAweDramFree;
    }
};
struct AweVec {
    double T;
    std::vector<int> n;
};

// Count vectors below `incumbent` whose bit estimate reaches the window (pruned depth-first traversal).
struct AweEnum {
    const AweSearch& s;
    double incumbent;
    bool dram;
    bool& dram_cut;
    std::vector<AweVec>& vecs;
    std::vector<int> n;
    void rec(int c, int S, double cost, double est, int npl, int mxo) {
        const int NC = (int)s.ks.size();
        if (vecs.size() >= kAweVecMax) return;
        if (c == NC) {
            if (est >= s.need && S > 0) {
                const double T = cost + awe_recon(s.C, S);
                if (T < incumbent) {
                    if (!dram || s.dram_ok(S, npl, mxo))
                        vecs.push_back({T, n});
                    else
                        dram_cut = true;
                }
            }
            return;
        }
        const double rem = std::max(0.0, s.need - est);
        if (cost + rem * s.minrate[c] + awe_recon(s.C, S) >= incumbent) return;
        const AweClass& k = s.ks[c];
        const int maxn = std::min<int>((int)k.est.size() - 1, s.max_moduli - S);
        for (int t = 0; t <= maxn; ++t) {
            n[c] = t;
            const double e2 = est + k.est[t];
            if (cost + t * k.cost + awe_recon(s.C, S + t) >= incumbent) break;
            if (t > 0 &&
                cost + t * k.cost + std::max(0.0, s.need - e2) * s.minrate[c + 1] + awe_recon(s.C, S + t) >= incumbent)
                continue;
            rec(c + 1, S + t, cost + t * k.cost, e2, npl + t * k.npl, (t && !k.one) ? std::max(mxo, k.nout) : mxo);
            if (e2 >= s.need + kAweOverNeedBits) break;
        }
        n[c] = 0;
    }
};

// Pairwise coprime moduli for one count vector with bits in [need, need + tol], least excess first.
struct AweAssign {
    const AweSearch& s;
    const std::vector<int>& ord;
    std::vector<int> cnt;
    std::vector<double> ubrest, lbrest;
    std::vector<int> pick, best;
    double bestex = 1e300;
    long nodes = 0;
    void dfs(int i, int start, int left, double bits) {
        const int NC = (int)s.ks.size();
        if (++nodes > kAweNodeMax || bestex <= 1e-4) return;
        if (i == NC) {
            const double ex = bits - s.need;
            if (ex >= 0 && ex <= s.tol && ex < bestex) {
                bestex = ex;
                best = pick;
            }
            return;
        }
        if (left == 0) {
            dfs(i + 1, 0, i + 1 < NC ? cnt[i + 1] : 0, bits);
            return;
        }
        const std::vector<AweCand>& v = s.ks[ord[i]].v;
        for (int j = start; j + left <= (int)v.size(); ++j) {
            double ubc = 0;
            for (int t = 0; t < left; ++t) ubc += v[j + t].bits;
            if (bits + ubc + ubrest[i + 1] < s.need) return;
            if (bits + v[j].bits + lbrest[i + 1] > s.need + s.tol && left == 1) continue;
            bool ok = true;
            for (int x : pick)
                if (std::gcd(x, v[j].m) != 1) {
                    ok = false;
                    break;
                }
            if (!ok) continue;
            pick.push_back(v[j].m);
            dfs(i, j + 1, left - 1, bits + v[j].bits);
            pick.pop_back();
            if (nodes > kAweNodeMax || bestex <= 1e-4) return;
        }
    }
};

std::vector<int> awe_assign(const AweSearch& s, const std::vector<int>& ord, const AweVec& vec, long& nodes) {
    const int NC = (int)s.ks.size();
    AweAssign a{s, ord, std::vector<int>(NC), std::vector<double>(NC + 1, 0.0), std::vector<double>(NC + 1, 0.0),
                {}, {}};
    for (int i = 0; i < NC; ++i) a.cnt[i] = vec.n[ord[i]];
    for (int i = NC - 1; i >= 0; --i) {
        const std::vector<AweCand>& v = s.ks[ord[i]].v;
        const int t = a.cnt[i];
        double ubs = 0, lbs = 0;
        for (int j = 0; j < t && j < (int)v.size(); ++j) {
            ubs += v[j].bits;
            lbs += v[v.size() - 1 - j].bits;
        }
        a.ubrest[i] = a.ubrest[i + 1] + ubs;
        a.lbrest[i] = a.lbrest[i + 1] + lbs;
    }
    a.dfs(0, 0, NC ? a.cnt[0] : 0, 0.0);
    nodes = a.nodes;
    return a.best;
}

std::vector<int> awe_search(const AweSearch& s, double ub, bool dram, bool& dram_cut, long budget) {
    const int NC = (int)s.ks.size();
    std::vector<AweVec> vecs;
    AweEnum e{s, ub, dram, dram_cut, vecs, std::vector<int>(NC, 0)};
    e.rec(0, 0, 0.0, 0.0, 0, 0);
    std::stable_sort(vecs.begin(), vecs.end(), [](const AweVec& a, const AweVec& b) { return a.T < b.T; });
    std::vector<int> ord(NC);
    for (int c = 0; c < NC; ++c) ord[c] = c;
    std::stable_sort(ord.begin(), ord.end(), [&](int a, int b) { return s.ks[a].v.size() < s.ks[b].v.size(); });
    long spent = 0;
    for (const AweVec& vec : vecs) {
        if (budget > 0 && spent > budget) break;
        long nodes = 0;
        std::vector<int> best = awe_assign(s, ord, vec, nodes);
        spent += nodes;
        if (!best.empty()) {
            std::sort(best.begin(), best.end(), std::greater<int>());
            return best;
        }
    }
    return {};
}

// The greedy solution by cost per bit (with a look-ahead that keeps the window reachable within the
// limit) times the slack; `unbounded` when the plain greedy solution reached the window.
double awe_upper_bound(const AweSearch& s, int mod_cap, bool& unbounded) {
    double ub = 1e300;
    std::vector<std::pair<double, std::pair<int, double>>> all;
    for (const AweClass& k : s.ks)
        for (const AweCand& c : k.v) all.push_back({k.cost / c.bits, {c.m, k.cost}});
    std::stable_sort(all.begin(), all.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
    const double maxbits = std::log2((double)mod_cap);
    std::vector<int> got;
    double bits = 0, cost = 0;
    bool skipped = false;
    for (const auto& a : all) {
        if (bits >= s.need || (int)got.size() >= s.max_moduli) break;
        bool ok = true;
        for (int g : got)
            if (std::gcd(g, a.second.first) != 1) {
                ok = false;
                break;
            }
        if (!ok) continue;
        const double lb = std::log2((double)a.second.first);
        if (bits + lb + (s.max_moduli - (int)got.size() - 1) * maxbits < s.need) {
            skipped = true;
            continue;
        }
        got.push_back(a.second.first);
        bits += lb;
        cost += a.second.second;
    }
    if (bits >= s.need) ub = (cost + awe_recon(s.C, (int)got.size())) * kAweUbSlack + 1e-9;
    unbounded = bits >= s.need && !skipped;
    return ub;
}

// The moduli set (descending) of the stage-time model for the window `need`, or empty. The search is
// deterministic in its arguments and can take seconds for large K, so its results are kept for the process.
std::vector<int> awe_search_set(int awe, const Path& p, int smax, double need, double tol, int max_moduli, uint32_t M,
                                uint32_t N, double slice_tile);
std::vector<int> awe_choose(int awe, const Path& p, int smax, double need, double tol, int max_moduli, uint32_t M,
                            uint32_t N, double slice_tile) {
    struct Key {
        int awe, mod_cap, dmax, smax, max_moduli;
        bool one;
        uint32_t K, M, N;
        double need, tol, slice_tile;
        bool operator==(const Key& o) const {
            return awe == o.awe && mod_cap == o.mod_cap && dmax == o.dmax && smax == o.smax &&
                   max_moduli == o.max_moduli && one == o.one && K == o.K && M == o.M && N == o.N && need == o.need &&
                   tol == o.tol && slice_tile == o.slice_tile;
        }
    };
    static std::mutex mu;
    static std::vector<std::pair<Key, std::vector<int>>> memo;
    const Key key{awe, p.mod_cap, p.dmax, smax, max_moduli, p.one, p.K, M, N, need, tol, slice_tile};
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const auto& e : memo)
            if (e.first == key) return e.second;
    }
    std::vector<int> set = awe_search_set(awe, p, smax, need, tol, max_moduli, M, N, slice_tile);
    std::lock_guard<std::mutex> lock(mu);
    if (memo.size() >= 256) memo.erase(memo.begin());
    memo.push_back({key, set});
    return set;
}

std::vector<int> awe_search_set(int awe, const Path& p, int smax, double need, double tol, int max_moduli, uint32_t M,
                                uint32_t N, double slice_tile) {
    const uint32_t K = p.K;
    const AweCoef C = awe_coef(awe, K);
    const std::vector<AweClass> ks = awe_classes(K, C, p, smax);
    if (ks.empty()) return {};
    const int NC = (int)ks.size();
    const double Md = M, Nd = N;
    AweSearch s{ks,
                C,
                need,
                tol,
                max_moduli,
                std::vector<double>(NC + 1, 1e300),
                (Md * K + (double)K * Nd) / 1024.0 * slice_tile,
                Md * Nd * 4.0,
                (Md * K + (double)K * Nd) * 8.0};
    for (int c = NC - 1; c >= 0; --c) s.minrate[c] = std::min(s.minrate[c + 1], ks[c].cost / ks[c].v[0].bits);
    bool unbounded = false;
    const double ub = awe_upper_bound(s, p.mod_cap, unbounded);
    bool dram_cut = false;
    std::vector<int> best = awe_search(s, ub, true, dram_cut, unbounded ? 0 : kAweNodeBudget);
    if (best.empty() && dram_cut) {
        bool unused = false;
        best = awe_search(s, ub, false, unused, kAweNodeBudget);
    }
    return best;
}

// ---- moduli selection (ozaki2_choose_moduli, moduli.hpp:700-770) ---------------------------------
struct Choice {
    bool ok = false, acc_ok = true, fold_first = false, model_set = false;
    int b = 0, m_cap = 0, ncand = 0, smax = 0;
    Path path{};
    std::vector<int> m, maxg;
    std::string acc_why;  // first failed accumulation condition ("digit", "one" or "compose")
    int acc_m = 0, acc_d = 0;
    double acc_val = 0;
};

Choice choose(const Route& rt, uint32_t M, uint32_t N, uint32_t K, int num_moduli, int b_cap) {
    int mod_cap = rt.mod_cap, smax = rt.smax;
    const double wlog2 = std::log2((double)K);
    if (smax && (double)K * smax * smax + mod_cap > kTwo24) {  // FP8: dense digits for large K
        smax = 0;
        mod_cap = std::min(mod_cap, (2 * rt.dmax + 1) * (2 * rt.dmax + 1));
    }
    Choice o;
    const Path p{K, mod_cap, rt.dmax, smax, rt.one};
    o.path = p;
    o.smax = smax;
    o.m_cap = mod_cap;
    double logM = 0;
    if (rt.awe) {
        const double need_awe = 2.0 * std::min(b_cap, kMaxDigit * kDigitBits) + 1.0 + wlog2 + kWinEps;
        const std::vector<int> ms =
            awe_choose(rt.awe, p, smax, need_awe, kTailTol, std::min(num_moduli, kMaxS), M, N, rt.slice_tile);
        if (!ms.empty()) {
            for (int mm : ms) {
                o.m.push_back(mm);
                logM += std::log2((double)mm);
            }
            o.model_set = true;
        }
    }
    if (!o.model_set) {
        const int* table = smax ? kTableF8S : (rt.dmax > 16 ? kTableB8 : kTableF8);
        const int tn = smax ? (int)std::size(kTableF8S)
                            : (rt.dmax > 16 ? (int)std::size(kTableB8) : (int)std::size(kTableF8));
        for (int t = 0; t < tn; ++t) {
            const int mm = table[t];
            if ((int)o.m.size() >= num_moduli) break;
            if (mm > mod_cap || !usable(mm, p, smax)) continue;
            o.m.push_back(mm);
            logM += std::log2((double)mm);
        }
    }
    o.ncand = (int)o.m.size();
    const double room = logM - 1.0 - wlog2 - kWinEps;
    o.b = std::min(std::min((int)std::floor(room / 2.0), kMaxDigit * kDigitBits), b_cap);
    const double need = 2.0 * o.b + 1.0 + wlog2 + kWinEps;
    if (!o.model_set) {
        // trim: drop moduli from the end while the window stays covered
        while (o.m.size() > 2) {
            const double l2 = std::log2((double)o.m.back());
            if (logM - l2 < need) break;
            o.m.pop_back();
            logM -= l2;
        }
        // reselect the last two (moduli.hpp:357-453)
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
                if (usable(mm, p, smax)) {
                    use_c[mm] = 1;
                    np_c[mm] = (int)product_terms(mm, p).size();
                    lay_c[mm] =
                        1000 * (int)product_groups(mm, p, maxg_for(mm, K, mod_cap, p, smax)).size() + planes_of(mm, p);
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
    // exact FP32 accumulation of the digit products (per-plane bounds with sparse digits or one-digit
    // moduli), and the reduction of a one-digit modulus's raw GEMM output (moduli.hpp:456-495)
    int deff = rt.dmax;
    if (smax || rt.one) {
        deff = 0;
        for (int mm : o.m)
            for (int pl = 0; pl < planes_of(mm, p); ++pl) deff = std::max(deff, plane_bound(mm, pl, p, smax));
    }
    if ((double)K * deff * deff > kTwo24) fail("digit", 0, deff, (double)K * deff * deff);
    if (rt.one)
        for (int mm : o.m)
            if (split_mode(mm, p, smax) == OZTT_SPLIT_ONE) {
                const double Rb = (double)resid_bound(mm);
                if ((double)K * Rb * Rb + mm > kTwo24) fail("one", mm, (int)Rb, (double)K * Rb * Rb + mm);
            }
    // concatenation and composition (oz2_plan_concat, moduli.hpp:520-600)
    int mmax = 0;
    for (int mm : o.m) mmax = std::max(mmax, mm);
    o.maxg.assign(S, 1);
    for (int i = 0; i < S; ++i)
        if (split_mode(o.m[i], p, smax) != OZTT_SPLIT_ONE) o.maxg[i] = maxg_for(o.m[i], K, mmax, p, smax);
    auto maxg_all = [&] {
        int g = 1;
        for (int x : o.maxg) g = std::max(g, x);
        return g;
    };
    auto compose_sum = [&](int i, bool fold) {
        const int mm = o.m[i];
        double sum = 0;
        for (const Group& g : product_groups(mm, p, o.maxg[i])) {
            const double hi = (double)((g.coeff * kComposeSplit) % mm);
            sum += fold ? std::fabs((double)g.coeff) * ((double)mm / 2.0 + 2.0)
                        : std::floor(group_bound(mm, g, (double)K, p, smax) / (double)kComposeSplit + 0.5) *
                                  std::fabs(hi) +
                              (double)(kComposeSplit / 2) * std::fabs((double)g.coeff);
        }
        return sum;
    };
    for (int attempt = 0; attempt < 2; ++attempt) {
        bool can_fold = true, grouped_ok = true;
        for (int i = 0; i < S; ++i) {
            const std::vector<Group> gr = product_groups(o.m[i], p, o.maxg[i]);
            if (gr.empty()) grouped_ok = false;
            double gmax = 0;
            for (const Group& g : gr) gmax = std::max(gmax, group_bound(o.m[i], g, (double)K, p, smax));
            if (gmax + o.m[i] > kTwo24 || compose_sum(i, true) >= kTwo22) can_fold = false;
        }
        if (maxg_all() > 1 && (!can_fold || !grouped_ok)) {
            o.maxg.assign(S, 1);
            continue;
        }
        o.fold_first = can_fold;
        if (!can_fold)
            for (int i = 0; i < S; ++i)
                if (const double cs = compose_sum(i, false); cs >= kTwo22) fail("compose", o.m[i], 0, cs);
        break;
    }
    return o;
}

std::string short_cause(const Route& rt, const Choice& mo, uint32_t S_req, uint32_t M, uint32_t N, uint32_t K,
                        int b_cap, int target) {
    const uint32_t want = std::min<uint32_t>(S_req, kMaxS);
    if ((uint32_t)mo.ncand < want)
        return "Every candidate modulus is in use (" + std::to_string(mo.ncand) +
               "), so a larger Options::max_moduli does not help; use a smaller K or a different format.";
    if (want >= (uint32_t)kMaxS) return "The maximum of 24 moduli is not enough; use a smaller K or a different format.";
    Choice t;
    for (uint32_t n = S_req + 1; n <= (uint32_t)kMaxS; ++n) {
        t = choose(rt, M, N, K, (int)n, b_cap);
        if (t.ok && t.b >= target)
            return "The limit of " + std::to_string(S_req) + " moduli is too small; set Options::max_moduli to " +
                   std::to_string(n) + " or more.";
    }
    return "The limit of " + std::to_string(S_req) + " moduli is too small, and the maximum of 24 moduli still gives only " +
           std::to_string(t.ok ? t.b : 0) + " bits; use a smaller K or a different format.";
}

}  // namespace digit

int plan_digit_with(int32_t format, const std::function<PolicyStats(uint32_t, uint32_t)>& stats, uint64_t m,
                    uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits,
                    oztt_digit_plan& p, std::string& err) {
    using namespace digit;
    std::memset(&p, 0, sizeof p);
    oztt_ii_plan& base = p.base;
    const Route* rtp = route_of(format);
    if (!rtp) {
        err = "format is unknown or was not built";
        return OZTT_EINVAL;
    }
    const Route& rt = *rtp;
    p.format = format;
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
    const uint32_t S_req = max_moduli ? max_moduli : (b_fixed ? rt.def_s : (uint32_t)kMaxS);
    if (b_fixed && reconstruction == OZTT_RECON_AUTO) st = stats(base.N, base.K);
    const Choice mo = choose(rt, base.M, base.N, base.K, (int)S_req, b_cap);
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
            } else if (mo.acc_why == "one") {
                std::snprintf(buf, sizeof buf,
                              "the product of the one-digit modulus %d (digits up to %d) plus the modulus, %.0f, "
                              "exceeds 2^24",
                              mo.acc_m, mo.acc_d, mo.acc_val);
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
                  std::to_string(base.K) + ". " +
                  short_cause(rt, mo, S_req, base.M, base.N, base.K, b_cap, b_fixed ? 1 : kTargetBits);
        }
        return OZTT_ERUNTIME;
    }
    if (!b_fixed && mo.b < kTargetBits) {
        err = "Ozaki II: for the padded inner dimension K=" + std::to_string(base.K) + " the " +
              std::to_string(mo.m.size()) + " selected moduli cover a width of only " + std::to_string(mo.b) +
              " bits, below the 53 bits of FP64-equivalent accuracy. " +
              short_cause(rt, mo, S_req, base.M, base.N, base.K, b_cap, kTargetBits);
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
    const Path& pa = mo.path;
    p.fold_first = mo.fold_first ? 1 : 0;
    int plane = 0, out = 0;
    for (int i = 0; i < (int)mo.m.size(); ++i) {
        const int mm = mo.m[i];
        p.q[i] = radix_of(mm, pa);
        p.mode[i] = split_mode(mm, pa, mo.smax);
        p.poff[i] = plane;
        p.npl[i] = planes_of(mm, pa);
        p.oout[i] = out;
        p.nprod += (int32_t)product_terms(mm, pa).size();
        for (const Group& g : product_groups(mm, pa, mo.maxg[i])) {
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

int plan_digit(int32_t format, const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
               uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_digit_plan& p,
               std::string& err) {
    return plan_digit_with(
        format, [&](uint32_t N, uint32_t K) { return measure_policy_stats(a, b, m, n, k, N, K); }, m, n, k, max_moduli,
        reconstruction, fixed_bits, p, err);
}

}  // namespace oztt

extern "C" int oztt_ii_digit_plan(int32_t format, const double* a, const double* b, uint64_t m, uint64_t n,
                                  uint64_t k, uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits,
                                  oztt_digit_plan* plan, char* err, size_t errlen) {
    std::string msg;
    int rc;
    try {
        if (!plan || (fixed_bits <= 0 && (!a || !b))) {
            msg = "null argument";
            rc = OZTT_EINVAL;
        } else {
            rc = oztt::plan_digit(format, a, b, m, n, k, max_moduli, reconstruction, fixed_bits, *plan, msg);
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
