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
#include <map>
#include <mutex>
#include <numeric>
#include <string>
#include <tuple>
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

// The model search chooses the moduli of the BF16 and FP16 routes (awe.hpp, oz2_awe_choose): the set whose
// modelled stage time is least among those covering the CRT window. Its decisions are the reference's, so
// the specification below fixes not only what is minimised but also the traversal orders and cutoffs that
// decide which set comes out when several cost the same or a cutoff is reached.
//
//  1. Families. Every usable modulus, taken from mod_cap down to 2, whose GEMM outputs stay exact binary32
//     integers (largest group bound + mod_cap <= 2^24) and whose composition sum sum|c| (m/2 + 2) stays
//     below 2^22, joins the family of moduli with the same (products, outputs, digit planes, slicer
//     operations, one-digit) signature; the signature fixes the family's modelled cost per modulus. A
//     family keeps its members in descending order; reach[t] is the number of bits of its first t members
//     that are pairwise coprime, taken greedily in that order. Families are ranked by cost per bit of their
//     largest member (ties: by cost).
//  2. Bound. All members of all families, in ascending cost per bit (stable: family rank, then member
//     order), are taken greedily when coprime to those taken, until the window is covered or the slots are
//     used up; a member whose bits, with every remaining slot holding log2(mod_cap) bits, could no longer
//     cover the window is passed over. If the window is covered the bound is 1.05 (cost + reconstruction)
//     + 1e-9, with no total budget for the assignments when nothing was passed over; else there is no bound.
//  3. Count vectors. Depth first over the families in rank order, the count of a family rising from 0 to
//     the smaller of its reach table's length - 1 and the slots left. A complete vector is kept when its reach
//     covers the window, it has a modulus, and its time (cost + reconstruction) is below the bound -- unless
//     the DRAM condition applies and fails, which drops it and records the drop. A family is not entered
//     when the cost so far plus the cheapest completion (missing bits x the least cost per bit of this and
//     later families) reaches the bound; its counting stops at the first count whose cost + reconstruction
//     reaches the bound, and after a count whose reach is 16 bits past the window; a count above zero is
//     passed over when its cost plus the cheapest completion by later families reaches the bound. At most
//     200000 vectors are kept; they are tried in ascending time (ties in the order kept).
//  4. Assignment of one vector. Families in ascending member count (ties: rank). A family's members are
//     chosen as ascending index combinations, each member coprime to all chosen before it. Trying index j
//     with `left` members still to choose: if the bits so far, the next `left` members from j and the most
//     the later families can add fall short of the window, no later index can do better (members descend)
//     and the choices at this depth end; for the family's last member, one whose bits and the least the
//     later families add overshoot the window by more than tol is passed over. A complete choice with an
//     excess over the window in [0, tol], below the best so far, becomes the best. Every state -- a member
//     chosen, the move to the next family, a complete choice, and the start -- counts one; the assignment
//     stops once more than 400000 states were counted or an excess of at most 1e-4 was found.
//  5. The first vector, in order, that has an assignment gives the set (sorted descending); with a total
//     budget, no further vector is started once the states counted exceed it. If no set was found and the
//     DRAM condition dropped some vector, the search runs again without the condition, with the budget 10^7.
struct ModelFamily {
    int nprod, nout, npl, ops;
    bool one;
    double cost;                // modelled cost of one member
    std::vector<int> members;   // descending
    std::vector<double> bits;   // log2 of each member
    std::vector<double> reach;  // reach[t]: bits of the first t pairwise coprime members
};

bool coprime_to_all(const std::vector<int>& set, int m) {
    return std::all_of(set.begin(), set.end(), [m](int x) { return std::gcd(x, m) == 1; });
}

std::vector<ModelFamily> model_families(uint32_t K, const AweCoef& C, const Path& p, int smax) {
    std::vector<ModelFamily> fam;
    const int mod_cap = p.mod_cap;
    for (int m = mod_cap; m >= 2; --m) {
        if (!usable(m, p, smax)) continue;
        const std::vector<Group> gr = product_groups(m, p, maxg_for(m, K, mod_cap, p, smax));
        if (gr.empty()) continue;
        double coeff_sum = 0, worst = 0;
        for (const Group& g : gr) {
            coeff_sum += std::fabs((double)g.coeff);
            worst = std::max(worst, group_bound(m, g, (double)K, p, smax));
        }
        if (worst + mod_cap > kTwo24 || coeff_sum * (m / 2.0 + 2.0) >= kTwo22) continue;
        const int nprod = (int)product_terms(m, p).size(), nout = (int)gr.size(), npl = planes_of(m, p);
        const int ops = awe_ops(m, p, smax);
        const bool one = split_mode(m, p, smax) == OZTT_SPLIT_ONE;
        auto same = [&](const ModelFamily& f) {
            return f.nprod == nprod && f.nout == nout && f.npl == npl && f.ops == ops && f.one == one;
        };
        auto it = std::find_if(fam.begin(), fam.end(), same);
        if (it == fam.end()) {
            // GEMM products and outputs, the composition, the slicer's operations and planes (summed in
            // this order: the costs are compared exactly); a one-digit modulus skips the composition and
            // costs one more ModRound in the reconstruction instead
            const double cost = one ? C.gp * nprod + C.go * nout + C.sop * (19 + ops) + C.spl * npl + kAweOneRecon * C.rb
                                    : C.gp * nprod + (C.go + C.co) * nout + C.cs + C.sop * (19 + ops) + C.spl * npl;
            fam.push_back({nprod, nout, npl, ops, one, cost, {}, {}, {}});
            it = fam.end() - 1;
        }
        it->members.push_back(m);
        it->bits.push_back(std::log2((double)m));
    }
    for (ModelFamily& f : fam) {
        std::vector<int> taken;
        f.reach.assign(1, 0.0);
        for (size_t j = 0; j < f.members.size(); ++j)
            if (coprime_to_all(taken, f.members[j])) {
                taken.push_back(f.members[j]);
                f.reach.push_back(f.reach.back() + f.bits[j]);
            }
    }
    std::sort(fam.begin(), fam.end(), [](const ModelFamily& x, const ModelFamily& y) {
        const double rx = x.cost / x.bits[0], ry = y.cost / y.bits[0];
        if (rx != ry) return rx < ry;
        return x.cost < y.cost;
    });
    return fam;
}

// The search's fixed data: the families, the window `need` and tolerance, the slots (max_moduli), the least
// cost per bit from each family on, and the byte counts of the DRAM estimate.
struct ModelProblem {
    std::vector<ModelFamily> fam;
    AweCoef C;
    double need, tol;
    int slots;
    std::vector<double> cheapest;  // cheapest[f]: least cost per bit among families f.. (1e300 past the end)
    double plane_bytes, out_bytes, free_bytes;
    double recon(int S) const { return awe_recon(C, S); }
    // S moduli with npl digit planes (largest composed output count mxo, 0: none) fit the model's free DRAM
    // without output bands.
    bool fits_dram(int S, int npl, int mxo) const {
        const double q = (compose_planes(mxo > 0, (uint32_t)mxo) + S) * out_bytes;
        return npl * plane_bytes + std::max(0.0, q - free_bytes) + kDramMargin <= kAweDramFree;
    }
};

struct CountVector {
    double time;
    std::vector<int> n;
};

// Step 3: the count vectors under `bound`; returns whether the DRAM condition dropped one.
bool count_vectors(const ModelProblem& P, double bound, bool dram, std::vector<CountVector>& kept) {
    const int F = (int)P.fam.size();
    struct Level {
        int t = -1, tmax = 0, S = 0, npl = 0, mxo = 0;
        double cost = 0, reach = 0;
        bool visited = false;  // the current count t was descended into
    };
    std::vector<Level> path;
    std::vector<int> n(F, 0);
    bool dropped = false, full = false;
    // Visits the node of family f (f == F: a complete vector); pushes a level when family f's counts are
    // to be tried.
    auto visit = [&](int f, int S, double cost, double reach, int npl, int mxo) {
        if (kept.size() >= kAweVecMax) {
            full = true;
            return;
        }
        if (f == F) {
            if (reach < P.need || S == 0) return;
            const double T = cost + P.recon(S);
            if (T >= bound) return;
            if (dram && !P.fits_dram(S, npl, mxo))
                dropped = true;
            else
                kept.push_back({T, n});
            return;
        }
        if (cost + std::max(0.0, P.need - reach) * P.cheapest[f] + P.recon(S) >= bound) return;
        Level lv;
        lv.tmax = std::min((int)P.fam[f].reach.size() - 1, P.slots - S);
        lv.S = S;
        lv.npl = npl;
        lv.mxo = mxo;
        lv.cost = cost;
        lv.reach = reach;
        path.push_back(lv);
    };
    visit(0, 0, 0.0, 0.0, 0, 0);
    while (!path.empty() && !full) {
        const int f = (int)path.size() - 1;
        const ModelFamily& g = P.fam[f];
        Level& lv = path.back();
        if (lv.visited && lv.reach + g.reach[lv.t] >= P.need + kAweOverNeedBits) lv.t = lv.tmax;  // counting ends
        lv.visited = false;
        if (++lv.t > lv.tmax) {
            n[f] = 0;
            path.pop_back();
            continue;
        }
        const int t = lv.t;
        n[f] = t;
        const double cost = lv.cost + t * g.cost, reach = lv.reach + g.reach[t];
        if (cost + P.recon(lv.S + t) >= bound) {
            lv.t = lv.tmax;  // no larger count can be cheaper
            continue;
        }
        if (t > 0 && cost + std::max(0.0, P.need - reach) * P.cheapest[f + 1] + P.recon(lv.S + t) >= bound) continue;
        lv.visited = true;
        const Level at = lv;  // visit() may grow `path`
        visit(f + 1, at.S + t, cost, reach, at.npl + t * g.npl, (t && !g.one) ? std::max(at.mxo, g.nout) : at.mxo);
    }
    return dropped;
}

// Step 4: the moduli for one count vector (empty if none); `states` receives the states counted.
std::vector<int> assign_moduli(const ModelProblem& P, const std::vector<int>& order, const std::vector<int>& counts,
                               long& states) {
    const int F = (int)P.fam.size();
    std::vector<int> want(F);
    std::vector<double> most(F + 1, 0.0), least(F + 1, 0.0);  // bits the families at positions i.. can add
    for (int i = 0; i < F; ++i) want[i] = counts[order[i]];
    for (int i = F - 1; i >= 0; --i) {
        const std::vector<double>& b = P.fam[order[i]].bits;
        const int use = std::min<int>(want[i], (int)b.size());
        double hi = 0, lo = 0;
        for (int j = 0; j < use; ++j) {
            hi += b[j];
            lo += b[b.size() - 1 - j];
        }
        most[i] = most[i + 1] + hi;
        least[i] = least[i + 1] + lo;
    }
    struct Choosing {
        int pos, next, left;
        double bits;
        bool rooted;  // entered by choosing a member (every frame but the first)
    };
    std::vector<Choosing> frames;
    std::vector<int> chosen, best;
    double best_excess = 1e300;
    bool stop = false;
    states = 0;
    auto finished = [&] { return states > kAweNodeMax || best_excess <= 1e-4; };
    // Enters a state: counts it, evaluates a complete choice, passes through family moves, and pushes a
    // frame when members are to be chosen.
    auto enter = [&](int pos, int next, int left, double bits, bool rooted) {
        for (;;) {
            ++states;
            if (finished()) {
                stop = true;
                return;
            }
            if (pos == F) {
                const double excess = bits - P.need;
                if (excess >= 0 && excess <= P.tol && excess < best_excess) {
                    best_excess = excess;
                    best = chosen;
                }
                return;
            }
            if (left > 0) break;
            ++pos;  // the move to the next family is a state of its own
            next = 0;
            left = pos < F ? want[pos] : 0;
        }
        frames.push_back({pos, next, left, bits, rooted});
    };
    enter(0, 0, F ? want[0] : 0, 0.0, false);
    while (!stop && !frames.empty()) {
        Choosing& fr = frames.back();
        const ModelFamily& g = P.fam[order[fr.pos]];
        const int size = (int)g.members.size();
        bool pushed = false;
        while (!stop && fr.next + fr.left <= size) {
            const int j = fr.next++;
            double upper = 0;
            for (int t = 0; t < fr.left; ++t) upper += g.bits[j + t];
            if (fr.bits + upper + most[fr.pos + 1] < P.need) {
                fr.next = size;  // nothing from j on can reach the window
                break;
            }
            if (fr.left == 1 && fr.bits + g.bits[j] + least[fr.pos + 1] > P.need + P.tol) continue;
            if (!coprime_to_all(chosen, g.members[j])) continue;
            chosen.push_back(g.members[j]);
            const Choosing here = fr;  // enter() may grow `frames`
            const size_t depth = frames.size();
            enter(here.pos, j + 1, here.left - 1, here.bits + g.bits[j], true);
            if (stop) break;
            if (frames.size() > depth) {
                pushed = true;
                break;
            }
            chosen.pop_back();
            if (finished()) stop = true;
        }
        if (stop || pushed) continue;
        const bool rooted = frames.back().rooted;
        frames.pop_back();
        if (rooted) {
            chosen.pop_back();
            if (finished()) stop = true;
        }
    }
    return best;
}

// Step 5 for one bound: the first assignable vector's moduli, descending (empty if none).
std::vector<int> model_search(const ModelProblem& P, double bound, bool dram, bool& dropped, long budget) {
    std::vector<CountVector> vecs;
    dropped = count_vectors(P, bound, dram, vecs) || dropped;
    std::stable_sort(vecs.begin(), vecs.end(), [](const CountVector& x, const CountVector& y) { return x.time < y.time; });
    std::vector<int> order(P.fam.size());
    for (size_t f = 0; f < order.size(); ++f) order[f] = (int)f;
    std::stable_sort(order.begin(), order.end(),
                     [&](int x, int y) { return P.fam[x].members.size() < P.fam[y].members.size(); });
    long spent = 0;
    for (const CountVector& v : vecs) {
        if (budget > 0 && spent > budget) break;
        long states = 0;
        std::vector<int> set = assign_moduli(P, order, v.n, states);
        spent += states;
        if (!set.empty()) {
            std::sort(set.begin(), set.end(), std::greater<int>());
            return set;
        }
    }
    return {};
}

// Step 2: the cost bound; `unbounded` when the plain greedy set covered the window.
double model_bound(const ModelProblem& P, int mod_cap, bool& unbounded) {
    struct Item {
        double rate, cost;
        int m;
    };
    std::vector<Item> items;
    for (const ModelFamily& f : P.fam)
        for (size_t j = 0; j < f.members.size(); ++j) items.push_back({f.cost / f.bits[j], f.cost, f.members[j]});
    std::stable_sort(items.begin(), items.end(), [](const Item& x, const Item& y) { return x.rate < y.rate; });
    const double widest = std::log2((double)mod_cap);
    std::vector<int> taken;
    double bits = 0, cost = 0;
    bool passed_over = false;
    for (const Item& it : items) {
        if (bits >= P.need || (int)taken.size() >= P.slots) break;
        if (!coprime_to_all(taken, it.m)) continue;
        const double b = std::log2((double)it.m);
        const int open_slots = P.slots - (int)taken.size() - 1;
        if (bits + b + open_slots * widest < P.need) {
            passed_over = true;
            continue;
        }
        taken.push_back(it.m);
        bits += b;
        cost += it.cost;
    }
    unbounded = bits >= P.need && !passed_over;
    return bits >= P.need ? (cost + P.recon((int)taken.size())) * kAweUbSlack + 1e-9 : 1e300;
}

std::vector<int> model_set_uncached(int awe, const Path& p, int smax, double need, double tol, int max_moduli, uint32_t M,
                                    uint32_t N, double slice_tile) {
    const uint32_t K = p.K;
    ModelProblem P;
    P.C = awe_coef(awe, K);
    P.fam = model_families(K, P.C, p, smax);
    if (P.fam.empty()) return {};
    P.need = need;
    P.tol = tol;
    P.slots = max_moduli;
    const int F = (int)P.fam.size();
    P.cheapest.assign(F + 1, 1e300);
    for (int f = F - 1; f >= 0; --f) P.cheapest[f] = std::min(P.cheapest[f + 1], P.fam[f].cost / P.fam[f].bits[0]);
    const double operand_elems = (double)M * K + (double)K * N;
    P.plane_bytes = operand_elems / 1024.0 * slice_tile;
    P.out_bytes = (double)M * N * 4.0;
    P.free_bytes = operand_elems * 8.0;
    bool unbounded = false;
    const double bound = model_bound(P, p.mod_cap, unbounded);
    bool dropped = false;
    std::vector<int> set = model_search(P, bound, true, dropped, unbounded ? 0 : kAweNodeBudget);
    if (set.empty() && dropped) {
        bool ignored = false;
        set = model_search(P, bound, false, ignored, kAweNodeBudget);
    }
    return set;
}

// The model's moduli set (descending) for the window `need`, or empty. The search is deterministic in its
// arguments and can take seconds for large K, so its results are kept for the process.
std::vector<int> awe_choose(int awe, const Path& p, int smax, double need, double tol, int max_moduli, uint32_t M,
                            uint32_t N, double slice_tile) {
    using Key = std::tuple<int, int, int, int, int, bool, uint32_t, uint32_t, uint32_t, double, double, double>;
    static std::mutex mu;
    static std::map<Key, std::vector<int>> memo;
    const Key key{awe, p.mod_cap, p.dmax, smax, max_moduli, p.one, p.K, M, N, need, tol, slice_tile};
    {
        std::lock_guard<std::mutex> lock(mu);
        const auto it = memo.find(key);
        if (it != memo.end()) return it->second;
    }
    std::vector<int> set = model_set_uncached(awe, p, smax, need, tol, max_moduli, M, N, slice_tile);
    std::lock_guard<std::mutex> lock(mu);
    if (memo.size() >= 256) memo.clear();
    memo.emplace(key, set);
    return set;
}

// Tail reselection (oz2_reselect_tail, moduli.hpp:365-451). The table's moduli step by several bits, so
// the last two of a set often overshoot the window; the excess buys no accuracy (the reconstruction solves
// C'/M to a fixed absolute accuracy) but costs products. Specification: keep the head (all but the last two
// moduli) and choose, as the new tail, one modulus a or a pair a < b -- usable, at most mod_cap, coprime to
// the head and to each other -- whose product with the head covers the window, minimising the key
//   (matrix products of the tail, 1 if the excess exceeds kTailTol, 1000 x GEMM outputs + digit planes of
//    the tail, log2 of the whole set)
// lexicographically. The current tail is the starting incumbent and only a strictly smaller key replaces
// it; candidates are met in the order a = 3, 4, ... (only odd a and b when the head has an even member),
// a alone before the pairs (a, b) with b ascending, so among equal keys the first met wins.
void reselect_tail(std::vector<int>& m, double& logM, double need, const Path& p, int smax, int mod_cap, uint32_t K) {
    if (m.size() < 2 || !(logM > need)) return;
    const std::vector<int> head(m.begin(), m.end() - 2);
    double base = 0;
    for (int x : head) base += std::log2((double)x);
    // per-modulus products and layout cost; `open`: usable and coprime to the head
    std::vector<int> products(mod_cap + 1, 0), layout(mod_cap + 1, 0);
    std::vector<char> open(mod_cap + 1, 0);
    for (int x = 3; x <= mod_cap; ++x)
        if (usable(x, p, smax)) {
            products[x] = (int)product_terms(x, p).size();
            layout[x] = 1000 * (int)product_groups(x, p, maxg_for(x, K, mod_cap, p, smax)).size() + planes_of(x, p);
            open[x] = coprime_to_all(head, x);
        }
    struct Key {
        int products, over, layout;
        double log2m;
        bool operator<(const Key& o) const {
            return std::tie(products, over, layout, log2m) < std::tie(o.products, o.over, o.layout, o.log2m);
        }
    };
    auto key = [&](int nprod, int lay, double l) { return Key{nprod, (l - need) > kTailTol ? 1 : 0, lay, l}; };
    auto cost_of = [&](int x) { return x >= 0 && x <= mod_cap ? products[x] : 0; };
    auto layout_of = [&](int x) { return x >= 0 && x <= mod_cap ? layout[x] : 0; };
    int ta = m[m.size() - 2], tb = m.back();
    Key best = key(cost_of(ta) + cost_of(tb), layout_of(ta) + layout_of(tb), logM);
    const bool head_even = std::any_of(head.begin(), head.end(), [](int x) { return x % 2 == 0; });
    const int step = head_even ? 2 : 1;
    for (int a = 3; a <= mod_cap; a += step) {
        if (!open[a]) continue;
        const double la = base + std::log2((double)a);
        if (la >= need) {
            const Key k = key(products[a], layout[a], la);
            if (k < best) {
                best = k;
                ta = a;
                tb = 0;
            }
        }
        for (int b = a + step; b <= mod_cap; b += step) {
            if (!open[b] || std::gcd(a, b) != 1) continue;
            const double lab = la + std::log2((double)b);
            if (lab < need) continue;
            const Key k = key(products[a] + products[b], layout[a] + layout[b], lab);
            if (k < best) {
                best = k;
                ta = a;
                tb = b;
            }
        }
    }
    m = head;
    m.push_back(ta);
    if (tb) m.push_back(tb);
    logM = best.log2m;
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
        reselect_tail(o.m, logM, need, p, smax, mod_cap, K);
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
