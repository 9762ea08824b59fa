// TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT (see oz2_oracle.h).
//
// CPU restatement of ozTTgemm's Ozaki-II INT8 path. Build with -ffp-contract=off and without
// fast-math: every FP32 step below is one IEEE binary32 operation rounded to nearest even, with
// the flush-to-zero rules of the reference's SFPU model (experiments/src/checks/sfpu_tf_emu.hpp:64-83).
#include "oz2_oracle.h"

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <numeric>
#include <quadmath.h>
#include <random>
#include <string>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

static_assert(LDBL_MANT_DIG == 64, "the oracle needs the x86 80-bit long double of the reference host code");

namespace {

// ---------------------------------------------------------------------------------------------
// One SFPU tile operation (sfpu_tf_emu.hpp:64-83): binary32 round-to-nearest-even, subnormal
// inputs and outputs flushed to signed zero, a product with a zero operand is +0, Rnd is
// round-half-even with a zero result returned as +0.
// ---------------------------------------------------------------------------------------------
inline float flush(float x) { return (x != 0.0f && std::fabs(x) < FLT_MIN) ? std::copysign(0.0f, x) : x; }
inline float fadd(float a, float b) { return flush(flush(a) + flush(b)); }
inline float fsub(float a, float b) { return flush(flush(a) - flush(b)); }
inline float fmul(float a, float b) {
    a = flush(a);
    b = flush(b);
    if (a == 0.0f || b == 0.0f) return 0.0f;
    return flush(a * b);
}
inline float frnd(float v) {
    v = flush(v);
    const float mag = std::fabs(v);
    if (!(mag < 8388608.0f)) return v;
    const float t = (mag + 8388608.0f) - 8388608.0f;
    return t == 0.0f ? 0.0f : std::copysign(t, v);
}
inline float bits_to_f(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
inline uint32_t f_to_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
inline uint64_t d_to_bits(double d) {
    uint64_t u;
    std::memcpy(&u, &d, 8);
    return u;
}

// Knuth TwoSum as the reference orders it (sfpu_tf_proc.h:61-64).
inline void two_sum(float x, float y, float& s, float& e) {
    s = fadd(x, y);
    const float bb = fsub(s, x);
    const float a = fsub(x, fsub(s, bb));
    e = fadd(a, fsub(y, bb));
}
// Dekker FastTwoSum (sfpu_tf_proc.h:71-74).
inline void fast_two_sum(float a, float b, float& s, float& t) {
    s = fadd(a, b);
    t = fsub(b, fsub(s, a));
}

// Triple-float times a power of two (tfMulP2, sfpu_tf_proc.h:160-169).
inline void tf_mul_p2(float& x0, float& x1, float& x2, float r) {
    x0 = fmul(x0, r);
    x1 = fmul(x1, r);
    x2 = fmul(x2, r);
    float s3, e4, s5, e6;
    two_sum(x1, x2, s3, e4);
    two_sum(x0, s3, s5, e6);
    x0 = s5;
    fast_two_sum(e6, e4, x1, x2);
}

// ModRound: d - Rnd(d*rinv)*m (sfpu_tf_proc.h:316-319).
inline float mod_round(float d, float m, float rinv) { return fsub(d, fmul(frnd(fmul(d, rinv)), m)); }

// Triple-float accumulation of one scalar (tfAddS<3>, sfpu_tf_proc.h:184-198).
inline void tf_add(float& a0, float& a1, float& a2, float v) {
    float s, e;
    two_sum(a0, v, s, e);
    a0 = s;
    float s2, e2;
    two_sum(a1, e, s2, e2);
    a1 = s2;
    a2 = fadd(a2, e2);
}
// Small-term accumulation (tfAddSmall<3>, sfpu_tf_proc.h:237-258).
inline void tf_add_small(float& a1, float& a2, float v) {
    float s, e;
    two_sum(a1, v, s, e);
    a1 = s;
    a2 = fadd(a2, e);
}

// ---------------------------------------------------------------------------------------------
// FP64 -> triple-float bit split (split_f64, f64_tf.h:141-168) and the SFPU assembly
// (tf_load_f64, slice_tf_core.h:67-75).
// ---------------------------------------------------------------------------------------------
void split_f64(uint64_t bits, int32_t d, uint32_t& hi, uint32_t& braw, uint32_t& craw, uint32_t& s) {
    const uint32_t w1 = (uint32_t)(bits >> 32), w0 = (uint32_t)bits;
    const uint32_t sgn = w1 & 0x80000000u;
    const int32_t E = (int32_t)((w1 >> 20) & 0x7FFu);
    if (E == 0) {
        hi = 0u;
        braw = craw = 0x4B000000u;
        s = 0u;
        return;
    }
    // 53-bit significand split 30/23/7 with the top part rounded to nearest (ties up).
    uint32_t top = 0x400000u | ((w1 & 0xFFFFFu) << 2) | (w0 >> 30);
    const uint32_t low30 = w0 & 0x3FFFFFFFu;
    int32_t rest = (int32_t)low30;
    if (low30 >= 0x20000000u) {
        top += 1u;
        rest = (int32_t)low30 - 0x40000000;
    }
    const int32_t mid = rest >> 7;           // [-2^22, 2^22)
    const uint32_t lo = (uint32_t)rest & 0x7Fu;
    const int32_t elsb = E - 1075 + d;      // exponent of the significand's last bit
    int32_t eh;
    uint32_t mh;
    if (top == 0x800000u) {
        eh = elsb + 180;
        mh = 0u;
    } else {
        eh = elsb + 179;
        mh = (top << 1) & 0x7FFFFFu;
    }
    const int32_t es = elsb + 134;
    hi = (eh > 0 && eh < 255) ? (sgn | ((uint32_t)eh << 23) | mh) : 0u;
    s = (es > 0 && es < 255) ? (sgn | ((uint32_t)es << 23)) : 0u;
    braw = 0x4B000000u | ((uint32_t)(mid + 0x400000) & 0x7FFFFFu);
    craw = 0x4B000000u | lo;
}

void tf_load(double x, int32_t d, float& x0, float& x1, float& x2) {
    uint32_t hi, braw, craw, s;
    split_f64(d_to_bits(x), d, hi, braw, craw, s);
    const float sc = bits_to_f(s);
    x0 = bits_to_f(hi);
    x1 = fmul(fadd(bits_to_f(braw), -12582912.0f), sc);
    x2 = fmul(fmul(fadd(bits_to_f(craw), -8388608.0f), sc), 0.0078125f);
}

// The nd radix-2^20 digits of A' (oz2_make_digits, digits.h:80-108); out[0] = d_{nd-1} (made first).
void make_digits(double x, int32_t d, int nd, float* out) {
    float x0, x1, x2;
    tf_load(x, d, x0, x1, x2);
    for (int i = 0; i < nd; ++i) {
        if (i > 0) tf_mul_p2(x0, x1, x2, 1048576.0f);
        const float dig = frnd(x0);
        out[i] = dig;
        x0 = fsub(x0, dig);
    }
}

// Residue of A' from its digits (oz2_residue, digits.h:165-179). dg[0] is the top digit.
float residue(const float* dg, int nd, float m, float rinv, const float* c) {
    const float d0 = dg[nd - 1], d1 = dg[nd - 2], d2 = dg[nd - 3];
    float acc = fadd(d0, fmul(mod_round(d1, m, rinv), c[0]));
    acc = fadd(acc, fmul(mod_round(d2, m, rinv), c[1]));
    if (nd >= 4) {
        acc = mod_round(acc, m, rinv);
        if (nd >= 5) {
            acc = fadd(acc, fmul(mod_round(dg[0], m, rinv), c[3]));
            acc = mod_round(acc, m, rinv);
        }
        acc = fadd(acc, fmul(mod_round(dg[nd - 4], m, rinv), c[2]));
    }
    return mod_round(acc, m, rinv);
}

// |x| of an FP64 pattern (sign cleared) -> BF16 rounded up (ceil 1) or truncated (ceil 0)
// (oz_absf64_to_bf16<CEIL>, scale_bits.h:33-44).
uint16_t abs_to_bf16(uint64_t mag, int ceil) {
    const uint32_t h = (uint32_t)(mag >> 32), l = (uint32_t)mag;
    const int32_t E = (int32_t)((h >> 20) & 0x7FFu);
    if (E == 0x7FF) return 0xFFC0u;
    const int32_t e8 = E - 896;
    if (e8 <= 0) return (h | l) ? 0xFF80u : 0u;
    if (e8 >= 255) return 0x7F80u;
    uint32_t v = ((uint32_t)e8 << 7) | ((h >> 13) & 0x7Fu);
    if (ceil == 1 && ((h & 0x1FFFu) || l)) v += 1u;
    return (uint16_t)v;
}
// e = ceil(log2 u) of the BF16 maximum with the out-of-range flags (oz_bf16_scale_exp, scale_bits.h:56-63).
int32_t bf16_scale_exp(uint16_t u, uint32_t& flags) {
    const uint32_t E = (u >> 7) & 0xFFu, mant = u & 0x7Fu;
    if (E == 0u) return 0;
    if (E == 0xFFu) {
        flags |= !(u & 0x8000u) ? 1u : (mant ? 4u : 2u);
        return 0;
    }
    return (int32_t)E - 127 + (mant ? 1 : 0);
}

// ---------------------------------------------------------------------------------------------
// Scheme II INT8 planner (moduli.hpp, plan.hpp, auto_precision.hpp, norm_estimate.hpp).
// ---------------------------------------------------------------------------------------------
constexpr int MAXS = 24;
constexpr int DIGIT_BITS = 20;
constexpr int MAXDIGIT = 5;
constexpr int TARGET_BITS = 53;
constexpr int B_DEFAULT = 54;
constexpr int ACC_BITS = 31;
constexpr double WIN_EPS = 1e-9;
constexpr double TAIL_EXCESS_TOL = 0.25;
constexpr int RGRAN = 64;
constexpr double RECON1_EPS_LOG2 = -70.0;
constexpr double RECON1_THR_LOG2 = -(TARGET_BITS + 2.0);
constexpr uint32_t DEF_S_INT8 = 16;  // OZ2_ROUTE_INT8.def_s (split.hpp:75)
// INT8 candidate table (moduli.hpp:180-182).
constexpr int TABLE_I8[] = {255, 254, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217,
                            211, 199, 197, 193, 191, 181, 179, 173, 167, 163, 157, 151};
constexpr int TABLE_I8_MIN = 151;

bool int8_fits(uint32_t K, int m) {
    const unsigned __int128 r = (unsigned)(m / 2);
    return (unsigned __int128)K * r * r <= (((unsigned __int128)1 << ACC_BITS) - 1);
}
long int8_rmax(uint32_t K) {
    const unsigned __int128 lim = ((unsigned __int128)1 << ACC_BITS) - 1;
    long r = (long)std::floor(std::sqrt((double)lim / (double)K));
    while (r > 0 && (unsigned __int128)K * r * r > lim) --r;
    while ((unsigned __int128)K * (r + 1) * (r + 1) <= lim) ++r;
    return r;
}
long inv_mod(long a, long mod) {
    long t = 0, nt = 1, r = mod, nr = a % mod;
    while (nr != 0) {
        const long q = r / nr;
        long tmp = t - q * nt;
        t = nt;
        nt = tmp;
        tmp = r - q * nr;
        r = nr;
        nr = tmp;
    }
    if (t < 0) t += mod;
    return t;
}

struct Moduli {
    bool ok = false, acc_ok = true;
    int m_cap = 0, ncand = 0, b = 23;
    std::vector<int> m;
    double logM = 0;
};

// ozaki2_choose_moduli for the INT8 route (moduli.hpp:719-769 with the steps at :255-451).
Moduli choose_moduli(uint32_t K, int num_moduli, int b_cap) {
    Moduli o;
    const double Wlog2 = std::log2((double)K);
    const int m_cap = (int)std::min<long>(255, 2 * int8_rmax(K) + 1);
    double logM = 0.0;
    for (int mm : TABLE_I8) {
        if ((int)o.m.size() >= num_moduli) break;
        if (mm > m_cap) continue;
        o.m.push_back(mm);
        logM += std::log2((double)mm);
    }
    const int want = std::min(num_moduli, MAXS);
    for (int mm = std::min(m_cap, TABLE_I8_MIN - 1); mm >= 3 && (int)o.m.size() < want; --mm) {
        bool cop = true;
        for (int x : o.m)
            if (std::gcd(x, mm) != 1) {
                cop = false;
                break;
            }
        if (!cop) continue;
        o.m.push_back(mm);
        logM += std::log2((double)mm);
    }
    o.m_cap = m_cap;
    o.ncand = (int)o.m.size();
    // Width from the window (moduli.hpp:338-342).
    {
        const double room = logM - 1.0 - Wlog2 - WIN_EPS;
        const int b_win = (int)std::floor(room / 2.0);
        o.b = std::min(std::min(b_win, MAXDIGIT * DIGIT_BITS), b_cap);
    }
    const int b = o.b;
    const double need = 2.0 * b + 1.0 + Wlog2 + WIN_EPS;
    // Drop surplus moduli from the end (oz2_trim_tail, moduli.hpp:347-354).
    while (o.m.size() > 2) {
        const double l2 = std::log2((double)o.m.back());
        if (logM - l2 < need) break;
        o.m.pop_back();
        logM -= l2;
    }
    // Reselect the last two (oz2_reselect_tail, moduli.hpp:365-451); every INT8 modulus is one
    // product and has no layout cost.
    if (o.m.size() >= 2 && logM > need) {
        std::vector<int> head(o.m.begin(), o.m.end() - 2);
        double base = 0.0;
        for (int x : head) base += std::log2((double)x);
        auto cop_head = [&](int mm) {
            for (int x : head)
                if (std::gcd(mm, x) != 1) return false;
            return true;
        };
        double best = logM;
        int bp = o.m[o.m.size() - 2], bq = o.m.back();
        int bcost = 2;
        auto over = [&](double l) { return (l - need) > TAIL_EXCESS_TOL ? 1 : 0; };
        auto better = [&](int c, double l) {
            if (c != bcost) return c < bcost;
            if (over(l) != over(best)) return over(l) < over(best);
            return l < best;
        };
        bool head_even = false;
        for (int x : head) head_even = head_even || (x % 2 == 0);
        const int step = head_even ? 2 : 1;
        for (int p = 3; p <= m_cap; p += step) {
            if (!cop_head(p)) continue;
            const double lp = base + std::log2((double)p);
            if (lp >= need && better(1, lp)) {
                best = lp;
                bp = p;
                bq = 0;
                bcost = 1;
            }
            for (int q = p + step; q <= m_cap; q += step) {
                if (std::gcd(p, q) != 1 || !cop_head(q)) continue;
                const double lq = lp + std::log2((double)q);
                if (lq >= need && better(2, lq)) {
                    best = lq;
                    bp = p;
                    bq = q;
                    bcost = 2;
                }
            }
        }
        o.m = head;
        o.m.push_back(bp);
        if (bq) o.m.push_back(bq);
        logM = best;
    }
    const int s = (int)o.m.size();
    o.ok = (logM >= need) && s > 0 && s <= MAXS && s <= num_moduli && b > 0;
    for (int i = 0; i < s; ++i)
        for (int j = i + 1; j < s; ++j)
            if (std::gcd(o.m[i], o.m[j]) != 1) o.ok = false;
    for (int mm : o.m)
        if (!int8_fits(K, mm)) o.ok = o.acc_ok = false;
    o.logM = logM;
    return o;
}

// Per-modulus constants (oz2_crt_constants, moduli.hpp:615-703) and the small-tail counts
// (oz2_choose_small_tail, moduli.hpp:804-826).
float top12(__float128 v) {
    const float p = (float)(double)v;
    if (p == 0.0f) return 0.0f;
    const float c = (float)((double)4097.0f * (double)p);
    return (float)((double)c - (double)(float)((double)c - (double)p));
}
int small_tail(const float (*rp)[OZO_MAXRP], int nrp, const int* m, int s) {
    float worst[8] = {0};
    float vmax = 0.f;
    for (int t = 0; t < nrp; ++t) {
        for (int i = 0; i < s; ++i) {
            const float v = std::fabs(rp[i][t]) * (float)(m[i] / 2 + 1);
            if (v > worst[t]) worst[t] = v;
        }
        if (worst[t] > vmax) vmax = worst[t];
    }
    const float scale = vmax < 1.f ? vmax : 1.f;
    const float eps = (float)std::ldexp((double)scale, -30);
    int n = 0;
    for (int t = nrp; t-- > 0;) {
        if (worst[t] <= eps)
            n++;
        else
            break;
    }
    return n;
}
void crt_constants(const Moduli& mo, ozo_plan& p) {
    const int s = (int)mo.m.size();
    p.S = s;
    for (int i = 0; i < s; ++i) {
        p.m[i] = mo.m[i];
        long P = 1, mi = mo.m[i];
        for (int j = 0; j < s; ++j)
            if (j != i) P = (P * (mo.m[j] % mi)) % mi;
        p.yi[i] = (int)inv_mod(P, mi);
    }
    long double Mld = 1.0L;
    for (int mm : mo.m) Mld *= (long double)mm;
    const long double KMl = Mld * std::pow(2.0L, -2.0 * mo.b);
    int e;
    const long double f = frexpl(KMl, &e);
    const unsigned long long W = (unsigned long long)ldexpl(f, 64);
    p.W_hi = (uint32_t)(W >> 32);
    p.W_lo = (uint32_t)W;
    p.qw = e - 64;
    for (int i = 0; i < s; ++i) {
        const int mm = mo.m[i];
        const __float128 r = (__float128)1 / (__float128)mm;
        const __float128 gran = powq((__float128)2, -(__float128)RGRAN);
        const __float128 Rg = roundq(r / gran) * gran;
        __float128 v = Rg;
        for (int t = 0; t < 5; ++t) {
            p.rp1[i][t] = top12(v);
            v -= (__float128)p.rp1[i][t];
        }
        const __float128 sum1 = Rg - v;
        v = r - sum1;
        for (int t = 0; t < 3; ++t) {
            p.rp2[i][t] = (t + 1 < 3) ? top12(v) : (float)(double)v;
            v -= (__float128)p.rp2[i][t];
        }
        v = r;
        for (int t = 0; t < 5; ++t) {
            p.rp0[i][t] = (t + 1 < 5) ? top12(v) : (float)(double)v;
            v -= (__float128)p.rp0[i][t];
        }
        p.rinv[i] = (float)(double)r;
        auto pow2mod = [](int ex, long mod) {
            long r2 = 1 % mod, base = 2 % mod;
            for (int q = 0; q < ex; ++q) r2 = (r2 * base) % mod;
            return (float)r2;
        };
        for (int j = 0; j < 4; ++j) p.c[j][i] = pow2mod(DIGIT_BITS * (j + 1), mm);
        p.m16[i] = pow2mod(16, mm);
    }
    p.nsmall0 = small_tail(p.rp0, 5, p.m, s);
    p.nsmall1 = small_tail(p.rp1, 5, p.m, s);
    p.nsmall2 = small_tail(p.rp2, 3, p.m, s);
}

// Power-of-two normalizer of a matrix (oz_pow2_scale, norm_estimate.hpp:20-28).
double pow2_scale(const double* v, size_t n) {
    double mx = 0;
    for (size_t i = 0; i < n; ++i) mx = std::max(mx, std::fabs(v[i]));
    if (!(mx > 0) || !std::isfinite(mx)) return 1.0;
    int e;
    std::frexp(mx, &e);
    e = std::min(std::max(e, -1000), 1000);
    return std::ldexp(1.0, e);
}

// Operand statistics and the Hutchinson estimate of ||C||_F^2 (auto_precision.hpp:24-80,
// norm_estimate.hpp:49-73).
void measure_stats(const double* A, const double* B, uint32_t M, uint32_t N, uint32_t K, ozo_plan& p) {
    const double rgA = 1.0 / pow2_scale(A, (size_t)M * K), rgB = 1.0 / pow2_scale(B, (size_t)K * N);
    double TA = 0, TB = 0, nA = 0, nB = 0;
    for (uint32_t r = 0; r < M; r++) {
        double mx = 0, s2 = 0;
        for (uint32_t c = 0; c < K; c++) {
            const double v = A[(size_t)r * K + c] * rgA;
            mx = std::max(mx, std::fabs(v));
            s2 += v * v;
        }
        if (mx > 0) {
            const double t = std::exp2(std::ceil(std::log2(mx)));
            TA += t * t;
        }
        nA += s2;
    }
    for (uint32_t c = 0; c < N; c++) {
        double mx = 0, s2 = 0;
        for (uint32_t r = 0; r < K; r++) {
            const double v = B[(size_t)r * N + c] * rgB;
            mx = std::max(mx, std::fabs(v));
            s2 += v * v;
        }
        if (mx > 0) {
            const double t = std::exp2(std::ceil(std::log2(mx)));
            TB += t * t;
        }
        nB += s2;
    }
    const uint32_t L = 8;
    std::mt19937 rg(12345);
    std::normal_distribution<double> nd(0.0, 1.0);
    std::vector<double> g(N), y(K);
    double cs2 = 0, cmax = 0;
    for (uint32_t l = 0; l < L; l++) {
        for (uint32_t j = 0; j < N; j++) g[j] = nd(rg);
        for (uint32_t k = 0; k < K; k++) {
            long double s = 0;
            for (uint32_t j = 0; j < N; j++) s += (long double)(B[(size_t)k * N + j] * rgB) * g[j];
            y[k] = (double)s;
        }
        double q = 0;
        for (uint32_t i = 0; i < M; i++) {
            long double s = 0;
            for (uint32_t k = 0; k < K; k++) s += (long double)(A[(size_t)i * K + k] * rgA) * y[k];
            q += (double)s * (double)s;
        }
        cs2 += q;
        cmax = std::max(cmax, q);
    }
    p.TA = TA;
    p.TB = TB;
    p.nA = nA;
    p.nB = nB;
    p.nC = (cs2 - cmax) / (L - 1) / (1.0 + 2.0 * std::sqrt(2.0 / (double)L));
}

void fill_plan(const Moduli& mo, ozo_plan& p) {
    p.ok = mo.ok;
    p.acc_ok = mo.acc_ok;
    p.b = mo.b;
    p.m_cap = mo.m_cap;
    p.ncand = mo.ncand;
    p.logM = mo.logM;
    crt_constants(mo, p);
    p.nd = (mo.b > 4 * DIGIT_BITS) ? 5 : ((mo.b > 3 * DIGIT_BITS) ? 4 : 3);
    p.shift = mo.b - (p.nd - 1) * DIGIT_BITS;
}

void set_err(char* err, size_t errlen, const std::string& s) {
    if (err && errlen) {
        std::strncpy(err, s.c_str(), errlen - 1);
        err[errlen - 1] = 0;
    }
}

// Exact CRT helpers: little-endian 32-bit words, 8 words (256 bits).
struct Big {
    uint32_t w[8] = {0};
};
void big_add(Big& a, const Big& b) {
    uint64_t c = 0;
    for (int i = 0; i < 8; ++i) {
        c += (uint64_t)a.w[i] + b.w[i];
        a.w[i] = (uint32_t)c;
        c >>= 32;
    }
}
void big_sub(Big& a, const Big& b) {
    int64_t br = 0;
    for (int i = 0; i < 8; ++i) {
        int64_t t = (int64_t)a.w[i] - b.w[i] - br;
        br = t < 0;
        a.w[i] = (uint32_t)(t + (br << 32));
    }
}
int big_cmp(const Big& a, const Big& b) {
    for (int i = 7; i >= 0; --i)
        if (a.w[i] != b.w[i]) return a.w[i] < b.w[i] ? -1 : 1;
    return 0;
}
Big big_mul_small(const Big& a, uint32_t k) {
    Big r;
    uint64_t c = 0;
    for (int i = 0; i < 8; ++i) {
        c += (uint64_t)a.w[i] * k;
        r.w[i] = (uint32_t)c;
        c >>= 32;
    }
    return r;
}
// value * 2^e2 with one round-to-nearest-even, results below 2^-1022 flushed to +-0.
double big_to_double(const Big& mag, bool neg, int e2) {
    int top = -1;
    for (int i = 7; i >= 0 && top < 0; --i)
        if (mag.w[i]) top = 32 * i + 31 - __builtin_clz(mag.w[i]);
    if (top < 0) return 0.0;
    auto bit = [&](int k) -> uint32_t { return k < 0 ? 0u : (mag.w[k >> 5] >> (k & 31)) & 1u; };
    uint64_t mant = 0;
    for (int k = top; k > top - 53; --k) mant = (mant << 1) | bit(k);
    const uint32_t guard = bit(top - 53);
    bool sticky = false;
    for (int k = top - 54; k >= 0 && !sticky; --k) sticky = bit(k) != 0;
    int ex = top + e2;  // exponent of the leading bit
    if (guard && (sticky || (mant & 1))) {
        mant += 1;
        if (mant >> 53) {
            mant >>= 1;
            ex += 1;
        }
    }
    const double sgn = neg ? -1.0 : 1.0;
    if (ex < -1022) return sgn * 0.0;
    if (ex > 1023) return sgn * INFINITY;
    return sgn * std::ldexp((double)mant, ex - 52);
}

}  // namespace

extern "C" {

int ozo_gen_inputs(double* a, double* b, uint64_t m, uint64_t n, uint64_t k, double phi, uint32_t seed) {
    std::mt19937 rng(seed);
    const size_t na = (size_t)m * k, nb = (size_t)k * n;
    if (phi < 0) {
        std::uniform_real_distribution<double> u(-1, 1);
        for (size_t i = 0; i < na; ++i) a[i] = u(rng);
        for (size_t i = 0; i < nb; ++i) b[i] = u(rng);
    } else {
        std::uniform_real_distribution<double> u(0, 1);
        std::normal_distribution<double> normal(0, 1);
        auto value = [&] {
            const double v = u(rng);
            const double z = normal(rng);
            return (v - 0.5) * std::exp(phi * z);
        };
        for (size_t i = 0; i < na; ++i) a[i] = value();
        for (size_t i = 0; i < nb; ++i) b[i] = value();
    }
    return 0;
}

int ozo_gen_pattern(double* a, double* b, uint64_t m, uint64_t n, uint64_t k, int mode) {
    std::mt19937_64 rng(42);
    std::uniform_real_distribution<double> uniform(-1, 1);
    for (size_t i = 0; i < m * k; ++i) a[i] = mode == 1 ? 0 : uniform(rng);
    for (size_t i = 0; i < k * n; ++i) b[i] = uniform(rng);
    if (mode == 2) {
        for (size_t i = 0; i < m * k; ++i) a[i] = std::abs(a[i]);
        for (size_t i = 0; i < k * n; ++i) b[i] = std::abs(b[i]);
    }
    if (mode == 3) {
        for (size_t i = 0; i < m; ++i)
            for (size_t j = 0; j < k; ++j) a[i * k + j] = std::ldexp(a[i * k + j], int(i % 31) - 15);
        for (size_t i = 0; i < k; ++i)
            for (size_t j = 0; j < n; ++j) b[i * n + j] = std::ldexp(b[i * n + j], int(j % 27) - 13);
    }
    if (mode == 4) {
        for (size_t i = 0; i < m; ++i)
            for (size_t j = 0; j < k; ++j) a[i * k + j] = j % 2 ? -1 : 1;
        std::fill(b, b + k * n, 1.0);
    }
    if (mode == 5) {
        for (size_t j = 0; j < k; ++j) a[j] = 0;
        for (size_t i = 0; i < k; ++i) b[i * n] = 0;
    }
    if (mode == 6) {
        std::fill(a, a + m * k, 0x1p-126);
        std::fill(b, b + k * n, 1.0);
    }
    if (mode == 7) {
        std::fill(a, a + m * k, 0x1.fep127);
        std::fill(b, b + k * n, 1.0);
    }
    return 0;
}

int ozo_choose_moduli_int8(uint32_t K, int num_moduli, int b_cap, ozo_plan* out) {
    std::memset(out, 0, sizeof(*out));
    const Moduli mo = choose_moduli(K, num_moduli, b_cap);
    fill_plan(mo, *out);
    out->b_cap = b_cap;
    out->S_req = num_moduli;
    return 0;
}

int ozo_plan_ii_int8(const double* a, const double* b, uint32_t M, uint32_t N, uint32_t K, uint32_t max_moduli,
                     int passes, int fixed_bits, ozo_plan* out, char* err, size_t errlen) {
    std::memset(out, 0, sizeof(*out));
    const bool b_fixed = fixed_bits > 0;
    int b_cap = B_DEFAULT;
    bool have_stats = false;
    if (b_fixed) {
        b_cap = fixed_bits;
    } else {
        measure_stats(a, b, M, N, K, *out);
        have_stats = true;
        const double k2 = std::min(
            std::sqrt((out->TA * out->nB + out->TB * out->nA) / std::max(12.0 * out->nC, 1e-300)), 1e18);
        b_cap = std::min(MAXDIGIT * DIGIT_BITS, TARGET_BITS + (int)std::ceil(std::log2(std::max(k2, 1.0))));
    }
    const uint32_t S_req = max_moduli ? max_moduli : (b_fixed ? DEF_S_INT8 : (uint32_t)MAXS);
    if (b_fixed && passes == 0) {
        measure_stats(a, b, M, N, K, *out);
        have_stats = true;
    }
    const double TA = out->TA, TB = out->TB, nA = out->nA, nB = out->nB, nC = out->nC;
    const Moduli mo = choose_moduli(K, (int)S_req, b_cap);
    fill_plan(mo, *out);
    out->TA = TA;
    out->TB = TB;
    out->nA = nA;
    out->nB = nB;
    out->nC = nC;
    out->b_cap = b_cap;
    out->S_req = (int)S_req;
    if (!mo.ok) {
        set_err(err, errlen, mo.acc_ok ? "Ozaki II: the available moduli do not cover the CRT window"
                                       : "Ozaki II: the padded inner dimension K is too large for this format");
        return 1;
    }
    if (!b_fixed && mo.b < TARGET_BITS) {
        set_err(err, errlen, "Ozaki II: the selected moduli cover a width below 53 bits");
        return 1;
    }
    // Passes (oz2_choose_passes, plan.hpp:245-251; oz2_recon1_log2, auto_precision.hpp:133-138).
    double r1 = -INFINITY;
    if (have_stats && nC > 0 && TA > 0 && TB > 0) {
        double l2m = 0;
        for (int mm : mo.m) l2m += std::log2((double)mm);
        r1 = RECON1_EPS_LOG2 + l2m - 2.0 * mo.b + 0.5 * (std::log2(TA) + std::log2(TB) - std::log2(nC));
    }
    out->recon1_log2 = r1;
    if (passes != 0)
        out->two_pass = passes == 2;
    else
        out->two_pass = !(r1 <= RECON1_THR_LOG2);
    return 0;
}

int ozo_scale(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, int32_t shift,
              uint16_t* bf16_max, int32_t* delta, uint32_t* flags) {
    return ozo_scale_mode(x, rows, cols, ld, col_mode, shift, 1, bf16_max, delta, flags);
}

int ozo_scale_mode(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, int32_t shift, int ceil,
                   uint16_t* bf16_max, int32_t* delta, uint32_t* flags) {
    uint32_t fl = 0;
    const uint64_t nout = col_mode ? cols : rows, nin = col_mode ? rows : cols;
    for (uint64_t o = 0; o < nout; ++o) {
        uint64_t mx = 0;
        for (uint64_t i = 0; i < nin; ++i) {
            const double v = col_mode ? x[i * ld + o] : x[o * ld + i];
            mx = std::max<uint64_t>(mx, d_to_bits(v) & 0x7FFFFFFFFFFFFFFFull);
        }
        const uint16_t u = abs_to_bf16(mx, ceil);
        if (bf16_max) bf16_max[o] = u;
        delta[o] = shift - bf16_scale_exp(u, fl);
    }
    if (flags) *flags = fl;
    return 0;
}

int ozo_digits(double x, int32_t delta, int nd, float* digits) {
    make_digits(x, delta, nd, digits);
    return 0;
}

int ozo_split(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, const int32_t* delta,
              const ozo_plan* plan, int8_t* planes) {
    const int S = plan->S, nd = plan->nd;
    const uint64_t plane = rows * cols;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; ++r)
        for (uint64_t c = 0; c < cols; ++c) {
            const double v = x[(uint64_t)r * ld + c];
            const int32_t d = col_mode ? delta[c] : delta[r];
            float dg[5];
            make_digits(v, d, nd, dg);
            const uint64_t idx = col_mode ? c * rows + (uint64_t)r : (uint64_t)r * cols + c;
            for (int s = 0; s < S; ++s) {
                const float cc[4] = {plan->c[0][s], plan->c[1][s], plan->c[2][s], plan->c[3][s]};
                const float res = residue(dg, nd, (float)plan->m[s], plan->rinv[s], cc);
                planes[(uint64_t)s * plane + idx] = (int8_t)(int)res;
            }
        }
    return 0;
}

int ozo_gemm_i32(const int8_t* ap, const int8_t* bp, uint64_t S, uint64_t M, uint64_t N, uint64_t K, int32_t* c) {
    int bad = 0;
#pragma omp parallel for collapse(2) schedule(static) reduction(| : bad)
    for (int64_t s = 0; s < (int64_t)S; ++s)
        for (int64_t i = 0; i < (int64_t)M; ++i) {
            const int8_t* ar = ap + ((uint64_t)s * M + (uint64_t)i) * K;
            for (uint64_t j = 0; j < N; ++j) {
                const int8_t* br = bp + ((uint64_t)s * N + j) * K;
                int64_t acc = 0;
                for (uint64_t k = 0; k < K; ++k) acc += (int32_t)ar[k] * (int32_t)br[k];
                if (acc > INT32_MAX || acc < -INT32_MAX) bad = 1;
                c[((uint64_t)s * M + (uint64_t)i) * N + j] = (int32_t)acc;
            }
        }
    return bad;
}

namespace {
// The reference's reconstruction of one element from its residues r_s (recon_crt.cpp:296-338 with
// recon_crt_proc.h and the assembly of recon_elem.h / f64_tf.h:296-400).
double recon_element_faithful(const float* r, const ozo_plan* plan, int32_t g) {
    const int S = plan->S;
    struct Pass {
        const float (*rp)[OZO_MAXRP];
        int nrp, nsmall;
    };
    Pass passes[2];
    int npass;
    if (plan->two_pass) {
        passes[0] = {plan->rp1, 5, plan->nsmall1};
        passes[1] = {plan->rp2, 3, plan->nsmall2};
        npass = 2;
    } else {
        passes[0] = {plan->rp0, 5, plan->nsmall0};
        npass = 1;
    }
    // 128-bit fixed point frac * 2^124 (recon_elem.h:28-60, f64_tf.h:296-400).
    unsigned __int128 fix = 0;
    for (int pi = 0; pi < npass; ++pi) {
        const Pass& ps = passes[pi];
        float a0 = 0.f, a1 = 0.f, a2 = 0.f;
        for (int s = 0; s < S; ++s) {
            const float m = (float)plan->m[s], ri = plan->rinv[s];
            // term_k and accumulate (recon_crt_proc.h:27-52).
            const float kk = mod_round(fmul(r[s], (float)plan->yi[s]), m, ri);
            for (int t = 0; t < ps.nrp; ++t) {
                const float v = fmul(kk, ps.rp[s][t]);
                if (t >= ps.nrp - ps.nsmall)
                    tf_add_small(a1, a2, v);
                else
                    tf_add(a0, a1, a2, v);
            }
            a0 = fsub(a0, frnd(a0));  // drop_integer (recon_crt_proc.h:56-59)
        }
        for (float limb : {a0, a1, a2}) {
            const uint32_t u = f_to_bits(limb);
            const int32_t ee = (int32_t)((u >> 23) & 0xFFu);
            if (ee == 0) continue;
            const int32_t mag = (int32_t)(0x800000u | (u & 0x7FFFFFu));
            const int32_t sh = ee - 26;
            if (sh <= -24 || sh >= 128) continue;  // below the fixed-point LSB / above bit 127
            const unsigned __int128 v =
                sh < 0 ? (unsigned __int128)((uint64_t)mag >> (uint32_t)(-sh)) : ((unsigned __int128)mag << sh);
            if (v == 0) continue;
            if (u & 0x80000000u)
                fix -= v;
            else
                fix += v;
        }
    }
    // Fold to [-1/2, 1/2] and assemble (a128_frac_to_f64, f64_tf.h:345-400).
    const uint32_t top = (uint32_t)(fix >> 96);
    if (top + 0x08000000u >= 0x10000000u || top == 0xF8000000u) {
        const unsigned __int128 one = (unsigned __int128)1 << 124;
        if ((int32_t)top >= 0x08000000)
            fix -= one;
        else if ((int32_t)top < -0x08000000 || (fix & (((unsigned __int128)1 << 96) - 1)) == 0)
            fix += one;
    }
    const bool neg = (fix >> 127) != 0;
    unsigned __int128 mag = neg ? (~fix + 1) : fix;
    double out = 0.0;
    if (mag != 0) {
        int lz = 0;
        {
            const uint64_t hi = (uint64_t)(mag >> 64), lo = (uint64_t)mag;
            lz = hi ? __builtin_clzll(hi) : 64 + __builtin_clzll(lo);
        }
        const uint64_t A = lz <= 64 ? (uint64_t)(mag >> (64 - lz)) : (uint64_t)(mag << (lz - 64));
        const int32_t total = plan->qw + g - lz - 60;
        // pack_f64 (f64_tf.h:189-213): top 64 bits of A*W, guard-bit rounding (ties away).
        const uint64_t W = ((uint64_t)plan->W_hi << 32) | plan->W_lo;
        const uint64_t hi = (uint64_t)(((unsigned __int128)A * W) >> 64);
        const int32_t nb = (hi >> 63) ? 63 : 62;
        int32_t exp2 = nb + 64 + total;
        uint64_t mant;
        bool up;
        if (nb == 63) {
            mant = hi >> 11;
            up = (hi & 0x400ull) != 0;
        } else {
            mant = hi >> 10;
            up = (hi & 0x200ull) != 0;
        }
        if (up) {
            mant += 1;
            if (mant >> 53) {
                mant >>= 1;
                exp2 += 1;
            }
        }
        const uint64_t sgn = neg ? 0x8000000000000000ull : 0ull;
        const int32_t eb = exp2 + 1023;
        uint64_t ub;
        if (eb <= 0)
            ub = sgn;
        else if (eb >= 2047)
            ub = sgn | 0x7FF0000000000000ull;
        else
            ub = sgn | ((uint64_t)eb << 52) | (mant & 0x000FFFFFFFFFFFFFull);
        std::memcpy(&out, &ub, 8);
    }
    return out;
}
}  // namespace

int ozo_recon_faithful(const int32_t* cs, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                       const ozo_plan* plan, double* c, uint64_t ldc) {
    const int S = plan->S;
    const int32_t sh2 = 2 * plan->shift;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)M; ++i)
        for (uint64_t j = 0; j < N; ++j) {
            // r_i per modulus from the sign-magnitude int32 word (decode_signmag_residue,
            // recon_crt.cpp:219-245; host model oz_sim.h:277-295).
            float r[OZO_MAXS];
            for (int s = 0; s < S; ++s) {
                const int32_t v = cs[((uint64_t)s * M + (uint64_t)i) * N + j];
                const uint32_t mag = (uint32_t)(v < 0 ? -(int64_t)v : v);
                const uint32_t w = (v < 0 ? 0x80000000u : 0u) | mag;
                const float m = (float)plan->m[s], ri = plan->rinv[s];
                const float sgn = v > 0 ? 1.f : (v < 0 ? -1.f : 0.f);
                float chi = fmul((float)(w & 0x7FFF0000u), 1.52587890625e-05f);
                const float kh = fmul(mod_round(chi, m, ri), plan->m16[s]);
                const float kl = mod_round((float)(w & 0x0000FFFFu), m, ri);
                r[s] = mod_round(fmul(fadd(kl, kh), sgn), m, ri);
            }
            c[(uint64_t)i * ldc + j] = recon_element_faithful(r, plan, sh2 - (dA[i] + dB[j]));
        }
    return 0;
}

int ozo_recon_faithful_residue(const float* rs, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                               const ozo_plan* plan, double* c, uint64_t ldc) {
    const int S = plan->S;
    const int32_t sh2 = 2 * plan->shift;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)M; ++i)
        for (uint64_t j = 0; j < N; ++j) {
            float r[OZO_MAXS];
            for (int s = 0; s < S; ++s) r[s] = rs[((uint64_t)s * M + (uint64_t)i) * N + j];
            c[(uint64_t)i * ldc + j] = recon_element_faithful(r, plan, sh2 - (dA[i] + dB[j]));
        }
    return 0;
}

int ozo_recon_exact(const int32_t* cs, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                    const ozo_plan* plan, double* c, uint64_t ldc) {
    const int S = plan->S;
    Big Mb;
    Mb.w[0] = 1;
    for (int s = 0; s < S; ++s) Mb = big_mul_small(Mb, (uint32_t)plan->m[s]);
    std::vector<Big> Q(S);
    for (int s = 0; s < S; ++s) {
        Big q;
        q.w[0] = 1;
        for (int t = 0; t < S; ++t)
            if (t != s) q = big_mul_small(q, (uint32_t)plan->m[t]);
        Q[s] = q;
    }
    Big half = Mb;  // floor(M/2)
    for (int i = 0; i < 8; ++i) half.w[i] = (half.w[i] >> 1) | (i < 7 ? (half.w[i + 1] << 31) : 0u);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)M; ++i)
        for (uint64_t j = 0; j < N; ++j) {
            Big X;
            for (int s = 0; s < S; ++s) {
                const int64_t m = plan->m[s];
                int64_t r = cs[((uint64_t)s * M + (uint64_t)i) * N + j] % m;
                if (r < 0) r += m;
                const uint32_t k = (uint32_t)((r * plan->yi[s]) % m);
                big_add(X, big_mul_small(Q[s], k));
                if (big_cmp(X, Mb) >= 0) big_sub(X, Mb);
            }
            bool neg = false;
            if (big_cmp(X, half) > 0) {
                Big t = Mb;
                big_sub(t, X);
                X = t;
                neg = true;
            }
            const int32_t g = 2 * plan->shift - (dA[i] + dB[j]);
            c[(uint64_t)i * ldc + j] = big_to_double(X, neg, g - 2 * plan->b);
        }
    return 0;
}

int ozo_ii_int8_emulate(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                        uint32_t max_moduli, int passes, int fixed_bits, int recon, ozo_plan* info_out, char* err,
                        size_t errlen) {
    auto pad = [](uint64_t v, uint64_t q) { return (v + q - 1) / q * q; };
    const uint64_t M = pad(m, 64), N = pad(n, 64), K = pad(k, 32);
    std::vector<double> ap(M * K, 0.0), bp(K * N, 0.0);
    for (uint64_t i = 0; i < m; ++i) std::copy_n(a + i * k, k, ap.data() + i * K);
    for (uint64_t i = 0; i < k; ++i) std::copy_n(b + i * n, n, bp.data() + i * N);
    ozo_plan plan;
    const int rc = ozo_plan_ii_int8(ap.data(), bp.data(), (uint32_t)M, (uint32_t)N, (uint32_t)K, max_moduli, passes,
                                    fixed_bits, &plan, err, errlen);
    if (info_out) *info_out = plan;
    if (rc) return rc;
    std::vector<int32_t> dA(M), dB(N);
    uint32_t fa = 0, fb = 0;
    ozo_scale(ap.data(), M, K, K, 0, plan.shift, nullptr, dA.data(), &fa);
    ozo_scale(bp.data(), K, N, N, 1, plan.shift, nullptr, dB.data(), &fb);
    if (fa | fb) {
        set_err(err, errlen, "out-of-range row or column maxima");
        return 1;
    }
    const uint64_t S = (uint64_t)plan.S;
    std::vector<int8_t> ra(S * M * K), rb(S * N * K);
    ozo_split(ap.data(), M, K, K, 0, dA.data(), &plan, ra.data());
    ozo_split(bp.data(), K, N, N, 1, dB.data(), &plan, rb.data());
    std::vector<int32_t> cs(S * M * N);
    if (ozo_gemm_i32(ra.data(), rb.data(), S, M, N, K, cs.data())) {
        set_err(err, errlen, "int32 overflow in the residue GEMM");
        return 1;
    }
    std::vector<double> cp(M * N);
    if (recon == 0)
        ozo_recon_faithful(cs.data(), M, N, dA.data(), dB.data(), &plan, cp.data(), N);
    else
        ozo_recon_exact(cs.data(), M, N, dA.data(), dB.data(), &plan, cp.data(), N);
    for (uint64_t i = 0; i < m; ++i) std::copy_n(cp.data() + i * N, n, c + i * n);
    return 0;
}

int ozo_dot2_gemm(const double* A, const double* B, uint64_t M, uint64_t N, uint64_t K, double* Chi, double* Clo) {
    std::fill(Chi, Chi + M * N, 0.0);
    std::fill(Clo, Clo + M * N, 0.0);
    constexpr uint64_t IB = 8, JB = 512;
#pragma omp parallel for schedule(static)
    for (int64_t ib = 0; ib < (int64_t)M; ib += IB) {
        const uint64_t i1 = std::min<uint64_t>((uint64_t)ib + IB, M);
        for (uint64_t j0 = 0; j0 < N; j0 += JB) {
            const uint64_t j1 = std::min<uint64_t>(j0 + JB, N);
            for (uint64_t kk = 0; kk < K; ++kk) {
                const double* Br = B + kk * N;
                for (uint64_t i = (uint64_t)ib; i < i1; ++i) {
                    const double av = A[i * K + kk];
                    double* chi = Chi + i * N;
                    double* clo = Clo + i * N;
                    for (uint64_t j = j0; j < j1; ++j) {
                        const double bv = Br[j];
                        const double p = av * bv, e = std::fma(av, bv, -p);
                        const double c0 = chi[j];
                        const double s = c0 + p, bb = s - c0;
                        clo[j] += (c0 - (s - bb)) + (p - bb) + e;
                        chi[j] = s;
                    }
                }
            }
        }
    }
    return 0;
}

int ozo_accuracy(const double* C, const double* Chi, const double* Clo, uint64_t count, double* rel_fro,
                 double* ebits) {
    auto ref = [](double hi, double lo, double& s, double& e) {
        s = hi + lo;
        const double bb = s - hi;
        e = (hi - (s - bb)) + (lo - bb);
    };
    double num = 0, den = 0, mx = 0;
    for (uint64_t z = 0; z < count; z++) {
        double hi, lo;
        ref(Chi[z], Clo[z], hi, lo);
        mx = std::max(mx, std::max(std::fabs(hi), std::fabs((C[z] - hi) - lo)));
    }
    const int sce = (mx > 0 && std::isfinite(mx)) ? -std::ilogb(mx) : 0;
    const int sce1 = std::min(sce, 1023);
    const double sc1 = std::ldexp(1.0, sce1), sc2 = std::ldexp(1.0, sce - sce1);
    for (uint64_t z = 0; z < count; z++) {
        double hi, lo;
        ref(Chi[z], Clo[z], hi, lo);
        const double dd = (C[z] - hi) - lo;
        const double ds = (dd * sc1) * sc2, gs = (hi * sc1) * sc2;
        num += ds * ds;
        den += gs * gs;
    }
    double rel;
    if (!std::isfinite(num) || !std::isfinite(den))
        rel = INFINITY;
    else if (den > 0)
        rel = std::sqrt(num) / std::sqrt(den);
    else
        rel = num > 0 ? INFINITY : 0.0;
    *rel_fro = rel;
    *ebits = std::isfinite(rel) ? (rel > 0 ? -std::log2(rel) : 99.0) : -1.0;
    return 0;
}

uint64_t ozo_output_hash(const double* C, uint64_t count) {
    uint64_t h = 1469598103934665603ull;
    for (uint64_t z = 0; z < count; z++) {
        const uint64_t u = d_to_bits(C[z]);
        for (int b = 0; b < 64; b += 8) {
            h ^= (u >> b) & 0xFFu;
            h *= 1099511628211ull;
        }
    }
    return h;
}

int ozo_maxrel_f128(const double* a, const double* b, const double* c, uint64_t m, uint64_t n, uint64_t k,
                    const uint64_t* rows, uint64_t nrows, double* maxrel) {
    const uint64_t nr = rows ? nrows : m;
    double worst = 0;
#pragma omp parallel for schedule(dynamic) reduction(max : worst)
    for (int64_t t = 0; t < (int64_t)nr; ++t) {
        const uint64_t i = rows ? rows[t] : (uint64_t)t;
        std::vector<__float128> acc(n, 0);
        for (uint64_t l = 0; l < k; ++l) {
            const __float128 av = a[i * k + l];
            const double* br = b + l * n;
            for (uint64_t j = 0; j < n; ++j) acc[j] += av * (__float128)br[j];
        }
        for (uint64_t j = 0; j < n; ++j) {
            const __float128 d = (__float128)c[i * n + j] - acc[j];
            const double ad = (double)(d < 0 ? -d : d);
            const double ar = (double)(acc[j] < 0 ? -acc[j] : acc[j]);
            const double e = ar > 0 ? ad / ar : ad;
            worst = std::max(worst, e);
        }
    }
    *maxrel = worst;
    return 0;
}

int ozo_maxrel_f128_rows(const double* a, const double* b, const double* const* cs, int nc, uint64_t m, uint64_t n,
                         uint64_t k, const uint64_t* rows, uint64_t nrows, double* maxrel) {
    if (nc < 1 || nc > 16) return 1;
    for (uint64_t t = 0; t < nrows; ++t)
        if (rows[t] >= m) return 1;
    double worst[16] = {};
    // rows in parallel, and each row's columns in chunks, so that a handful of rows still fills the cores
    const uint64_t chunk = 512, nchunk = (n + chunk - 1) / chunk;
#pragma omp parallel
    {
        double mine[16] = {};
#pragma omp for schedule(dynamic) collapse(2)
        for (int64_t t = 0; t < (int64_t)nrows; ++t)
            for (int64_t q = 0; q < (int64_t)nchunk; ++q) {
                const uint64_t i = rows[t], j0 = (uint64_t)q * chunk, j1 = std::min(n, j0 + chunk);
                std::vector<__float128> acc(j1 - j0, 0);
                for (uint64_t l = 0; l < k; ++l) {
                    const __float128 av = a[i * k + l];
                    const double* br = b + l * n;
                    for (uint64_t j = j0; j < j1; ++j) acc[j - j0] += av * (__float128)br[j];
                }
                for (int r = 0; r < nc; ++r)
                    for (uint64_t j = j0; j < j1; ++j) {
                        const __float128 ref = acc[j - j0];
                        const __float128 d = (__float128)cs[r][(uint64_t)t * n + j] - ref;
                        const double ad = (double)(d < 0 ? -d : d);
                        const double ar = (double)(ref < 0 ? -ref : ref);
                        mine[r] = std::max(mine[r], ar > 0 ? ad / ar : ad);
                    }
            }
#pragma omp critical
        for (int r = 0; r < nc; ++r) worst[r] = std::max(worst[r], mine[r]);
    }
    for (int r = 0; r < nc; ++r) maxrel[r] = worst[r];
    return 0;
}

double ozo_time_dot2_rows(const double* a, const double* b, uint64_t rows, uint64_t n, uint64_t k, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
    const double t0 = omp_get_wtime();
#endif
    std::vector<double> hi(rows * n), lo(rows * n);
    ozo_dot2_gemm(a, b, rows, n, k, hi.data(), lo.data());
#ifdef _OPENMP
    return omp_get_wtime() - t0;
#else
    return -1.0;
#endif
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Scheme II with FP8 (e4m3) digits.
// ---------------------------------------------------------------------------------------------
namespace {
// Integers e4m3 holds exactly (the digit sets of modslice_digit.cpp: |x| <= 16, or even with |x| <= 32).
bool e4m3_integer(float v) {
    const float a = std::fabs(v);
    if (a != std::floor(a)) return false;
    if (a <= 16.0f) return true;
    return a <= 32.0f && std::fmod(a, 2.0f) == 0.0f;
}
// Parity of an integer-valued float through the units bit of |x| + 2^23 (sparse_fix.h:55-70).
bool odd_integer(float a) { return (f_to_bits(a + 8388608.0f) & 1u) != 0; }

// Digits of one residue r of a modulus with splitting mode `mode` (modslice_digit.cpp:193-226,
// sparse_fix.h:52-72); returns the number of digits (l, h[, s]).
int split_residue(float r, int mode, float q, float qinv, float* dg) {
    if (mode == OZTT_SPLIT_ONE) {  // one digit: the residue itself (modslice_digit.cpp:207-211)
        dg[0] = r;
        return 1;
    }
    if (mode == OZTT_SPLIT_KAR) {
        // h = round((r + sign(r) (q/2 - 1/2)) / q), the sign from Ltz: +1 for r >= 0
        const float ltz = r < 0.0f ? 1.0f : 0.0f;
        const float sgn = fadd(fmul(ltz, -2.0f), 1.0f);
        const float t = fmul(sgn, q * 0.5f - 0.5f);
        const float h = frnd(fmul(fadd(r, t), qinv));
        const float l = fsub(r, fmul(h, q));
        dg[0] = l;
        dg[1] = h;
        dg[2] = fadd(h, l);
        return 3;
    }
    float h = frnd(fmul(r, qinv));
    float l = fsub(r, fmul(h, q));
    if (mode == OZTT_SPLIT_SQS) {
        const float al = std::fabs(l);
        if (al > 16.5f && odd_integer(al)) {
            if (l < 0.0f) {
                l = l + q;
                h = h - 1.0f;
            } else {
                l = l - q;
                h = h + 1.0f;
            }
        }
        const float ah = std::fabs(h);
        if (ah > 16.5f && odd_integer(ah)) h = h < 0.0f ? h + q : h - q;
    }
    dg[0] = l;
    dg[1] = h;
    return 2;
}
}  // namespace

extern "C" {

int ozo_crt_plan(const int32_t* m, int S, int b, int two_pass, ozo_plan* out) {
    if (S < 1 || S > OZO_MAXS) return 1;
    Moduli mo;
    mo.ok = true;
    mo.b = b;
    mo.m.assign(m, m + S);
    mo.logM = 0;
    for (int i = 0; i < S; ++i) mo.logM += std::log2((double)m[i]);
    mo.m_cap = *std::max_element(m, m + S);
    mo.ncand = S;
    *out = ozo_plan{};
    fill_plan(mo, *out);
    out->two_pass = two_pass;
    out->S_req = S;
    return 0;
}

int ozo_digit_split(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, const int32_t* delta,
                  const ozo_plan* crt, const oztt_digit_plan* fp, int8_t* planes) {
    const int S = crt->S, nd = crt->nd;
    const uint64_t plane = rows * cols;
    float qinv[OZO_MAXS];
    for (int s = 0; s < S; ++s) qinv[s] = 1.0f / (float)fp->q[s];  // sl_qinv, stages.hpp:223
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t r = 0; r < (int64_t)rows; ++r)
        for (uint64_t c = 0; c < cols; ++c) {
            const double v = x[(uint64_t)r * ld + c];
            const int32_t d = col_mode ? delta[c] : delta[r];
            float dg[5];
            make_digits(v, d, nd, dg);
            const uint64_t idx = col_mode ? c * rows + (uint64_t)r : (uint64_t)r * cols + c;
            for (int s = 0; s < S; ++s) {
                const float cc[4] = {crt->c[0][s], crt->c[1][s], crt->c[2][s], crt->c[3][s]};
                const float res = residue(dg, nd, (float)crt->m[s], crt->rinv[s], cc);
                float digit[3];
                const int nd2 = split_residue(res, fp->mode[s], (float)fp->q[s], qinv[s], digit);
                for (int j = 0; j < nd2; ++j) {
                    if (fp->format == OZTT_FMT_FP8 ? !e4m3_integer(digit[j]) : std::fabs(digit[j]) > 32.0f) bad = 1;
                    planes[(uint64_t)(fp->poff[s] + j) * plane + idx] = (int8_t)(int)digit[j];
                }
            }
        }
    return bad;
}

int ozo_digit_gemm(const int8_t* ap, const int8_t* bp, const oztt_digit_plan* fp, uint64_t M, uint64_t N, uint64_t K,
                 int32_t* out) {
    int bad = 0;
    const int64_t nout = fp->nout;
#pragma omp parallel for collapse(2) schedule(static) reduction(| : bad)
    for (int64_t o = 0; o < nout; ++o)
        for (int64_t i = 0; i < (int64_t)M; ++i)
            for (uint64_t j = 0; j < N; ++j) {
                int64_t acc = 0;
                for (int t = 0; t < fp->out_g[o]; ++t) {
                    const int8_t* ar = ap + ((uint64_t)(fp->out_a[o] + t) * M + (uint64_t)i) * K;
                    const int8_t* br = bp + ((uint64_t)(fp->out_b[o] - t) * N + j) * K;
                    for (uint64_t k = 0; k < K; ++k) acc += (int32_t)ar[k] * (int32_t)br[k];
                }
                if (acc > (1 << 24) || acc < -(1 << 24)) bad = 1;
                out[((uint64_t)o * M + (uint64_t)i) * N + j] = (int32_t)acc;
            }
    return bad;
}

int ozo_digit_compose(const int32_t* P, const oztt_digit_plan* fp, const ozo_plan* crt, uint64_t M, uint64_t N, float* r) {
    const int S = crt->S;
    const uint64_t plane = M * N;
    for (int s = 0; s < S; ++s) {
        const float m = (float)crt->m[s], ri = crt->rinv[s];
        const int o0 = fp->oout[s], o1 = fp->oout[s + 1];
        float lo[OZTT_MAXOUT], hi[OZTT_MAXOUT];
        for (int o = o0; o < o1; ++o) {
            lo[o] = (float)fp->coeff[o];                                   // c mod m (coeff_lo)
            hi[o] = (float)(((int64_t)fp->coeff[o] * 4096) % crt->m[s]);  // c 2^12 mod m (coeff_hi)
        }
        if (fp->mode[s] == OZTT_SPLIT_ONE) {
            // a one-digit modulus bypasses the composition; the reconstruction reduces its product first
            // (RAWMASK, recon_crt_proc.h:28-33)
#pragma omp parallel for schedule(static)
            for (int64_t e = 0; e < (int64_t)plane; ++e)
                r[(uint64_t)s * plane + (uint64_t)e] = mod_round((float)P[(uint64_t)o0 * plane + (uint64_t)e], m, ri);
            continue;
        }
#pragma omp parallel for schedule(static)
        for (int64_t e = 0; e < (int64_t)plane; ++e) {
            float acc = 0.0f;
            for (int o = o0; o < o1; ++o) {
                const float p = (float)P[(uint64_t)o * plane + (uint64_t)e];
                float v;
                if (fp->fold_first) {
                    v = fmul(mod_round(p, m, ri), lo[o]);
                } else {
                    const float h = frnd(fmul(p, 1.0f / 4096.0f));
                    const float l = fsub(p, fmul(h, 4096.0f));
                    v = fadd(fmul(h, hi[o]), fmul(l, lo[o]));
                }
                acc = (o == o0) ? v : fadd(acc, v);
            }
            r[(uint64_t)s * plane + (uint64_t)e] = mod_round(acc, m, ri);
        }
    }
    return 0;
}

int ozo_digit_emulate(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                    const oztt_digit_plan* fp, int exact, char* err, size_t errlen) {
    auto pad = [](uint64_t v, uint64_t q) { return (v + q - 1) / q * q; };
    const uint64_t M = pad(m, 64), N = pad(n, 64), K = pad(k, 32);
    std::vector<double> ap(M * K, 0.0), bp(K * N, 0.0);
    for (uint64_t i = 0; i < m; ++i) std::copy_n(a + i * k, k, ap.data() + i * K);
    for (uint64_t i = 0; i < k; ++i) std::copy_n(b + i * n, n, bp.data() + i * N);
    ozo_plan crt;
    if (ozo_crt_plan(fp->base.moduli, fp->base.S, fp->base.b, fp->base.two_pass, &crt)) {
        set_err(err, errlen, "bad moduli set");
        return 1;
    }
    std::vector<int32_t> dA(M), dB(N);
    uint32_t fa = 0, fb = 0;
    ozo_scale(ap.data(), M, K, K, 0, crt.shift, nullptr, dA.data(), &fa);
    ozo_scale(bp.data(), K, N, N, 1, crt.shift, nullptr, dB.data(), &fb);
    if (fa | fb) {
        set_err(err, errlen, "out-of-range row or column maxima");
        return 1;
    }
    const uint64_t NP = (uint64_t)fp->nplane;
    std::vector<int8_t> da(NP * M * K), db(NP * N * K);
    if (ozo_digit_split(ap.data(), M, K, K, 0, dA.data(), &crt, fp, da.data()) |
        ozo_digit_split(bp.data(), K, N, N, 1, dB.data(), &crt, fp, db.data())) {
        set_err(err, errlen, "a digit outside the digit set of the format");
        return 1;
    }
    std::vector<int32_t> P((uint64_t)fp->nout * M * N);
    if (ozo_digit_gemm(da.data(), db.data(), fp, M, N, K, P.data())) {
        set_err(err, errlen, "a digit product above 2^24");
        return 1;
    }
    std::vector<float> r((uint64_t)crt.S * M * N);
    ozo_digit_compose(P.data(), fp, &crt, M, N, r.data());
    std::vector<double> cp(M * N);
    if (exact) {
        std::vector<int32_t> ri(r.size());
        for (size_t e = 0; e < r.size(); ++e) ri[e] = (int32_t)r[e];
        ozo_recon_exact(ri.data(), M, N, dA.data(), dB.data(), &crt, cp.data(), N);
    } else {
        ozo_recon_faithful_residue(r.data(), M, N, dA.data(), dB.data(), &crt, cp.data(), N);
    }
    for (uint64_t i = 0; i < m; ++i) std::copy_n(cp.data() + i * N, n, c + i * n);
    return 0;
}

}  // extern "C"

// =================================================================================================
// Scheme I INT8 (src/ozaki1.cpp, src/backend/ozaki1/*): radix 254, digits +-127, target 2^-1.
// =================================================================================================
namespace {

// Triple-float times a radix that is not a power of two, with Dekker splits (tfMulR,
// sfpu_tf_proc.h:108-133); the constant of the split is 4097.
void tf_mul_r(float& x0, float& x1, float& x2, float r) {
    const float spl = 4097.0f;
    const float lo_r = fmul(x2, r);
    float t1 = fmul(x1, spl);
    float t2 = fsub(t1, x1);
    float hm = fsub(t1, t2);
    float lm = fsub(x1, hm);
    hm = fmul(hm, r);
    lm = fmul(lm, r);
    const float P1 = fadd(hm, lm);
    float kk = fsub(P1, hm);
    const float F1 = fsub(lm, kk);
    t1 = fmul(x0, spl);
    t2 = fsub(t1, x0);
    float hh = fsub(t1, t2);
    float lh = fsub(x0, hh);
    hh = fmul(hh, r);
    lh = fmul(lh, r);
    const float P0 = fadd(hh, lh);
    kk = fsub(P0, hh);
    const float F0 = fsub(lh, kk);
    const float G1 = fadd(F1, lo_r);
    float sa, ea, sb, eb, r0, ec;
    two_sum(P1, G1, sa, ea);
    two_sum(F0, sa, sb, eb);
    two_sum(P0, sb, r0, ec);
    const float G = fadd(ea, eb);
    x0 = r0;
    fast_two_sum(ec, G, x1, x2);
}

// Radix and digit bound of a scheme I format (ozaki1/param.hpp:47-70): INT8 (5) 254 / 127, FP8 (4) 32 / 16,
// BF16 (0), FP16 (1) and TF32 (2) 64 / 32.
struct I1Fmt {
    float radix, dmax;
    bool pow2;  // radix multiplication by tfMulP2 (sfpu_tf.h:121-134)
};
I1Fmt i1_fmt(int format) {
    if (format == 4) return I1Fmt{32.0f, 16.0f, true};
    if (format == 0 || format == 1 || format == 2) return I1Fmt{64.0f, 32.0f, true};
    return I1Fmt{254.0f, 127.0f, false};
}

// The p slices of one element (slice_tf_body.h): t *= radix; d = clamp(Rnd(t0), +-dmax); t0 -= d.
void make_slices(double x, int32_t d, int p, const I1Fmt& f, int8_t* out, uint64_t stride) {
    float x0, x1, x2;
    tf_load(x, d, x0, x1, x2);
    for (int i = 0; i < p; ++i) {
        if (f.pow2)
            tf_mul_p2(x0, x1, x2, f.radix);
        else
            tf_mul_r(x0, x1, x2, f.radix);
        float dig = frnd(x0);
        if (dig < -f.dmax)
            dig = -f.dmax;
        else if (dig >= f.dmax)
            dig = f.dmax;
        out[(uint64_t)i * stride] = (int8_t)(int)dig;
        x0 = fsub(x0, dig);
    }
}

// 64-bit significand and exponent of radix^-(L+2) in long double (recon_scale, ozaki1/plan.hpp:437-465).
void radix_scale(int L, float radix, uint64_t& W, int32_t& q) {
    long double w = 1.0L;
    for (int i = 0; i < L + 2; ++i) w /= (long double)radix;
    int e;
    const long double f = frexpl(w, &e);
    W = (unsigned long long)ldexpl(f, 64);
    q = e - 64;
}

// Rounds +-A * W * 2^total to FP64 the way pack_f64 does (f64_tf.h:189-213): top 64 bits of the
// product, guard-bit rounding, subnormals flushed.
double pack_like_reference(uint64_t A, uint64_t W, int32_t total, bool neg) {
    const uint64_t hi = (uint64_t)(((unsigned __int128)A * W) >> 64);
    const int32_t nb = (hi >> 63) ? 63 : 62;
    int32_t exp2 = nb + 64 + total;
    uint64_t mant;
    bool up;
    if (nb == 63) {
        mant = hi >> 11;
        up = (hi & 0x400ull) != 0;
    } else {
        mant = hi >> 10;
        up = (hi & 0x200ull) != 0;
    }
    if (up) {
        mant += 1;
        if (mant >> 53) {
            mant >>= 1;
            exp2 += 1;
        }
    }
    const uint64_t sgn = neg ? 0x8000000000000000ull : 0ull;
    const int32_t eb = exp2 + 1023;
    uint64_t ub;
    if (eb <= 0)
        ub = sgn;
    else if (eb >= 2047)
        ub = sgn | 0x7FF0000000000000ull;
    else
        ub = sgn | ((uint64_t)eb << 52) | (mant & 0x000FFFFFFFFFFFFFull);
    double out;
    std::memcpy(&out, &ub, 8);
    return out;
}

// The scheme I exit (assemble_tf_f64, f64_tf.h:269-300): three limbs collected in a 64-bit window
// 37 bits above the largest exponent, re-collected when the window cancels to zero.
int64_t acc64_term(int32_t sig, int32_t sh) {
    if (!sig) return 0;
    if (sh >= 0) return (int64_t)((uint64_t)(int64_t)sig << sh);
    if (sh <= -32) return 0;
    const uint32_t nsh = (uint32_t)(-sh);
    const int32_t mg = sig < 0 ? -sig : sig;
    const int64_t q = (int64_t)(mg >> nsh);
    return sig < 0 ? -q : q;
}
void dec32(uint32_t u, int32_t& e, int32_t& sig) {
    const int32_t ee = (int32_t)((u >> 23) & 0xFFu);
    if (ee == 0) {
        e = 0;
        sig = 0;
        return;
    }
    e = ee;
    const int32_t s = (int32_t)(0x800000u | (u & 0x7FFFFFu));
    sig = (u & 0x80000000u) ? -s : s;
}
double assemble_tf(uint32_t hb, uint32_t mb, uint32_t lb, int32_t g, uint64_t W, int32_t qw) {
    int32_t eh, em, el, gh, gm, gl;
    dec32(hb, eh, gh);
    dec32(mb, em, gm);
    dec32(lb, el, gl);
    if (gh == 0 && gm == 0 && gl == 0) return 0.0;
    int32_t eb = std::max(eh, std::max(em, el));
    const int64_t ch = acc64_term(gh, eh - eb + 37), cm = acc64_term(gm, em - eb + 37), cl = acc64_term(gl, el - eb + 37);
    int64_t acc = ch + cm + cl;
    if (acc == 0) {
        if (ch) eh = gh = 0;
        if (cm) em = gm = 0;
        if (cl) el = gl = 0;
        if (gh == 0 && gm == 0 && gl == 0) return 0.0;
        eb = std::max(eh, std::max(em, el));
        acc = acc64_term(gh, eh - eb + 37) + acc64_term(gm, em - eb + 37) + acc64_term(gl, el - eb + 37);
    }
    if (acc == 0) return 0.0;
    const bool neg = acc < 0;
    uint64_t A = neg ? (uint64_t)(-acc) : (uint64_t)acc;
    const int32_t shA = __builtin_clzll(A);
    A <<= shA;
    return pack_like_reference(A, W, qw + g + (eb - 187) - shA, neg);
}

}  // namespace

extern "C" {

int ozo_i_slice(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, const int32_t* delta, int p,
                int8_t* planes) {
    return ozo_i_slice_fmt(x, rows, cols, ld, col_mode, delta, p, 5, planes);
}

int ozo_i_slice_fmt(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, const int32_t* delta,
                    int p, int format, int8_t* planes) {
    const uint64_t plane = rows * cols;
    const I1Fmt f = i1_fmt(format);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; ++r)
        for (uint64_t c = 0; c < cols; ++c) {
            const uint64_t idx = col_mode ? c * rows + (uint64_t)r : (uint64_t)r * cols + c;
            make_slices(x[(uint64_t)r * ld + c], col_mode ? delta[c] : delta[r], p, f, planes + idx, plane);
        }
    return 0;
}

int ozo_i_gemm(const int8_t* ap, const int8_t* bp, int p, uint64_t M, uint64_t N, uint64_t K, int32_t* pd) {
    int bad = 0;
#pragma omp parallel for collapse(2) schedule(static) reduction(| : bad)
    for (int64_t d = 0; d < (int64_t)p; ++d)
        for (int64_t i = 0; i < (int64_t)M; ++i)
            for (uint64_t j = 0; j < N; ++j) {
                int64_t acc = 0;
                for (int64_t s = 0; s <= d; ++s) {
                    const int8_t* ar = ap + ((uint64_t)s * M + (uint64_t)i) * K;
                    const int8_t* br = bp + ((uint64_t)(d - s) * N + j) * K;
                    for (uint64_t kk = 0; kk < K; ++kk) acc += (int32_t)ar[kk] * (int32_t)br[kk];
                }
                if (acc > INT32_MAX || acc < -INT32_MAX) bad = 1;
                pd[((uint64_t)d * M + (uint64_t)i) * N + j] = (int32_t)acc;
            }
    return bad;
}

int ozo_i_recon_faithful(const int32_t* pd, int p, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                         double* c, uint64_t ldc) {
    const int L = p - 1;
    uint64_t W;
    int32_t qw;
    radix_scale(L, 254.0f, W, qw);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)M; ++i)
        for (uint64_t j = 0; j < N; ++j) {
            float a0 = 0.f, a1 = 0.f, a2 = 0.f;
            for (int d = 0; d < p; ++d) {
                if (d > 0) tf_mul_r(a0, a1, a2, 254.0f);
                // Sign-magnitude decoding into two exact FP32 values (recon_tf_i32in.cpp decode,
                // masks 0x7FFFFF00 / 0xFF of recon_reader_i32in.cpp:34-35).
                const int32_t v = pd[((uint64_t)d * M + (uint64_t)i) * N + j];
                const uint32_t mag = (uint32_t)(v < 0 ? -(int64_t)v : v);
                const uint32_t w = (v < 0 ? 0x80000000u : 0u) | mag;
                const float sgn = v > 0 ? 1.f : (v < 0 ? -1.f : 0.f);
                const float vh = fmul((float)(w & 0x7FFFFF00u), sgn), vl = fmul((float)(w & 0xFFu), sgn);
                if (d == 0) a0 = a1 = a2 = 0.f;
                tf_add(a0, a1, a2, vh);
                tf_add(a0, a1, a2, vl);
            }
            c[(uint64_t)i * ldc + j] =
                assemble_tf(f_to_bits(a0), f_to_bits(a1), f_to_bits(a2), -(dA[i] + dB[j]), W, qw);
        }
    return 0;
}

int ozo_i_recon_faithful_deferred(const int32_t* pd, int p, int format, uint64_t K, uint64_t M, uint64_t N,
                                  const int32_t* dA, const int32_t* dB, double* c, uint64_t ldc) {
    const I1Fmt f = i1_fmt(format);
    const int L = p - 1;
    uint64_t W;
    int32_t qw;
    radix_scale(L, f.radix, W, qw);
    // recon_nsmall (ozaki1/plan.hpp:428-433): leading diagonals with (d+1) K dmax^2 <= 2^24 are read with
    // one conversion; the others are split into (v & 0xFFFFFF00) and (v & 0xFF), two's complement
    // (recon_reader_i32in.cpp:34-35 with SIGNMAG = 0).
    const uint64_t per = K * (uint64_t)f.dmax * (uint64_t)f.dmax;
    const int nsingle = per ? (int)std::min<uint64_t>((1ull << 24) / per, (uint64_t)p) : 0;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)M; ++i)
        for (uint64_t j = 0; j < N; ++j) {
            float a0 = 0.f, a1 = 0.f, a2 = 0.f;
            for (int d = 0; d < p; ++d) {
                if (d > 0) {
                    if (f.pow2)
                        tf_mul_p2(a0, a1, a2, f.radix);
                    else
                        tf_mul_r(a0, a1, a2, f.radix);
                }
                const int32_t v = pd[((uint64_t)d * M + (uint64_t)i) * N + j];
                if (d < nsingle) {
                    if (d == 0) {
                        a0 = (float)v;
                        a1 = a2 = 0.f;
                    } else {
                        tf_add(a0, a1, a2, (float)v);
                    }
                    continue;
                }
                const float vh = (float)(int32_t)((uint32_t)v & 0xFFFFFF00u), vl = (float)((uint32_t)v & 0xFFu);
                if (d == 0) a0 = a1 = a2 = 0.f;
                tf_add(a0, a1, a2, vh);
                tf_add(a0, a1, a2, vl);
            }
            c[(uint64_t)i * ldc + j] =
                assemble_tf(f_to_bits(a0), f_to_bits(a1), f_to_bits(a2), -(dA[i] + dB[j]), W, qw);
        }
    return 0;
}

int ozo_i_recon_exact(const int32_t* pd, int p, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                      double* c, uint64_t ldc) {
    return ozo_i_recon_exact_fmt(pd, p, 5, M, N, dA, dB, c, ldc);
}

int ozo_i_recon_exact_fmt(const int32_t* pd, int p, int format, uint64_t M, uint64_t N, const int32_t* dA,
                          const int32_t* dB, double* c, uint64_t ldc) {
    const I1Fmt f = i1_fmt(format);
    const uint32_t radix = (uint32_t)f.radix;
    const int L = p - 1;
    uint64_t W;
    int32_t qw;
    radix_scale(L, f.radix, W, qw);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)M; ++i)
        for (uint64_t j = 0; j < N; ++j) {
            // S = sum_d P_d radix^(L-d) by Horner in exact 256-bit two's complement.
            Big S;
            bool negS = false;
            for (int d = 0; d < p; ++d) {
                if (d > 0) S = big_mul_small(S, radix);
                const int32_t v = pd[((uint64_t)d * M + (uint64_t)i) * N + j];
                Big t;
                t.w[0] = (uint32_t)(v < 0 ? -(int64_t)v : v);
                if (v < 0)
                    big_sub(S, t);
                else
                    big_add(S, t);
            }
            negS = (S.w[7] >> 31) != 0;
            if (negS) {
                Big z;
                big_sub(z, S);
                S = z;
            }
            int top = -1;
            for (int w = 7; w >= 0 && top < 0; --w)
                if (S.w[w]) top = 32 * w + 31 - __builtin_clz(S.w[w]);
            double out = 0.0;
            if (top >= 0) {
                // top 64 bits of |S| with a sticky bit, times W (64 bits), one rounding to 53 bits.
                auto bit = [&](int kbit) -> uint64_t { return kbit < 0 ? 0 : (S.w[kbit >> 5] >> (kbit & 31)) & 1u; };
                uint64_t A = 0;
                for (int kbit = top; kbit > top - 64; --kbit) A = (A << 1) | bit(kbit);
                bool sticky = false;
                for (int kbit = top - 64; kbit >= 0 && !sticky; --kbit) sticky = bit(kbit) != 0;
                const unsigned __int128 prod = (unsigned __int128)A * W;  // |S| * W / 2^(top-63)
                // product bits: leading bit at 127 or 126; keep 64 + sticky
                const uint64_t ph = (uint64_t)(prod >> 64), pl = (uint64_t)prod;
                const int lead = (ph >> 63) ? 127 : 126;
                const int sh = lead - 63;  // bits dropped below the 64-bit window
                const uint64_t win = (uint64_t)(prod >> sh);
                const bool st = sticky || (sh == 64 ? pl != 0 : (pl & ((1ull << sh) - 1)) != 0);
                // value = win * 2^(sh + (top - 63) + qw - (dA+dB))
                int32_t e2 = sh + (top - 63) + qw - (dA[i] + dB[j]);
                // round win (64 bits, leading bit 63) to 53 bits, ties to even with the sticky bit
                uint64_t mant = win >> 11;
                const uint64_t rem = win & 0x7FF;
                const bool half = rem == 0x400 && !st;
                if (rem > 0x400 || (rem == 0x400 && st) || (half && (mant & 1))) {
                    mant += 1;
                    if (mant >> 53) {
                        mant >>= 1;
                        e2 += 1;
                    }
                }
                const int lead_exp = 52 + 11 + e2;  // exponent of the leading bit of mant * 2^(11+e2)
                if (lead_exp < -1022)
                    out = 0.0;
                else if (lead_exp > 1023)
                    out = INFINITY;
                else
                    out = std::ldexp((double)mant, 11 + e2);
                if (negS) out = -out;
            }
            c[(uint64_t)i * ldc + j] = out;
        }
    return 0;
}

int ozo_i_emulate(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k, int p, int exact) {
    return ozo_i_emulate_fmt(a, b, c, m, n, k, p, 5, exact);
}

int ozo_i_emulate_fmt(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k, int p,
                      int format, int exact) {
    auto pad = [](uint64_t v, uint64_t q) { return (v + q - 1) / q * q; };
    const uint64_t M = pad(m, 64), N = pad(n, 64), K = pad(k, 32);
    std::vector<double> ap(M * K, 0.0), bp(K * N, 0.0);
    for (uint64_t i = 0; i < m; ++i) std::copy_n(a + i * k, k, ap.data() + i * K);
    for (uint64_t i = 0; i < k; ++i) std::copy_n(b + i * n, n, bp.data() + i * N);
    std::vector<int32_t> dA(M), dB(N);
    uint32_t fa = 0, fb = 0;
    const int ceil = format == 5 ? 1 : 0;  // OZ1_CEIL_MODE: INT8 rounds the maxima up, the FP formats truncate
    ozo_scale_mode(ap.data(), M, K, K, 0, -1, ceil, nullptr, dA.data(), &fa);
    ozo_scale_mode(bp.data(), K, N, N, 1, -1, ceil, nullptr, dB.data(), &fb);
    if (fa | fb) return 1;
    std::vector<int8_t> sa((uint64_t)p * M * K), sb((uint64_t)p * N * K);
    ozo_i_slice_fmt(ap.data(), M, K, K, 0, dA.data(), p, format, sa.data());
    ozo_i_slice_fmt(bp.data(), K, N, N, 1, dB.data(), p, format, sb.data());
    std::vector<int32_t> pd((uint64_t)p * M * N);
    if (ozo_i_gemm(sa.data(), sb.data(), p, M, N, K, pd.data())) return 1;
    std::vector<double> cp(M * N);
    if (exact)
        ozo_i_recon_exact_fmt(pd.data(), p, format, M, N, dA.data(), dB.data(), cp.data(), N);
    else if (format != 5)
        ozo_i_recon_faithful_deferred(pd.data(), p, format, K, M, N, dA.data(), dB.data(), cp.data(), N);
    else
        ozo_i_recon_faithful(pd.data(), p, M, N, dA.data(), dB.data(), cp.data(), N);
    for (uint64_t i = 0; i < m; ++i) std::copy_n(cp.data() + i * N, n, c + i * n);
    return 0;
}

}  // extern "C"
