// SPDX-License-Identifier: Apache-2.0
//
// Scheme II reconstruction on sm_100a: exact Chinese-remainder reconstruction of C' from the CRT
// digits k_s written by the GEMM epilogue, one rounding to FP64, exact power-of-two scale.
//
// Reference counterpart: recon_crt.cpp:219-338 with recon_crt_proc.h and the assembly of
// recon_elem.h / f64_tf.h:296-400. The reference evaluates frac = sum_s k_s/m_s mod 1 in FP32
// triple-float because its device has no FP64 (absolute error about 2^-67 for one pass), folds it in
// 128-bit fixed point and multiplies by M*2^-2b. Here the same quantity is computed without error:
//     X  = sum_s k_s * (M/m_s)                  (multiword integer, NW 32-bit words, X < S*M < 2^(32 NW);
//                                                formed two moduli at a time on the FP64 pipe, recon_pair_kernel)
//     q  = rint(top 64 bits of X * 2^t / M)     (FP64; the window margin |C'|/M <= 1/2 - 2^-31.4
//                                                makes this q = round(X/M) exactly)
//     C' = X - q*M                              (|C'| < M/2, two's complement in NW words)
//     C  = C' * 2^(2 shift - dA_i - dB_j - 2b)  (one round-to-nearest-even; below 2^-1022 -> +-0,
//                                                as pack_f64 of the reference flushes)
// One pass and two passes of the reference therefore give the same B200 result, which is at least as
// accurate as either; the tests bound |C - C_reference| componentwise.
//
// HBM traffic per output element: S bytes of digits in, 8 bytes out, plus the two deltas.
#include <algorithm>
#include <cstdlib>

#include "oztt_common.cuh"

namespace oztt {


constexpr int kMaxPairs = (OZTT_MAXS + 1) / 2;
constexpr int kPairLimbs = 6;  // M/(m_s m_t) < 2^192 in 32-bit limbs

struct ReconConst {
    uint32_t S;
    int32_t two_b, sh2;
    uint32_t M[8];
    uint32_t Q[OZTT_MAXS][8];
    double top_scale;  // 2^(32 (NW-3)) / M: X/M from the top three words of X
    // the moduli in pairs (s, t) = (2p, 2p+1), the last one alone when S is odd: u_p = (k_s m_t + k_t m_s) mod
    // m_s m_t and M/(m_s m_t) (or M/m_s) in 32-bit limbs as doubles (exact): X = sum_p u_p M/(m_s m_t) mod M
    uint32_t P;
    uint32_t pm_s[kMaxPairs], pm_t[kMaxPairs];  // the multipliers of k_t and k_s: m_s and m_t (m_s = 0 alone)
    uint32_t pm_st[kMaxPairs];                   // m_s m_t (m_s alone)
    double Qp[kMaxPairs][kPairLimbs];
    // for q in the finish of the limb sums: 2^(32 l) / M (rounded)
    double Rl[kPairLimbs];
};

template <int NW>
__device__ __forceinline__ double round_scaled(uint32_t (&y)[NW], int32_t g, const ReconConst& rc);

// Finishes one element from its column sums acc (X = sum_w acc[w] 2^(32w)).
template <int NW>
__device__ __forceinline__ double crt_finish(const uint64_t (&acc)[NW], int32_t g, const ReconConst& rc) {
    // X in words (carry the column sums).
    uint32_t x[NW];
    uint64_t cx = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        const uint64_t sx = acc[w] + cx;
        x[w] = (uint32_t)sx;
        cx = sx >> 32;
    }
    // q = round(X/M) from the top three words of X: the dropped words change X/M by less than
    // 2^(32(NW-3))/M <= 2^-40, far inside the window margin.
    const double xtop = fma(__ull2double_rn(((uint64_t)x[NW - 1] << 32) | x[NW - 2]), 4294967296.0,
                            (double)x[NW - 3]);
    const uint32_t q = (uint32_t)rint(xtop * rc.top_scale);
    // y = X - q*M modulo 2^(32 NW).
    uint32_t y[NW];
    int64_t br = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        const int64_t d = (int64_t)x[w] - (int64_t)((uint64_t)q * rc.M[w]) + br;
        y[w] = (uint32_t)d;
        br = d >> 32;
    }
    return round_scaled<NW>(y, g, rc);
}

// C' * 2^(g - 2b) rounded to nearest even, from C' in two's complement in NW words (|C'| < 2^(32 NW - 1)):
// below 2^-1022 -> +-0, as pack_f64 of the reference flushes, above the range -> +-inf.
template <int NW>
__device__ __forceinline__ double round_scaled(uint32_t (&y)[NW], int32_t g, const ReconConst& rc) {
    const bool neg = (y[NW - 1] >> 31) != 0;
    if (neg) {
        uint32_t c = 1;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const uint64_t t = (uint64_t)(~y[w]) + c;
            y[w] = (uint32_t)t;
            c = (uint32_t)(t >> 32);
        }
    }
    // |C'| in 64-bit halves, low first; the top nonzero half t0, the one below it t1 and whether any half
    // under those is nonzero, found in one upward pass (constant indices only, so the words stay in registers)
    constexpr int NH = (NW + 1) / 2;
    int hh = -1;
    uint64_t t0 = 0, t1 = 0, a = 0;
    bool sticky = false, below = false;
#pragma unroll
    for (int i = 0; i < NH; ++i) {
        const uint64_t h = ((uint64_t)(2 * i + 1 < NW ? y[2 * i + 1 < NW ? 2 * i + 1 : 0] : 0u) << 32) | y[2 * i];
        if (h) {
            hh = i;
            t0 = h;
            t1 = a;
            sticky = below;
        }
        below = below || a != 0;
        a = h;
    }
    if (hh < 0) return 0.0;
    // the top 64 bits from the leading one, and a sticky bit for every bit under them (bit 0 is far below
    // the rounding position, so setting it decides a tie without moving any other rounding)
    const int lz = __clzll((long long)t0);
    const uint64_t top64 = lz ? ((t0 << lz) | (t1 >> (64 - lz))) : t0;
    sticky = sticky || (t1 << lz) != 0;
    const double v = __ull2double_rn(top64 | (sticky ? 1ull : 0ull));  // in [2^63, 2^64]
    const int p = 64 * hh + 63 - lz;                                    // position of the leading bit
    const int lead = p + g - rc.two_b + (v == 18446744073709551616.0 ? 1 : 0);
    double r;
    if (lead < -1022)
        r = 0.0;
    else if (lead > 1023)
        r = __longlong_as_double(0x7FF0000000000000ll);
    else  // v * 2^(p - 63 + g - 2b), a normal number: add the scale to the exponent field
        r = __longlong_as_double(__double_as_longlong(v) + ((long long)(p - 63 + g - rc.two_b) << 52));
    return neg ? -r : r;
}

// Finishes one element from its limb sums. Each limb was accumulated on top of 2^52: lim[l] = 2^52 + L_l
// with L_l < 2^52 an exact integer, so the low 52 bits of its pattern are L_l, and X' = sum_l L_l 2^(32 l)
// (X' < P M, P pairs).
//   q  = rint(sum_l L_l * fl(2^(32 l)/M)) over the limbs l >= L-3 (as doubles, L_l = lim[l] - 2^52 exactly):
//        the limbs below add less than 2^52 2^(32(L-4)) / 2^(32(L-1)) = 2^-44 to X'/M (M >= 2^(32(L-1))) and
//        the rounding errors are below 2^-45, while the window margin keeps X'/M 2^-31.4 from a half-integer,
//        so q = round(X'/M) (at most P, taken from the low word of q + 1.5 2^52);
//   C' = X' - q M in L 32-bit words, two's complement: every limb difference L_l - q M_l plus the carry is
//        below 2^53 in magnitude, and |C'| <= M/2 < 2^(32 L - 1), so the words modulo 2^(32 L) hold C';
//   then the rounding of crt_finish (round_scaled): the same result bit for bit.
template <int NL, int L>
__device__ __forceinline__ double crt_finish_biased(const double (&lim)[NL], int32_t g, const ReconConst& rc) {
    constexpr double two52 = 4503599627370496.0, magic = 6755399441055744.0;  // 2^52, 1.5 * 2^52
    constexpr int LQ = L > 3 ? L - 3 : 0;
    double xm = 0.0;
#pragma unroll
    for (int l = NL - 1; l >= LQ; --l) xm = __fma_rn(__dsub_rn(lim[l], two52), rc.Rl[l], xm);
    const uint32_t q = (uint32_t)__double2loint(__dadd_rn(xm, magic));
    uint32_t y[L];
    int64_t cr = 0;
#pragma unroll
    for (int l = 0; l < L; ++l) {
        int64_t v = cr - (int64_t)((uint64_t)q * rc.M[l]);
        if (l < NL) v += (int64_t)((uint64_t)__double_as_longlong(lim[l < NL ? l : 0]) & 0xFFFFFFFFFFFFFull);
        y[l] = (uint32_t)v;
        cr = v >> 32;
    }
    return round_scaled<L>(y, g, rc);
}

// Four consecutive digits of one plane in one load (uint8 digits of the INT8 path, uint16 digits of
// the FP8 path), the first in the low bits.
template <typename D>
__device__ __forceinline__ uint64_t load_digits4(const D* p) {
    if constexpr (sizeof(D) == 1) {
        return __ldg(reinterpret_cast<const uint32_t*>(p));
    } else {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
        return ((uint64_t)v.y << 32) | v.x;
    }
}

// One thread = 4 consecutive columns of one row: the S digit words (one load per plane) are all
// requested before any is used, so the loads of a thread overlap instead of waiting one by one; then
// X = sum_s k_s (M/m_s) column by column (k_s < 2^12, so each column sum stays below 2^50); 32 bytes out.
template <int NW, typename D = uint8_t>
__global__ void __launch_bounds__(256) recon_kernel(const D* __restrict__ kp, uint64_t mp, uint64_t np,
                                                    const int32_t* __restrict__ dA, const int32_t* __restrict__ dB,
                                                    double* __restrict__ c, uint64_t m, uint64_t n, uint64_t ldc,
                                                    const ReconConst rc) {
    constexpr int BITS = 8 * (int)sizeof(D);
    constexpr uint64_t MASK = (1ull << BITS) - 1;
    const uint64_t nq = (n + 3) >> 2, total = m * nq, plane = mp * np;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t i = t / nq, j0 = (t - i * nq) << 2;
        const D* base = kp + i * np + j0;
        uint64_t kw[OZTT_MAXS];
#pragma unroll
        for (int s = 0; s < OZTT_MAXS; ++s) kw[s] = (uint32_t)s < rc.S ? load_digits4<D>(base + s * plane) : 0u;
        uint64_t acc[4][NW];
#pragma unroll
        for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int w = 0; w < NW; ++w) acc[e][w] = 0;
#pragma unroll
        for (int s = 0; s < OZTT_MAXS; ++s) {
            if ((uint32_t)s >= rc.S) break;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t k = (uint32_t)((kw[s] >> (BITS * e)) & MASK);
#pragma unroll
                for (int w = 0; w < NW; ++w) acc[e][w] += (uint64_t)k * rc.Q[s][w];
            }
        }
        const int32_t da = __ldg(dA + i);
        double* crow = c + i * ldc + j0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (j0 + e < n) {
                const int32_t g = rc.sh2 - (da + __ldg(dB + j0 + e));
                crow[e] = crt_finish<NW>(acc[e], g, rc);
            }
        }
    }
}

// The same with X accumulated on the FP64 pipe, two moduli at a time. For a pair (s, t),
// k_s (M/m_s) + k_t (M/m_t) = (k_s m_t + k_t m_s) (M/(m_s m_t)), and only X mod M matters (q is taken from
// X itself), so u = (k_s m_t + k_t m_s) mod (m_s m_t) < 2^16 -- one integer, formed on the integer pipe, against
// one multiplier: the pairs halve the FP64 work. The sum X' = sum_p u_p M/(m_s m_t) < (S/2) M is X plus a
// multiple of M. M/(m_s m_t) is held in NL 32-bit limbs; each limb sum starts at 2^52 and stays below
// 2^52 + 12 * 2^16 * 2^32 <= 2^53, exact in binary64 (every fused multiply-add of integers below 2^53 whose sum
// stays below 2^53 is exact), so the sum itself is the low 52 bits of the limb's pattern. The limbs, 32 bits
// apart, then go through the integer finish (crt_finish_biased); L is the number of M's 32-bit words.
template <int NL, int L>
__global__ void __launch_bounds__(256) recon_pair_kernel(const uint8_t* __restrict__ kp, uint64_t mp, uint64_t np,
                                                         const int32_t* __restrict__ dA,
                                                         const int32_t* __restrict__ dB, double* __restrict__ c,
                                                         uint64_t m, uint64_t n, uint64_t ldc, const ReconConst rc) {
    static_assert(NL <= L && L <= kPairLimbs, "limbs");
    const uint64_t nq = (n + 3) >> 2, total = m * nq, plane = mp * np;
    constexpr double two52 = 4503599627370496.0;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t i = t / nq, j0 = (t - i * nq) << 2;
        const uint8_t* base = kp + i * np + j0;
        uint32_t kw[OZTT_MAXS];
#pragma unroll
        for (int s = 0; s < OZTT_MAXS; ++s)
            kw[s] = (uint32_t)s < rc.S ? __ldg(reinterpret_cast<const uint32_t*>(base + s * plane)) : 0u;
        double lim[4][NL];
#pragma unroll
        for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int l = 0; l < NL; ++l) lim[e][l] = two52;
#pragma unroll
        for (int p = 0; p < kMaxPairs; ++p) {
            if ((uint32_t)p >= rc.P) break;
            const uint32_t ws = kw[2 * p], wt = kw[2 * p + 1];
            const uint32_t mm = rc.pm_st[p];
            const uint32_t mts = rc.pm_t[p] | (rc.pm_s[p] << 8);  // the multipliers as bytes: m_t, m_s, 0, 0
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                // k_s and k_t of element e in bytes 0 and 1 (bytes 2 and 3 meet zero multipliers): one byte dot
                // product gives u2 = k_s m_t + k_t m_s < 2 mm (the moduli and the digits are below 256)
                const uint32_t u2 = __dp4a(__byte_perm(ws, wt, (uint32_t)(e | ((4 + e) << 4))), mts, 0u);
                const uint32_t u = min(u2, u2 - mm);  // u2 mod mm (u2 - mm wraps above u2 when u2 < mm)
                // u as a double: 2^52 + u has u in its low significand bits; subtracting 2^52 is exact
                const double ud = __dsub_rn(__hiloint2double(0x43300000, (int)u), two52);
#pragma unroll
                for (int l = 0; l < NL; ++l) lim[e][l] = __fma_rn(ud, rc.Qp[p][l], lim[e][l]);
            }
        }
        const int32_t da = __ldg(dA + i);
        double* crow = c + i * ldc + j0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (j0 + e < n) {
                const int32_t g = rc.sh2 - (da + __ldg(dB + j0 + e));
                crow[e] = crt_finish_biased<NL, L>(lim[e], g, rc);
            }
        }
    }
}

// ---- host side -------------------------------------------------------------------------------
namespace {
struct Big {
    uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
};
Big big_mul(const Big& a, uint32_t k) {
    Big r;
    uint64_t c = 0;
    for (int i = 0; i < 8; ++i) {
        c += (uint64_t)a.w[i] * k;
        r.w[i] = (uint32_t)c;
        c >>= 32;
    }
    if (c) throw Error(OZTT_EINVAL, "recon: the product of the moduli exceeds 256 bits");
    return r;
}
int big_bits_of(const uint32_t (&w)[8]) {
    for (int i = 7; i >= 0; --i)
        if (w[i]) return 32 * i + 32 - __builtin_clz(w[i]);
    return 0;
}
int big_bits(const Big& a) {
    for (int i = 7; i >= 0; --i)
        if (a.w[i]) return 32 * i + 32 - __builtin_clz(a.w[i]);
    return 0;
}
}  // namespace

// Constants of the reconstruction for the moduli of p, the word count nw of X and the limb count nl
// of the largest M/m_s.
static ReconConst recon_const(const oztt_ii_plan& p, int& nw, int& nl) {
    ReconConst rc{};
    rc.S = (uint32_t)p.S;
    rc.two_b = 2 * p.b;
    rc.sh2 = 2 * p.shift;
    Big M;
    M.w[0] = 1;
    for (int s = 0; s < p.S; ++s) M = big_mul(M, (uint32_t)p.moduli[s]);
    for (int w = 0; w < 8; ++w) rc.M[w] = M.w[w];
    for (int s = 0; s < p.S; ++s) {
        Big q;
        q.w[0] = 1;
        for (int t = 0; t < p.S; ++t)
            if (t != s) q = big_mul(q, (uint32_t)p.moduli[t]);
        for (int w = 0; w < 8; ++w) rc.Q[s][w] = q.w[w];
    }
    // the pairs: u_p = k_s m_t + k_t m_s against M/(m_s m_t); the last modulus alone (u = k_s) when S is odd
    rc.P = (uint32_t)((p.S + 1) / 2);
    int pair_bits = 0;
    for (int q = 0; q < (int)rc.P && q < kMaxPairs; ++q) {
        const int s0 = 2 * q, s1 = 2 * q + 1;
        Big qp;
        qp.w[0] = 1;
        for (int t = 0; t < p.S; ++t)
            if (t != s0 && t != s1) qp = big_mul(qp, (uint32_t)p.moduli[t]);
        if (s1 < p.S) {
            rc.pm_s[q] = (uint32_t)p.moduli[s0];
            rc.pm_t[q] = (uint32_t)p.moduli[s1];
            rc.pm_st[q] = (uint32_t)(p.moduli[s0] * p.moduli[s1]);
        } else {
            rc.pm_s[q] = 0;
            rc.pm_t[q] = 1;
            rc.pm_st[q] = (uint32_t)p.moduli[s0];
        }
        for (int l = 0; l < kPairLimbs; ++l) rc.Qp[q][l] = (double)qp.w[l];  // limbs above 192 bits: u16 path only
        pair_bits = std::max(pair_bits, big_bits(qp));
    }
    // X = sum_s k_s (M/m_s) < S*M must fit the words, and the three top words must carry X/M to
    // better than the window margin: 32 (NW-3) <= bits(M) - 40 holds for this choice of NW.
    int sbits = 0;
    while ((1 << sbits) < p.S) ++sbits;
    nw = std::max(3, (big_bits(M) + sbits + 31) / 32);
    if (nw > 8) throw Error(OZTT_EINVAL, "recon: the product of the moduli is too large");
    if (32 * (nw - 3) > big_bits(M) - 40) throw Error(OZTT_EINVAL, "recon: the moduli product is too small");
    {
        long double Ml = 0;
        for (int w = 7; w >= 0; --w) Ml = Ml * 4294967296.0L + (long double)M.w[w];
        rc.top_scale = (double)(ldexpl(1.0L, 32 * (nw - 3)) / Ml);
    }
    // 32-bit limbs of the largest pair multiplier (at most kPairLimbs for moduli below 256)
    nl = std::max(1, (pair_bits + 31) / 32);
    {
        long double Mld = 0;
        for (int w = 7; w >= 0; --w) Mld = Mld * 4294967296.0L + (long double)M.w[w];
        for (int l = 0; l < kPairLimbs; ++l) {
            rc.Rl[l] = (double)(ldexpl(1.0L, 32 * l) / Mld);
        }
    }
    return rc;
}

static unsigned recon_blocks(uint64_t total) {
    int dev = 0, sms = 148;
    OZTT_CUDA(cudaGetDevice(&dev));
    OZTT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    return (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)sms * 16);
}

void launch_recon(const uint8_t* kp, uint64_t mp, uint64_t np, const int32_t* dA, const int32_t* dB,
                  const oztt_ii_plan& p, double* c, uint64_t m, uint64_t n, uint64_t ldc, cudaStream_t st) {
    if (p.S < 1 || p.S > OZTT_MAXS) throw Error(OZTT_EINVAL, "recon: bad number of moduli");
    if (np % 4 || (reinterpret_cast<uintptr_t>(kp) & 3)) throw Error(OZTT_EINVAL, "recon: np must be a multiple of 4");
    if (m > mp || n > np) throw Error(OZTT_EINVAL, "recon: output larger than the digit planes");
    for (int s = 0; s < p.S; ++s)
        if (p.moduli[s] < 2 || p.moduli[s] > 255) throw Error(OZTT_EINVAL, "recon: uint8 digits need moduli below 256");
    int nw = 0, nl = 0;
    const ReconConst rc = recon_const(p, nw, nl);
    const uint64_t total = m * ((n + 3) / 4);
    if (total == 0) return;
    const unsigned blocks = recon_blocks(total);
    // the FP64-pipe kernel unless oztt_set_option(OZTT_OPT_RECON_INT, 1) asks for the integer-pipe one
    // (identical results)
    const bool fp64 = option_value(OZTT_OPT_RECON_INT) != 1;
    if (fp64) {
#define OZTT_RECON_PAIR(NL_, L_) \
    case NL_ * 10 + L_: \
        recon_pair_kernel<NL_, L_><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); \
        break
        const int words_m = std::max(1, (big_bits_of(rc.M) + 31) / 32);
        switch (nl * 10 + words_m) {
            OZTT_RECON_PAIR(1, 1); OZTT_RECON_PAIR(1, 2); OZTT_RECON_PAIR(2, 2); OZTT_RECON_PAIR(2, 3);
            OZTT_RECON_PAIR(3, 3); OZTT_RECON_PAIR(3, 4); OZTT_RECON_PAIR(4, 4); OZTT_RECON_PAIR(4, 5);
            OZTT_RECON_PAIR(5, 5); OZTT_RECON_PAIR(5, 6); OZTT_RECON_PAIR(6, 6);
        default: throw Error(OZTT_EINVAL, "recon: no kernel for these moduli");
        }
#undef OZTT_RECON_PAIR
    } else {
        switch (nw) {
        case 3: recon_kernel<3><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
        case 4: recon_kernel<4><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
        case 5: recon_kernel<5><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
        case 6: recon_kernel<6><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
        case 7: recon_kernel<7><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
        default: recon_kernel<8><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
        }
    }
    OZTT_CUDA(cudaGetLastError());
}

// The same reconstruction from uint16 CRT digits (the FP8 path's moduli reach 2401), on the integer
// pipe: k_s < 2^12 times a 32-bit word of M/m_s, summed over at most 24 moduli, stays below 2^50.
void launch_recon_u16(const uint16_t* kp, uint64_t mp, uint64_t np, const int32_t* dA, const int32_t* dB,
                      const oztt_ii_plan& p, double* c, uint64_t m, uint64_t n, uint64_t ldc, cudaStream_t st) {
    if (p.S < 1 || p.S > OZTT_MAXS) throw Error(OZTT_EINVAL, "recon: bad number of moduli");
    if (np % 4 || (reinterpret_cast<uintptr_t>(kp) & 7)) throw Error(OZTT_EINVAL, "recon: np must be a multiple of 4");
    if (m > mp || n > np) throw Error(OZTT_EINVAL, "recon: output larger than the digit planes");
    for (int s = 0; s < p.S; ++s)
        if (p.moduli[s] < 2 || p.moduli[s] > 4096) throw Error(OZTT_EINVAL, "recon: moduli must be in 2..4096");
    int nw = 0, nl = 0;
    const ReconConst rc = recon_const(p, nw, nl);
    const uint64_t total = m * ((n + 3) / 4);
    if (total == 0) return;
    const unsigned blocks = recon_blocks(total);
    switch (nw) {
    case 3: recon_kernel<3, uint16_t><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
    case 4: recon_kernel<4, uint16_t><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
    case 5: recon_kernel<5, uint16_t><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
    case 6: recon_kernel<6, uint16_t><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
    case 7: recon_kernel<7, uint16_t><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
    default: recon_kernel<8, uint16_t><<<blocks, 256, 0, st>>>(kp, mp, np, dA, dB, c, m, n, ldc, rc); break;
    }
    OZTT_CUDA(cudaGetLastError());
}

}  // namespace oztt
