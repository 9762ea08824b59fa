// SPDX-License-Identifier: Apache-2.0
//
// Ozaki scheme I with INT8, FP8, BF16, FP16 or TF32 slices on sm_100a (reference: src/ozaki1.cpp:192-282).
//
//   scale        the scheme II scaling kernels with the scheme I target: delta = -1 - e
//                (OZ1_NSHIFT = -1; the maxima rounded up to BF16 for INT8, CEIL mode 1, truncated for
//                FP8, BF16, FP16 and TF32, CEIL mode 0: ozaki1/format.hpp:79-97)
//   slice        p slices per element: INT8 radix 254, digits in [-127, 127], t *= 254 by the
//                Dekker-split triple-float product (tfMulR of sfpu_tf_proc.h:108-133); FP8 radix 32,
//                digits in [-16, 16], and BF16/FP16/TF32 radix 64, digits in [-32, 32] (integers the
//                formats hold; stored as int8), t *= radix by tfMulP2 (sfpu_tf_proc.h:160-169); then
//                d = clamp(rint(t0)), t0 -= d (slice_tf_body.h). The
//                binary32 operation sequence is the reference's, with round-to-nearest-even and
//                flush-to-zero, two elements per packed-FP32 instruction, so the slices are
//                bit-identical. Layout: A [p][mp][kp], B transposed [p][np][kp].
//   diagonals    P_d = sum_{i=0..d} A_i B_{d-i}^T for d = 0..p-1 on the tensor cores (gemm_i8.cu,
//                mode 2): the concatenated GEMMs of issue_panel_diagonals with K_eff = (d+1) K,
//                exact in s32 because (L+1) K dmax^2 < 2^31 (the planner's condition for INT8; for
//                FP8 the condition of the reference's Int32 accumulation, checked here)
//   recon        S = sum_d P_d r^(L-d) exactly (Horner in 192-bit two's complement), then
//                C = S * r^-(L+2) * 2^-(dA_i + dB_j): the top 64 bits of |S| times the 64-bit
//                significand W of r^-(L+2) (the reference's long double constant, recon_scale in
//                ozaki1/plan.hpp:437-465), one round-to-nearest-even, results below 2^-1022 -> +-0.
//                The reference accumulates S in binary32 triple-float (recon_tf_i32in.cpp) and
//                assembles in a 64-bit window (assemble_tf_f64); the B200 result is within that
//                error of the reference's.
#include <algorithm>
#include <functional>
#include <string>
#include <vector>

#include "oztt_common.cuh"

namespace oztt {

namespace {

// Triple-float times 254 with Dekker splits (the constant of the split is 4097), in the
// reference's operation order, for two elements at once (packed FP32; each half rounds as the
// scalar binary32 operation would).
__device__ __forceinline__ void two_sum2(f32x2 x, f32x2 y, f32x2& s, f32x2& e) {
    s = add2(x, y);
    const f32x2 bb = sub2(s, x);
    e = add2(sub2(x, sub2(s, bb)), sub2(y, bb));
}
__device__ __forceinline__ void tf_mul_254(f32x2& x0, f32x2& x1, f32x2& x2, f32x2 nz) {
    const f32x2 r = splat2(254.0f), spl = splat2(4097.0f);
    const f32x2 lo_r = mul2(x2, r, nz);
    f32x2 t1 = mul2(x1, spl, nz);
    f32x2 t2 = sub2(t1, x1);
    f32x2 hm = sub2(t1, t2);
    f32x2 lm = sub2(x1, hm);
    hm = mul2(hm, r, nz);
    lm = mul2(lm, r, nz);
    const f32x2 P1 = add2(hm, lm);
    f32x2 kk = sub2(P1, hm);
    const f32x2 F1 = sub2(lm, kk);
    t1 = mul2(x0, spl, nz);
    t2 = sub2(t1, x0);
    f32x2 hh = sub2(t1, t2);
    f32x2 lh = sub2(x0, hh);
    hh = mul2(hh, r, nz);
    lh = mul2(lh, r, nz);
    const f32x2 P0 = add2(hh, lh);
    kk = sub2(P0, hh);
    const f32x2 F0 = sub2(lh, kk);
    const f32x2 G1 = add2(F1, lo_r);
    f32x2 sa, ea, sb, eb, r0, ec;
    two_sum2(P1, G1, sa, ea);
    two_sum2(F0, sa, sb, eb);
    two_sum2(P0, sb, r0, ec);
    const f32x2 G = add2(ea, eb);
    x0 = r0;
    x1 = add2(ec, G);
    x2 = sub2(G, sub2(x1, ec));
}

// Triple-float times a power-of-two radix (tfMulP2, sfpu_tf_proc.h:160-169): the three products are
// exact, then TwoSum(x1, x2), TwoSum(x0, s3) and FastTwoSum renormalise.
__device__ __forceinline__ void tf_mul_p2(f32x2& x0, f32x2& x1, f32x2& x2, f32x2 r, f32x2 nz) {
    x0 = mul2(x0, r, nz);
    x1 = mul2(x1, r, nz);
    x2 = mul2(x2, r, nz);
    f32x2 s3, e4, s5, e6;
    two_sum2(x1, x2, s3, e4);
    two_sum2(x0, s3, s5, e6);
    x0 = s5;
    x1 = add2(e6, e4);
    x2 = sub2(e4, sub2(x1, e6));
}

// FP64 x*2^d -> triple-float (the split of split.cu, repeated here so that this file stands alone).
__device__ __forceinline__ void tf_load1(double xv, int32_t d, float& x0, float& x1, float& x2) {
    const uint64_t bits = (uint64_t)__double_as_longlong(xv);
    const uint32_t w1 = (uint32_t)(bits >> 32), w0 = (uint32_t)bits;
    const uint32_t sgn = w1 & 0x80000000u;
    const int32_t E = (int32_t)((w1 >> 20) & 0x7FFu);
    uint32_t hi, braw, craw, s;
    if (E == 0) {
        hi = 0u;
        braw = craw = 0x4B000000u;
        s = 0u;
    } else {
        uint32_t top = 0x400000u | ((w1 & 0xFFFFFu) << 2) | (w0 >> 30);
        const uint32_t low30 = w0 & 0x3FFFFFFFu;
        int32_t rest = (int32_t)low30;
        if (low30 >= 0x20000000u) {
            top += 1u;
            rest = (int32_t)low30 - 0x40000000;
        }
        const int32_t mid = rest >> 7;
        const uint32_t lo = (uint32_t)rest & 0x7Fu;
        const int32_t elsb = E - 1075 + d;
        const bool carry = top == 0x800000u;
        const int32_t eh = elsb + (carry ? 180 : 179);
        const uint32_t mh = carry ? 0u : ((top << 1) & 0x7FFFFFu);
        const int32_t es = elsb + 134;
        hi = (eh > 0 && eh < 255) ? (sgn | ((uint32_t)eh << 23) | mh) : 0u;
        s = (es > 0 && es < 255) ? (sgn | ((uint32_t)es << 23)) : 0u;
        braw = 0x4B000000u | ((uint32_t)(mid + 0x400000) & 0x7FFFFFu);
        craw = 0x4B000000u | lo;
    }
    const float sc = __uint_as_float(s);
    x0 = __uint_as_float(hi);
    x1 = f32_mul(f32_add(__uint_as_float(braw), -12582912.0f), sc);
    x2 = f32_mul(f32_mul(f32_add(__uint_as_float(craw), -8388608.0f), sc), 0.0078125f);
}

// One slice of two elements: t *= radix (P2: 32 or 64 by tfMulP2; else 254 by tfMulR), d = clamp(rint(t0),
// +-dmax), t0 -= d. |t0| <= radix here, inside the range of rint2 (the 1.5*2^23 rounding, whose values
// equal cvt.rni's).
template <bool P2>
__device__ __forceinline__ f32x2 next_digit2(f32x2& x0, f32x2& x1, f32x2& x2, float radix, float dmax, f32x2 nz) {
    if constexpr (P2)
        tf_mul_p2(x0, x1, x2, splat2(radix), nz);
    else
        tf_mul_254(x0, x1, x2, nz);
    float da, db;
    unpk2(rint2(x0), da, db);
    da = fminf(fmaxf(da, -dmax), dmax);
    db = fminf(fmaxf(db, -dmax), dmax);
    const f32x2 d = pk2(da, db);
    x0 = sub2(x0, d);
    return d;
}

// Bytes of four integer digits in [-127, 127]: the low byte of the binary32 pattern of d + 1.5*2^23.
__device__ __forceinline__ uint32_t pack_digits4(f32x2 d01, f32x2 d23) {
    const f32x2 m = splat2(kRoundMagic);
    float f0, f1, f2, f3;
    unpk2(add2(d01, m), f0, f1);
    unpk2(add2(d23, m), f2, f3);
    const uint32_t lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x0040);
    const uint32_t hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x0040);
    return __byte_perm(lo, hi, 0x5410);
}

// 16 elements -> p slices of 16 bytes each; element states stay in registers across the slices.
template <bool P2>
__device__ __forceinline__ void slice16(const double (&x)[16], int32_t d, int p, float radix, float dmax, float nzf,
                                        int8_t* dst, uint64_t plane) {
    const f32x2 nz = splat2(nzf);
    f32x2 s0[8], s1[8], s2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        float a0, a1, a2, b0, b1, b2;
        tf_load1(x[2 * e], d, a0, a1, a2);
        tf_load1(x[2 * e + 1], d, b0, b1, b2);
        s0[e] = pk2(a0, b0);
        s1[e] = pk2(a1, b1);
        s2[e] = pk2(a2, b2);
    }
    for (int i = 0; i < p; ++i) {
        f32x2 dg[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) dg[e] = next_digit2<P2>(s0[e], s1[e], s2[e], radix, dmax, nz);
        *reinterpret_cast<uint4*>(dst + (uint64_t)i * plane) =
            make_uint4(pack_digits4(dg[0], dg[1]), pack_digits4(dg[2], dg[3]), pack_digits4(dg[4], dg[5]),
                       pack_digits4(dg[6], dg[7]));
    }
}

template <bool P2>
__global__ void __launch_bounds__(256) slice_rows_kernel(const double* __restrict__ a, uint64_t m, uint64_t k,
                                                         uint64_t lda, const int32_t* __restrict__ delta, int p,
                                                         float radix, float dmax, float nz,
                                                         int8_t* __restrict__ planes, uint64_t mp, uint64_t kp) {
    const uint64_t chunks = kp >> 4, total = mp * chunks, plane = mp * kp;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = t / chunks, k0 = (t - row * chunks) << 4;
        const bool in_row = row < m;
        const double* src = a + row * lda + k0;
        double x[16];
        if (in_row && k0 + 16 <= k && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
                const double2 v = __ldg(reinterpret_cast<const double2*>(src + e));
                x[e] = v.x;
                x[e + 1] = v.y;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] = (in_row && k0 + e < k) ? __ldg(src + e) : 0.0;
        }
        slice16<P2>(x, in_row ? __ldg(delta + row) : 0, p, radix, dmax, nz, planes + row * kp + k0, plane);
    }
}

template <bool P2>
__global__ void __launch_bounds__(256) slice_cols_kernel(const double* __restrict__ b, uint64_t k, uint64_t n,
                                                         uint64_t ldb, const int32_t* __restrict__ delta, int p,
                                                         float radix, float dmax, float nz,
                                                         int8_t* __restrict__ planes, uint64_t np, uint64_t kp) {
    const int lane = threadIdx.x & 31;
    const uint64_t col_groups = np >> 4, total = col_groups * (kp >> 5), plane = np * kp;
    for (uint64_t w = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total;
         w += ((uint64_t)gridDim.x * blockDim.x) >> 5) {
        const uint64_t cg = w % col_groups, rg = w / col_groups;
        const uint64_t col = (cg << 4) + (lane & 15), r0 = (rg << 5) + ((lane >> 4) << 4);
        const bool in_col = col < n;
        double x[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = (in_col && r0 + e < k) ? __ldg(b + (r0 + e) * ldb + col) : 0.0;
        slice16<P2>(x, in_col ? __ldg(delta + col) : 0, p, radix, dmax, nz, planes + col * kp + r0, plane);
    }
}

// ---- exact Horner reconstruction ------------------------------------------------------------
constexpr int HW = 6;  // 192-bit two's complement: |S| < 2^32 r^(p-1): < 2^152 for r = 254, p <= 16,
                       // < 2^187 for r = 32, p <= 32, < 2^188 for r = 64, p <= 27

struct HornerConst {
    int32_t p;
    uint32_t radix;  // 254 or 32
    uint64_t W;      // 64-bit significand of radix^-(L+2)
    int32_t qw;      // its exponent
};

// T: int32_t diagonals (one K block), or int64_t diagonals summed over K blocks; NW words of two's
// complement (HW = 6, or 7 for the K-blocked sums: |S| < 2^45 r^(p-1) < 2^204 for every format).
template <typename T = int32_t, int NW = HW>
__device__ __forceinline__ double horner_element(const T* pd, uint64_t plane, const HornerConst& hc, int32_t g) {
    constexpr int HW = NW;
    uint32_t s[HW];
#pragma unroll
    for (int w = 0; w < HW; ++w) s[w] = 0;
    for (int d = 0; d < hc.p; ++d) {
        // s = s * radix + P_d  (mod 2^(32 NW))
        const int64_t v = (int64_t)__ldg(pd + (uint64_t)d * plane);
        uint64_t carry = 0;
#pragma unroll
        for (int w = 0; w < HW; ++w) {
            const uint64_t t = (uint64_t)s[w] * hc.radix + carry;
            s[w] = (uint32_t)t;
            carry = t >> 32;
        }
        int64_t add = v;
#pragma unroll
        for (int w = 0; w < HW; ++w) {
            const int64_t t = (int64_t)s[w] + add;
            s[w] = (uint32_t)t;
            add = t >> 32;
        }
    }
    const bool neg = (s[HW - 1] >> 31) != 0;
    if (neg) {
        uint32_t c = 1;
#pragma unroll
        for (int w = 0; w < HW; ++w) {
            const uint64_t t = (uint64_t)(~s[w]) + c;
            s[w] = (uint32_t)t;
            c = (uint32_t)(t >> 32);
        }
    }
    int hw = -1;
#pragma unroll
    for (int w = 0; w < HW; ++w)
        if (s[w]) hw = w;
    if (hw < 0) return 0.0;
    uint32_t w0 = 0, w1 = 0, w2 = 0;
    bool sticky = false;
#pragma unroll
    for (int w = 0; w < HW; ++w) {
        if (w == hw) w0 = s[w];
        if (w == hw - 1) w1 = s[w];
        if (w == hw - 2) w2 = s[w];
        if (w < hw - 2 && s[w]) sticky = true;
    }
    const int lz = __clz(w0);
    const uint64_t top = ((uint64_t)w0 << 32) | w1;
    const uint64_t A = lz ? ((top << lz) | (w2 >> (32 - lz))) : top;
    sticky = sticky || (lz ? (w2 << lz) : w2) != 0u;
    const int topbit = 32 * hw + 31 - lz;
    // A * W, 128 bits; keep a 64-bit window with its leading bit at 63, plus a sticky bit.
    const uint64_t ph = __umul64hi(A, hc.W), pl = A * hc.W;
    const int lead = (ph >> 63) ? 127 : 126;
    const int sh = lead - 63;  // 63 or 64
    uint64_t win;
    bool st;
    if (sh == 64) {
        win = ph;
        st = sticky || pl != 0;
    } else {
        win = (ph << 1) | (pl >> 63);
        st = sticky || (pl << 1) != 0;
    }
    int32_t e2 = sh + (topbit - 63) + hc.qw + g;
    uint64_t mant = win >> 11;
    const uint64_t rem = win & 0x7FFull;
    if (rem > 0x400ull || (rem == 0x400ull && (st || (mant & 1ull)))) {
        mant += 1;
        if (mant >> 53) {
            mant >>= 1;
            e2 += 1;
        }
    }
    const int lead_exp = 63 + e2;
    double r;
    if (lead_exp < -1022)
        r = 0.0;
    else if (lead_exp > 1023)
        r = __longlong_as_double(0x7FF0000000000000ll);
    else
        r = ldexp((double)mant, 11 + e2);
    return neg ? -r : r;
}

template <typename T = int32_t, int NW = HW>
__global__ void __launch_bounds__(256) horner_kernel(const T* __restrict__ pd, uint64_t mp, uint64_t np,
                                                     const int32_t* __restrict__ dA, const int32_t* __restrict__ dB,
                                                     double* __restrict__ c, uint64_t m, uint64_t n, uint64_t ldc,
                                                     const HornerConst hc) {
    const uint64_t total = m * n, plane = mp * np;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t i = t / n, j = t - i * n;
        const int32_t g = -(__ldg(dA + i) + __ldg(dB + j));
        c[i * ldc + j] = horner_element<T, NW>(pd + i * np + j, plane, hc, g);
    }
}

// acc[i] += part[i] (the diagonals of one K block into their running 64-bit sums), four at a time.
__global__ void __launch_bounds__(256) accumulate_kernel(const int32_t* __restrict__ part, int64_t* __restrict__ acc,
                                                         uint64_t count4) {
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < count4;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const int4 v = __ldg(reinterpret_cast<const int4*>(part) + t);
        longlong2* a = reinterpret_cast<longlong2*>(acc) + 2 * t;
        longlong2 lo = a[0], hi = a[1];
        lo.x += v.x;
        lo.y += v.y;
        hi.x += v.z;
        hi.y += v.w;
        a[0] = lo;
        a[1] = hi;
    }
}

int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace

// 64-bit significand and exponent of radix^-(L+2), from the long double quotient as the reference
// forms it (exact for the power-of-two radices 32 and 64).
void scheme1_radix_scale(int p, uint32_t radix, uint64_t& W, int32_t& qw) {
    long double w = 1.0L;
    for (int i = 0; i < p + 1; ++i) w /= (long double)radix;
    int e;
    const long double f = frexpl(w, &e);
    W = (unsigned long long)ldexpl(f, 64);
    qw = e - 64;
}

// Format constants of the device stages: radix, digit bound, BF16 rounding of the maxima, and the
// largest p the exact Horner word count allows.
struct I1Dev {
    uint32_t radix;
    float dmax;
    uint32_t ceil;
    int pmax;
};
I1Dev i1_dev(int format) {
    if (format == OZTT_FMT_FP8) return {32u, 16.0f, 0u, 32};
    if (format == OZTT_FMT_INT8) return {254u, 127.0f, 1u, 16};
    // BF16, FP16, TF32: radix 64, digits +-32 (|S| < 2^32 64^26 < 2^188 for p <= 27)
    if (format == OZTT_FMT_BF16 || format == OZTT_FMT_FP16 || format == OZTT_FMT_TF32) return {64u, 32.0f, 0u, 27};
    throw Error(OZTT_EINVAL, "scheme I: the format must be INT8, FP8, BF16, FP16 or TF32");
}

void launch_slice_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta, int p, int format,
                       int8_t* planes, uint64_t mp, uint64_t kp, cudaStream_t st) {
    const I1Dev f = i1_dev(format);
    if (mp % 16 || kp % 16) throw Error(OZTT_EINVAL, "slice_rows: padded dimensions must be multiples of 16");
    const uint64_t total = mp * (kp / 16);
    if (!total) return;
    const unsigned blocks = (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 32);
    if (f.radix != 254u)
        slice_rows_kernel<true><<<blocks, 256, 0, st>>>(a, m, k, lda, delta, p, (float)f.radix, f.dmax, -0.0f, planes,
                                                        mp, kp);
    else
        slice_rows_kernel<false><<<blocks, 256, 0, st>>>(a, m, k, lda, delta, p, (float)f.radix, f.dmax, -0.0f, planes,
                                                         mp, kp);
    OZTT_CUDA(cudaGetLastError());
}

void launch_slice_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta, int p, int format,
                       int8_t* planes, uint64_t np, uint64_t kp, cudaStream_t st) {
    const I1Dev f = i1_dev(format);
    if (np % 16 || kp % 32) throw Error(OZTT_EINVAL, "slice_cols: np must be a multiple of 16 and kp of 32");
    const uint64_t warps = (np / 16) * (kp / 32);
    if (!warps) return;
    const unsigned blocks = (unsigned)std::min<uint64_t>((warps + 7) / 8, (uint64_t)sm_count() * 32);
    if (f.radix != 254u)
        slice_cols_kernel<true><<<blocks, 256, 0, st>>>(b, k, n, ldb, delta, p, (float)f.radix, f.dmax, -0.0f, planes,
                                                        np, kp);
    else
        slice_cols_kernel<false><<<blocks, 256, 0, st>>>(b, k, n, ldb, delta, p, (float)f.radix, f.dmax, -0.0f, planes,
                                                         np, kp);
    OZTT_CUDA(cudaGetLastError());
}

// pd: int32 diagonals [p][mp][np]; pd64 (instead, when not NULL): their int64 sums over K blocks.
void launch_horner(const int32_t* pd, uint64_t mp, uint64_t np, const int32_t* dA, const int32_t* dB, int p,
                   int format, double* c, uint64_t m, uint64_t n, uint64_t ldc, cudaStream_t st,
                   const int64_t* pd64 = nullptr) {
    const I1Dev f = i1_dev(format);
    if (p < 1 || p > f.pmax)
        throw Error(OZTT_EINVAL, "horner: the number of slices must be 1.." + std::to_string(f.pmax));
    HornerConst hc{};
    hc.p = p;
    hc.radix = f.radix;
    scheme1_radix_scale(p, f.radix, hc.W, hc.qw);
    const uint64_t total = m * n;
    if (!total) return;
    const unsigned blocks = (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 16);
    if (pd64)
        horner_kernel<int64_t, HW + 1><<<blocks, 256, 0, st>>>(pd64, mp, np, dA, dB, c, m, n, ldc, hc);
    else
        horner_kernel<<<blocks, 256, 0, st>>>(pd, mp, np, dA, dB, c, m, n, ldc, hc);
    OZTT_CUDA(cudaGetLastError());
}

void launch_accumulate(const int32_t* part, int64_t* acc, uint64_t count, cudaStream_t st) {
    if (count % 4) throw Error(OZTT_EINVAL, "accumulate: count must be a multiple of 4");
    const uint64_t c4 = count / 4;
    if (!c4) return;
    accumulate_kernel<<<(unsigned)std::min<uint64_t>((c4 + 255) / 256, (uint64_t)sm_count() * 16), 256, 0, st>>>(
        part, acc, c4);
    OZTT_CUDA(cudaGetLastError());
}

namespace {
uint64_t g_kblock_cap = 0;  // test hook: the largest K block (0: as exactness allows)
}

// K blocks of the diagonal products: one block over all of kp when (L+1) K dmax^2 fits the s32
// accumulators (K the reference's padded k, to 32: the further zero columns add nothing); else blocks of
// kb columns, a multiple of 128 with p kb dmax^2 <= 2^31 - 1, whose int32 diagonals are summed in int64.
uint64_t scheme1_kblock(int p, uint64_t k, uint64_t kp, uint64_t d2) {
    uint64_t kb = kp;
    if ((uint64_t)p * round_up(k, 32) > (uint64_t)INT32_MAX / d2)
        kb = std::max<uint64_t>(128, ((uint64_t)INT32_MAX / ((uint64_t)p * d2)) / 128 * 128);
    if (g_kblock_cap) kb = std::min(kb, std::max<uint64_t>(128, g_kblock_cap / 128 * 128));
    return std::min(kb, kp);
}

}  // namespace oztt

// ---- pipeline and C ABI ---------------------------------------------------------------------------
#include "runtime.cuh"

namespace oztt {

void launch_scale_rows_mode(const double* a, uint64_t m, uint64_t k, uint64_t lda, int32_t shift, uint32_t ceil,
                            int32_t* delta, uint16_t* bfmax, uint32_t* flags, cudaStream_t st);
void launch_scale_cols_mode(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift, uint32_t ceil,
                            int32_t* delta, uint16_t* bfmax, uint32_t* flags, unsigned long long* colmax,
                            cudaStream_t st);
void launch_diag_gemm(const int8_t* ap, const int8_t* bp, uint64_t mp, uint64_t np, uint64_t kp, int p,
                      int32_t* out, int* err_word, cudaStream_t st, uint64_t a_plane_rows = 0, uint64_t k0 = 0,
                      uint64_t kw = 0);

// The exact diagonal products of a band of rows_p rows (planes rows kp long; A planes a_plane_rows tall when
// nonzero): into pd (int32) in one launch, or, K blocked, block by block into pd (int32) summed into pd64.
void diag_products(const int8_t* ap, const int8_t* bp, uint64_t rows_p, uint64_t np, uint64_t kp, uint64_t kb,
                   int p, int32_t* pd, int64_t* pd64, int* err_word, cudaStream_t st, uint64_t a_plane_rows) {
    if (kb >= kp) {
        launch_diag_gemm(ap, bp, rows_p, np, kp, p, pd, err_word, st, a_plane_rows);
        return;
    }
    const uint64_t count = (uint64_t)p * rows_p * np;
    OZTT_CUDA(cudaMemsetAsync(pd64, 0, count * 8, st));
    for (uint64_t k0 = 0; k0 < kp; k0 += kb) {
        launch_diag_gemm(ap, bp, rows_p, np, kp, p, pd, err_word, st, a_plane_rows, k0, std::min(kb, kp - k0));
        launch_accumulate(pd, pd64, count, st);
    }
}

void run_i_device(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                  const oztt_i_plan& plan, cudaStream_t st, double* stage_ms) {
    const int p = plan.p, format = plan.format;
    const I1Dev f = i1_dev(format);
    if (p < 1 || p > f.pmax)
        throw Error(OZTT_EINVAL, "scheme I: the number of slices must be 1.." + std::to_string(f.pmax) +
                                     " for radix " + std::to_string(f.radix));
    if (plan.radix != (int32_t)f.radix || plan.dmax != (int32_t)f.dmax)
        throw Error(OZTT_EINVAL, "scheme I: the plan's radix and digit bound do not match its format");
    // The diagonal sums are exact in the s32 accumulators while (L+1) K dmax^2 <= 2^31 - 1 (the planner
    // guarantees it for INT8, whose K blocking the reference rejects); beyond it (FP8, BF16, FP16, TF32 with
    // a long K) the products run in K blocks summed exactly in int64, where the reference sums FP32 partial
    // products block by block (src/ozaki1.cpp:238-262).
    const uint64_t d2 = (uint64_t)f.dmax * (uint64_t)f.dmax;
    const uint64_t mp = round_up(m, 128), np = round_up(n, 256), kp = round_up(k, 128);
    const uint64_t kb = scheme1_kblock(p, k, kp, d2);
    const uint64_t P = (uint64_t)p;
    DevBuf dA(st, mp * 4), dB(st, np * 4), colmax(st, n * 8), words(st, 16);
    DevBuf sa(st, P * mp * kp), sb(st, P * np * kp), pd(st, P * mp * np * 4), pd64(st, kb < kp ? P * mp * np * 8 : 8);
    OZTT_CUDA(cudaMemsetAsync(words.p, 0, 16, st));
    uint32_t* flags = words.as<uint32_t>();
    int* gemm_err = words.as<int>() + 1;
    // The evaluator's Scheme I has no scale stage: the scaling belongs to the slice stage, as in the
    // reference's slicing programs (src/ozaki1.cpp:113-118).
    Pipeline pl;
    pl.add(kSlice, kHead, 0,
           [&] { launch_scale_rows_mode(a, m, k, k, -1, f.ceil, dA.as<int32_t>(), nullptr, flags, st); });
    pl.add(kSlice, kHead, 1, [&] {
        launch_scale_cols_mode(b, k, n, n, -1, f.ceil, dB.as<int32_t>(), nullptr, flags,
                               colmax.as<unsigned long long>(), st);
    });
    pl.add(kSlice, kHead, 2,
           [&] { launch_slice_rows(a, m, k, k, dA.as<int32_t>(), p, format, sa.as<int8_t>(), mp, kp, st); });
    pl.add(kSlice, kHead, 2,
           [&] { launch_slice_cols(b, k, n, n, dB.as<int32_t>(), p, format, sb.as<int8_t>(), np, kp, st); });
    int64_t* wide = kb < kp ? pd64.as<int64_t>() : nullptr;
    pl.add(kGemm, kGemmStep, 3, [&] {
        diag_products(sa.as<int8_t>(), sb.as<int8_t>(), mp, np, kp, kb, p, pd.as<int32_t>(), wide, gemm_err, st, 0);
    });
    pl.add(kRecon, kReconStep, 4, [&] {
        launch_horner(pd.as<int32_t>(), mp, np, dA.as<int32_t>(), dB.as<int32_t>(), p, format, c, m, n, n, st, wide);
    });
    pl.writes(dA.p, mp * 4);
    pl.writes(dB.p, np * 4);
    pl.writes(sa.p, P * mp * kp);
    pl.writes(sb.p, P * np * kp);
    pl.writes(pd.p, P * mp * np * 4);
    if (wide) pl.writes(pd64.p, P * mp * np * 8);
    pl.writes(c, m * n * 8);
    pl.out = c;
    pl.out_bytes = m * n * 8;
    pl.partial_products = (unsigned)(P * (P + 1) / 2 * ((kp + kb - 1) / kb));
    if (!run_profiled(pl, st)) pl.run(st, stage_ms, 5);
    uint32_t host_words[2] = {0, 0};
    OZTT_CUDA(cudaMemcpyAsync(host_words, words.p, 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaStreamSynchronize(st));
    check_flags(host_words[0], (int)host_words[1]);
}

void run_i_host(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                const oztt_i_plan& plan) {
    open_device(device_id);
    cudaStream_t st;
    OZTT_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    struct StreamGuard {
        cudaStream_t s;
        ~StreamGuard() {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
    } guard{st};
    DevBuf da(st, m * k * 8), db(st, k * n * 8), dc(st, m * n * 8);
    OZTT_CUDA(cudaMemcpyAsync(da.p, a, m * k * 8, cudaMemcpyHostToDevice, st));
    OZTT_CUDA(cudaMemcpyAsync(db.p, b, k * n * 8, cudaMemcpyHostToDevice, st));
    run_i_device(da.as<double>(), db.as<double>(), dc.as<double>(), m, n, k, plan, st, nullptr);
    OZTT_CUDA(cudaMemcpyAsync(c, dc.p, m * n * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaStreamSynchronize(st));
}

}  // namespace oztt

using oztt::Error;
using oztt::guarded;

// Test hook: caps the K blocks of the Scheme I diagonal products at kb columns (0: only as exactness
// requires), so that the blocked path can be checked against the unblocked one at small sizes.
extern "C" void oztt_test_scheme1_kblock(uint64_t kb) { oztt::g_kblock_cap = kb; }

extern "C" {

int oztt_i_int8_run(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                    const oztt_i_plan* plan, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !c || !plan) throw Error(OZTT_EINVAL, "null argument");
        if (!m || !n || !k) throw Error(OZTT_EINVAL, "matrix dimensions are zero");
        oztt::run_i_host(device_id, a, b, c, m, n, k, *plan);
    });
}

int oztt_i_int8_run_device(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                           uint64_t k, const oztt_i_plan* plan, void* stream, double* stage_ms, char* err,
                           size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !c || !plan) throw Error(OZTT_EINVAL, "null argument");
        if (!m || !n || !k) throw Error(OZTT_EINVAL, "matrix dimensions are zero");
        oztt::open_device(device_id);
        oztt::run_i_device(a, b, c, m, n, k, *plan, reinterpret_cast<cudaStream_t>(stream), stage_ms);
    });
}

int oztt_i_scale_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, int32_t format, int32_t* delta,
                      uint32_t* flags, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !delta || !flags || lda < k) throw Error(OZTT_EINVAL, "i_scale_rows: bad arguments");
        oztt::launch_scale_rows_mode(a, m, k, lda, -1, oztt::i1_dev(format).ceil, delta, nullptr, flags,
                                     reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_i_scale_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t format, int32_t* delta,
                      uint32_t* flags, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!b || !delta || !flags || ldb < n) throw Error(OZTT_EINVAL, "i_scale_cols: bad arguments");
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        oztt::DevBuf colmax(st, n * 8);
        oztt::launch_scale_cols_mode(b, k, n, ldb, -1, oztt::i1_dev(format).ceil, delta, nullptr, flags,
                                     colmax.as<unsigned long long>(), st);
    });
}

int oztt_i_slice_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta, int32_t p,
                      int32_t format, int8_t* planes, uint64_t mp, uint64_t kp, void* stream, char* err,
                      size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !delta || !planes || lda < k || mp < m || kp < k || p < 1 || p > 64)
            throw Error(OZTT_EINVAL, "slice_rows: bad arguments");
        oztt::launch_slice_rows(a, m, k, lda, delta, p, format, planes, mp, kp,
                                reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_i_slice_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta, int32_t p,
                      int32_t format, int8_t* planes, uint64_t np, uint64_t kp, void* stream, char* err,
                      size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!b || !delta || !planes || ldb < n || np < n || kp < k || p < 1 || p > 64)
            throw Error(OZTT_EINVAL, "slice_cols: bad arguments");
        oztt::launch_slice_cols(b, k, n, ldb, delta, p, format, planes, np, kp,
                                reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_i_diag_gemm(const int8_t* a_planes, const int8_t* b_planes, uint64_t mp, uint64_t np, uint64_t kp, int32_t p,
                     int32_t* out, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a_planes || !b_planes || !out) throw Error(OZTT_EINVAL, "diag_gemm: null argument");
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        oztt::DevBuf word(st, 16);
        OZTT_CUDA(cudaMemsetAsync(word.p, 0, 16, st));
        oztt::launch_diag_gemm(a_planes, b_planes, mp, np, kp, p, out, word.as<int>(), st);
        int host_err = 0;
        OZTT_CUDA(cudaMemcpyAsync(&host_err, word.p, 4, cudaMemcpyDeviceToHost, st));
        OZTT_CUDA(cudaStreamSynchronize(st));
        oztt::check_flags(0, host_err);
    });
}

int oztt_i_recon(const int32_t* diag, uint64_t mp, uint64_t np, const int32_t* delta_a, const int32_t* delta_b,
                 int32_t p, int32_t format, double* c, uint64_t m, uint64_t n, uint64_t ldc, void* stream, char* err,
                 size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!diag || !delta_a || !delta_b || !c || ldc < n || m > mp || n > np)
            throw Error(OZTT_EINVAL, "recon: bad arguments");
        oztt::launch_horner(diag, mp, np, delta_a, delta_b, p, format, c, m, n, ldc,
                            reinterpret_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"

// ---- Context::gemm's Scheme I call from host buffers, transfers overlapped ---------------------------
namespace oztt {

int plan_i_measured(const double* a_dev, const double* b_dev, uint64_t m, uint64_t n, uint64_t k, uint32_t slices,
                    const I1Format& f, const I1Normalization& nm, double nC, oztt_i_plan& p, std::string& err,
                    cudaStream_t st);

// The upload with the statistics measured on the way (StreamedCall), the caller's value checks from the
// measured maxima, the slice count (when not fixed) selected from those statistics and the device's model
// sums, then scale and slice, and the diagonal GEMM and the Horner evaluation in bands of about 2048 rows
// (up to 8), each band of C read back while the next is computed.
static int run_i_streamed_impl(int device_id, int32_t format, const double* a, const double* b, double* c,
                               uint64_t m, uint64_t n, uint64_t k, uint32_t slices,
                               const std::function<void(const uint64_t*, const uint64_t*)>& check, oztt_i_plan& plan,
                               std::string& err) {
    const I1Format* fp = i1_format(format);
    if (!fp) throw Error(OZTT_EINVAL, "format is unknown or was not built");
    const I1Format& fmt = *fp;
    StreamedCall call(device_id, a, b, m, n, k);
    StreamedPhases& ph = call.phases();
    cudaStream_t st = call.work();
    std::vector<uint64_t> row_max, col_max;
    std::vector<double> nrA, nrB;
    double rg[2] = {1.0, 1.0};
    const PolicyStats ps = call.upload(row_max, col_max, &nrA, &nrB, rg);
    double t = call.ms_since_start();
    check(row_max.data(), col_max.data());
    ph.check_ms = call.ms_since_start() - t;
    t = call.ms_since_start();
    const I1Normalization nm =
        i1_normalization(rg[0], rg[1], row_max.data(), col_max.data(), nrA.data(), nrB.data(), m, n, fmt);
    const int rc = plan_i_measured(call.a_dev(), call.b_dev(), m, n, k, slices, fmt, nm, ps.nC, plan, err, st);
    if (rc != OZTT_OK) return rc;
    ph.plan_ms = call.ms_since_start() - t;
    t = call.ms_since_start();
    const int p = plan.p;
    const I1Dev f = i1_dev(format);
    if (p < 1 || p > f.pmax)
        throw Error(OZTT_EINVAL, "scheme I: the number of slices must be 1.." + std::to_string(f.pmax) +
                                     " for radix " + std::to_string(f.radix));
    const uint64_t d2 = (uint64_t)f.dmax * (uint64_t)f.dmax;
    const uint64_t mp = round_up(m, 128), np = round_up(n, 256), kp = round_up(k, 128), P = (uint64_t)p;
    const uint64_t kb = scheme1_kblock(p, k, kp, d2);
    const uint64_t bands = std::min<uint64_t>(8, std::max<uint64_t>(1, mp / 2048));
    const uint64_t bm = round_up((mp + bands - 1) / bands, 128);
    const double *da = call.a_dev(), *db = call.b_dev();
    double* dc = call.c_dev();
    DevBuf dA(st, mp * 4), dB(st, np * 4), colmax(st, n * 8), words(st, 16);
    DevBuf sa(st, P * mp * kp), sb(st, P * np * kp), pd(st, P * bm * np * 4), pd64(st, kb < kp ? P * bm * np * 8 : 8);
    int64_t* wide = kb < kp ? pd64.as<int64_t>() : nullptr;
    OZTT_CUDA(cudaMemsetAsync(words.p, 0, 16, st));
    uint32_t* flags = words.as<uint32_t>();
    int* gemm_err = words.as<int>() + 1;
    launch_scale_rows_mode(da, m, k, k, -1, f.ceil, dA.as<int32_t>(), nullptr, flags, st);
    launch_scale_cols_mode(db, k, n, n, -1, f.ceil, dB.as<int32_t>(), nullptr, flags, colmax.as<unsigned long long>(),
                           st);
    launch_slice_rows(da, m, k, k, dA.as<int32_t>(), p, format, sa.as<int8_t>(), mp, kp, st);
    launch_slice_cols(db, k, n, n, dB.as<int32_t>(), p, format, sb.as<int8_t>(), np, kp, st);
    for (uint64_t r0 = 0; r0 < mp; r0 += bm) {
        const uint64_t rows_p = std::min(bm, mp - r0);
        diag_products(sa.as<int8_t>() + r0 * kp, sb.as<int8_t>(), rows_p, np, kp, kb, p, pd.as<int32_t>(), wide,
                      gemm_err, st, mp);
        if (r0 >= m) continue;
        const uint64_t rows = std::min(m, r0 + rows_p) - r0;
        launch_horner(pd.as<int32_t>(), rows_p, np, dA.as<int32_t>() + r0, dB.as<int32_t>(), p, format, dc + r0 * n,
                      rows, n, n, st, wide);
        call.band_done(r0, rows);
    }
    call.read_back(c);
    uint32_t host_words[2] = {0, 0};
    OZTT_CUDA(cudaMemcpyAsync(host_words, words.p, 8, cudaMemcpyDeviceToHost, st));
    call.finish(t);
    check_flags(host_words[0], (int)host_words[1]);
    return OZTT_OK;
}

int run_i_streamed(int device_id, int32_t format, const double* a, const double* b, double* c, uint64_t m,
                   uint64_t n, uint64_t k, uint32_t slices,
                   const std::function<void(const uint64_t*, const uint64_t*)>& check, oztt_i_plan& plan,
                   std::string& err) {
    char buf[1024];
    int inner = OZTT_OK;
    const int rc = guarded(buf, sizeof buf, [&] {
        inner = run_i_streamed_impl(device_id, format, a, b, c, m, n, k, slices, check, plan, err);
    });
    if (rc != OZTT_OK) err = buf;
    return rc != OZTT_OK ? rc : inner;
}

}  // namespace oztt
