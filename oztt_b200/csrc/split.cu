// SPDX-License-Identifier: Apache-2.0
//
// Scheme II scaling and slicing on sm_100a (HBM-bound stages of the INT8 pipeline).
//
//   scale_rows / scale_cols   max |x| per row of A / column of B on the 63-bit FP64 patterns, BF16
//                             rounded up, e = ceil(log2), delta = shift - e, range flags
//                             (reference: scale_f64_reader.cpp:129-198, scale_bits.h:33-63,
//                             expdelta.cpp:44-91)
//   split_rows / split_cols   the S residues of every element in one pass over the FP64 operand
//                             (reference: slice_f64_reader.cpp with split_f64, f64_tf.h:141-168;
//                             tf_load_f64, slice_tf_core.h:67-75; oz2_make_digits and oz2_residue,
//                             ozaki2/kernels/digits.h:80-179; modslice_int8.cpp)
//
// The residues must be bit-identical to the reference's. Its integer A' is not the rounded value of
// x*2^(b-e): only the top limb of a triple-float is rounded (|A' - X| <= 1), and for an even modulus
// the sign of a residue of m/2 depends on the binary32 rounding inside ModRound. The digit kernel
// therefore executes the reference's binary32 operation sequence with round-to-nearest-even and
// flush-to-zero (oztt_common.cuh), two elements per instruction on the packed FP32 pipe. Rounding to
// an integer uses the 1.5*2^23 addition instead of the conversion unit (a quarter-rate pipe that
// would otherwise bound the kernel); its values equal the reference's, and like the rest of the
// sequence they differ at most in the sign of a zero, which no later step can turn into a different
// number. The residue bytes come from the binary32 patterns directly, again without conversions.
//
// Layout in HBM: A is read row-major (m x k, lda) and written as S planes [S][mp][kp] int8 (K
// contiguous). B is read row-major (k x n, ldb) and written transposed, [S][np][kp] int8, so that
// both GEMM operands are K-major for the tensor cores. Padding rows/columns are written as zeros.
//
// Digit formats (the DIG variants; FP8, BF16, FP16, TF32): the same residues are then split into the one to
// three digits of their modulus (modslice_digit.cpp:193-226 with sparse_fix.h:52-72) and written as nplane
// digit planes [nplane][mp][kp] / [nplane][np][kp], plane poff_s + 0 = l (or the residue of a one-digit
// modulus), + 1 = h, + 2 = s. Every digit is an integer in [-32, 32] that the format represents exactly; the
// planes hold it as an int8, the operand type of the tensor-core products (which are then exact in s32 for
// any K).
#include <algorithm>

#include "oztt_common.cuh"

namespace oztt {

struct SplitConst {
    int32_t S;
    float nz;  // -0.0, the run-time addend of the packed multiplies (mul2 in oztt_common.cuh)
    float m[OZTT_MAXS], rinv[OZTT_MAXS];
    float c[4][OZTT_MAXS];
    // odd moduli (bit s): their residues from one exact sum of weighted digit terms (store_residues);
    // w[j][s] = the symmetric residue of 2^e mod m_s for the j-th weighted term (split_const)
    uint32_t odd;
    float w[8][OZTT_MAXS];
    // FP8 digits: radix q, fl(1/q) (stages.hpp:222-223), splitting method, first digit plane
    float q[OZTT_MAXS], qinv[OZTT_MAXS];
    int32_t mode[OZTT_MAXS], poff[OZTT_MAXS];
};

// ---- scaling -------------------------------------------------------------------------------
// |x| pattern (sign cleared) -> BF16, rounded up (ceil = 1; Scheme II and Scheme I INT8) or truncated
// (ceil = 0; Scheme I FP8, whose span 16/31 absorbs the truncation: ozaki1/format.hpp:79-97); out-of-range
// markers 0xFFC0 (Inf/NaN), 0xFF80 (nonzero below 2^-126), 0x7F80 (above BF16).
__device__ __forceinline__ uint32_t bf16_of_max(uint64_t mag, uint32_t ceil) {
    const uint32_t h = (uint32_t)(mag >> 32), l = (uint32_t)mag;
    const int32_t E = (int32_t)((h >> 20) & 0x7FFu);
    if (E == 0x7FF) return 0xFFC0u;
    const int32_t e8 = E - 896;
    if (e8 <= 0) return (h | l) ? 0xFF80u : 0u;
    if (e8 >= 255) return 0x7F80u;
    uint32_t v = ((uint32_t)e8 << 7) | ((h >> 13) & 0x7Fu);
    if (ceil && ((h & 0x1FFFu) || l)) v += 1u;
    return v;
}
// e = ceil(log2 u); flags for the markers.
__device__ __forceinline__ int32_t bf16_ceil_log2(uint32_t u, uint32_t& flags) {
    const uint32_t E = (u >> 7) & 0xFFu, mant = u & 0x7Fu;
    if (E == 0u) return 0;
    if (E == 0xFFu) {
        flags |= !(u & 0x8000u) ? 1u : (mant ? 4u : 2u);
        return 0;
    }
    return (int32_t)E - 127 + (mant ? 1 : 0);
}

__device__ __forceinline__ void finish_scale(uint64_t mx, int32_t shift, uint32_t ceil, int32_t* delta,
                                             uint16_t* bfmax, uint32_t* flags, uint64_t idx) {
    const uint32_t u = bf16_of_max(mx, ceil);
    uint32_t fl = 0;
    const int32_t e = bf16_ceil_log2(u, fl);
    delta[idx] = shift - e;
    if (bfmax) bfmax[idx] = (uint16_t)u;
    if (fl) atomicOr(flags, fl);
}

__device__ __forceinline__ uint64_t mx64(uint64_t a, uint64_t b) { return a > b ? a : b; }

// One warp per row; 16-byte loads when the row is 16-byte aligned.
__global__ void __launch_bounds__(256) scale_rows_kernel(const double* __restrict__ a, uint64_t m, uint64_t k,
                                                         uint64_t lda, int32_t shift, uint32_t ceil,
                                                         int32_t* __restrict__ delta,
                                                         uint16_t* __restrict__ bfmax, uint32_t* flags) {
    const int lane = threadIdx.x & 31;
    const uint64_t nwarps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    constexpr uint64_t MASK = 0x7FFFFFFFFFFFFFFFull;
    for (uint64_t row = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < m; row += nwarps) {
        const double* p = a + row * lda;
        uint64_t mx = 0;
        uint64_t j0 = 0;
        if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
            const ulonglong2* p2 = reinterpret_cast<const ulonglong2*>(p);
            const uint64_t n2 = k >> 1;
            uint64_t j = lane;
            for (; j + 96 < n2; j += 128) {
                const ulonglong2 v0 = __ldg(p2 + j), v1 = __ldg(p2 + j + 32), v2 = __ldg(p2 + j + 64),
                                 v3 = __ldg(p2 + j + 96);
                mx = mx64(mx, mx64(mx64(v0.x & MASK, v0.y & MASK), mx64(v1.x & MASK, v1.y & MASK)));
                mx = mx64(mx, mx64(mx64(v2.x & MASK, v2.y & MASK), mx64(v3.x & MASK, v3.y & MASK)));
            }
            for (; j < n2; j += 32) {
                const ulonglong2 v = __ldg(p2 + j);
                mx = mx64(mx, mx64(v.x & MASK, v.y & MASK));
            }
            j0 = n2 << 1;
        }
        const unsigned long long* pu = reinterpret_cast<const unsigned long long*>(p);
        for (uint64_t j = j0 + lane; j < k; j += 32) mx = mx64(mx, (uint64_t)__ldg(pu + j) & MASK);
        for (int o = 16; o; o >>= 1) mx = mx64(mx, (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)mx, o));
        if (lane == 0) finish_scale(mx, shift, ceil, delta, bfmax, flags, row);
    }
}

// Column maxima: each thread reduces one column over a chunk of rows, then atomicMax into colmax
// (non-negative FP64 patterns order like unsigned integers).
__global__ void __launch_bounds__(256) col_max_kernel(const double* __restrict__ b, uint64_t k, uint64_t n,
                                                      uint64_t ldb, uint64_t rows_per_chunk,
                                                      unsigned long long* __restrict__ colmax) {
    const uint64_t col = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= n) return;
    const uint64_t r0 = (uint64_t)blockIdx.y * rows_per_chunk, r1 = min(k, r0 + rows_per_chunk);
    const unsigned long long* pu = reinterpret_cast<const unsigned long long*>(b);
    uint64_t mx = 0;
    uint64_t r = r0;
    for (; r + 4 <= r1; r += 4) {
        const uint64_t v0 = __ldg(pu + r * ldb + col), v1 = __ldg(pu + (r + 1) * ldb + col),
                       v2 = __ldg(pu + (r + 2) * ldb + col), v3 = __ldg(pu + (r + 3) * ldb + col);
        constexpr uint64_t MASK = 0x7FFFFFFFFFFFFFFFull;
        mx = mx64(mx, mx64(mx64(v0 & MASK, v1 & MASK), mx64(v2 & MASK, v3 & MASK)));
    }
    for (; r < r1; ++r) mx = mx64(mx, (uint64_t)__ldg(pu + r * ldb + col) & 0x7FFFFFFFFFFFFFFFull);
    if (mx) atomicMax(colmax + col, (unsigned long long)mx);
}

__global__ void col_finish_kernel(const unsigned long long* __restrict__ colmax, uint64_t n, int32_t shift,
                                  uint32_t ceil,
                                  int32_t* __restrict__ delta, uint16_t* __restrict__ bfmax, uint32_t* flags) {
    const uint64_t col = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (col < n) finish_scale(colmax[col], shift, ceil, delta, bfmax, flags, col);
}

// ---- digits and residues -------------------------------------------------------------------
// FP64 -> triple-float (x0, x1, x2) of x*2^d, integer bit split then binary32 assembly.
__device__ __forceinline__ void tf_load(double xv, int32_t d, float& x0, float& x1, float& x2) {
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
        // 53-bit significand split into 30 (rounded to nearest, ties up) / 23 / 7 bits.
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

// TwoSum (Knuth) in the reference's operation order.
__device__ __forceinline__ void two_sum(float x, float y, float& s, float& e) {
    s = f32_add(x, y);
    const float bb = f32_sub(s, x);
    const float a = f32_sub(x, f32_sub(s, bb));
    e = f32_add(a, f32_sub(y, bb));
}

// The ND radix-2^20 digits of two elements, top digit first: round the top limb, subtract, multiply
// the triple by 2^20 and renormalise (TwoSum, TwoSum, FastTwoSum); every operation on both elements
// at once. |x0| < 2^21 wherever it is rounded (the top limb is below 2^shift <= 2^20, later ones
// below 2^19 + 1), inside the range of rint2.
template <int ND>
__device__ __forceinline__ void make_digits2(double xa, double xb, int32_t d, f32x2 nz, f32x2* dg) {
    float a0, a1, a2, b0, b1, b2;
    tf_load(xa, d, a0, a1, a2);
    tf_load(xb, d, b0, b1, b2);
    f32x2 x0 = pk2(a0, b0), x1 = pk2(a1, b1), x2 = pk2(a2, b2);
    const f32x2 radix = splat2(1048576.0f);
#pragma unroll
    for (int i = 0; i < ND; ++i) {
        if (i > 0) {
            x0 = mul2(x0, radix, nz);
            x1 = mul2(x1, radix, nz);
            x2 = mul2(x2, radix, nz);
            // TwoSum(x1, x2) -> (s3, e4); TwoSum(x0, s3) -> (s5, e6)
            const f32x2 s3 = add2(x1, x2);
            f32x2 bb = sub2(s3, x1);
            const f32x2 e4 = add2(sub2(x1, sub2(s3, bb)), sub2(x2, bb));
            const f32x2 s5 = add2(x0, s3);
            bb = sub2(s5, x0);
            const f32x2 e6 = add2(sub2(x0, sub2(s5, bb)), sub2(s3, bb));
            x0 = s5;
            x1 = add2(e6, e4);
            x2 = sub2(e4, sub2(x1, e6));
        }
        const f32x2 dig = rint2(x0);
        dg[i] = dig;
        x0 = sub2(x0, dig);
    }
}

// ModRound d - rint(d*rinv)*m for two values; the products and sums are exact integers below 2^22.
__device__ __forceinline__ f32x2 mod_round2(f32x2 d, f32x2 negm, f32x2 rinv, f32x2 nz) {
    return fma2(rint2(mul2(d, rinv, nz)), negm, d);
}

// ModRound of an exact integer x for an odd m, with the product and the rounding to an integer in one fused
// operation (x * fl(1/m) + 1.5*2^23, then - 1.5*2^23): x * fl(1/m) is within 1/(4m) of x/m, and x/m is at least
// 1/(2m) from a half-integer when m is odd, so rounding once or twice gives the same quotient, and the
// residue x - q m is exact. (The even modulus keeps mod_round2, whose two roundings decide its ties.)
__device__ __forceinline__ f32x2 mod_round2_odd(f32x2 x, f32x2 negm, f32x2 rinv) {
    const f32x2 mg = splat2(kRoundMagic);
    return fma2(sub2(fma2(x, rinv, mg), mg), negm, x);
}

// Residues of A' from its digits (top first), the reference's chain; products of a reduced digit
// and a weight, and the partial sums, are exact integers below 2^22.
template <int ND>
__device__ __forceinline__ f32x2 residue2(const f32x2* dg, f32x2 negm, f32x2 ri, f32x2 c0, f32x2 c1, f32x2 c2,
                                          f32x2 c3, f32x2 nz) {
    f32x2 acc = fma2(mod_round2(dg[ND - 2], negm, ri, nz), c0, dg[ND - 1]);
    acc = fma2(mod_round2(dg[ND - 3], negm, ri, nz), c1, acc);
    if constexpr (ND >= 4) {
        acc = mod_round2(acc, negm, ri, nz);
        if constexpr (ND >= 5) {
            acc = fma2(mod_round2(dg[0], negm, ri, nz), c3, acc);
            acc = mod_round2(acc, negm, ri, nz);
        }
        acc = fma2(mod_round2(dg[ND - 4], negm, ri, nz), c2, acc);
    }
    return mod_round2(acc, negm, ri, nz);
}

// The low bytes of four integer-valued residues r + 1.5*2^23 (binary32 patterns whose low 22 bits are
// the two's complement integer), packed into one word, first residue in the low byte.
__device__ __forceinline__ uint32_t pack4(f32x2 r01, f32x2 r23) {
    const f32x2 m = splat2(kRoundMagic);
    float f0, f1, f2, f3;
    unpk2(add2(r01, m), f0, f1);
    unpk2(add2(r23, m), f2, f3);
    const uint32_t lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x0040);
    const uint32_t hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x0040);
    return __byte_perm(lo, hi, 0x5410);
}

// Writes the S residue planes of 16 elements whose digits are in dg (8 pairs x ND) to dst + s*plane.
//
// An even modulus follows the reference's chain (residue2), whose binary32 roundings decide the sign of a
// residue of m/2. For an odd modulus the residue is the symmetric one, r in [-(m-1)/2, (m-1)/2], whatever the
// chain; it is computed here with fewer operations, as one exact integer sum and one ModRound: A' = sum_i
// d_i 2^(20 (ND-1-i)), and every digit whose product with a weight 2^e mod m (symmetric, |.| <= 127) could
// leave the exact range of binary32 is first split into 10-bit halves (d = 1024 h + l, h = rint(d/1024),
// both exact). The lower digits are below 2^19 + 1, so they are split; the top digit is below 2^shift and
// is split only when shift > 16 (TOP): with it whole the sum is below 2^16 * 127 + 6 * 513 * 127 + 2^19 + 1
// < 2^24, exact. ModRound of that exact integer gives the symmetric residue (x * fl(1/m) is within 1/(4m)
// of x/m, and x/m is at least 1/(2m) from a half-integer when m is odd). The residues are the reference's,
// bit for bit. The terms of a pair: the top digit or its halves, the halves of the middle digits, the last
// digit (weight 1); NT of them carry a weight w[j][s] (split_const).
template <int ND, bool TOP>
struct ResidueTerms {
    static constexpr int NT = TOP ? 2 * (ND - 1) : 2 * ND - 3;
};

// The terms of pairs E0 .. E0+NPAIR-1, then their residues: 2*NPAIR bytes per plane at dst + s*plane +
// 2*E0. Rows of A store 8 bytes twice (fewer live registers); the transposed planes of B store 16 bytes
// at once (a whole half sector per lane).
template <int ND, bool TOP, int E0, int NPAIR>
__device__ __forceinline__ void store_residues_part(const f32x2 (&dg)[8][ND], const SplitConst& sc, int8_t* dst,
                                                    uint64_t plane) {
    const f32x2 nz = splat2(sc.nz);
    constexpr int NT = ResidueTerms<ND, TOP>::NT;
    constexpr int I0 = TOP ? 0 : 1;  // the first digit that is split
    f32x2 t[NPAIR][NT + 1];
    {
        const f32x2 inv = splat2(0.0009765625f), neg = splat2(-1024.0f);
#pragma unroll
        for (int e = 0; e < NPAIR; ++e) {
            if constexpr (!TOP) t[e][0] = dg[E0 + e][0];
#pragma unroll
            for (int i = I0; i < ND - 1; ++i) {
                const f32x2 h = rint2(mul2(dg[E0 + e][i], inv, nz));
                t[e][2 * i - I0] = h;
                t[e][2 * i - I0 + 1] = fma2(h, neg, dg[E0 + e][i]);
            }
            t[e][NT] = dg[E0 + e][ND - 1];
        }
    }
    const f32x2 k1024 = splat2(1024.0f);
    for (int s = 0; s < sc.S; ++s) {
        const f32x2 negm = splat2(-sc.m[s]), ri = splat2(sc.rinv[s]);
        f32x2 r[NPAIR];
        if ((sc.odd >> s) & 1u) {
#pragma unroll
            for (int e = 0; e < NPAIR; ++e) {
                f32x2 acc = t[e][NT];
#pragma unroll
                for (int j = 0; j < NT; ++j) acc = fma2(t[e][j], splat2(sc.w[j][s]), acc);
                r[e] = mod_round2_odd(acc, negm, ri);
            }
        } else {
            const f32x2 c0 = splat2(sc.c[0][s]), c1 = splat2(sc.c[1][s]), c2 = splat2(sc.c[2][s]),
                        c3 = splat2(sc.c[3][s]);
#pragma unroll
            for (int e = 0; e < NPAIR; ++e) {
                f32x2 d[ND];
                if constexpr (!TOP) d[0] = t[e][0];
#pragma unroll
                for (int i = I0; i < ND - 1; ++i) d[i] = fma2(t[e][2 * i - I0], k1024, t[e][2 * i - I0 + 1]);
                d[ND - 1] = t[e][NT];
                r[e] = residue2<ND>(d, negm, ri, c0, c1, c2, c3, nz);
            }
        }
        int8_t* o = dst + (uint64_t)s * plane + 2 * E0;
        if constexpr (NPAIR == 4)
            *reinterpret_cast<uint2*>(o) = make_uint2(pack4(r[0], r[1]), pack4(r[2], r[3]));
        else
            *reinterpret_cast<uint4*>(o) =
                make_uint4(pack4(r[0], r[1]), pack4(r[2], r[3]), pack4(r[4], r[5]), pack4(r[6], r[7]));
    }
}

template <int ND, bool TOP, bool ROWS>
__device__ __forceinline__ void store_residues(const f32x2 (&dg)[8][ND], const SplitConst& sc, int8_t* dst,
                                               uint64_t plane) {
    if constexpr (ROWS) {
        store_residues_part<ND, TOP, 0, 4>(dg, sc, dst, plane);
        store_residues_part<ND, TOP, 4, 4>(dg, sc, dst, plane);
    } else {
        store_residues_part<ND, TOP, 0, 8>(dg, sc, dst, plane);
    }
}

// ---- FP8 digits ------------------------------------------------------------------------------
// Sparse-digit fix of one element (method (E), sparse_fix.h:52-72): an odd digit of magnitude 17 or
// more is moved by q into the even integers of e4m3 (l -= sgn(l) q carrying sgn(l) into h; then
// h -= sgn(h) q, which q^2 = 0 (mod m) allows). Parity is the units bit of |x| + 2^23. Exact.
__device__ __forceinline__ void sqs_fix(float& l, float& h, float q) {
    const float al = fabsf(l);
    if (al > 16.5f && (__float_as_uint(f32_add(al, 8388608.0f)) & 1u)) {
        if (l < 0.0f) {
            l = f32_add(l, q);
            h = f32_sub(h, 1.0f);
        } else {
            l = f32_sub(l, q);
            h = f32_add(h, 1.0f);
        }
    }
    const float ah = fabsf(h);
    if (ah > 16.5f && (__float_as_uint(f32_add(ah, 8388608.0f)) & 1u)) h = h < 0.0f ? f32_add(h, q) : f32_sub(h, q);
}

// Writes the digit planes of 16 elements (8 pairs x ND digits of A') for every modulus.
//   one digit (ONE): the residue r itself (|r| <= 32)
//   rounding to nearest (SQ, WIDE, SQS): h = rint(fl(r * qinv)), l = r - q h (exact); SQS then sqs_fix
//   Karatsuba (KAR): h = rint((r + sgn(r) (q/2 - 1/2)) * qinv), l = r - q h, s = h + l, sgn(+-0) = +1
// The products r*qinv are single roundings like the reference's MulS; everything else is exact.
template <int ND>
__device__ __forceinline__ void store_digits(const f32x2 (&dg)[8][ND], const SplitConst& sc, int8_t* dst,
                                             uint64_t plane) {
    const f32x2 nz = splat2(sc.nz);
    for (int s = 0; s < sc.S; ++s) {
        const f32x2 negm = splat2(-sc.m[s]), ri = splat2(sc.rinv[s]);
        const f32x2 c0 = splat2(sc.c[0][s]), c1 = splat2(sc.c[1][s]), c2 = splat2(sc.c[2][s]),
                    c3 = splat2(sc.c[3][s]);
        const float q = sc.q[s];
        const f32x2 qi = splat2(sc.qinv[s]), negq = splat2(-q);
        const int mode = sc.mode[s];
        f32x2 l[8], h[8], t[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const f32x2 r = residue2<ND>(dg[e], negm, ri, c0, c1, c2, c3, nz);
            if (mode == OZTT_SPLIT_ONE) {
                l[e] = r;
            } else if (mode == OZTT_SPLIT_KAR) {
                float r0, r1;
                unpk2(r, r0, r1);
                const float half = q * 0.5f - 0.5f;
                const f32x2 off = pk2(r0 < 0.0f ? -half : half, r1 < 0.0f ? -half : half);
                h[e] = rint2(mul2(add2(r, off), qi, nz));
                l[e] = fma2(h[e], negq, r);
                t[e] = add2(h[e], l[e]);
            } else {
                h[e] = rint2(mul2(r, qi, nz));
                l[e] = fma2(h[e], negq, r);
                if (mode == OZTT_SPLIT_SQS) {
                    float l0, l1, h0, h1;
                    unpk2(l[e], l0, l1);
                    unpk2(h[e], h0, h1);
                    sqs_fix(l0, h0, q);
                    sqs_fix(l1, h1, q);
                    l[e] = pk2(l0, l1);
                    h[e] = pk2(h0, h1);
                }
            }
        }
        int8_t* p = dst + (uint64_t)sc.poff[s] * plane;
        *reinterpret_cast<uint4*>(p) =
            make_uint4(pack4(l[0], l[1]), pack4(l[2], l[3]), pack4(l[4], l[5]), pack4(l[6], l[7]));
        if (mode == OZTT_SPLIT_ONE) continue;
        *reinterpret_cast<uint4*>(p + plane) =
            make_uint4(pack4(h[0], h[1]), pack4(h[2], h[3]), pack4(h[4], h[5]), pack4(h[6], h[7]));
        if (mode == OZTT_SPLIT_KAR)
            *reinterpret_cast<uint4*>(p + 2 * plane) =
                make_uint4(pack4(t[0], t[1]), pack4(t[2], t[3]), pack4(t[4], t[5]), pack4(t[6], t[7]));
    }
}

// What a split kernel stores: residues with the top digit split (kTopSplit) or whole (kTopWhole), or the
// digit planes of the digit formats (kDigits).
constexpr int kTopSplit = 0, kTopWhole = 1, kDigits = 2;

template <int ND, int MODE, bool ROWS>
__device__ __forceinline__ void store_planes(const f32x2 (&dg)[8][ND], const SplitConst& sc, int8_t* dst,
                                             uint64_t plane) {
    if constexpr (MODE == kDigits)
        store_digits<ND>(dg, sc, dst, plane);
    else
        store_residues<ND, MODE == kTopSplit, ROWS>(dg, sc, dst, plane);
}

// A: one thread = 16 consecutive elements of one row; the planes are `plane` bytes apart (mp * kp, or more
// for a band of the rows of taller planes). (ND = 3 with the top digit whole, the widths of the
// usual plans: at most 85 registers, so that three blocks share an SM -- measured 2.78 against 3.08 ms at
// 16384^2 x 17 moduli with two.)
template <int ND, int MODE>
__global__ void __launch_bounds__(256, (ND == 3 && MODE == kTopWhole) ? 3 : 1) split_rows_kernel(const double* __restrict__ a, uint64_t m, uint64_t k,
                                                         uint64_t lda, const int32_t* __restrict__ delta,
                                                         int8_t* __restrict__ planes, uint64_t mp, uint64_t kp,
                                                         uint64_t plane, const SplitConst sc) {
    const uint64_t chunks = kp >> 4, total = mp * chunks;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = t / chunks, k0 = (t - row * chunks) << 4;
        double x[16];
        const bool in_row = row < m;
        const double* p = a + row * lda + k0;
        if (in_row && k0 + 16 <= k && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
                const double2 v = __ldg(reinterpret_cast<const double2*>(p + e));
                x[e] = v.x;
                x[e + 1] = v.y;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] = (in_row && k0 + e < k) ? __ldg(p + e) : 0.0;
        }
        const int32_t d = in_row ? __ldg(delta + row) : 0;
        f32x2 dg[8][ND];
#pragma unroll
        for (int e = 0; e < 8; ++e) make_digits2<ND>(x[2 * e], x[2 * e + 1], d, splat2(sc.nz), dg[e]);
        store_planes<ND, MODE, true>(dg, sc, planes + row * kp + k0, plane);
    }
}

// B: a warp covers 16 columns x 32 rows of B; lane l takes column (l & 15) and the 16 rows of half
// (l >> 4), so lanes l and l+16 write the two halves of one 32-byte sector of the transposed plane. The
// planes are `plane` bytes apart (np * kp, or more for a block of the columns of wider planes).
template <int ND, int MODE>
__global__ void __launch_bounds__(256) split_cols_kernel(const double* __restrict__ b, uint64_t k, uint64_t n,
                                                         uint64_t ldb, const int32_t* __restrict__ delta,
                                                         int8_t* __restrict__ planes, uint64_t np, uint64_t kp,
                                                         uint64_t plane, const SplitConst sc) {
    const int lane = threadIdx.x & 31;
    const uint64_t col_groups = np >> 4, row_groups = kp >> 5, total = col_groups * row_groups;
    for (uint64_t w = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total;
         w += ((uint64_t)gridDim.x * blockDim.x) >> 5) {
        const uint64_t cg = w % col_groups, rg = w / col_groups;
        const uint64_t col = (cg << 4) + (lane & 15), r0 = (rg << 5) + ((lane >> 4) << 4);
        const bool in_col = col < n;
        double x[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = (in_col && r0 + e < k) ? __ldg(b + (r0 + e) * ldb + col) : 0.0;
        const int32_t d = in_col ? __ldg(delta + col) : 0;
        f32x2 dg[8][ND];
#pragma unroll
        for (int e = 0; e < 8; ++e) make_digits2<ND>(x[2 * e], x[2 * e + 1], d, splat2(sc.nz), dg[e]);
        store_planes<ND, MODE, false>(dg, sc, planes + col * kp + r0, plane);
    }
}

// B transposed (bt[j][i] = b[i][j], k x n to n x k) through 32 x 32 tiles in shared memory, so that B's columns
// are split as rows (split_rows_kernel), whose loads and stores are contiguous, instead of through the column
// kernel's strided loads and scattered 16-byte stores. The maxima of |B|'s columns (B^T's rows) are taken on
// the way, so that B^T needs no separate pass for its scale (col_finish_kernel turns them into deltas and
// flags, as scale_rows_kernel would). Blocks of 32 x 8 threads take 32 columns over kTransposeTiles tiles of
// 32 rows, 4 elements per thread and tile; at the store a warp's lanes hold the
// 32 rows of one column of a tile, four columns per warp, so each column's maximum is kept per lane across
// the tiles, reduced across the warp once and given to one atomicMax per block (non-negative FP64 patterns
// order like unsigned integers, NaN patterns above infinity, as in scale_rows_kernel).
constexpr int kTransposeTiles = 2;
__global__ void __launch_bounds__(256) transpose_max_kernel(const double* __restrict__ b, uint64_t k, uint64_t n,
                                                            uint64_t ldb, double* __restrict__ bt,
                                                            unsigned long long* __restrict__ colmax) {
    __shared__ double tile[32][33];
    constexpr uint64_t MASK = 0x7FFFFFFFFFFFFFFFull;
    const uint64_t c0 = (uint64_t)blockIdx.x * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;
    uint64_t mx[4] = {0, 0, 0, 0};
    for (int it = 0; it < kTransposeTiles; ++it) {
        const uint64_t r0 = ((uint64_t)blockIdx.y * kTransposeTiles + it) * 32;
        if (r0 >= k) break;  // the same for the whole block
        if (it) __syncthreads();  // the previous tile read out before it is overwritten
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
            const uint64_t r = r0 + ty + j, c = c0 + tx;
            tile[ty + j][tx] = (r < k && c < n) ? __ldg(b + r * ldb + c) : 0.0;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
            const uint64_t c = c0 + ty + j, r = r0 + tx;
            const double v = tile[tx][ty + j];
            mx[j >> 3] = mx64(mx[j >> 3], (uint64_t)__double_as_longlong(v) & MASK);
            if (c < n && r < k) bt[c * k + r] = v;
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint64_t v = mx[j];
        for (int o = 16; o; o >>= 1) v = mx64(v, (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v, o));
        const uint64_t c = c0 + ty + 8 * j;
        if (tx == 0 && v && c < n) atomicMax(colmax + c, (unsigned long long)v);
    }
}

// ---- host side -------------------------------------------------------------------------------
static int device_sms() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

// The residue mode of a plan: the top digit whole when it is below 2^16 (shift <= 16; store_residues).
static int residue_mode(const oztt_ii_plan& p) { return p.shift <= 16 ? kTopWhole : kTopSplit; }

// 2^e mod m as the symmetric residue in [-(m-1)/2, m/2].
static float pow2_mod_symmetric(int e, int32_t m) {
    int64_t r = 1 % m;
    for (int t = 0; t < e; ++t) r = (r * 2) % m;
    if (r > m / 2) r -= m;
    return (float)r;
}

static SplitConst split_const(const oztt_ii_plan& p) {
    SplitConst sc{};
    sc.S = p.S;
    sc.nz = -0.0f;
    const bool top_whole = residue_mode(p) == kTopWhole;
    for (int s = 0; s < p.S; ++s) {
        sc.m[s] = (float)p.moduli[s];
        sc.rinv[s] = p.rinv[s];
        for (int j = 0; j < 4; ++j) sc.c[j][s] = p.c[j][s];
        const int32_t m = p.moduli[s];
        if (m % 2 == 1 && p.nd >= 3 && p.nd <= 5) {
            sc.odd |= 1u << s;
            // the weighted terms of store_residues_part, top first: the top digit (exponent 20 (nd-1)) or
            // its halves, then the halves of digits 1 .. nd-2 (exponents 20 (nd-1-i) + 10 and 20 (nd-1-i))
            int j = 0;
            if (top_whole) sc.w[j++][s] = pow2_mod_symmetric(20 * (p.nd - 1), m);
            for (int i = top_whole ? 1 : 0; i < p.nd - 1; ++i) {
                sc.w[j++][s] = pow2_mod_symmetric(20 * (p.nd - 1 - i) + 10, m);
                sc.w[j++][s] = pow2_mod_symmetric(20 * (p.nd - 1 - i), m);
            }
        }
    }
    return sc;
}

void launch_scale_rows_mode(const double* a, uint64_t m, uint64_t k, uint64_t lda, int32_t shift, uint32_t ceil,
                            int32_t* delta, uint16_t* bfmax, uint32_t* flags, cudaStream_t st) {
    if (m == 0) return;
    const uint64_t warps_needed = m;
    const uint64_t blocks = std::min<uint64_t>((warps_needed + 7) / 8, (uint64_t)device_sms() * 16);
    scale_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(a, m, k, lda, shift, ceil, delta, bfmax, flags);
    OZTT_CUDA(cudaGetLastError());
}

void launch_scale_cols_mode(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift, uint32_t ceil,
                            int32_t* delta, uint16_t* bfmax, uint32_t* flags, unsigned long long* colmax,
                            cudaStream_t st) {
    if (n == 0) return;
    OZTT_CUDA(cudaMemsetAsync(colmax, 0, n * sizeof(unsigned long long), st));
    const uint64_t colblocks = (n + 255) / 256;
    // Enough row chunks to give every SM several blocks.
    const uint64_t want = std::max<uint64_t>(1, ((uint64_t)device_sms() * 8 + colblocks - 1) / colblocks);
    const uint64_t chunks = std::min<uint64_t>(std::min<uint64_t>(want, 65535), std::max<uint64_t>(1, k));
    const uint64_t rows_per_chunk = (k + chunks - 1) / chunks;
    const uint64_t nchunks = (k + rows_per_chunk - 1) / rows_per_chunk;
    if (k > 0) {
        col_max_kernel<<<dim3((unsigned)colblocks, (unsigned)nchunks), 256, 0, st>>>(b, k, n, ldb, rows_per_chunk,
                                                                                   colmax);
        OZTT_CUDA(cudaGetLastError());
    }
    col_finish_kernel<<<(unsigned)colblocks, 256, 0, st>>>(colmax, n, shift, ceil, delta, bfmax, flags);
    OZTT_CUDA(cudaGetLastError());
}

void launch_scale_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, int32_t shift, int32_t* delta,
                       uint16_t* bfmax, uint32_t* flags, cudaStream_t st) {
    launch_scale_rows_mode(a, m, k, lda, shift, 1u, delta, bfmax, flags, st);
}

// B^T = B transposed into bt (n x k), and the exponent deltas and flags of B's columns (B^T's rows) from the
// maxima taken on the way; colmax: n words of scratch.
void launch_transpose_scale(const double* b, uint64_t k, uint64_t n, uint64_t ldb, double* bt, int32_t shift,
                            int32_t* delta, uint32_t* flags, unsigned long long* colmax, cudaStream_t st) {
    if (n == 0) return;
    const uint64_t rows_per_block = 32ull * kTransposeTiles;
    if ((n + 31) / 32 > 0x7FFFFFFFull || (k + rows_per_block - 1) / rows_per_block > 65535)
        throw Error(OZTT_EINVAL, "transpose: too large");
    OZTT_CUDA(cudaMemsetAsync(colmax, 0, n * sizeof(unsigned long long), st));
    if (k > 0) {
        transpose_max_kernel<<<dim3((unsigned)((n + 31) / 32), (unsigned)((k + rows_per_block - 1) / rows_per_block)),
                               dim3(32, 8), 0, st>>>(b, k, n, ldb, bt, colmax);
        OZTT_CUDA(cudaGetLastError());
    }
    col_finish_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(colmax, n, shift, 1u, delta, nullptr, flags);
    OZTT_CUDA(cudaGetLastError());
}

void launch_scale_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift, int32_t* delta,
                       uint16_t* bfmax, uint32_t* flags, unsigned long long* colmax, cudaStream_t st) {
    launch_scale_cols_mode(b, k, n, ldb, shift, 1u, delta, bfmax, flags, colmax, st);
}

template <int MODE>
static void split_rows_nd(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta, int nd,
                          const SplitConst& sc, int8_t* planes, uint64_t mp, uint64_t kp, uint64_t plane_rows,
                          cudaStream_t st) {
    if (mp % 16 || kp % 16) throw Error(OZTT_EINVAL, "split_rows: padded dimensions must be multiples of 16");
    if (plane_rows < mp) throw Error(OZTT_EINVAL, "split_rows: band taller than its planes");
    const uint64_t plane = plane_rows * kp;
    const uint64_t total = mp * (kp / 16);
    const unsigned blocks = (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)device_sms() * 32);
    if (total == 0) return;
    switch (nd) {
    case 3: split_rows_kernel<3, MODE><<<blocks, 256, 0, st>>>(a, m, k, lda, delta, planes, mp, kp, plane, sc); break;
    case 4: split_rows_kernel<4, MODE><<<blocks, 256, 0, st>>>(a, m, k, lda, delta, planes, mp, kp, plane, sc); break;
    case 5: split_rows_kernel<5, MODE><<<blocks, 256, 0, st>>>(a, m, k, lda, delta, planes, mp, kp, plane, sc); break;
    default: throw Error(OZTT_EINVAL, "split: the number of digits must be 3, 4 or 5");
    }
    OZTT_CUDA(cudaGetLastError());
}

template <int MODE>
static void split_cols_nd(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta, int nd,
                          const SplitConst& sc, int8_t* planes, uint64_t np, uint64_t kp, uint64_t plane_rows,
                          cudaStream_t st) {
    if (np % 16 || kp % 32) throw Error(OZTT_EINVAL, "split_cols: np must be a multiple of 16 and kp of 32");
    if (plane_rows < np) throw Error(OZTT_EINVAL, "split_cols: block wider than its planes");
    const uint64_t warps = (np / 16) * (kp / 32);
    if (warps == 0) return;
    const unsigned blocks = (unsigned)std::min<uint64_t>((warps + 7) / 8, (uint64_t)device_sms() * 32);
    const uint64_t plane = plane_rows * kp;
    switch (nd) {
    case 3: split_cols_kernel<3, MODE><<<blocks, 256, 0, st>>>(b, k, n, ldb, delta, planes, np, kp, plane, sc); break;
    case 4: split_cols_kernel<4, MODE><<<blocks, 256, 0, st>>>(b, k, n, ldb, delta, planes, np, kp, plane, sc); break;
    case 5: split_cols_kernel<5, MODE><<<blocks, 256, 0, st>>>(b, k, n, ldb, delta, planes, np, kp, plane, sc); break;
    default: throw Error(OZTT_EINVAL, "split: the number of digits must be 3, 4 or 5");
    }
    OZTT_CUDA(cudaGetLastError());
}

// plane_rows: when nonzero, planes points at row r0 of planes that are plane_rows tall (rows r0 .. r0+mp-1 of
// taller planes: a band of A's rows, split as it lands).
void launch_split_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta,
                       const oztt_ii_plan& p, int8_t* planes, uint64_t mp, uint64_t kp, cudaStream_t st,
                       uint64_t plane_rows) {
    const uint64_t pr = plane_rows ? plane_rows : mp;
    if (residue_mode(p) == kTopWhole)
        split_rows_nd<kTopWhole>(a, m, k, lda, delta, p.nd, split_const(p), planes, mp, kp, pr, st);
    else
        split_rows_nd<kTopSplit>(a, m, k, lda, delta, p.nd, split_const(p), planes, mp, kp, pr, st);
}

// plane_rows: when nonzero, planes points at row c0 of planes that are plane_rows tall (columns c0 ..
// c0+np-1 of wider planes: a block of B's columns, split as it lands).
void launch_split_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta,
                       const oztt_ii_plan& p, int8_t* planes, uint64_t np, uint64_t kp, cudaStream_t st,
                       uint64_t plane_rows) {
    const uint64_t pr = plane_rows ? plane_rows : np;
    if (residue_mode(p) == kTopWhole)
        split_cols_nd<kTopWhole>(b, k, n, ldb, delta, p.nd, split_const(p), planes, np, kp, pr, st);
    else
        split_cols_nd<kTopSplit>(b, k, n, ldb, delta, p.nd, split_const(p), planes, np, kp, pr, st);
}

static SplitConst digit_const(const oztt_digit_plan& fp) {
    SplitConst sc = split_const(fp.base);
    for (int s = 0; s < fp.base.S; ++s) {
        sc.q[s] = (float)fp.q[s];
        sc.qinv[s] = 1.0f / (float)fp.q[s];
        sc.mode[s] = fp.mode[s];
        sc.poff[s] = fp.poff[s];
    }
    return sc;
}

// Digit planes of A ([nplane][mp][kp]) and of B transposed ([nplane][np][kp]).
void launch_digit_split_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta,
                             const oztt_digit_plan& fp, int8_t* planes, uint64_t mp, uint64_t kp, cudaStream_t st) {
    split_rows_nd<kDigits>(a, m, k, lda, delta, fp.base.nd, digit_const(fp), planes, mp, kp, mp, st);
}

void launch_digit_split_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta,
                             const oztt_digit_plan& fp, int8_t* planes, uint64_t np, uint64_t kp, cudaStream_t st) {
    split_cols_nd<kDigits>(b, k, n, ldb, delta, fp.base.nd, digit_const(fp), planes, np, kp, np, st);
}

}  // namespace oztt
