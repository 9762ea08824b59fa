// SPDX-License-Identifier: Apache-2.0
//
// Binary floating point with a 64-bit significand and round-to-nearest-even: the arithmetic of the
// x86 "long double" (x87 extended precision, precision control 64 bits), in integer code that compiles
// for the host and for the GPU.
//
// The reference's precision policy sums its random-projection products in long double on the host
// (estimate_product_norm, src/backend/common/norm_estimate.hpp:48-73: acc += (long double)x * g). To
// compute the same sums on the device bit for bit, each product of two doubles is rounded to 64
// significand bits and added to the accumulator with one rounding to 64 bits, as the x87 unit does.
// Only what those sums need is here: conversion from double, the product of two values converted
// from doubles, addition, and conversion back to double (round to nearest even, as the host's
// (double) cast). Exponents are kept in an int32, so nothing overflows or becomes subnormal on the way
// (the extended range of the x87 format is not reached by products of doubles); zero keeps its sign
// with the IEEE rules for sums of zeros.
#pragma once
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define OZTT_HD __host__ __device__ __forceinline__
#else
#define OZTT_HD inline
#endif

namespace oztt {
namespace ext80 {

// value = (-1)^neg * m * 2^(e - 63); m has bit 63 set, or m == 0 for a zero.
struct Ext {
    uint64_t m;
    int32_t e;
    uint32_t neg;
};

OZTT_HD uint64_t mulhi64(uint64_t a, uint64_t b) {
#if defined(__CUDA_ARCH__)
    return __umul64hi(a, b);
#else
    return (uint64_t)(((unsigned __int128)a * b) >> 64);
#endif
}
OZTT_HD int clz64(uint64_t x) {
#if defined(__CUDA_ARCH__)
    return __clzll((long long)x);
#else
    return x ? __builtin_clzll(x) : 64;
#endif
}
OZTT_HD uint64_t bits_of(double x) {
#if defined(__CUDA_ARCH__)
    return (uint64_t)__double_as_longlong(x);
#else
    uint64_t u;
    memcpy(&u, &x, 8);
    return u;
#endif
}
OZTT_HD double double_of(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
    double x;
    memcpy(&x, &u, 8);
    return x;
#endif
}

OZTT_HD Ext zero() { return Ext{0, 0, 0}; }

// x >> s and x << s for s in [0, 64], 0 at s = 64 (C++ leaves a 64-bit shift by 64 undefined).
OZTT_HD uint64_t shr64(uint64_t x, uint32_t s) { return s < 64 ? x >> s : 0; }
OZTT_HD uint64_t shl64(uint64_t x, uint32_t s) { return s < 64 ? x << s : 0; }

// The operations below are written without data-dependent branches (every case is computed and the
// result selected), so that the lanes of a warp, which hold different operands, never diverge.

// Exact conversion of a finite double.
OZTT_HD Ext from_double(double x) {
    const uint64_t u = bits_of(x);
    const int32_t E = (int32_t)((u >> 52) & 0x7FF);
    const uint64_t f = u & 0xFFFFFFFFFFFFFull;
    const int lz = clz64(f);  // subnormal: value = f * 2^-1074
    Ext r;
    r.neg = (uint32_t)(u >> 63);
    r.m = E ? (f | 0x10000000000000ull) << 11 : shl64(f, (uint32_t)lz);
    r.e = E ? E - 1023 : (f ? -1074 + 63 - lz : 0);
    return r;
}

// Rounds the 128-bit magnitude (hi:lo, bit 127 set) to 64 bits, ties to even; `sticky` says that
// nonzero bits lie below lo. Returns the significand and adds the carry of the rounding to e.
OZTT_HD uint64_t round128(uint64_t hi, uint64_t lo, bool sticky, int32_t& e) {
    const uint64_t guard = lo >> 63;
    const uint64_t rest = ((lo << 1) != 0 || sticky) ? 1u : 0u;
    const uint64_t inc = guard & (rest | (hi & 1));
    const uint64_t r = hi + inc;
    const bool wrap = r == 0 && inc;  // carried out of 64 bits: the significand becomes 2^63
    e += wrap ? 1 : 0;
    return wrap ? 0x8000000000000000ull : r;
}

// a * b rounded once to 64 significand bits (a, b from doubles or any Ext values).
OZTT_HD Ext mul(const Ext& a, const Ext& b) {
    const bool zero = a.m == 0 || b.m == 0;
    const uint64_t hi = mulhi64(a.m, b.m), lo = a.m * b.m;
    // a.m * b.m in [2^126, 2^128): value = (hi:lo) * 2^(ea + eb - 126)
    const bool top = (hi >> 63) != 0;
    int32_t e = a.e + b.e + (top ? 1 : 0);
    const uint64_t h = top ? hi : (hi << 1) | (lo >> 63);
    const uint64_t l = top ? lo : lo << 1;
    Ext r;
    r.neg = a.neg ^ b.neg;
    r.m = round128(h, l, false, e);
    r.m = zero ? 0 : r.m;
    r.e = zero ? 0 : e;
    return r;
}

// a + b rounded once to 64 significand bits. Zeros keep the IEEE signs: -0 + -0 = -0, any other sum
// of zeros and an exact cancellation give +0.
OZTT_HD Ext add(const Ext& a, const Ext& b) {
    const bool az = a.m == 0, bz = b.m == 0;
    // x: the operand of larger magnitude (a zero is the smaller)
    const bool a_big = bz || (!az && (a.e > b.e || (a.e == b.e && a.m >= b.m)));
    const uint64_t xm = a_big ? a.m : b.m, ym = a_big ? b.m : a.m;
    const int32_t xe = a_big ? a.e : b.e, ye = a_big ? b.e : a.e;
    const uint32_t xn = a_big ? a.neg : b.neg, yn = a_big ? b.neg : a.neg;
    // Y = y.m * 2^(64 - d) beside X = x.m * 2^64 as 128-bit fixed point; the bits of Y below the window
    // become the sticky flag. d = 128 stands for "entirely below" (and for a zero y).
    const int64_t dd = (int64_t)xe - (int64_t)ye;
    const uint32_t d = (ym == 0 || dd >= 128) ? 128u : (uint32_t)dd;
    const uint64_t yh = shr64(ym, d);
    const uint64_t yl = d == 0 ? 0 : (d <= 64 ? shl64(ym, 64 - d) : shr64(ym, d - 64));
    const bool sticky = d > 64 && (d < 128 ? shl64(ym, 128 - d) != 0 : ym != 0);
    // same signs: X + Y, then one right shift on a carry out of bit 127
    const uint64_t sh = xm + yh;
    const bool carry = sh < xm;
    const uint64_t add_hi = carry ? (sh >> 1) | 0x8000000000000000ull : sh;
    const uint64_t add_lo = carry ? (yl >> 1) | (sh << 63) : yl;
    const bool add_sticky = sticky || (carry && (yl & 1));
    const int32_t add_e = xe + (carry ? 1 : 0);
    // opposite signs: X - Y - (sticky ? 1 : 0) -- with discarded bits of Y the exact difference lies
    // strictly between this value and the next, which the sticky flag records -- then normalised
    const uint64_t sub = yl + (sticky ? 1u : 0u);  // wraps to 0 only when yl = 2^64 - 1 and sticky
    const uint64_t d_lo = 0 - sub;
    const uint64_t d_hi = xm - yh - ((yl != 0 || sticky) ? 1u : 0u);
    const bool cancel = d_hi == 0 && d_lo == 0;  // exact (sticky is then false)
    const bool hz = d_hi == 0;
    const uint64_t h1 = hz ? d_lo : d_hi, l1 = hz ? 0 : d_lo;
    const uint32_t lz = cancel ? 0u : (uint32_t)clz64(h1);
    const uint64_t sub_hi = shl64(h1, lz) | (lz ? shr64(l1, 64 - lz) : 0);
    const uint64_t sub_lo = shl64(l1, lz);
    const int32_t sub_e = xe - (hz ? 64 : 0) - (int32_t)lz;
    const bool same = xn == yn;
    int32_t e = same ? add_e : sub_e;
    const uint64_t m = round128(same ? add_hi : sub_hi, same ? add_lo : sub_lo, same ? add_sticky : sticky, e);
    const bool zero = xm == 0 || (!same && cancel);
    Ext r;
    r.m = zero ? 0 : m;
    r.e = zero ? 0 : e;
    r.neg = zero ? (xm == 0 ? (a.neg & b.neg) : 0u) : xn;
    return r;
}

// Round to the nearest double, ties to even (the value range of the sums here stays normal).
OZTT_HD double to_double(const Ext& a) {
    if (a.m == 0) return a.neg ? -0.0 : 0.0;
    const uint64_t sign = (uint64_t)a.neg << 63;
    if (a.e < -1022) {
        // subnormal result: value = a.m * 2^(a.e - 63), rounded at the position 2^-1074
        const int drop = 11 + (-1022 - a.e);
        if (drop > 64) return double_of(sign);
        const uint64_t q0 = drop < 64 ? a.m >> drop : 0;
        const uint64_t r2 = drop < 64 ? a.m & ((1ull << drop) - 1) : a.m;
        const uint64_t half = 1ull << (drop - 1);
        const uint64_t q = q0 + ((r2 > half || (r2 == half && (q0 & 1))) ? 1 : 0);
        return double_of(sign | q);  // q may reach 2^52: the smallest normal number
    }
    int32_t e = a.e;
    uint64_t m = a.m >> 11;
    const uint64_t rem = a.m & 0x7FF;
    if (rem > 0x400 || (rem == 0x400 && (m & 1))) {
        ++m;
        if (m >> 53) {
            m >>= 1;
            ++e;
        }
    }
    if (e > 1023) return double_of(sign | 0x7FF0000000000000ull);
    return double_of(sign | ((uint64_t)(e + 1023) << 52) | (m & 0xFFFFFFFFFFFFFull));
}

}  // namespace ext80
}  // namespace oztt
