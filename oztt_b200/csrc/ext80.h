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

// Exact conversion of a finite double.
OZTT_HD Ext from_double(double x) {
    const uint64_t u = bits_of(x);
    Ext r;
    r.neg = (uint32_t)(u >> 63);
    const int32_t E = (int32_t)((u >> 52) & 0x7FF);
    uint64_t f = u & 0xFFFFFFFFFFFFFull;
    if (E == 0) {
        if (f == 0) {
            r.m = 0;
            r.e = 0;
            return r;
        }
        const int lz = clz64(f);  // subnormal: value = f * 2^-1074
        r.m = f << lz;
        r.e = -1074 + 63 - lz;
        return r;
    }
    r.m = (f | 0x10000000000000ull) << 11;
    r.e = E - 1023;
    return r;
}

// Rounds the 128-bit magnitude (hi:lo, bit 127 set) to 64 bits, ties to even; `sticky` says that
// nonzero bits lie below lo. Returns the significand and adds the carry of the rounding to e.
OZTT_HD uint64_t round128(uint64_t hi, uint64_t lo, bool sticky, int32_t& e) {
    const bool guard = (lo >> 63) != 0;
    const bool rest = (lo << 1) != 0 || sticky;
    if (guard && (rest || (hi & 1))) {
        ++hi;
        if (hi == 0) {  // carried out of 64 bits: the significand becomes 2^63 with a larger exponent
            hi = 0x8000000000000000ull;
            ++e;
        }
    }
    return hi;
}

// a * b rounded once to 64 significand bits (a, b from doubles or any Ext values).
OZTT_HD Ext mul(const Ext& a, const Ext& b) {
    Ext r;
    r.neg = a.neg ^ b.neg;
    if (a.m == 0 || b.m == 0) {
        r.m = 0;
        r.e = 0;
        return r;
    }
    uint64_t hi = mulhi64(a.m, b.m), lo = a.m * b.m;
    // a.m * b.m in [2^126, 2^128): value = (hi:lo) * 2^(ea + eb - 126)
    int32_t e = a.e + b.e + 1;
    if (!(hi >> 63)) {
        hi = (hi << 1) | (lo >> 63);
        lo <<= 1;
        e -= 1;
    }
    r.m = round128(hi, lo, false, e);
    r.e = e;
    return r;
}

// a + b rounded once to 64 significand bits.
OZTT_HD Ext add(const Ext& a, const Ext& b) {
    if (b.m == 0) {
        if (a.m == 0) return Ext{0, 0, a.neg & b.neg};  // -0 + -0 = -0, otherwise +0
        return a;
    }
    if (a.m == 0) return b;
    // x: the operand of larger magnitude.
    const bool a_big = a.e > b.e || (a.e == b.e && a.m >= b.m);
    const Ext& x = a_big ? a : b;
    const Ext& y = a_big ? b : a;
    const uint32_t d = (uint32_t)(x.e - y.e);
    // X = x.m * 2^64, Y = y.m * 2^(64 - d), both as 128-bit fixed point, with the bits of Y that fall
    // below the window kept as a sticky flag.
    uint64_t yh, yl;
    bool sticky = false;
    if (d == 0) {
        yh = y.m;
        yl = 0;
    } else if (d < 64) {
        yh = y.m >> d;
        yl = y.m << (64 - d);
    } else if (d == 64) {
        yh = 0;
        yl = y.m;
    } else if (d < 128) {
        yh = 0;
        yl = y.m >> (d - 64);
        sticky = (y.m << (128 - d)) != 0;
    } else {
        yh = 0;
        yl = 0;
        sticky = true;
    }
    int32_t e = x.e;
    uint64_t hi, lo;
    if (x.neg == y.neg) {
        lo = yl;  // x's low half is zero
        hi = x.m + yh;
        if (hi < x.m) {  // carry out of bit 127: shift right by one
            sticky = sticky || (lo & 1);
            lo = (lo >> 1) | (hi << 63);
            hi = (hi >> 1) | 0x8000000000000000ull;
            ++e;
        }
    } else {
        // X - Y - (sticky ? 1 : 0): with discarded bits of Y, the exact difference lies strictly between
        // this value and the next, which the sticky flag records.
        const uint64_t sub = yl + (sticky ? 1u : 0u);  // wraps to 0 only when yl = 2^64 - 1 and sticky
        lo = 0 - sub;
        const uint64_t borrow = (yl != 0 || sticky) ? 1u : 0u;
        hi = x.m - yh - borrow;
        if (hi == 0 && lo == 0) return Ext{0, 0, 0};  // exact cancellation (sticky is then false): +0
        // normalize: shift left until bit 127 is set
        if (hi == 0) {
            hi = lo;
            lo = 0;
            e -= 64;
        }
        const int lz = clz64(hi);
        if (lz) {
            hi = (hi << lz) | (lo >> (64 - lz));
            lo <<= lz;
            e -= lz;
        }
    }
    Ext r;
    r.neg = x.neg;
    r.m = round128(hi, lo, sticky, e);
    r.e = e;
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
