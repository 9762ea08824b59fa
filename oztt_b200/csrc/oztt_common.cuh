// SPDX-License-Identifier: Apache-2.0
// Shared helpers of the B200 Ozaki kernels: error plumbing of the C ABI and the binary32 operations
// with explicit rounding and flush-to-zero that the bit-exact split kernel is built from.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>

#include "oztt_cuda.h"

namespace oztt {

// Error carrying the C-ABI code.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

inline void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Error(OZTT_ERUNTIME, std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
}
#define OZTT_CUDA(call) ::oztt::check_cuda((call), #call)

inline void set_err(char* err, size_t errlen, const char* msg) {
    if (err && errlen) {
        std::strncpy(err, msg, errlen - 1);
        err[errlen - 1] = 0;
    }
}

// Runs f, translating exceptions into C-ABI codes.
template <class F>
int guarded(char* err, size_t errlen, F&& f) {
    try {
        f();
        set_err(err, errlen, "");
        return OZTT_OK;
    } catch (const Error& e) {
        set_err(err, errlen, e.what());
        return e.code;
    } catch (const std::invalid_argument& e) {
        set_err(err, errlen, e.what());
        return OZTT_EINVAL;
    } catch (const std::bad_alloc&) {
        set_err(err, errlen, "host memory exhausted");
        return OZTT_ENOMEM;
    } catch (const std::exception& e) {
        set_err(err, errlen, e.what());
        return OZTT_ERUNTIME;
    }
}

inline uint64_t round_up(uint64_t v, uint64_t q) { return (v + q - 1) / q * q; }

// Current value of a process-wide kernel-variant option (OZTT_OPT_*, set by oztt_set_option; 0 by default).
int option_value(int option);

// ---- binary32 with round-to-nearest-even and flush-to-zero, never contracted -----------------
// Each is one PTX instruction with an explicit rounding modifier, so the compiler can neither fuse
// nor reorder them; .ftz flushes subnormal inputs and results to signed zero.
__device__ __forceinline__ float f32_add(float a, float b) {
    float r;
    asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float f32_sub(float a, float b) {
    float r;
    asm("sub.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float f32_mul(float a, float b) {
    float r;
    asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
// Round to the nearest integer, ties to even.
__device__ __forceinline__ float f32_rint(float a) {
    float r;
    asm("cvt.rni.ftz.f32.f32 %0, %1;" : "=f"(r) : "f"(a));
    return r;
}
// a*b + c rounded once. Used only where a*b and the sum are exact integers below 2^24, where it
// equals the separate multiply and add.
__device__ __forceinline__ float f32_fma(float a, float b, float c) {
    float r;
    asm("fma.rn.ftz.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// ---- the same operations on pairs of binary32 values (sm_100 packed FP32 pipe) ---------------
// A pair lives in one 64-bit register, first element in the low half. Each operation is one
// f32x2 instruction with the same rounding (.rn) and flushing (.ftz) as the scalar forms above, so
// each half is bit-identical to the scalar operation on that half.
typedef uint64_t f32x2;
__device__ __forceinline__ f32x2 pk2(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpk2(f32x2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 splat2(float v) { return pk2(v, v); }
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// a*b + c rounded once.
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 r;
    asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// a*b rounded once, for two values. The assembler treats a packed multiply followed by an addition
// as a candidate for fusion (one rounding instead of two), which would change the reference's
// results; the product is therefore formed as fma(a, b, nz) with nz = -0.0 that the caller receives
// at run time (a kernel argument), so nothing can be folded into it. a*b + (-0) equals a*b in every
// case, the sign of a zero product included.
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b, f32x2 nz) { return fma2(a, b, nz); }
// Round to the nearest integer, ties to even, for |x| < 2^22: adding 1.5 * 2^23 moves x into the
// binade where the spacing is 1, so the addition itself rounds to an integer (ties to even, since the
// added constant is even), and subtracting the constant again is exact. The value equals
// cvt.rni.f32.f32; only the sign of a zero result can differ (+0 where cvt.rni would give -0).
constexpr float kRoundMagic = 12582912.0f;
__device__ __forceinline__ f32x2 rint2(f32x2 x) {
    const f32x2 m = splat2(kRoundMagic);
    return sub2(add2(x, m), m);
}

// Global nanosecond timer, for bounded waits.
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

}  // namespace oztt
