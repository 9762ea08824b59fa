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

// Global nanosecond timer, for bounded waits.
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

}  // namespace oztt
