// SPDX-License-Identifier: Apache-2.0
//
// The input statistics of the Scheme II precision policy on the device, bit-identical to the
// reference's host computation (choose_precision_policy / oz2_measure_stats and estimate_product_norm,
// src/backend/ozaki2/auto_precision.hpp:24-108, src/backend/common/norm_estimate.hpp:20-73), so that the
// plan made from them is the reference's. Once A and B are resident in HBM this replaces seconds of
// host work at 16384^3 by a few milliseconds.
//
//   absmax     exact max |a| per row of A and per column of B (order-free, so any reduction order)
//   sumsq      sum_c (a*rgA)^2 per row of A and sum_r (b*rgB)^2 per column of B, each summed
//              sequentially in the reference's order by one thread, one rounding per multiply and add
//   sketch     y_l[r] = (double) sum_j (long double)(x[r][j]*rg) * v_l[j] for the 8 random vectors, with
//              the x87 extended-precision product and sum emulated exactly (ext80.h); one thread per
//              (row, vector), the row walked in the reference's order
// The host finishes the reductions over rows and columns in the reference's order (device_policy_stats
// below): the sums over M and N terms are cheap, and doing them there keeps their order exact.
#include <algorithm>
#include <cmath>
#include <memory>
#include <mutex>
#include <random>
#include <vector>

#include "ext80.h"
#include "oztt_common.cuh"
#include "planner.hpp"
#include "runtime.cuh"

namespace oztt {

constexpr int kVectors = 8;

namespace {

// One warp per row: the largest |a| over `cols` columns of rows lda apart, as the 63-bit pattern
// (nonnegative doubles order like integers); with `carry` also over out[row] (earlier columns).
__global__ void __launch_bounds__(256) row_absmax_kernel(const double* __restrict__ a, uint64_t m, uint64_t cols,
                                                         uint64_t lda, unsigned long long* __restrict__ out,
                                                         int carry) {
    const int lane = threadIdx.x & 31;
    const uint64_t nwarps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    const unsigned long long* pu = reinterpret_cast<const unsigned long long*>(a);
    for (uint64_t row = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < m; row += nwarps) {
        unsigned long long mx = (carry && lane == 0) ? out[row] : 0ull;
        for (uint64_t j = lane; j < cols; j += 32) {
            const unsigned long long v = __ldg(pu + row * lda + j) & 0x7FFFFFFFFFFFFFFFull;
            mx = v > mx ? v : mx;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
            mx = t > mx ? t : mx;
        }
        if (lane == 0) out[row] = mx;
    }
}

// Column maxima of n columns of rows ldb apart: a thread per column over a chunk of rows, combined with
// atomicMax.
__global__ void __launch_bounds__(256) col_absmax_kernel(const double* __restrict__ b, uint64_t k, uint64_t n,
                                                         uint64_t ldb, uint64_t rows_per_chunk,
                                                         unsigned long long* __restrict__ out) {
    const uint64_t col = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= n) return;
    const uint64_t r0 = (uint64_t)blockIdx.y * rows_per_chunk, r1 = min(k, r0 + rows_per_chunk);
    const unsigned long long* pu = reinterpret_cast<const unsigned long long*>(b);
    unsigned long long mx = 0;
    for (uint64_t r = r0; r < r1; ++r) {
        const unsigned long long v = __ldg(pu + r * ldb + col) & 0x7FFFFFFFFFFFFFFFull;
        mx = v > mx ? v : mx;
    }
    if (mx) atomicMax(out + col, mx);
}

// Nonzero magnitudes below 2^-383 are the only inputs (with row and column maxima in the validated
// range, so that the scale rg lies in [2^-128, 2^125]) for which the sums of squares and sketches taken
// on the unscaled values, scaled by rg afterwards, could differ from the reference's scale-first sums:
// above that bound x*rg, x^2 and (x*rg)^2 are all normal doubles, so scaling by a power of two commutes
// with every rounding. The chunked path raises a matrix's `tiny` word when it meets one, and the matrix
// is then measured again scale-first once its scale is known.
constexpr double kTinyBound = 0x1p-383;

__device__ __forceinline__ bool is_tiny(double x) { return x != 0.0 && fabs(x) < kTinyBound; }

// Each of the sequential sums below runs as one dependent chain per thread, so its speed is set by
// the latency of a step, not by bandwidth: the loads of a batch of kBatch steps are issued together
// (and those of the next batch before the current one is summed), so that a step waits for the
// arithmetic only.
constexpr int kBatch = 16;
constexpr int kSketchBatch = 8;  // the sketch's steps hold more registers
constexpr int kSketchThreads = 128;

// sum over `len` terms at stride `stride` from p of (x*rg)^2, continuing from sq; raises `small` for a
// tiny element.
// B is the batch; a column chain (stride of a whole row) waits on DRAM for every batch, so it takes a
// larger one.
template <int B = kBatch>
__device__ __forceinline__ double sumsq_chain(const double* __restrict__ p, uint64_t len, uint64_t stride, double rg,
                                              double sq, bool& small) {
    double cur[B], nxt[B];
#pragma unroll
    for (int u = 0; u < B; ++u) cur[u] = (uint64_t)u < len ? __ldg(p + (uint64_t)u * stride) : 0.0;
    for (uint64_t j0 = 0; j0 < len; j0 += B) {
        const uint64_t j1 = j0 + B;
#pragma unroll
        for (int u = 0; u < B; ++u) nxt[u] = j1 + u < len ? __ldg(p + (j1 + u) * stride) : 0.0;
        const int cnt = len - j0 < (uint64_t)B ? (int)(len - j0) : B;
#pragma unroll
        for (int u = 0; u < B; ++u) {
            if (u < cnt) {
                small |= is_tiny(cur[u]);
                const double v = __dmul_rn(cur[u], rg);
                sq = __dadd_rn(sq, __dmul_rn(v, v));
            }
        }
#pragma unroll
        for (int u = 0; u < B; ++u) cur[u] = nxt[u];
    }
    return sq;
}

// sum_c (a[i][c]*rg)^2 over `cols` columns of each row i (rows lda apart), c ascending, one rounding
// per operation; with `carry` the sum continues from out[i] (earlier columns). The scale is rg, or
// *rgp when rgp is set; gate, when set, skips the kernel unless *gate is nonzero; tiny, when set,
// receives 1 if a row holds a tiny element.
__global__ void __launch_bounds__(128) row_sumsq_kernel(const double* __restrict__ a, uint64_t m, uint64_t cols,
                                                        uint64_t lda, double rg, const double* __restrict__ rgp,
                                                        double* __restrict__ out, int carry,
                                                        uint32_t* __restrict__ tiny,
                                                        const uint32_t* __restrict__ gate) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m || (gate && *gate == 0u)) return;
    if (rgp) rg = *rgp;
    bool small = false;
    out[i] = sumsq_chain<>(a + i * lda, cols, 1, rg, carry ? out[i] : 0.0, small);
    if (tiny && small) atomicOr(tiny, 1u);
}

// sum_r (b[r][j]*rg)^2 for each of n columns j (rows ldb apart), r ascending over the `rows` rows given;
// with `carry` the sum continues from out[j] (the rows of an earlier chunk).
__global__ void __launch_bounds__(128) col_sumsq_kernel(const double* __restrict__ b, uint64_t rows, uint64_t n,
                                                        uint64_t ldb, double rg, const double* __restrict__ rgp,
                                                        double* __restrict__ out, int carry,
                                                        uint32_t* __restrict__ tiny,
                                                        const uint32_t* __restrict__ gate) {
    const uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n || (gate && *gate == 0u)) return;
    if (rgp) rg = *rgp;
    bool small = false;
    out[j] = sumsq_chain<32>(b + j, rows, ldb, rg, carry ? out[j] : 0.0, small);
    if (tiny && small) atomicOr(tiny, 1u);
}

// out[l][r] = (double) sum_{j < cols} ext((x[r][j]*rg)) * ext(v[l][j]), the sum in 64-bit-significand
// arithmetic, j ascending. Thread t handles row t / 8 and vector t % 8, so a warp reads 4 rows and
// the 8 vectors. The products are independent of the running sum, so only the additions form the
// chain. UNSCALED: the elements enter as they are. EXT_OUT: the extended-precision sums are stored
// (eout) instead of their rounding to double -- for scaling later (UNSCALED) or for a later stretch of
// columns, on this device or another (the tiled statistics).
// Rows of x lie ldx apart; the sum runs over `cols` columns and, EXT_OUT with `carry`, continues from
// eout (earlier columns).
template <bool UNSCALED, bool EXT_OUT = UNSCALED>
__global__ void __launch_bounds__(128) sketch_kernel(const double* __restrict__ x, uint64_t rows, uint64_t cols,
                                                     uint64_t ldx, double rg, const double* __restrict__ rgp,
                                                     const double* __restrict__ v, uint64_t vstride,
                                                     double* __restrict__ out, ext80::Ext* __restrict__ eout,
                                                     uint64_t ostride, int carry, const uint32_t* __restrict__ gate) {
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t r = t / kVectors, l = t % kVectors;
    if (r >= rows || (gate && *gate == 0u)) return;
    if (rgp) rg = *rgp;
    const double* xr = x + r * ldx;
    const double* vl = v + l * vstride;
    ext80::Ext acc = (EXT_OUT && carry) ? eout[l * ostride + r] : ext80::zero();
    constexpr int B = kSketchBatch;
    double cx[B], cv[B], nx[B], nv[B];
#pragma unroll
    for (int u = 0; u < B; ++u) {
        cx[u] = (uint64_t)u < cols ? __ldg(xr + u) : 0.0;
        cv[u] = (uint64_t)u < cols ? __ldg(vl + u) : 0.0;
    }
    for (uint64_t j0 = 0; j0 < cols; j0 += B) {
        const uint64_t j1 = j0 + B;
#pragma unroll
        for (int u = 0; u < B; ++u) {
            nx[u] = j1 + u < cols ? __ldg(xr + j1 + u) : 0.0;
            nv[u] = j1 + u < cols ? __ldg(vl + j1 + u) : 0.0;
        }
        const int cnt = cols - j0 < (uint64_t)B ? (int)(cols - j0) : B;
#pragma unroll
        for (int u = 0; u < B; ++u) {
            const double xs = UNSCALED ? cx[u] : __dmul_rn(cx[u], rg);
            const ext80::Ext prod = ext80::mul(ext80::from_double(xs), ext80::from_double(cv[u]));
            if (u < cnt) acc = ext80::add(acc, prod);
        }
#pragma unroll
        for (int u = 0; u < B; ++u) {
            cx[u] = nx[u];
            cv[u] = nv[u];
        }
    }
    if constexpr (EXT_OUT)
        eout[l * ostride + r] = acc;
    else
        out[l * ostride + r] = ext80::to_double(acc);
}

// Bounded statistics of rows of A (x: rows x k, row-major), for deciding the plan without the reference's
// sequential long-double sums: per row, into out[r*kCertW ..]:
//   [0]          the largest magnitude as its bit pattern (NaN and Inf patterns order above every number)
//   [1]          sum x^2            [2 .. 9]   sum x * y_l            [10 .. 17]  sum |x * y_l|
//   [18]         sum |x| * ew       (0 when ew is null)
// all unscaled, in FP64 (in the lanes', then the warp's order); the host turns them into bounds that contain
// the reference's values. y: the 8 x k sketch y_l = B g_l (scaled), as the reference has it or as
// bcert_finish_kernel bounds it (then ew[j] bounds |y_l[j] - the reference's y_l[j]| over l). flags |= 1
// when a nonzero element below 2^-383 makes the scaled squares leave the normal range (no bounds then).
// A block of 8 warps takes 8 rows, one per warp, the lanes striding the columns four at a time (all four
// loads in flight before any is used); the sketch and ew go through shared memory a chunk of kCertChunk
// columns at a time, so that each value is read from L2 once per 8 rows, in two buffers: the next chunk's
// asynchronous copies are in flight while this one is summed. 36 KB of shared memory a block.
constexpr int kCertW = 19;
constexpr int kCertWarps = 8, kCertRows = kCertWarps;
constexpr int kCertChunk = 256;
// An 8-byte asynchronous copy from global into shared memory; when !valid nothing is read (src is then any
// valid address) and the 8 bytes are zero-filled.
__device__ __forceinline__ void cp_async8(double* dst, const double* src, bool valid) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(src), "r"(valid ? 8 : 0) : "memory");
}
__global__ void __launch_bounds__(256) band_certify_kernel(const double* __restrict__ x, uint64_t rows, uint64_t k,
                                                           const double* __restrict__ y,
                                                           const double* __restrict__ ew, double* __restrict__ out,
                                                           uint32_t* __restrict__ flags) {
    // per row V = kCertW - 1 sums: s2, sl[8], al[8], se (slots 1 .. 18 of the row's output; slot 0 the maximum)
    constexpr int V = 1 + 2 * kVectors + 1;
    static_assert(V + 1 == kCertW, "the sums and the maximum fill a row of the output");
    __shared__ double ys[2][kVectors][kCertChunk];
    __shared__ double es[2][kCertChunk];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t row = (uint64_t)blockIdx.x * kCertWarps + warp;
    const bool live = row < rows;
    const double* xr = x + (live ? row : 0) * k;
    unsigned long long mx = 0;
    double acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0.0;
    bool tiny = false;
    const auto add = [&](double v, int j, int b) {
        const unsigned long long pat = (unsigned long long)__double_as_longlong(v) & 0x7FFFFFFFFFFFFFFFull;
        mx = pat > mx ? pat : mx;
        tiny = tiny || (pat != 0 && pat < 0x1800000000000000ull);  // 0 < |v| < 2^-383
        acc[0] = fma(v, v, acc[0]);
        acc[V - 1] = fma(fabs(v), es[b][j], acc[V - 1]);
        // the products fused into the sums: one rounding per term instead of two, within the same
        // gamma(k) bound of sum |x y_l| that the host's bounds take for these sums
#pragma unroll
        for (int l = 0; l < kVectors; ++l) {
            const double yl = ys[b][l][j];
            acc[1 + l] = fma(v, yl, acc[1 + l]);
            acc[1 + kVectors + l] = fma(fabs(v), fabs(yl), acc[1 + kVectors + l]);
        }
    };
    // the sketch and ew of chunk c into buffer c & 1, asynchronously (zeros past k)
    const auto stage = [&](uint64_t j0, int b) {
        for (int i = threadIdx.x; i < kVectors * kCertChunk; i += blockDim.x) {
            const int l = i / kCertChunk, j = i % kCertChunk;
            const bool in = j0 + j < k;
            cp_async8(&ys[b][l][j], in ? y + (uint64_t)l * k + j0 + j : y, in);
        }
        for (int j = threadIdx.x; j < kCertChunk; j += blockDim.x) {
            const bool in = ew && j0 + j < k;
            cp_async8(&es[b][j], in ? ew + j0 + j : y, in);
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    stage(0, 0);
    for (uint64_t j0 = 0, c = 0; j0 < k; j0 += kCertChunk, ++c) {
        const int b = (int)(c & 1);
        const int cw = k - j0 < (uint64_t)kCertChunk ? (int)(k - j0) : kCertChunk;
        // the next chunk's copies go out before this one is summed (an empty group after the last chunk);
        // its buffer was last read in the previous iteration, which every warp has left (the barrier below)
        if (j0 + kCertChunk < k)
            stage(j0 + kCertChunk, b ^ 1);
        else
            asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");  // this chunk's copies (this thread's) landed
        __syncthreads();                                           // ... and every thread's
        if (live) {
            for (int j = lane; j < cw; j += 128) {
                double v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = j + 32 * u < cw ? __ldg(xr + j0 + j + 32 * u) : 0.0;
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (j + 32 * u < cw) add(v[u], j + 32 * u, b);
            }
        }
        __syncthreads();  // every warp done with buffer b before the next iteration's copies refill it
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    // the lanes' sums (any order: the bounds hold for every order of the k terms)
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long om = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
        mx = om > mx ? om : mx;
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] += __shfl_xor_sync(0xFFFFFFFFu, acc[v], o);
    }
    if (__any_sync(0xFFFFFFFFu, tiny) && lane == 0) atomicOr(flags, 1u);
    if (!live) return;
    // lane v < V writes sum v into slot 1 + v, lane V the maximum into slot 0
    double* o = out + row * kCertW;
#pragma unroll
    for (int v = 0; v < V; ++v)
        if (lane == v) o[1 + v] = acc[v];
    if (lane == V) o[0] = __longlong_as_double((long long)mx);
}

// Bounded statistics of B, a block of columns at a time as the blocks land (b: k rows of w elements from the
// block's first column, rows ldb apart; g: the probe vectors from the block's first column, gstride apart);
// one warp per row r of B, accumulating into acc[r*kBCertW ..] (zeroed before the first block):
//   [0 .. 7]  sum b g_l        [8 .. 15]  sum |b g_l|        [16]  sum b^2
// unscaled, in FP64 (the warp's order, the blocks one after another). flags |= 1 when a nonzero element
// below 2^-383 is met (the scaled values could leave the normal range: no bounds then).
constexpr int kBCertW = 17;
__global__ void __launch_bounds__(256) bcert_block_kernel(const double* __restrict__ b, uint64_t k, uint64_t w,
                                                          uint64_t ldb, const double* __restrict__ g, uint64_t gstride,
                                                          double* __restrict__ acc, uint32_t* __restrict__ flags) {
    // the probe vectors over the block's columns go through shared memory kCertChunk columns at a time, in two
    // buffers (the next chunk's asynchronous copies in flight while this one is summed), read from L2 once
    // per 8 rows instead of once per row
    __shared__ double gs[2][kVectors][kCertChunk];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t r = (uint64_t)blockIdx.x * kCertWarps + warp;
    const bool live = r < k;
    const double* br = b + (live ? r : 0) * ldb;
    bool tiny = false;
    double s2 = 0.0, sl[kVectors], al[kVectors];
#pragma unroll
    for (int l = 0; l < kVectors; ++l) sl[l] = al[l] = 0.0;
    const auto stage = [&](uint64_t c0, int buf) {
        for (int i = threadIdx.x; i < kVectors * kCertChunk; i += blockDim.x) {
            const int l = i / kCertChunk, c = i % kCertChunk;
            const bool in = c0 + c < w;
            cp_async8(&gs[buf][l][c], in ? g + (uint64_t)l * gstride + c0 + c : g, in);
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    stage(0, 0);
    for (uint64_t c0 = 0, ch = 0; c0 < w; c0 += kCertChunk, ++ch) {
        const int buf = (int)(ch & 1);
        const int cw = w - c0 < (uint64_t)kCertChunk ? (int)(w - c0) : kCertChunk;
        if (c0 + kCertChunk < w)
            stage(c0 + kCertChunk, buf ^ 1);
        else
            asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        __syncthreads();
        if (live) {
            for (int c = lane; c < cw; c += 32) {
                const double v = __ldg(br + c0 + c);
                const unsigned long long pat = (unsigned long long)__double_as_longlong(v) & 0x7FFFFFFFFFFFFFFFull;
                tiny = tiny || (pat != 0 && pat < 0x1800000000000000ull);
                s2 = fma(v, v, s2);
#pragma unroll
                for (int l = 0; l < kVectors; ++l) {
                    const double t = v * gs[buf][l][c];
                    sl[l] += t;
                    al[l] += fabs(t);
                }
            }
        }
        __syncthreads();
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        s2 += __shfl_xor_sync(0xFFFFFFFFu, s2, o);
#pragma unroll
        for (int l = 0; l < kVectors; ++l) {
            sl[l] += __shfl_xor_sync(0xFFFFFFFFu, sl[l], o);
            al[l] += __shfl_xor_sync(0xFFFFFFFFu, al[l], o);
        }
    }
    if (__any_sync(0xFFFFFFFFu, tiny) && lane == 0) atomicOr(flags, 1u);
    if (live && lane == 0) {
        double* o = acc + r * kBCertW;
#pragma unroll
        for (int l = 0; l < kVectors; ++l) {
            o[l] += sl[l];
            o[kVectors + l] += al[l];
        }
        o[16] += s2;
    }
}

// After B's last block: the scaled sketch y_l[r] = acc_l[r] * rgB (8 x k, as band_certify_kernel reads it)
// and ew[r], a bound of |y_l[r] - the reference's y_l[r]| over l: c1 * sum |b g_l| * rgB + u |y_l[r]|, with
// c1 covering this FP64 sum and the reference's long-double one (bcert_error_factor).
__global__ void __launch_bounds__(256) bcert_finish_kernel(const double* __restrict__ acc, uint64_t k,
                                                           const double* __restrict__ rgp, double c1,
                                                           double* __restrict__ y, double* __restrict__ ew) {
    const double rg = *rgp;
    for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < k; r += (uint64_t)gridDim.x * blockDim.x) {
        const double* o = acc + r * kBCertW;
        double e = 0.0;
#pragma unroll
        for (int l = 0; l < kVectors; ++l) {
            const double v = o[l] * rg;
            y[(uint64_t)l * k + r] = v;
            e = fmax(e, c1 * (o[kVectors + l] * rg) + 0x1p-53 * fabs(v));
        }
        ew[r] = e;
    }
}

// out[i] = the extended sum e[i] rounded to double (the end of a chain of sketch stretches).
__global__ void __launch_bounds__(256) round_ext_kernel(const ext80::Ext* __restrict__ e, uint64_t count,
                                                        double* __restrict__ out) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = ext80::to_double(e[i]);
}

inline unsigned sketch_blocks(uint64_t rows) {
    return (unsigned)((rows * kVectors + kSketchThreads - 1) / kSketchThreads);
}

// The exponent s of a scale rg = 2^s.
__device__ __forceinline__ int pow2_exponent(double rg) {
    return (int)((__double_as_longlong(rg) >> 52) & 0x7FF) - 1023;
}

// Unscaled sums of squares -> scaled: s * rg * rg, both products exact (the results are normal
// doubles when the matrix held no tiny element). Skipped when *tiny is set.
__global__ void __launch_bounds__(256) finish_sumsq_kernel(double* __restrict__ s, uint64_t count,
                                                           const double* __restrict__ rgp,
                                                           const uint32_t* __restrict__ tiny) {
    if (*tiny) return;
    const double rg = *rgp;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x)
        s[i] = __dmul_rn(__dmul_rn(s[i], rg), rg);
}

// Unscaled extended sums -> the scaled sums rounded to double: the scale is an exact shift of the
// exponent. Skipped when *tiny is set.
__global__ void __launch_bounds__(256) finish_sketch_kernel(const ext80::Ext* __restrict__ e, uint64_t count,
                                                            const double* __restrict__ rgp,
                                                            const uint32_t* __restrict__ tiny,
                                                            double* __restrict__ out) {
    if (*tiny) return;
    const int sh = pow2_exponent(*rgp);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (uint64_t)gridDim.x * blockDim.x) {
        ext80::Ext t = e[i];
        if (t.m) t.e += sh;
        out[i] = ext80::to_double(t);
    }
}

// rg = 1 / 2^e for the exponent e of the largest of `count` magnitude patterns, e clamped to
// [-1000, 1000], and 1 when that largest is zero or infinite (oz_pow2_scale,
// src/backend/common/norm_estimate.hpp:20-28). NaN patterns are passed over, as the host's std::max
// over the maxima passes them over. One block.
__global__ void __launch_bounds__(1024) pow2_scale_kernel(const unsigned long long* __restrict__ maxima,
                                                          uint64_t count, double* __restrict__ rg) {
    __shared__ unsigned long long part[32];
    constexpr unsigned long long kInf = 0x7FF0000000000000ull;
    unsigned long long mx = 0;
    for (uint64_t i = threadIdx.x; i < count; i += blockDim.x) {
        const unsigned long long v = maxima[i];
        if (v <= kInf && v > mx) mx = v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
        mx = t > mx ? t : mx;
    }
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x >= 32) return;
    mx = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0ull;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
        mx = t > mx ? t : mx;
    }
    if (threadIdx.x == 0) {
        double r = 1.0;
        if (mx != 0 && mx < kInf) {
            int e;
            frexp(__longlong_as_double((long long)mx), &e);
            e = min(max(e, -1000), 1000);
            r = __longlong_as_double((long long)(1023 - e) << 52);  // 2^-e, exact
        }
        *rg = r;
    }
}

// The 8 Gaussian vectors of length N from mt19937(12345), in the reference's draw order, kept for the
// last few N of the process (drawing them costs milliseconds at N = 16384).
std::shared_ptr<const std::vector<double>> policy_vectors(uint32_t N) {
    static std::mutex mu;
    static std::vector<std::pair<uint32_t, std::shared_ptr<const std::vector<double>>>> cache;
    std::lock_guard<std::mutex> lock(mu);
    for (auto& e : cache)
        if (e.first == N) return e.second;
    auto g = std::make_shared<std::vector<double>>((size_t)kVectors * N);
    std::mt19937 rng(12345);
    std::normal_distribution<double> normal(0.0, 1.0);
    for (int l = 0; l < kVectors; ++l)
        for (uint32_t j = 0; j < N; ++j) (*g)[(size_t)l * N + j] = normal(rng);
    if (cache.size() >= 4) cache.erase(cache.begin());
    cache.emplace_back(N, g);
    return g;
}

}  // namespace

// The host's part of the statistics, in the reference's order (choose_precision_policy and
// estimate_product_norm): TA, nA over the rows of A and TB, nB over the columns of B, each a sequential
// sum; ||C||_F^2 from the eight sketches s_l (8 x m, l-th row at sstride*l) -- each ||s_l||^2 a
// sequential sum -- dropping the largest, over 7, divided by 1 + 2 sqrt(2/8). The maxima are |values|
// (their bit patterns are the ones the absmax stages write).
PolicyStats combine_policy_stats(const double* row_max, uint64_t m, const double* col_max, uint64_t n,
                                 const double* row_sumsq, const double* col_sumsq, const double* s, uint64_t sstride,
                                 double rgA, double rgB) {
    PolicyStats ps;
    for (uint64_t r = 0; r < m; ++r) {
        const double mx = row_max[r] * rgA;
        if (mx > 0) {
            const double t = std::exp2(std::ceil(std::log2(mx)));
            ps.TA += t * t;
        }
        ps.nA += row_sumsq[r];
    }
    for (uint64_t c = 0; c < n; ++c) {
        const double mx = col_max[c] * rgB;
        if (mx > 0) {
            const double t = std::exp2(std::ceil(std::log2(mx)));
            ps.TB += t * t;
        }
        ps.nB += col_sumsq[c];
    }
    double cs2 = 0, cmx = 0;
    for (int l = 0; l < kVectors; ++l) {
        double q = 0;
        const double* sv = s + (size_t)l * sstride;
        for (uint64_t i = 0; i < m; ++i) q += sv[i] * sv[i];
        cs2 += q;
        cmx = std::max(cmx, q);
    }
    ps.nC = (cs2 - cmx) / (kVectors - 1) / (1.0 + 2.0 * std::sqrt(2.0 / (double)kVectors));
    ps.measured = true;
    return ps;
}

// The statistics in stages on stream st, every stage stream-ordered; collect() is the one
// synchronisation. Chunk stages measure unscaled values; the finishing stage of
// each matrix scales them once its scale is known (or, after a tiny element, recomputes scale-first).
struct PolicyStatsRun::Bufs {
    Bufs(cudaStream_t st, uint64_t m, uint64_t n, uint64_t k, uint32_t N)
        : rmax(st, m * 8), cmax(st, n * 8), rg(st, 16), words(st, 16), s2r(st, m * 8), s2c(st, n * 8),
          dg(st, (uint64_t)kVectors * N * 8), dy(st, (uint64_t)kVectors * k * 8), ds(st, (uint64_t)kVectors * m * 8),
          ey(st, (uint64_t)kVectors * k * sizeof(ext80::Ext)), es(st, (uint64_t)kVectors * m * sizeof(ext80::Ext)) {}
    DevBuf rmax, cmax, rg, words, s2r, s2c, dg, dy, ds, ey, es;
    uint32_t* tiny_a() { return words.as<uint32_t>(); }
    uint32_t* tiny_b() { return words.as<uint32_t>() + 1; }
};

PolicyStatsRun::PolicyStatsRun(uint64_t m, uint64_t n, uint64_t k, uint32_t N, cudaStream_t st)
    : m_(m), n_(n), k_(k), N_(N), st_(st) {
    // The row stages of A's bands run beside the persistent residue GEMM, whose CTAs hold most of each SM's
    // shared memory: ask for the same carveout, so that their blocks can share the SMs instead of waiting
    // for the GEMM to end (they use no shared memory themselves).
    static std::once_flag carveout;
    std::call_once(carveout, [] {
        const int shared = cudaSharedmemCarveoutMaxShared;
        cudaFuncSetAttribute(row_absmax_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, shared);
        cudaFuncSetAttribute(row_sumsq_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, shared);
        cudaFuncSetAttribute(sketch_kernel<true, true>, cudaFuncAttributePreferredSharedMemoryCarveout, shared);
        cudaGetLastError();
    });
    int dev = 0;
    OZTT_CUDA(cudaGetDevice(&dev));
    OZTT_CUDA(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, dev));
    OZTT_CUDA(cudaStreamCreateWithFlags(&cols_st_, cudaStreamNonBlocking));
    for (cudaEvent_t* e : {&landed_, &cols_done_}) OZTT_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    bufs_ = std::make_unique<Bufs>(st, m, n, k, N);
    OZTT_CUDA(cudaMemsetAsync(bufs_->cmax.p, 0, n * 8, st));
    OZTT_CUDA(cudaMemsetAsync(bufs_->words.p, 0, 16, st));
    g_ = policy_vectors(N);
    OZTT_CUDA(cudaMemcpyAsync(bufs_->dg.p, g_->data(), g_->size() * 8, cudaMemcpyHostToDevice, st));
}

PolicyStatsRun::~PolicyStatsRun() {
    if (cols_st_) cudaStreamSynchronize(cols_st_);
    bufs_.reset();  // freed on st, after the column stages
    for (cudaEvent_t e : {landed_, cols_done_})
        if (e) cudaEventDestroy(e);
    if (cols_st_) cudaStreamDestroy(cols_st_);
}

void PolicyStatsRun::b_cols(const double* b, uint64_t c0, uint64_t c1) {
    if (c1 <= c0) return;
    const uint64_t w = c1 - c0;
    // Each column of the block is complete, so its maximum and its sum of squares (a chain over all k
    // rows, latency-bound for a narrow block) depend on no other block: they run on their own stream,
    // beside the sketch sums, which continue from block to block on st.
    OZTT_CUDA(cudaEventRecord(landed_, st_));
    OZTT_CUDA(cudaStreamWaitEvent(cols_st_, landed_, 0));
    const uint64_t col_blocks = (w + 255) / 256;
    const uint64_t want = std::max<uint64_t>(1, (uint64_t)sms_ * 8 / std::max<uint64_t>(col_blocks, 1));
    const uint64_t chunks = std::min<uint64_t>(std::min<uint64_t>(want, k_), 65535);
    const uint64_t rpc = (k_ + chunks - 1) / chunks;
    col_absmax_kernel<<<dim3((unsigned)col_blocks, (unsigned)((k_ + rpc - 1) / rpc)), 256, 0, cols_st_>>>(
        b + c0, k_, w, n_, rpc, bufs_->cmax.as<unsigned long long>() + c0);
    OZTT_CUDA(cudaGetLastError());
    col_sumsq_kernel<<<(unsigned)((w + 127) / 128), 128, 0, cols_st_>>>(b + c0, k_, w, n_, 1.0, nullptr,
                                                                       bufs_->s2c.as<double>() + c0, 0,
                                                                       bufs_->tiny_b(), nullptr);
    OZTT_CUDA(cudaGetLastError());
    // y_l = B g_l over these columns (the padded ones add exact zeros), unscaled, continuing the sums of
    // the earlier columns
    sketch_kernel<true><<<sketch_blocks(k_), kSketchThreads, 0, st_>>>(b + c0, k_, w, n_, 1.0, nullptr,
                                                                      bufs_->dg.as<double>() + c0, N_, nullptr,
                                                                      bufs_->ey.as<ext80::Ext>(), k_, c0 > 0 ? 1 : 0,
                                                                      nullptr);
    OZTT_CUDA(cudaGetLastError());
}

void PolicyStatsRun::b_done(const double* b) {
    OZTT_CUDA(cudaEventRecord(cols_done_, cols_st_));
    OZTT_CUDA(cudaStreamWaitEvent(st_, cols_done_, 0));
    double* rgB = bufs_->rg.as<double>() + 1;
    const uint32_t* tiny = bufs_->tiny_b();
    pow2_scale_kernel<<<1, 1024, 0, st_>>>(bufs_->cmax.as<unsigned long long>(), n_, rgB);
    OZTT_CUDA(cudaGetLastError());
    finish_sumsq_kernel<<<(unsigned)std::min<uint64_t>((n_ + 255) / 256, 1024), 256, 0, st_>>>(bufs_->s2c.as<double>(),
                                                                                               n_, rgB, tiny);
    OZTT_CUDA(cudaGetLastError());
    const uint64_t ny = (uint64_t)kVectors * k_;
    finish_sketch_kernel<<<(unsigned)std::min<uint64_t>((ny + 255) / 256, 1024), 256, 0, st_>>>(
        bufs_->ey.as<ext80::Ext>(), ny, rgB, tiny, bufs_->dy.as<double>());
    OZTT_CUDA(cudaGetLastError());
    // after a tiny element: B again, scale first
    col_sumsq_kernel<<<(unsigned)((n_ + 127) / 128), 128, 0, st_>>>(b, k_, n_, n_, 0.0, rgB, bufs_->s2c.as<double>(),
                                                                    0, nullptr, tiny);
    OZTT_CUDA(cudaGetLastError());
    sketch_kernel<false><<<sketch_blocks(k_), kSketchThreads, 0, st_>>>(
        b, k_, n_, n_, 0.0, rgB, bufs_->dg.as<double>(), N_, bufs_->dy.as<double>(), nullptr, k_, 0, tiny);
    OZTT_CUDA(cudaGetLastError());
}

void PolicyStatsRun::a_cols(const double* a, uint64_t c0, uint64_t c1) {
    if (c1 <= c0) return;
    const uint64_t w = c1 - c0;
    const int carry = c0 > 0 ? 1 : 0;
    row_absmax_kernel<<<(unsigned)std::min<uint64_t>((m_ + 7) / 8, (uint64_t)sms_ * 32), 256, 0, st_>>>(
        a + c0, m_, w, k_, bufs_->rmax.as<unsigned long long>(), carry);
    OZTT_CUDA(cudaGetLastError());
    row_sumsq_kernel<<<(unsigned)((m_ + 127) / 128), 128, 0, st_>>>(a + c0, m_, w, k_, 1.0, nullptr,
                                                                    bufs_->s2r.as<double>(), carry, bufs_->tiny_a(),
                                                                    nullptr);
    OZTT_CUDA(cudaGetLastError());
    // s_l = A y_l over these columns, unscaled, continuing the sums of the earlier columns
    sketch_kernel<true><<<sketch_blocks(m_), kSketchThreads, 0, st_>>>(a + c0, m_, w, k_, 1.0, nullptr,
                                                                      bufs_->dy.as<double>() + c0, k_, nullptr,
                                                                      bufs_->es.as<ext80::Ext>(), m_, carry, nullptr);
    OZTT_CUDA(cudaGetLastError());
}

void PolicyStatsRun::a_rows(const double* a, uint64_t r0, uint64_t r1) {
    if (r1 <= r0) return;
    const uint64_t rows = r1 - r0;
    const double* ab = a + r0 * k_;
    // whole rows: the maxima, the unscaled sums of squares and the unscaled sketch sums of these rows are
    // complete in one pass each (the same sequential sums as a_cols over all column blocks)
    row_absmax_kernel<<<(unsigned)std::min<uint64_t>((rows + 7) / 8, (uint64_t)sms_ * 32), 256, 0, st_>>>(
        ab, rows, k_, k_, bufs_->rmax.as<unsigned long long>() + r0, 0);
    OZTT_CUDA(cudaGetLastError());
    row_sumsq_kernel<<<(unsigned)((rows + 127) / 128), 128, 0, st_>>>(ab, rows, k_, k_, 1.0, nullptr,
                                                                     bufs_->s2r.as<double>() + r0, 0, bufs_->tiny_a(),
                                                                     nullptr);
    OZTT_CUDA(cudaGetLastError());
    sketch_kernel<true><<<sketch_blocks(rows), kSketchThreads, 0, st_>>>(ab, rows, k_, k_, 1.0, nullptr,
                                                                        bufs_->dy.as<double>(), k_, nullptr,
                                                                        bufs_->es.as<ext80::Ext>() + r0, m_, 0,
                                                                        nullptr);
    OZTT_CUDA(cudaGetLastError());
}


void PolicyStatsRun::a_done(const double* a) {
    double* rgA = bufs_->rg.as<double>();
    const uint32_t* tiny = bufs_->tiny_a();
    pow2_scale_kernel<<<1, 1024, 0, st_>>>(bufs_->rmax.as<unsigned long long>(), m_, rgA);
    OZTT_CUDA(cudaGetLastError());
    finish_sumsq_kernel<<<(unsigned)std::min<uint64_t>((m_ + 255) / 256, 1024), 256, 0, st_>>>(bufs_->s2r.as<double>(),
                                                                                               m_, rgA, tiny);
    OZTT_CUDA(cudaGetLastError());
    const uint64_t ns = (uint64_t)kVectors * m_;
    finish_sketch_kernel<<<(unsigned)std::min<uint64_t>((ns + 255) / 256, 1024), 256, 0, st_>>>(
        bufs_->es.as<ext80::Ext>(), ns, rgA, tiny, bufs_->ds.as<double>());
    OZTT_CUDA(cudaGetLastError());
    // after a tiny element: A again, scale first
    row_sumsq_kernel<<<(unsigned)((m_ + 127) / 128), 128, 0, st_>>>(a, m_, k_, k_, 0.0, rgA, bufs_->s2r.as<double>(),
                                                                    0, nullptr, tiny);
    OZTT_CUDA(cudaGetLastError());
    sketch_kernel<false><<<sketch_blocks(m_), kSketchThreads, 0, st_>>>(
        a, m_, k_, k_, 0.0, rgA, bufs_->dy.as<double>(), k_, bufs_->ds.as<double>(), nullptr, m_, 0, tiny);
    OZTT_CUDA(cudaGetLastError());
}

PolicyStats PolicyStatsRun::collect(std::vector<uint64_t>* row_max, std::vector<uint64_t>* col_max,
                                    std::vector<double>* row_sumsq, std::vector<double>* col_sumsq, double* rg_out) {
    const uint64_t m = m_, n = n_;
    std::vector<unsigned long long> hr(m), hc(n);
    std::vector<double> h2r(m), h2c(n), hs((size_t)kVectors * m);
    double rg[2] = {0, 0};
    OZTT_CUDA(cudaMemcpyAsync(hr.data(), bufs_->rmax.p, m * 8, cudaMemcpyDeviceToHost, st_));
    OZTT_CUDA(cudaMemcpyAsync(hc.data(), bufs_->cmax.p, n * 8, cudaMemcpyDeviceToHost, st_));
    OZTT_CUDA(cudaMemcpyAsync(rg, bufs_->rg.p, 16, cudaMemcpyDeviceToHost, st_));
    OZTT_CUDA(cudaMemcpyAsync(h2r.data(), bufs_->s2r.p, m * 8, cudaMemcpyDeviceToHost, st_));
    OZTT_CUDA(cudaMemcpyAsync(h2c.data(), bufs_->s2c.p, n * 8, cudaMemcpyDeviceToHost, st_));
    OZTT_CUDA(cudaMemcpyAsync(hs.data(), bufs_->ds.p, hs.size() * 8, cudaMemcpyDeviceToHost, st_));
    OZTT_CUDA(cudaStreamSynchronize(st_));
    const double rgA = rg[0], rgB = rg[1];
    PolicyStats ps = combine_policy_stats(reinterpret_cast<const double*>(hr.data()), m,
                                          reinterpret_cast<const double*>(hc.data()), n, h2r.data(), h2c.data(),
                                          hs.data(), m, rgA, rgB);
    if (row_max) row_max->assign(hr.begin(), hr.end());
    if (col_max) col_max->assign(hc.begin(), hc.end());
    if (row_sumsq) *row_sumsq = h2r;
    if (col_sumsq) *col_sumsq = h2c;
    if (rg_out) {
        rg_out[0] = rgA;
        rg_out[1] = rgB;
    }
    return ps;
}

// The statistics stages on one whole matrix (x: rows x cols, row-major), as the C ABI and the resident
// operands use them: |maxima| per row (mode 0) or column (mode 1), scaled sums of squares, the sketch.
void launch_stats_absmax(const double* x, uint64_t rows, uint64_t cols, int mode, double* out, cudaStream_t st) {
    if (!rows || !cols) return;
    int dev = 0, sms = 148;
    OZTT_CUDA(cudaGetDevice(&dev));
    OZTT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    auto* o = reinterpret_cast<unsigned long long*>(out);  // nonnegative doubles order like their patterns
    if (mode == 0) {
        row_absmax_kernel<<<(unsigned)std::min<uint64_t>((rows + 7) / 8, (uint64_t)sms * 32), 256, 0, st>>>(
            x, rows, cols, cols, o, 0);
    } else {
        OZTT_CUDA(cudaMemsetAsync(out, 0, cols * 8, st));
        const uint64_t col_blocks = (cols + 255) / 256;
        const uint64_t want = std::max<uint64_t>(1, (uint64_t)sms * 8 / std::max<uint64_t>(col_blocks, 1));
        const uint64_t chunks = std::min<uint64_t>(std::min<uint64_t>(want, rows), 65535);
        const uint64_t rpc = (rows + chunks - 1) / chunks;
        col_absmax_kernel<<<dim3((unsigned)col_blocks, (unsigned)((rows + rpc - 1) / rpc)), 256, 0, st>>>(
            x, rows, cols, cols, rpc, o);
    }
    OZTT_CUDA(cudaGetLastError());
}

void launch_stats_sumsq(const double* x, uint64_t rows, uint64_t cols, int mode, double rg, double* out,
                        cudaStream_t st) {
    if (!rows || !cols) return;
    if (mode == 0)
        row_sumsq_kernel<<<(unsigned)((rows + 127) / 128), 128, 0, st>>>(x, rows, cols, cols, rg, nullptr, out, 0,
                                                                         nullptr, nullptr);
    else
        col_sumsq_kernel<<<(unsigned)((cols + 127) / 128), 128, 0, st>>>(x, rows, cols, cols, rg, nullptr, out, 0,
                                                                         nullptr, nullptr);
    OZTT_CUDA(cudaGetLastError());
}

void launch_stats_sketch(const double* x, uint64_t rows, uint64_t cols, double rg, const double* v, uint64_t vstride,
                         double* out, uint64_t ostride, cudaStream_t st) {
    if (!rows) return;
    sketch_kernel<false><<<sketch_blocks(rows), kSketchThreads, 0, st>>>(x, rows, cols, cols, rg, nullptr, v, vstride,
                                                                        out, nullptr, ostride, 0, nullptr);
    OZTT_CUDA(cudaGetLastError());
}

std::vector<double> policy_vectors_host(uint32_t N) { return *policy_vectors(N); }

void launch_band_certify(const double* x, uint64_t rows, uint64_t k, const double* y, const double* ew, double* out,
                         uint32_t* flags, cudaStream_t st) {
    if (!rows) return;
    band_certify_kernel<<<(unsigned)((rows + kCertRows - 1) / kCertRows), 256, 0, st>>>(x, rows, k, y, ew, out, flags);
    OZTT_CUDA(cudaGetLastError());
}

// Column maxima (magnitude patterns) of k rows of w columns, rows ldb apart, merged into out (atomic maxima:
// out holds zeros or earlier maxima).
void launch_col_absmax(const double* b, uint64_t k, uint64_t w, uint64_t ldb, unsigned long long* out,
                       cudaStream_t st) {
    if (!k || !w) return;
    int dev = 0, sms = 148;
    OZTT_CUDA(cudaGetDevice(&dev));
    OZTT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const uint64_t col_blocks = (w + 255) / 256;
    const uint64_t want = std::max<uint64_t>(1, (uint64_t)sms * 8 / col_blocks);
    const uint64_t chunks = std::min<uint64_t>(std::min<uint64_t>(want, k), 65535);
    const uint64_t rpc = (k + chunks - 1) / chunks;
    col_absmax_kernel<<<dim3((unsigned)col_blocks, (unsigned)((k + rpc - 1) / rpc)), 256, 0, st>>>(b, k, w, ldb, rpc,
                                                                                                 out);
    OZTT_CUDA(cudaGetLastError());
}

void launch_bcert_block(const double* b, uint64_t k, uint64_t w, uint64_t ldb, const double* g, uint64_t gstride,
                        double* acc, uint32_t* flags, cudaStream_t st) {
    if (!k || !w) return;
    bcert_block_kernel<<<(unsigned)((k + kCertWarps - 1) / kCertWarps), 256, 0, st>>>(b, k, w, ldb, g, gstride, acc,
                                                                                       flags);
    OZTT_CUDA(cudaGetLastError());
}

// B's scale from its column maxima (patterns, n of them) into *rgB, then the scaled sketch and the bounds of
// its error (bcert_finish_kernel).
void launch_bcert_finish(const unsigned long long* col_max, uint64_t n, const double* acc, uint64_t k, double c1,
                         double* rgB, double* y, double* ew, cudaStream_t st) {
    pow2_scale_kernel<<<1, 1024, 0, st>>>(col_max, n, rgB);
    OZTT_CUDA(cudaGetLastError());
    bcert_finish_kernel<<<(unsigned)std::min<uint64_t>((k + 255) / 256, 1024), 256, 0, st>>>(acc, k, rgB, c1, y, ew);
    OZTT_CUDA(cudaGetLastError());
}

// c1 of bcert_finish_kernel for rows of n elements: this pass's FP64 sum (products and additions in a
// lane, the warp's shuffles, the blocks' partial sums: fewer than n + 64 roundings on any term's path) and
// the reference's long-double sum (n products and additions, gamma(n + 2, 2^-64)), with room for the final
// rounding of the reference's sum to double.
double bcert_error_factor(uint64_t n) {
    auto gamma = [](double cnt, double u) { return cnt * u / (1.0 - cnt * u); };
    const double u = 0x1p-53;
    return (gamma((double)n + 64, u) + gamma((double)n + 2, 0x1p-64)) * (1 + 4 * u) + 2 * u;
}

// Bounds of the reference's nB (per column a sequential double sum of the scaled squares, then a sequential
// sum over the columns) from the bounded pass: acc[r*kBCertW + 16] = the unscaled sum of row r's squares.
// With T the exact sum, the reference's value is within (gamma(k+1) + gamma(n+1) + their product) T of
// T, and the sum formed here (row sums in FP64, then over the rows) within gamma(n + k + 64) T.
void bounded_nb(const double* acc, uint64_t k, uint64_t n, double rgB, double& lo, double& hi) {
    auto gamma = [](double cnt, double u) { return cnt * u / (1.0 - cnt * u); };
    const double u = 0x1p-53;
    double t = 0;
    for (uint64_t r = 0; r < k; ++r) t += acc[r * kBCertW + 16] * rgB * rgB;
    const double gk = gamma((double)k + 1, u), gn = gamma((double)n + 1, u);
    const double e = gk + gn + gk * gn + gamma((double)(n + k) + 64, u) + 4 * u;
    lo = t * (1 - e);
    hi = t * (1 + e);
}

// Bounds of nA, nB and nC around the reference's values from the rows' bounded statistics (cert: m x kCertW as
// band_certify_kernel writes them), B's column maxima (exact) and bounds of B's nB; TA, TB exact. Error terms,
// with gamma(n, u) = n u / (1 - n u), u = 2^-53 for binary64 and 2^-64 for the reference's long double:
//   a row's sum of squares: each side (the reference's sequential one, this warp-order one) is within
//     gamma(k+1, u) of the exact sum of positive terms;
//   a sketch value s_l[r]: the reference's long-double sum is within gamma(k+1, 2^-64) sum |t| of the exact
//     sum and is rounded once to double, this one within gamma(k+1, u) sum |t|; when y is this pass's bound
//     of B's sketch rather than the reference's (cert[18] nonzero), the two sums differ by a further
//     sum_j |x_j| ew_j at most;
//   the sums over rows (nA, each ||s_l||^2) gain gamma(m+1, u) on each side; nC's last few operations
//     16 u. The bounds are widened by these, so the reference's values lie inside.
PolicyBounds certified_policy_bounds(const double* cert, uint64_t m, uint64_t k, const double* col_max, uint64_t n,
                                     double nB_lo, double nB_hi, double rgB) {
    PolicyBounds pb;
    auto gamma = [](double cnt, double u) { return cnt * u / (1.0 - cnt * u); };
    const double u = 0x1p-53, ue = 0x1p-64;
    unsigned long long top = 0;
    for (uint64_t r = 0; r < m; ++r) {
        unsigned long long pat;
        std::memcpy(&pat, cert + r * kCertW, 8);
        if (pat >= 0x7FF0000000000000ull) return pb;  // NaN or Inf: the value checks report it
        top = std::max(top, pat);
    }
    double topv;
    std::memcpy(&topv, &top, 8);
    double rgA = 1.0;
    if (topv > 0) {
        int e = 0;
        std::frexp(topv, &e);
        rgA = std::ldexp(1.0, -std::min(std::max(e, -1000), 1000));
    }
    // TA and TB exactly as the reference sums them (combine_policy_stats with zero placeholders for the sums)
    std::vector<double> row_max(m), zeros(std::max(m, n), 0.0), zs(8 * m, 0.0);
    for (uint64_t r = 0; r < m; ++r) row_max[r] = cert[r * kCertW];
    const PolicyStats exact = combine_policy_stats(row_max.data(), m, col_max, n, zeros.data(), zeros.data(),
                                                   zs.data(), m, rgA, rgB);
    const double g_row = gamma((double)k + 1, u), g_rowe = gamma((double)k + 1, ue), g_sum = gamma((double)m + 1, u);
    long double nA = 0, q_lo[8] = {}, q_hi[8] = {};
    const double s2scale = rgA * rgA;
    for (uint64_t r = 0; r < m; ++r) {
        const double* c = cert + r * kCertW;
        nA += (long double)(c[1] * s2scale);
        for (int l = 0; l < 8; ++l) {
            const double sv = c[2 + l] * rgA, av = c[10 + l] * rgA, ev = c[18] * rgA;
            const double d = ((g_row * (1 + u) + g_rowe) * (av + ev) + ev + u * std::fabs(sv)) * (1 + 4 * u) + 0x1p-1000;
            const double lo = std::max(0.0, std::fabs(sv) - d), hi = std::fabs(sv) + d;
            q_lo[l] += (long double)lo * lo;
            q_hi[l] += (long double)hi * hi;
        }
    }
    const double e_nA = 2 * g_row + g_sum + 4 * u;
    auto nc_of = [](const long double* q) {
        long double cs2 = 0, cmx = 0;
        for (int l = 0; l < 8; ++l) {
            cs2 += q[l];
            cmx = std::max(cmx, q[l]);
        }
        return (double)((cs2 - cmx) / 7 / (1.0L + 2.0L * std::sqrt(2.0L / 8)));
    };
    pb.lo = pb.hi = exact;
    pb.lo.measured = pb.hi.measured = true;
    pb.lo.nB = nB_lo;
    pb.hi.nB = nB_hi;
    pb.lo.nA = (double)nA * (1 - e_nA);
    pb.hi.nA = (double)nA * (1 + e_nA);
    pb.lo.nC = nc_of(q_lo) * (1 - g_sum - 16 * u);
    pb.hi.nC = nc_of(q_hi) * (1 + g_sum + 16 * u);
    pb.usable = std::isfinite(pb.hi.nA) && std::isfinite(pb.hi.nC) && std::isfinite(nB_hi) && nB_lo >= 0 &&
                pb.lo.nC > 0 && rgA * topv < 2.0;
    return pb;
}


// ---- a first estimate from parts of A and B ------------------------------------------------------------------
// For a block of B's columns (k rows of w elements, rows ldb apart), one warp per row r: the row's sum of
// squares over the block and y_l[r] = sum_c b[r][c] g_l[c] (the sketch of the block), unscaled, in FP64.
__global__ void __launch_bounds__(256) block_rows_kernel(const double* __restrict__ b, uint64_t k, uint64_t w,
                                                         uint64_t ldb, const double* __restrict__ g, uint64_t gstride,
                                                         double* __restrict__ y, double* __restrict__ sq) {
    const uint64_t r = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= k) return;
    const double* br = b + r * ldb;
    double s2 = 0.0, sl[kVectors];
#pragma unroll
    for (int l = 0; l < kVectors; ++l) sl[l] = 0.0;
    for (uint64_t c = lane; c < w; c += 32) {
        const double v = __ldg(br + c);
        s2 = fma(v, v, s2);
#pragma unroll
        for (int l = 0; l < kVectors; ++l) sl[l] = fma(v, __ldg(g + (uint64_t)l * gstride + c), sl[l]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        s2 += __shfl_xor_sync(0xFFFFFFFFu, s2, o);
#pragma unroll
        for (int l = 0; l < kVectors; ++l) sl[l] += __shfl_xor_sync(0xFFFFFFFFu, sl[l], o);
    }
    if (lane == 0) {
        sq[r] = s2;
#pragma unroll
        for (int l = 0; l < kVectors; ++l) y[(uint64_t)l * k + r] = sl[l];
    }
}

// An estimate of the policy statistics with rows [0, rows_a) of A (row-major, k columns) standing for the
// whole A and columns [0, cols_b) of B (rows ldb apart) for the whole B: each part is measured as if it
// were the matrix (the statistics enter the width cap through the size-free ratio (TA nB + TB nA) / nC).
// It is what the first plan of a call that computes while its operands are still uploading is made from,
// and is then confirmed by the reference's statistics. The steps follow the upload: b_block measures B's
// block as soon as it lands (its column maxima, its rows' sums of squares and its sketch y_l = B g_l, g the
// probe vectors on the device), a_band each band of A's rows as it lands (band_certify_kernel with that
// sketch), finish combines them on the host.
PrefixEstimate::PrefixEstimate(uint64_t rows_a, uint64_t k, uint64_t cols_b, cudaStream_t st)
    : rows_a_(rows_a), k_(k), cols_b_(cols_b), st_(st), cmax_(st, cols_b * 8), y_(st, (uint64_t)kVectors * k * 8),
      sq_(st, k * 8), cert_(st, rows_a * kCertW * 8), flags_(st, 16) {
    OZTT_CUDA(cudaMemsetAsync(cmax_.p, 0, cols_b * 8, st));
    OZTT_CUDA(cudaMemsetAsync(flags_.p, 0, 16, st));
}

void PrefixEstimate::b_block(const double* b, uint64_t ldb, const double* g, uint64_t gstride) {
    launch_col_absmax(b, k_, cols_b_, ldb, cmax_.as<unsigned long long>(), st_);
    block_rows_kernel<<<(unsigned)((k_ * 32 + 255) / 256), 256, 0, st_>>>(b, k_, cols_b_, ldb, g, gstride,
                                                                         y_.as<double>(), sq_.as<double>());
    OZTT_CUDA(cudaGetLastError());
}

void PrefixEstimate::a_band(const double* a, uint64_t r0, uint64_t rows) {
    if (!rows) return;
    band_certify_kernel<<<(unsigned)((rows + kCertRows - 1) / kCertRows), 256, 0, st_>>>(
        a + r0 * k_, rows, k_, y_.as<double>(), nullptr, cert_.as<double>() + r0 * kCertW, flags_.as<uint32_t>());
    OZTT_CUDA(cudaGetLastError());
}

PolicyStats PrefixEstimate::finish(bool& ok, std::vector<uint64_t>* row_max) {
    ok = false;
    const uint64_t rows_a = rows_a_, k = k_, cols_b = cols_b_;
    std::vector<double> hcmax(cols_b), hsq(k), hcert(rows_a * kCertW);
    OZTT_CUDA(cudaMemcpyAsync(hcmax.data(), cmax_.p, cols_b * 8, cudaMemcpyDeviceToHost, st_));
    OZTT_CUDA(cudaMemcpyAsync(hsq.data(), sq_.p, k * 8, cudaMemcpyDeviceToHost, st_));
    OZTT_CUDA(cudaMemcpyAsync(hcert.data(), cert_.p, hcert.size() * 8, cudaMemcpyDeviceToHost, st_));
    OZTT_CUDA(cudaStreamSynchronize(st_));
    if (row_max) {
        row_max->resize(rows_a);
        for (uint64_t r = 0; r < rows_a; ++r) std::memcpy(&(*row_max)[r], &hcert[r * kCertW], 8);
    }
    // the power-of-two scale of each part (the magnitude patterns order like the magnitudes)
    const auto scale_of = [](double top) {
        if (!(top > 0) || !std::isfinite(top)) return 1.0;
        int e = 0;
        std::frexp(top, &e);
        return std::ldexp(1.0, -std::min(std::max(e, -1000), 1000));
    };
    double top_a = 0, top_b = 0;
    for (uint64_t r = 0; r < rows_a; ++r) top_a = std::max(top_a, hcert[r * kCertW]);
    for (uint64_t c = 0; c < cols_b; ++c) top_b = std::max(top_b, hcmax[c]);
    if (!std::isfinite(top_a) || !std::isfinite(top_b)) return {};
    const double rgA = scale_of(top_a), rgB = scale_of(top_b);
    double nb = 0;
    for (uint64_t r = 0; r < k; ++r) nb += hsq[r];
    std::vector<double> hmax(rows_a), hs2(rows_a), hsk((uint64_t)kVectors * rows_a);
    for (uint64_t r = 0; r < rows_a; ++r) {
        const double* c = hcert.data() + r * kCertW;
        hmax[r] = c[0];
        hs2[r] = c[1] * rgA * rgA;
        for (int l = 0; l < kVectors; ++l) hsk[(uint64_t)l * rows_a + r] = c[2 + l] * rgA * rgB;
    }
    std::vector<double> cs2(cols_b, 0.0);
    cs2[0] = nb * rgB * rgB;  // only the sum over the block's columns enters the statistics
    const PolicyStats ps =
        combine_policy_stats(hmax.data(), rows_a, hcmax.data(), cols_b, hs2.data(), cs2.data(), hsk.data(), rows_a,
                             rgA, rgB);
    ok = std::isfinite(ps.TA) && std::isfinite(ps.TB) && std::isfinite(ps.nA) && std::isfinite(ps.nB) &&
         std::isfinite(ps.nC) && ps.nC > 0;
    return ps;
}

PolicyStats device_policy_stats(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                                cudaStream_t st) {
    PolicyStatsRun run(m, n, k, N, st);
    run.b_cols(b, 0, n);
    run.b_done(b);
    run.a_cols(a, 0, k);
    run.a_done(a);
    return run.collect();
}

}  // namespace oztt

// Test hook: the certified decision from host copies of the bounded row statistics (m x 19, as
// band_certify_kernel writes them) and B's exact parts; bounds5 (NULL or 4 doubles) receives nA lo/hi and nC
// lo/hi, *decided whether the bounds decided the plan (which is then in *plan).
extern "C" int oztt_test_certified_plan(const double* cert, uint64_t m, uint64_t n, uint64_t k, const double* col_max,
                                        double nB_lo, double nB_hi, double rgB, uint32_t max_moduli,
                                        int32_t reconstruction, oztt_ii_plan* plan, int32_t* decided, double* bounds6,
                                        char* err, size_t errlen) {
    return oztt::guarded(err, errlen, [&] {
        const oztt::PolicyBounds pb = oztt::certified_policy_bounds(cert, m, k, col_max, n, nB_lo, nB_hi, rgB);
        if (bounds6) {
            bounds6[0] = pb.lo.nA;
            bounds6[1] = pb.hi.nA;
            bounds6[2] = pb.lo.nC;
            bounds6[3] = pb.hi.nC;
            bounds6[4] = pb.lo.nB;
            bounds6[5] = pb.hi.nB;
        }
        bool ok = false;
        std::string msg;
        const int rc = oztt::plan_ii_int8_certified(pb, m, n, k, max_moduli, reconstruction, *plan, msg, ok);
        if (rc != OZTT_OK) throw oztt::Error(rc, msg);
        *decided = ok ? 1 : 0;
    });
}

// Test hook: band_certify_kernel on device rows x (rows x k), the device sketch y (8 x k) and ew (k, or NULL),
// into the device rows out (rows x 19: the maximum's pattern, then the sums) and the device flag word.
extern "C" int oztt_test_band_certify(const double* x, uint64_t rows, uint64_t k, const double* y, const double* ew,
                                      double* out, uint32_t* flags, void* stream, char* err, size_t errlen) {
    return oztt::guarded(err, errlen, [&] {
        oztt::launch_band_certify(x, rows, k, y, ew, out, flags, reinterpret_cast<cudaStream_t>(stream));
    });
}

// Test hook: the bounds of nB and the error factor of the bounded pass over B, from its accumulators
// (k x 17 as bcert_block_kernel leaves them); out3 = {nB low, nB high, c1}.
extern "C" int oztt_test_bounded_nb(const double* acc, uint64_t k, uint64_t n, double rgB, double* out3, char* err,
                                    size_t errlen) {
    return oztt::guarded(err, errlen, [&] {
        oztt::bounded_nb(acc, k, n, rgB, out3[0], out3[1]);
        out3[2] = oztt::bcert_error_factor(n);
    });
}

// ---- C ABI: the statistics stages, for callers that hold panels of A and B on several devices ------
using oztt::Error;
using oztt::guarded;

extern "C" {

int oztt_stats_absmax(const double* x, uint64_t rows, uint64_t cols, int32_t mode, double* out, void* stream,
                      char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!x || !out || (mode != 0 && mode != 1)) throw Error(OZTT_EINVAL, "stats_absmax: bad arguments");
        oztt::launch_stats_absmax(x, rows, cols, mode, out, reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_stats_sumsq(const double* x, uint64_t rows, uint64_t cols, int32_t mode, double rg, double* out,
                     void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!x || !out || (mode != 0 && mode != 1)) throw Error(OZTT_EINVAL, "stats_sumsq: bad arguments");
        oztt::launch_stats_sumsq(x, rows, cols, mode, rg, out, reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_stats_sketch(const double* x, uint64_t rows, uint64_t cols, double rg, const double* v, uint64_t vstride,
                      double* out, uint64_t ostride, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!x || !v || !out || vstride < cols || ostride < rows) throw Error(OZTT_EINVAL, "stats_sketch: bad arguments");
        oztt::launch_stats_sketch(x, rows, cols, rg, v, vstride, out, ostride, reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_stats_sketch_chain(const double* x, uint64_t rows, uint64_t cols, uint64_t ldx, double rg, const double* v,
                            uint64_t vstride, void* state, int32_t carry, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!x || !v || !state || vstride < cols || ldx < cols) throw Error(OZTT_EINVAL, "stats_sketch_chain: bad arguments");
        if (!rows) return;
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        auto* e = reinterpret_cast<oztt::ext80::Ext*>(state);
        if (!cols) {
            if (!carry) OZTT_CUDA(cudaMemsetAsync(state, 0, rows * oztt::kVectors * sizeof(oztt::ext80::Ext), st));
            return;
        }
        oztt::sketch_kernel<false, true><<<oztt::sketch_blocks(rows), oztt::kSketchThreads, 0, st>>>(
            x, rows, cols, ldx, rg, nullptr, v, vstride, nullptr, e, rows, carry ? 1 : 0, nullptr);
        OZTT_CUDA(cudaGetLastError());
    });
}

int oztt_stats_sketch_round(const void* state, uint64_t count, double* out, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!state || !out) throw Error(OZTT_EINVAL, "stats_sketch_round: bad arguments");
        if (!count) return;
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        oztt::round_ext_kernel<<<(unsigned)std::min<uint64_t>((count + 255) / 256, 1024), 256, 0, st>>>(
            reinterpret_cast<const oztt::ext80::Ext*>(state), count, out);
        OZTT_CUDA(cudaGetLastError());
    });
}

int oztt_policy_stats_combine(const double* row_max, uint64_t m, const double* col_max, uint64_t n,
                              const double* row_sumsq, const double* col_sumsq, const double* sketch_s, double rgA,
                              double rgB, double* out5, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!row_max || !col_max || !row_sumsq || !col_sumsq || !sketch_s || !out5)
            throw Error(OZTT_EINVAL, "policy_stats_combine: null argument");
        const oztt::PolicyStats ps =
            oztt::combine_policy_stats(row_max, m, col_max, n, row_sumsq, col_sumsq, sketch_s, m, rgA, rgB);
        out5[0] = ps.TA;
        out5[1] = ps.TB;
        out5[2] = ps.nA;
        out5[3] = ps.nB;
        out5[4] = ps.nC;
    });
}

int oztt_ii_int8_plan_from_stats(uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction,
                                 int32_t fixed_bits, double TA, double TB, double nA, double nB, double nC,
                                 oztt_ii_plan* plan, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!plan) throw Error(OZTT_EINVAL, "null argument");
        oztt::PolicyStats ps;
        ps.TA = TA;
        ps.TB = TB;
        ps.nA = nA;
        ps.nB = nB;
        ps.nC = nC;
        ps.measured = true;
        std::string msg;
        const int rc = oztt::plan_ii_int8_with([&](uint32_t, uint32_t) { return ps; }, m, n, k, max_moduli,
                                               reconstruction, fixed_bits, *plan, msg);
        if (rc != OZTT_OK) throw Error(rc, msg);
    });
}

}  // extern "C"

// The 8 Gaussian vectors of the precision policy's norm estimate: 8 x N values of
// std::normal_distribution<double> over std::mt19937(12345), vector after vector, as the reference draws
// them (estimate_product_norm, src/backend/common/norm_estimate.hpp:48-73).
extern "C" void oztt_policy_vectors(uint32_t N, double* out) {
    std::mt19937 rng(12345);
    std::normal_distribution<double> normal(0.0, 1.0);
    for (int l = 0; l < oztt::kVectors; ++l)
        for (uint32_t j = 0; j < N; ++j) out[(size_t)l * N + j] = normal(rng);
}
