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
#include <random>
#include <vector>

#include "ext80.h"
#include "oztt_common.cuh"
#include "planner.hpp"
#include "runtime.cuh"

namespace oztt {

constexpr int kVectors = 8;

namespace {

// One warp per row: the largest |a| as the 63-bit pattern (nonnegative doubles order like integers).
__global__ void __launch_bounds__(256) row_absmax_kernel(const double* __restrict__ a, uint64_t m, uint64_t k,
                                                         unsigned long long* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const uint64_t nwarps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    const unsigned long long* pu = reinterpret_cast<const unsigned long long*>(a);
    for (uint64_t row = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < m; row += nwarps) {
        unsigned long long mx = 0;
        for (uint64_t j = lane; j < k; j += 32) {
            const unsigned long long v = __ldg(pu + row * k + j) & 0x7FFFFFFFFFFFFFFFull;
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

// Column maxima: a thread per column over a chunk of rows, combined with atomicMax.
__global__ void __launch_bounds__(256) col_absmax_kernel(const double* __restrict__ b, uint64_t k, uint64_t n,
                                                         uint64_t rows_per_chunk, unsigned long long* __restrict__ out) {
    const uint64_t col = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= n) return;
    const uint64_t r0 = (uint64_t)blockIdx.y * rows_per_chunk, r1 = min(k, r0 + rows_per_chunk);
    const unsigned long long* pu = reinterpret_cast<const unsigned long long*>(b);
    unsigned long long mx = 0;
    for (uint64_t r = r0; r < r1; ++r) {
        const unsigned long long v = __ldg(pu + r * n + col) & 0x7FFFFFFFFFFFFFFFull;
        mx = v > mx ? v : mx;
    }
    if (mx) atomicMax(out + col, mx);
}

// sum_c (a[i][c]*rg)^2 for each row i, c ascending, one rounding per operation.
__global__ void __launch_bounds__(128) row_sumsq_kernel(const double* __restrict__ a, uint64_t m, uint64_t k,
                                                        double rg, double* __restrict__ out) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const double* p = a + i * k;
    double sq = 0.0;
    for (uint64_t c = 0; c < k; ++c) {
        const double v = __dmul_rn(__ldg(p + c), rg);
        sq = __dadd_rn(sq, __dmul_rn(v, v));
    }
    out[i] = sq;
}

// sum_r (b[r][j]*rg)^2 for each column j, r ascending.
__global__ void __launch_bounds__(128) col_sumsq_kernel(const double* __restrict__ b, uint64_t k, uint64_t n,
                                                        double rg, double* __restrict__ out) {
    const uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    double sq = 0.0;
    for (uint64_t r = 0; r < k; ++r) {
        const double v = __dmul_rn(__ldg(b + r * n + j), rg);
        sq = __dadd_rn(sq, __dmul_rn(v, v));
    }
    out[j] = sq;
}

// out[l][r] = (double) sum_{j < cols} ext((x[r][j]*rg)) * ext(v[l][j]), the sum in 64-bit-significand
// arithmetic, j ascending. Thread t handles row t / 8 and vector t % 8, so a warp reads 4 rows and
// the 8 vectors; the rows stay in L1 while the warp walks them.
__global__ void __launch_bounds__(256) sketch_kernel(const double* __restrict__ x, uint64_t rows, uint64_t cols,
                                                     double rg, const double* __restrict__ v, uint64_t vstride,
                                                     double* __restrict__ out, uint64_t ostride) {
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t r = t / kVectors, l = t % kVectors;
    if (r >= rows) return;
    const double* xr = x + r * cols;
    const double* vl = v + l * vstride;
    ext80::Ext acc = ext80::zero();
    for (uint64_t j = 0; j < cols; ++j) {
        const double xs = __dmul_rn(__ldg(xr + j), rg);
        acc = ext80::add(acc, ext80::mul(ext80::from_double(xs), ext80::from_double(__ldg(vl + j))));
    }
    out[l * ostride + r] = ext80::to_double(acc);
}

double pattern_to_double(unsigned long long u) { return ext80::double_of(u); }

// 1 / (2^e) for the exponent e of the largest magnitude, e clamped to [-1000, 1000] (oz_pow2_scale).
double inverse_pow2_scale(double mx) {
    if (!(mx > 0) || !std::isfinite(mx)) return 1.0;
    int e;
    std::frexp(mx, &e);
    e = std::min(std::max(e, -1000), 1000);
    return 1.0 / std::ldexp(1.0, e);
}

}  // namespace

PolicyStats device_policy_stats(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                                cudaStream_t st) {
    PolicyStats ps;
    int dev = 0, sms = 148;
    OZTT_CUDA(cudaGetDevice(&dev));
    OZTT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // maxima
    DevBuf rmax(st, m * 8), cmax(st, n * 8);
    OZTT_CUDA(cudaMemsetAsync(cmax.p, 0, n * 8, st));
    row_absmax_kernel<<<(unsigned)std::min<uint64_t>((m + 7) / 8, (uint64_t)sms * 32), 256, 0, st>>>(
        a, m, k, rmax.as<unsigned long long>());
    OZTT_CUDA(cudaGetLastError());
    {
        const uint64_t col_blocks = (n + 255) / 256;
        const uint64_t want = std::max<uint64_t>(1, (uint64_t)sms * 8 / std::max<uint64_t>(col_blocks, 1));
        const uint64_t chunks = std::min<uint64_t>(std::min<uint64_t>(want, k), 65535);
        const uint64_t rpc = (k + chunks - 1) / chunks;
        col_absmax_kernel<<<dim3((unsigned)col_blocks, (unsigned)((k + rpc - 1) / rpc)), 256, 0, st>>>(
            b, k, n, rpc, cmax.as<unsigned long long>());
        OZTT_CUDA(cudaGetLastError());
    }
    std::vector<unsigned long long> hr(m), hc(n);
    OZTT_CUDA(cudaMemcpyAsync(hr.data(), rmax.p, m * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaMemcpyAsync(hc.data(), cmax.p, n * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaStreamSynchronize(st));
    double gA = 0, gB = 0;
    for (auto u : hr) gA = std::max(gA, pattern_to_double(u));
    for (auto u : hc) gB = std::max(gB, pattern_to_double(u));
    const double rgA = inverse_pow2_scale(gA), rgB = inverse_pow2_scale(gB);
    // sums of squares per row / column on the device
    DevBuf s2r(st, m * 8), s2c(st, n * 8);
    row_sumsq_kernel<<<(unsigned)((m + 127) / 128), 128, 0, st>>>(a, m, k, rgA, s2r.as<double>());
    OZTT_CUDA(cudaGetLastError());
    col_sumsq_kernel<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(b, k, n, rgB, s2c.as<double>());
    OZTT_CUDA(cudaGetLastError());
    // the 8 Gaussian vectors of length N from mt19937(12345), in the reference's draw order
    std::vector<double> g((size_t)kVectors * N);
    {
        std::mt19937 rng(12345);
        std::normal_distribution<double> normal(0.0, 1.0);
        for (int l = 0; l < kVectors; ++l)
            for (uint32_t j = 0; j < N; ++j) g[(size_t)l * N + j] = normal(rng);
    }
    DevBuf dg(st, g.size() * 8), dy(st, (uint64_t)kVectors * k * 8), ds(st, (uint64_t)kVectors * m * 8);
    OZTT_CUDA(cudaMemcpyAsync(dg.p, g.data(), g.size() * 8, cudaMemcpyHostToDevice, st));
    // y_l = B g_l over the real columns (the padded ones add exact zeros), then s_l = A y_l
    sketch_kernel<<<(unsigned)((k * kVectors + 255) / 256), 256, 0, st>>>(b, k, n, rgB, dg.as<double>(), N,
                                                                          dy.as<double>(), k);
    OZTT_CUDA(cudaGetLastError());
    sketch_kernel<<<(unsigned)((m * kVectors + 255) / 256), 256, 0, st>>>(a, m, k, rgA, dy.as<double>(), k,
                                                                          ds.as<double>(), m);
    OZTT_CUDA(cudaGetLastError());
    std::vector<double> h2r(m), h2c(n), hs((size_t)kVectors * m);
    OZTT_CUDA(cudaMemcpyAsync(h2r.data(), s2r.p, m * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaMemcpyAsync(h2c.data(), s2c.p, n * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaMemcpyAsync(hs.data(), ds.p, hs.size() * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaStreamSynchronize(st));
    // the host's part, in the reference's order
    for (uint64_t r = 0; r < m; ++r) {
        const double mx = pattern_to_double(hr[r]) * rgA;
        if (mx > 0) {
            const double t = std::exp2(std::ceil(std::log2(mx)));
            ps.TA += t * t;
        }
        ps.nA += h2r[r];
    }
    for (uint64_t c = 0; c < n; ++c) {
        const double mx = pattern_to_double(hc[c]) * rgB;
        if (mx > 0) {
            const double t = std::exp2(std::ceil(std::log2(mx)));
            ps.TB += t * t;
        }
        ps.nB += h2c[c];
    }
    double cs2 = 0, cmx = 0;
    for (int l = 0; l < kVectors; ++l) {
        double q = 0;
        const double* s = hs.data() + (size_t)l * m;
        for (uint64_t i = 0; i < m; ++i) q += s[i] * s[i];
        cs2 += q;
        cmx = std::max(cmx, q);
    }
    ps.nC = (cs2 - cmx) / (kVectors - 1) / (1.0 + 2.0 * std::sqrt(2.0 / (double)kVectors));
    ps.measured = true;
    return ps;
}

}  // namespace oztt

// ---- C ABI: the statistics stages, for callers that hold panels of A and B on several devices ------
using oztt::Error;
using oztt::guarded;

extern "C" {

int oztt_stats_absmax(const double* x, uint64_t rows, uint64_t cols, int32_t mode, double* out, void* stream,
                      char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!x || !out || (mode != 0 && mode != 1)) throw Error(OZTT_EINVAL, "stats_absmax: bad arguments");
        if (!rows || !cols) return;
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        int dev = 0, sms = 148;
        OZTT_CUDA(cudaGetDevice(&dev));
        OZTT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        auto* o = reinterpret_cast<unsigned long long*>(out);  // nonnegative doubles order like their patterns
        if (mode == 0) {
            oztt::row_absmax_kernel<<<(unsigned)std::min<uint64_t>((rows + 7) / 8, (uint64_t)sms * 32), 256, 0, st>>>(
                x, rows, cols, o);
        } else {
            OZTT_CUDA(cudaMemsetAsync(out, 0, cols * 8, st));
            const uint64_t col_blocks = (cols + 255) / 256;
            const uint64_t want = std::max<uint64_t>(1, (uint64_t)sms * 8 / std::max<uint64_t>(col_blocks, 1));
            const uint64_t chunks = std::min<uint64_t>(std::min<uint64_t>(want, rows), 65535);
            const uint64_t rpc = (rows + chunks - 1) / chunks;
            oztt::col_absmax_kernel<<<dim3((unsigned)col_blocks, (unsigned)((rows + rpc - 1) / rpc)), 256, 0, st>>>(
                x, rows, cols, rpc, o);
        }
        OZTT_CUDA(cudaGetLastError());
    });
}

int oztt_stats_sumsq(const double* x, uint64_t rows, uint64_t cols, int32_t mode, double rg, double* out,
                     void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!x || !out || (mode != 0 && mode != 1)) throw Error(OZTT_EINVAL, "stats_sumsq: bad arguments");
        if (!rows || !cols) return;
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        if (mode == 0)
            oztt::row_sumsq_kernel<<<(unsigned)((rows + 127) / 128), 128, 0, st>>>(x, rows, cols, rg, out);
        else
            oztt::col_sumsq_kernel<<<(unsigned)((cols + 127) / 128), 128, 0, st>>>(x, rows, cols, rg, out);
        OZTT_CUDA(cudaGetLastError());
    });
}

int oztt_stats_sketch(const double* x, uint64_t rows, uint64_t cols, double rg, const double* v, uint64_t vstride,
                      double* out, uint64_t ostride, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!x || !v || !out || vstride < cols || ostride < rows) throw Error(OZTT_EINVAL, "stats_sketch: bad arguments");
        if (!rows) return;
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        oztt::sketch_kernel<<<(unsigned)((rows * oztt::kVectors + 255) / 256), 256, 0, st>>>(x, rows, cols, rg, v,
                                                                                             vstride, out, ostride);
        OZTT_CUDA(cudaGetLastError());
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
