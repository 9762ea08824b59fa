// SPDX-License-Identifier: Apache-2.0
//
// Evaluation utilities of the C ABI: the reference evaluator's seeded input generator and output hash
// (evaluation/numerics.hpp:19-57), so that benchmarks and users can reproduce the reference's inputs
// (seed 7 for its published tables) and compare outputs by hash. The generator consumes the Mersenne
// twister exactly as the reference does (libstdc++ uniform_real_distribution and the polar-method
// normal_distribution), element by element, all of A before B.
#include <cmath>
#include <cstring>
#include <random>

#include "oztt_cuda.h"

extern "C" void oztt_eval_inputs(double* a, double* b, uint64_t m, uint64_t n, uint64_t k, double phi,
                                 uint32_t seed) {
    std::mt19937 rng(seed);
    const uint64_t na = m * k, nb = k * n;
    if (phi < 0) {
        std::uniform_real_distribution<double> u(-1, 1);
        for (uint64_t i = 0; i < na; ++i) a[i] = u(rng);
        for (uint64_t i = 0; i < nb; ++i) b[i] = u(rng);
        return;
    }
    std::uniform_real_distribution<double> u(0, 1);
    std::normal_distribution<double> normal(0, 1);
    const auto next = [&] {
        const double v = u(rng);
        const double z = normal(rng);
        return (v - 0.5) * std::exp(phi * z);
    };
    for (uint64_t i = 0; i < na; ++i) a[i] = next();
    for (uint64_t i = 0; i < nb; ++i) b[i] = next();
}

extern "C" uint64_t oztt_eval_output_hash(const double* c, uint64_t count) {
    uint64_t h = 1469598103934665603ull;
    for (uint64_t z = 0; z < count; ++z) {
        uint64_t u;
        std::memcpy(&u, &c[z], 8);
        for (int sh = 0; sh < 64; sh += 8) {
            h ^= (u >> sh) & 0xFFu;
            h *= 1099511628211ull;
        }
    }
    return h;
}

// Host model of one row of the device's long-double sketch (stats.cu, sketch_kernel): the sum
// (double) sum_j (long double)(x[j]*rg) * g[j] in the 64-bit-significand arithmetic of ext80.h, for
// the CPU tests of that arithmetic against the host's own long double.
#include "ext80.h"
extern "C" double oztt_test_ext80_dot(const double* x, const double* g, uint64_t n, double rg) {
    namespace e = oztt::ext80;
    e::Ext acc = e::zero();
    for (uint64_t j = 0; j < n; ++j) acc = e::add(acc, e::mul(e::from_double(x[j] * rg), e::from_double(g[j])));
    return e::to_double(acc);
}
