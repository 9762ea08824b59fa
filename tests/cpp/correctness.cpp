// SPDX-License-Identifier: Apache-2.0
//
// Acceptance test of the public C++ API on a B200, written against include/ozTTgemm/ozTTgemm.hpp
// only. It exercises the cases of the reference's tests/correctness.cpp (host validation :49-85,
// check() patterns :174-237, overlap, forced two-pass reconstruction, the max_moduli=2 rejection)
// for every available format and scheme, with the reference's bar: relative Frobenius error of C
// at most 8 DBL_EPSILON against a long-double reference. `--host-only` stops after the validation.
#include <ozTTgemm/ozTTgemm.hpp>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <iostream>
#include <limits>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

void expect(bool ok, const std::string& what) {
    if (!ok) throw std::runtime_error(what);
}
template <class F>
void expect_invalid(F&& f, const char* what) {
    try {
        f();
    } catch (const std::invalid_argument&) {
        return;
    }
    throw std::runtime_error(std::string("accepted invalid input: ") + what);
}
template <class F>
void expect_unsupported(F&& f, const char* what) {
    try {
        f();
    } catch (const std::invalid_argument&) {
        throw std::runtime_error(std::string("unsupported configuration reported as invalid input: ") + what);
    } catch (const std::runtime_error&) {
        return;
    }
    throw std::runtime_error(std::string("accepted an unsupported configuration: ") + what);
}

void validation(ozTTgemm::Context& ctx, ozTTgemm::Format fmt) {
    std::vector<double> a(4, 1), b(4, 1), c(4, 123);
    ozTTgemm::Options o;
    o.format = fmt;
    expect_invalid([&] { ctx.gemm(a, b, c, 0, 2, 2, o); }, "zero dimension");
    expect_invalid([&] { ctx.gemm(a, b, c, 2, 3, 2, o); }, "span size");
    expect_invalid(
        [&] {
            auto x = o;
            x.scheme = static_cast<ozTTgemm::Scheme>(7);
            ctx.gemm(a, b, c, 2, 2, 2, x);
        },
        "scheme enum");
    expect_invalid(
        [&] {
            auto x = o;
            x.format = static_cast<ozTTgemm::Format>(99);
            ctx.gemm(a, b, c, 2, 2, 2, x);
        },
        "format enum");
    expect_invalid(
        [&] {
            auto x = o;
            x.slices = 4;
            ctx.gemm(a, b, c, 2, 2, 2, x);
        },
        "slices with scheme II");
    expect_invalid(
        [&] {
            auto x = o;
            x.scheme = ozTTgemm::Scheme::I;
            x.reconstruction = ozTTgemm::Reconstruction::TwoPass;
            ctx.gemm(a, b, c, 2, 2, 2, x);
        },
        "reconstruction with scheme I");
    a[1] = std::numeric_limits<double>::quiet_NaN();
    expect_invalid([&] { ctx.gemm(a, b, c, 2, 2, 2, o); }, "NaN in A");
    a[1] = 1;
    b[2] = -std::numeric_limits<double>::infinity();
    expect_invalid([&] { ctx.gemm(a, b, c, 2, 2, 2, o); }, "Inf in B");
    b[2] = 1;
    a.assign(4, 0x1p-130);
    expect_invalid([&] { ctx.gemm(a, b, c, 2, 2, 2, o); }, "row maximum below 2^-126");
    expect(std::all_of(c.begin(), c.end(), [](double x) { return x == 123; }), "rejected call wrote C");
}

enum class Pattern { Uniform, ZeroA, Nonnegative, Scaled, Cancellation, ZeroRowColumn, Smallest, Largest };

double check(ozTTgemm::Context& ctx, const ozTTgemm::Options& o, std::size_t m, std::size_t n, std::size_t k,
             Pattern p) {
    std::mt19937_64 rng(42);
    std::uniform_real_distribution<double> u(-1, 1);
    std::vector<double> a(m * k), b(k * n), c(m * n, 123);
    for (auto& x : a) x = p == Pattern::ZeroA ? 0 : u(rng);
    for (auto& x : b) x = u(rng);
    switch (p) {
    case Pattern::Nonnegative:
        for (auto& x : a) x = std::abs(x);
        for (auto& x : b) x = std::abs(x);
        break;
    case Pattern::Scaled:
        for (std::size_t i = 0; i < m; ++i)
            for (std::size_t j = 0; j < k; ++j) a[i * k + j] = std::ldexp(a[i * k + j], int(i % 31) - 15);
        for (std::size_t i = 0; i < k; ++i)
            for (std::size_t j = 0; j < n; ++j) b[i * n + j] = std::ldexp(b[i * n + j], int(j % 27) - 13);
        break;
    case Pattern::ZeroRowColumn:
        for (std::size_t j = 0; j < k; ++j) a[j] = 0;
        for (std::size_t i = 0; i < k; ++i) b[i * n] = 0;
        break;
    case Pattern::Smallest:
        std::fill(a.begin(), a.end(), 0x1p-126);
        std::fill(b.begin(), b.end(), 1);
        break;
    case Pattern::Largest:
        std::fill(a.begin(), a.end(), 0x1.fep127);
        std::fill(b.begin(), b.end(), 1);
        break;
    case Pattern::Cancellation:
        for (std::size_t i = 0; i < m; ++i)
            for (std::size_t j = 0; j < k; ++j) a[i * k + j] = (j & 1) ? -1.0 : 1.0;
        std::fill(b.begin(), b.end(), 1);
        break;
    default: break;
    }
    const ozTTgemm::Info info = ctx.gemm(a, b, c, m, n, k, o);
    expect(info.padded_m % 64 == 0 && info.padded_n % 64 == 0 && info.padded_k % 32 == 0, "padded dimensions");
    long double err = 0, norm = 0;
    for (std::size_t i = 0; i < m; ++i)
        for (std::size_t j = 0; j < n; ++j) {
            long double ref = 0;
            for (std::size_t l = 0; l < k; ++l) ref += static_cast<long double>(a[i * k + l]) * b[l * n + j];
            expect(std::isfinite(c[i * n + j]), "nonfinite output");
            const long double d = c[i * n + j] - ref;
            err += d * d;
            norm += ref * ref;
        }
    const double rel = norm > 0 ? double(std::sqrt(err / norm)) : double(std::sqrt(err));
    std::cout << (o.scheme == ozTTgemm::Scheme::I ? "I " : "II ") << ozTTgemm::format_name(o.format) << ' ' << m
              << 'x' << n << 'x' << k << " pattern=" << int(p) << " error=" << rel << " slices=" << info.slices
              << " moduli=" << info.moduli << " bits=" << info.integer_bits << " passes=" << info.reconstruction_passes
              << '\n';
    expect(rel <= 8 * std::numeric_limits<double>::epsilon(), "error above 8 eps");
    return rel;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        const bool host_only = argc == 2 && std::string(argv[1]) == "--host-only";
        const ozTTgemm::Format formats[] = {ozTTgemm::Format::BF16, ozTTgemm::Format::FP16, ozTTgemm::Format::TF32,
                                            ozTTgemm::Format::BFP8, ozTTgemm::Format::FP8,  ozTTgemm::Format::INT8,
                                            ozTTgemm::Format::BFP4, ozTTgemm::Format::BFP2};
        ozTTgemm::Context ctx;
        ozTTgemm::Format first = ozTTgemm::Format::INT8;
        for (auto f : formats)
            if (ozTTgemm::is_available(f)) {
                first = f;
                break;
            }
        validation(ctx, first);
        if (host_only) {
            std::cout << "input validation passed\n";
            return 0;
        }
        // every available format with both schemes (the reference's tests/correctness.cpp:259-267)
        for (auto f : formats)
            if (ozTTgemm::is_available(f))
                for (auto scheme : {ozTTgemm::Scheme::I, ozTTgemm::Scheme::II}) {
                    ozTTgemm::Options o;
                    o.format = f;
                    o.scheme = scheme;
                    check(ctx, o, 64, 64, 64, Pattern::Uniform);
                    check(ctx, o, 3, 5, 7, Pattern::Nonnegative);
                }
        for (auto f : formats) {
            if (!ozTTgemm::is_available(f)) continue;
            for (auto scheme : {ozTTgemm::Scheme::I, ozTTgemm::Scheme::II}) {
                ozTTgemm::Options o;
                o.format = f;
                o.scheme = scheme;
                check(ctx, o, 65, 67, 97, Pattern::Scaled);
                check(ctx, o, 9, 11, 17, Pattern::ZeroA);
                check(ctx, o, 3, 5, 64, Pattern::Cancellation);
                check(ctx, o, 3, 5, 7, Pattern::ZeroRowColumn);
                check(ctx, o, 1, 1, 1, Pattern::Smallest);
                check(ctx, o, 1, 1, 1, Pattern::Largest);
            }
            // the fixed slice counts of the reference's test per format (tests/correctness.cpp:280)
            const unsigned fixed_slices[] = {10, 10, 10, 10, 12, 8, 16, 59};
            ozTTgemm::Options o;
            o.format = f;
            o.scheme = ozTTgemm::Scheme::I;
            o.slices = fixed_slices[static_cast<unsigned>(f)];
            check(ctx, o, 3, 5, 7, Pattern::Uniform);
            o = {};
            o.format = f;
            o.scheme = ozTTgemm::Scheme::II;
            check(ctx, o, 5056, 64, 32, Pattern::Uniform);
            o.reconstruction = ozTTgemm::Reconstruction::TwoPass;
            check(ctx, o, 64, 64, 64, Pattern::Uniform);
        }
        if (ozTTgemm::is_available(ozTTgemm::Format::BF16)) {
            ozTTgemm::Options o;
            o.scheme = ozTTgemm::Scheme::I;
            o.format = ozTTgemm::Format::BF16;
            check(ctx, o, 64, 64, 32768, Pattern::Nonnegative);  // beyond the reference's exact FP32 K block
        }
        ozTTgemm::Options o;
        o.format = first;
        std::vector<double> overlap{1, 2, 3, 4};
        const std::vector<double> identity{1, 0, 0, 1};
        ctx.gemm(overlap, identity, overlap, 2, 2, 2, o);
        expect(overlap == std::vector<double>{1, 2, 3, 4}, "output aliasing the input");
        o.max_moduli = 2;
        std::vector<double> a(64 * 64, 1), b(64 * 64, 1), c(64 * 64, 123);
        expect_unsupported([&] { ctx.gemm(a, b, c, 64, 64, 64, o); }, "two moduli");
        expect(std::all_of(c.begin(), c.end(), [](double x) { return x == 123; }), "rejected call wrote C");
        std::cout << "all correctness checks passed\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "FAILED: " << e.what() << '\n';
        return 1;
    }
}
