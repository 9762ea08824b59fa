// SPDX-License-Identifier: Apache-2.0
//
// Public C++ API (include/ozTTgemm/ozTTgemm.hpp) on top of the CUDA backend, and its C-ABI form
// oztt_gemm. Front-end semantics follow the reference's src/context.cpp:
//   * the same checks in the same order, before the device is touched and before C is written
//     (the options :82-93, span sizes and padding to 64/64/32 :103-110, finiteness and the
//     [2^-126, largest BF16] range of every nonzero row maximum of A and column maximum of B :37-62),
//     with the same exception types and messages; the Tensix tile-offset bound (:111-114) is a limit of
//     that device and is not applied;
//   * one process-wide mutex serialises the calls of all contexts (:19, :152);
//   * the device is opened on the first valid call; Info reports the padded dimensions (:176-180);
//   * all input is consumed before C is written, so C may overlap A or B.
// The finiteness and range checks are made from the device-measured row and column maxima once A and B
// are uploaded, before the plan is made and C is written.
// Under an evaluation Scope (include/evaluation_hooks.hpp, the reference's src/evaluation_hooks.hpp) a
// call runs its device pipeline through the evaluator's phase timing and whole-pass check, with the
// Ozaki II width the Scope fixes (src/ozaki2.cpp:447).
// Dispatch (src/dispatch.cpp:18-50): INT8, FP8 (e4m3 digits), BF16, FP16 and TF32 are built, both schemes;
// the Tenstorrent block formats BFP8/BFP4/BFP2 are not available on this hardware.
#include <ozTTgemm/ozTTgemm.hpp>
#include <evaluation_hooks.hpp>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>

#include "oztt_cuda.h"
#include "planner.hpp"

namespace oztt {
int run_ii_digit_planned(int device_id, int32_t format, const double* a, const double* b, double* c, uint64_t m,
                         uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits,
                         oztt_digit_plan& p, std::string& err);
}  // namespace oztt

namespace ozTTgemm {
namespace {

namespace ev = detail::evaluation;

std::mutex runtime_mutex;

std::size_t round_up_to(std::size_t v, std::size_t q) { return (v + q - 1) / q * q; }

// Finiteness and the range of every nonzero row maximum of A and column maximum of B, with the
// reference's order of reports (context.cpp:37-62): A's rows in order (a row's NaN/Inf before its
// maximum), then any NaN/Inf in B, then B's column maxima. The scans run on the process's host
// threads; each records per row (per column block) what it found, and the reports are made in order
// after. One unsigned maximum of the magnitude patterns (the sign bit cleared) gives both answers:
// nonnegative doubles order like their bit patterns, and a pattern at or above that of +Inf is an Inf
// or a NaN.
constexpr std::uint64_t kMagnitude = 0x7FFFFFFFFFFFFFFFull, kInfPattern = 0x7FF0000000000000ull;

std::uint64_t max_pattern(const std::uint64_t* p, std::size_t count) {
    std::uint64_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
    std::size_t j = 0;
    for (; j + 4 <= count; j += 4) {
        m0 = std::max(m0, p[j] & kMagnitude);
        m1 = std::max(m1, p[j + 1] & kMagnitude);
        m2 = std::max(m2, p[j + 2] & kMagnitude);
        m3 = std::max(m3, p[j + 3] & kMagnitude);
    }
    for (; j < count; ++j) m0 = std::max(m0, p[j] & kMagnitude);
    return std::max(std::max(m0, m1), std::max(m2, m3));
}

double pattern_value(std::uint64_t u) {
    double x;
    std::memcpy(&x, &u, sizeof x);
    return x;
}

// The reports from the magnitude-pattern maxima of A's rows and B's columns, in the reference's order.
void report_maxima(const std::uint64_t* row_max, std::size_t m, const std::uint64_t* col_max, std::size_t n) {
    constexpr double maximum = 0x1.fep127;
    constexpr double minimum = 0x1p-126;
    const auto out_of_range = [&](double x) { return x != 0 && (x < minimum || x > maximum); };
    const char* range_msg = "each nonzero row maximum of A and column maximum of B must be in [2^-126, max_BF16]";
    for (std::size_t i = 0; i < m; ++i) {
        if (row_max[i] >= kInfPattern) throw std::invalid_argument("A contains NaN or infinity");
        if (out_of_range(pattern_value(row_max[i]))) throw std::invalid_argument(range_msg);
    }
    for (std::size_t j = 0; j < n; ++j)
        if (col_max[j] >= kInfPattern) throw std::invalid_argument("B contains NaN or infinity");
    for (std::size_t j = 0; j < n; ++j)
        if (out_of_range(pattern_value(col_max[j]))) throw std::invalid_argument(range_msg);
}

void check_values(std::span<const double> a, std::span<const double> b, std::size_t m, std::size_t n, std::size_t k) {
    const auto* pa = reinterpret_cast<const std::uint64_t*>(a.data());
    const auto* pb = reinterpret_cast<const std::uint64_t*>(b.data());
    std::vector<std::uint64_t> row_max(m);
    oztt::parallel_ranges(m, [&](std::uint64_t r0, std::uint64_t r1) {
        for (std::uint64_t i = r0; i < r1; ++i) row_max[i] = max_pattern(pa + i * k, k);
    });
    std::vector<std::uint64_t> col_max(n, 0);
    oztt::parallel_ranges(n, [&](std::uint64_t c0, std::uint64_t c1) {
        std::uint64_t* mx = col_max.data();
        for (std::size_t i = 0; i < k; ++i) {
            const std::uint64_t* p = pb + i * n;
            for (std::uint64_t j = c0; j < c1; ++j) mx[j] = std::max(mx[j], p[j] & kMagnitude);
        }
    });
    report_maxima(row_max.data(), m, col_max.data(), n);
}
// The option rules in the order the reference examines them (src/context.cpp:79-93); the first one that
// holds is reported. The enum values are range-checked because a caller can cast any integer to them.
using OptionRule = std::pair<bool (*)(const Options&), const char*>;
const OptionRule kOptionRules[] = {
    {[](const Options& o) { return o.scheme != Scheme::I && o.scheme != Scheme::II; }, "unknown Ozaki scheme"},
    {[](const Options& o) { return !is_available(o.format); }, "format is unknown or was not built"},
    {[](const Options& o) {
         return o.reconstruction != Reconstruction::Automatic && o.reconstruction != Reconstruction::OnePass &&
                o.reconstruction != Reconstruction::TwoPass;
     },
     "unknown reconstruction mode"},
    {[](const Options& o) { return o.slices > 256; }, "slices must be zero (automatic) or at most 256"},
    {[](const Options& o) { return o.max_moduli > 24; }, "max_moduli exceeds the supported bound of 24"},
    {[](const Options& o) {
         return o.scheme == Scheme::I && (o.max_moduli != 0 || o.reconstruction != Reconstruction::Automatic);
     },
     "max_moduli and reconstruction apply only to Ozaki II"},
    {[](const Options& o) { return o.scheme == Scheme::II && o.slices != 0; }, "slices applies only to Ozaki I"},
};

void check_options(const Options& o) {
    for (const auto& [broken, message] : kOptionRules)
        if (broken(o)) throw std::invalid_argument(message);
}

// The size rules (src/context.cpp:103-110), in the reference's order: A's span, then B's, then C's; a zero
// dimension or an element count whose byte size overflows size_t is reported where the reference computes
// that count, so a wrong span of A is reported before a zero n. Then each padded dimension must stay in
// the signed 32-bit index range that the planner's dimensions use.
constexpr const char* kBadDims = "matrix dimensions are zero or overflow the address space";
constexpr const char* kBadSpans = "matrix span sizes do not match m, n, k";

std::size_t elements_or_throw(std::size_t rows, std::size_t cols) {
    const bool bad = rows == 0 || cols == 0 || rows > std::numeric_limits<std::size_t>::max() / sizeof(double) / cols;
    if (bad) throw std::invalid_argument(kBadDims);
    return rows * cols;
}

std::uint32_t padded_dim(std::size_t value, std::size_t quantum) {
    const std::size_t top = (std::size_t)std::numeric_limits<std::int32_t>::max() - quantum;
    if (value == 0 || value > top) throw std::invalid_argument("matrix dimension exceeds the supported device index range");
    return (std::uint32_t)round_up_to(value, quantum);
}
struct Checked {
    std::uint32_t mp, np, kp;
    std::size_t c_size;
};
// An ordinary call (either scheme, any format) makes the value checks from the row and column maxima
// that the device measures for the plan statistics (the same magnitude patterns, so the same reports in
// the same order), before the plan and before C is written; should the device or a fixed-slice plan fail
// before that, the host checks run after all, so that an invalid input is still the error reported.
// Profiled calls (an evaluation Scope) run the host checks here, before the device is touched.
bool checks_during_upload(const Options&) { return ev::active == nullptr; }

Checked validate(const Options& options, std::span<const double> a, std::span<const double> b,
                 std::optional<std::size_t> c_size, std::size_t m, std::size_t n, std::size_t k) {
    check_options(options);
    if (a.size() != elements_or_throw(m, k)) throw std::invalid_argument(kBadSpans);
    if (b.size() != elements_or_throw(k, n)) throw std::invalid_argument(kBadSpans);
    const std::size_t mn = elements_or_throw(m, n);
    if (c_size && *c_size != mn) throw std::invalid_argument(kBadSpans);
    Checked v{};
    v.mp = padded_dim(m, 64);
    v.np = padded_dim(n, 64);
    v.kp = padded_dim(k, 32);
    v.c_size = mn;
    // (The reference also bounds the Tensix tile offsets of the padded matrices, src/context.cpp:111-114; the
    // B200 kernels index HBM with 64-bit offsets, so that device limit does not apply here.)
    if (!checks_during_upload(options)) check_values(a, b, m, n, k);
    return v;
}
Info ii_info(const oztt_ii_plan& plan, const Options& opt, const Checked& v) {
    Info info{Scheme::II, opt.format};
    info.moduli = (std::uint32_t)plan.S;
    info.integer_bits = (std::uint32_t)plan.b;
    info.reconstruction_passes = plan.two_pass ? 2u : 1u;
    info.padded_m = v.mp;
    info.padded_n = v.np;
    info.padded_k = v.kp;
    return info;
}
// The Ozaki II width an evaluation Scope open on this thread fixes (0: none).
std::int32_t evaluation_fixed_bits() { return ev::active ? (std::int32_t)ev::active->fixed_bits : 0; }
int32_t recon_code(Reconstruction r) {
    return r == Reconstruction::OnePass ? OZTT_RECON_ONE : (r == Reconstruction::TwoPass ? OZTT_RECON_TWO : OZTT_RECON_AUTO);
}
[[noreturn]] void rethrow(int code, const std::string& msg) {
    if (code == OZTT_EINVAL) throw std::invalid_argument(msg);
    if (code == OZTT_ENOMEM) throw std::bad_alloc();
    throw std::runtime_error(msg);
}

}  // namespace

bool is_available(Format format) noexcept {
    return format == Format::INT8 || format == Format::FP8 || format == Format::BF16 || format == Format::FP16 ||
           format == Format::TF32;
}

const char* format_name(Format format) noexcept {
    switch (format) {
    case Format::BF16: return "BF16";
    case Format::FP16: return "FP16";
    case Format::TF32: return "TF32";
    case Format::BFP8: return "BFP8";
    case Format::FP8: return "FP8";
    case Format::INT8: return "INT8";
    case Format::BFP4: return "BFP4";
    case Format::BFP2: return "BFP2";
    default: return "unknown";
    }
}

struct Context::Impl {
    explicit Impl(DeviceOptions o) : options(std::move(o)) {
        if (options.device_id < 0) throw std::invalid_argument("device_id must be nonnegative");
    }
    Info execute(std::span<const double> a, std::span<const double> b, std::span<double> c, std::size_t m,
                 std::size_t n, std::size_t k, const Options& opt, const Checked& v);
    DeviceOptions options;
    bool opened = false;
};

Context::Context(DeviceOptions options) : impl_(std::make_unique<Impl>(std::move(options))) {}
Context::~Context() = default;

Info Context::Impl::execute(std::span<const double> a, std::span<const double> b, std::span<double> c, std::size_t m,
                            std::size_t n, std::size_t k, const Options& opt, const Checked& v) {
    std::lock_guard lock(runtime_mutex);
    // The value checks of an ordinary call are made from the maxima the device measures while A and B are
    // uploaded; should the device (or a fixed-slice plan) fail first, the host checks run after all.
    bool checked = false;
    const auto check_maxima = [&](const std::uint64_t* row_max, const std::uint64_t* col_max) {
        checked = true;
        report_maxima(row_max, m, col_max, n);
    };
    const auto fail = [&](int rc, const std::string& msg) {
        if (!checked && checks_during_upload(opt)) check_values(a, b, m, n, k);
        rethrow(rc, msg);
    };
    if (opt.format != Format::INT8 && opt.scheme == Scheme::II) {  // the digit formats
        oztt_digit_plan plan;
        std::string msg;
        const int rc =
            ev::active ? oztt::run_ii_digit_planned(options.device_id, (int32_t)opt.format, a.data(), b.data(),
                                                    c.data(), m, n, k, opt.max_moduli, recon_code(opt.reconstruction),
                                                    evaluation_fixed_bits(), plan, msg)
                       : oztt::run_ii_digit_streamed(options.device_id, (int32_t)opt.format, a.data(), b.data(),
                                                     c.data(), m, n, k, opt.max_moduli, recon_code(opt.reconstruction),
                                                     check_maxima, plan, msg);
        if (rc != OZTT_OK) fail(rc, msg);
        opened = true;
        return ii_info(plan.base, opt, v);
    }
    if (opt.scheme == Scheme::I) {
        const oztt::I1Format& fmt = *oztt::i1_format((int32_t)opt.format);
        oztt_i_plan plan;
        std::string msg;
        if (opt.slices) {
            // a fixed slice count: the feasibility checks before any device work, as the reference (an invalid
            // value is still the error reported first)
            const int rc = oztt::plan_i(a.data(), b.data(), m, n, k, opt.slices, fmt, plan, msg);
            if (rc != OZTT_OK) fail(rc, msg);
        }
        // the slice count (when not fixed) selected from statistics measured on the device: during the
        // streamed upload, or after one plain upload under an evaluation Scope
        const int rc = ev::active ? oztt::run_i_uploaded(options.device_id, a.data(), b.data(), c.data(), m, n, k,
                                                         opt.slices, fmt, plan, msg)
                                  : oztt::run_i_streamed(options.device_id, (int32_t)opt.format, a.data(), b.data(),
                                                         c.data(), m, n, k, opt.slices, check_maxima, plan, msg);
        if (rc != OZTT_OK) fail(rc, msg);
        opened = true;
        Info info{Scheme::I, opt.format};
        info.slices = (std::uint32_t)plan.p;
        info.padded_m = v.mp;
        info.padded_n = v.np;
        info.padded_k = v.kp;
        return info;
    }
    if (ev::active) {
        // a profiled call of the evaluator (its values were checked on the host in validate): the plain
        // upload and the pipeline under the Scope's phase timing and whole-pass check
        oztt_ii_plan plan;
        std::string msg;
        const int rc = oztt::run_ii_int8_uploaded(options.device_id, a.data(), b.data(), c.data(), m, n, k,
                                                  opt.max_moduli, recon_code(opt.reconstruction),
                                                  evaluation_fixed_bits(), plan, msg);
        if (rc != OZTT_OK) rethrow(rc, msg);
        opened = true;
        return ii_info(plan, opt, v);
    }
    // A and B go to the device in chunks; the precision policy measures them there (bit-identical to the
    // host measurement), the values are checked from the measured maxima and the host makes the
    // decisions; C is written only after that.
    oztt_ii_plan plan;
    std::string msg;
    const int rc = oztt::run_ii_int8_streamed(options.device_id, a.data(), b.data(), c.data(), m, n, k, opt.max_moduli,
                                              recon_code(opt.reconstruction), check_maxima, plan, msg);
    if (rc != OZTT_OK) fail(rc, msg);
    opened = true;
    return ii_info(plan, opt, v);
}

Info Context::gemm(std::span<const double> a, std::span<const double> b, std::span<double> c, std::size_t m,
                   std::size_t n, std::size_t k, const Options& options) {
    const Checked v = validate(options, a, b, c.size(), m, n, k);
    return impl_->execute(a, b, c, m, n, k, options, v);
}

std::vector<double> Context::multiply(std::span<const double> a, std::span<const double> b, std::size_t m,
                                      std::size_t n, std::size_t k, const Options& options) {
    const Checked v = validate(options, a, b, std::nullopt, m, n, k);
    std::vector<double> c(v.c_size);
    impl_->execute(a, b, c, m, n, k, options, v);
    return c;
}

}  // namespace ozTTgemm

extern "C" int oztt_is_available(int32_t format) {
    return ozTTgemm::is_available(static_cast<ozTTgemm::Format>(format)) ? 1 : 0;
}
extern "C" const char* oztt_format_name(int32_t format) {
    return ozTTgemm::format_name(static_cast<ozTTgemm::Format>(format));
}

extern "C" int oztt_gemm(int device_id, const double* a, uint64_t a_len, const double* b, uint64_t b_len, double* c,
                         uint64_t c_len, uint64_t m, uint64_t n, uint64_t k, const oztt_options* opt, oztt_info* info,
                         char* err, size_t errlen) {
    auto put = [&](const char* s) {
        if (err && errlen) {
            std::strncpy(err, s, errlen - 1);
            err[errlen - 1] = 0;
        }
    };
    try {
        if (!opt) throw std::invalid_argument("null options");
        ozTTgemm::Options o;
        o.scheme = static_cast<ozTTgemm::Scheme>(opt->scheme);
        o.format = static_cast<ozTTgemm::Format>(opt->format);
        o.slices = opt->slices;
        o.max_moduli = opt->max_moduli;
        o.reconstruction = static_cast<ozTTgemm::Reconstruction>(opt->reconstruction);
        ozTTgemm::DeviceOptions d;
        d.device_id = device_id;
        ozTTgemm::Context ctx(d);
        const ozTTgemm::Info in = ctx.gemm(std::span<const double>(a, a ? a_len : 0),
                                           std::span<const double>(b, b ? b_len : 0), std::span<double>(c, c ? c_len : 0),
                                           m, n, k, o);
        if (info) {
            info->scheme = (int32_t)in.scheme;
            info->format = (int32_t)in.format;
            info->slices = in.slices;
            info->moduli = in.moduli;
            info->integer_bits = in.integer_bits;
            info->reconstruction_passes = in.reconstruction_passes;
            info->padded_m = in.padded_m;
            info->padded_n = in.padded_n;
            info->padded_k = in.padded_k;
        }
        put("");
        return OZTT_OK;
    } catch (const std::invalid_argument& e) {
        put(e.what());
        return OZTT_EINVAL;
    } catch (const std::bad_alloc&) {
        put("host memory exhausted");
        return OZTT_ENOMEM;
    } catch (const std::exception& e) {
        put(e.what());
        return OZTT_ERUNTIME;
    }
}

extern "C" int oztt_ii_int8_last_phases(double* out, int32_t count) {
    if (!out || count < 1) return OZTT_EINVAL;
    const oztt::StreamedPhases ph = oztt::last_streamed_phases();
    const double v[16] = {ph.upload_ms,       ph.stats_ms,         ph.check_ms,         ph.plan_ms,
                          ph.pipeline_ms,     ph.total_ms,         (double)ph.bands,    ph.first_plan_ms,
                          (double)ph.replanned, (double)ph.exact_stats, (double)ph.early_readback,
                          ph.gpu_prefix_ms,   ph.gpu_compute_ms,   ph.gpu_readback_ms,  ph.gpu_bounds_ms,
                          ph.host_checked_ms};
    for (int32_t i = 0; i < count && i < 16; ++i) out[i] = v[i];
    return OZTT_OK;
}
