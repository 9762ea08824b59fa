// SPDX-License-Identifier: Apache-2.0
//
// Resident operands: Scheme II INT8 products of matrices kept in HBM between calls, with what the pipeline
// derives from each operand alone cached beside it.
//
// The reference rebuilds its buffers and programs on every call and offers no persistent operand
// (README.md:81-85); Context::gemm here does the same, as the drop-in contract requires. This is an
// extension for callers that multiply by the same matrix many times (a fixed right-hand side, a fixed
// basis): the matrix is uploaded once, and of the precision policy's input statistics
// (choose_precision_policy, src/backend/ozaki2/auto_precision.hpp:24-108, norm_estimate.hpp:20-73) the
// parts that depend on one operand only are measured once:
//   A (m x k)   the magnitude patterns of its row maxima, its scale rgA, the scaled sums of squares of its rows
//   B (k x n)   the same per column, rgB, and the sketch y_l = B g_l (8 x k, the reference's long-double sums)
// A product needs the pair's s_l = A y_l (one pass over A) before the host sums everything in the
// reference's order, so its plan is byte for byte the plan Context::gemm makes for the same values. Each
// operand also keeps the exponent deltas and residue planes of the plans it was last used with (two), so a
// repeated product with an unchanged plan starts at the residue GEMM.
#include <algorithm>
#include <memory>
#include <mutex>
#include <vector>

#include "ext80.h"
#include "oztt_common.cuh"
#include "planner.hpp"
#include "runtime.cuh"

namespace oztt {

void launch_scale_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, int32_t shift, int32_t* delta,
                       uint16_t* bfmax, uint32_t* flags, cudaStream_t st);
void launch_scale_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift, int32_t* delta,
                       uint16_t* bfmax, uint32_t* flags, unsigned long long* colmax, cudaStream_t st);
void launch_split_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta,
                       const oztt_ii_plan& p, int8_t* planes, uint64_t mp, uint64_t kp, cudaStream_t st,
                       uint64_t plane_rows = 0);
void launch_split_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta,
                       const oztt_ii_plan& p, int8_t* planes, uint64_t np, uint64_t kp, cudaStream_t st,
                       uint64_t plane_rows = 0);
void launch_residue_gemm(const int8_t* ap, const int8_t* bp, uint64_t mp, uint64_t np, uint64_t kp,
                         const oztt_ii_plan& p, int mode, void* out, int* err_word, cudaStream_t st,
                         uint64_t a_plane_rows, uint64_t b_plane_rows = 0);
void launch_recon(const uint8_t* kp, uint64_t mp, uint64_t np, const int32_t* dA, const int32_t* dB,
                  const oztt_ii_plan& p, double* c, uint64_t m, uint64_t n, uint64_t ldc, cudaStream_t st);
void check_plan(const oztt_ii_plan& p);
PolicyStats combine_policy_stats(const double* row_max, uint64_t m, const double* col_max, uint64_t n,
                                 const double* row_sumsq, const double* col_sumsq, const double* s, uint64_t sstride,
                                 double rgA, double rgB);
std::vector<double> policy_vectors_host(uint32_t N);

namespace {

// Device memory owned by a resident operand (not stream-ordered: it outlives every call's streams).
struct Mem {
    void* p = nullptr;
    Mem() = default;
    explicit Mem(size_t bytes) {
        const cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 256));
        if (e != cudaSuccess) {
            cudaGetLastError();
            p = nullptr;
            throw Error(OZTT_ERUNTIME, "device memory allocation of " + std::to_string(bytes) +
                                           " bytes for a resident operand failed: " + cudaGetErrorString(e));
        }
    }
    ~Mem() {
        if (p) cudaFree(p);
    }
    Mem(const Mem&) = delete;
    Mem& operator=(const Mem&) = delete;
    template <class T>
    T* as() const {
        return reinterpret_cast<T*>(p);
    }
};

// The residue planes of one plan (moduli set and shift) with the exponent deltas they were split with.
struct PlanePack {
    std::vector<int32_t> moduli;
    int32_t shift = 0;
    std::unique_ptr<Mem> delta, planes;
    uint64_t last_use = 0;
};

double magnitude(uint64_t pattern) {
    double x;
    std::memcpy(&x, &pattern, sizeof x);
    return x;
}

// The reference's power-of-two normaliser 1 / 2^e of the largest magnitude (oz_pow2_scale,
// src/backend/common/norm_estimate.hpp:20-28), e clamped to [-1000, 1000]; 1 for zero.
double pow2_scale_of(double mx) {
    if (!(mx > 0) || !std::isfinite(mx)) return 1.0;
    int e = 0;
    std::frexp(mx, &e);
    e = std::min(std::max(e, -1000), 1000);
    return std::ldexp(1.0, -e);
}

}  // namespace

void launch_stats_absmax(const double* x, uint64_t rows, uint64_t cols, int mode, double* out, cudaStream_t st);
void launch_stats_sumsq(const double* x, uint64_t rows, uint64_t cols, int mode, double rg, double* out,
                        cudaStream_t st);
void launch_stats_sketch(const double* x, uint64_t rows, uint64_t cols, double rg, const double* v, uint64_t vstride,
                         double* out, uint64_t ostride, cudaStream_t st);

}  // namespace oztt

struct oztt_resident {
    int device = 0;
    int32_t role = OZTT_ROLE_A;
    uint64_t rows = 0, cols = 0;  // A: m x k; B: k x n
    std::unique_ptr<oztt::Mem> x;  // the matrix, row-major
    // the single-operand statistics: maxima (|values|), the scale, scaled sums of squares per row of A or
    // column of B; for B the sketch y (8 x k doubles, on the device) and the padded width N it was drawn for
    std::vector<double> maxima, sumsq;
    double rg = 1.0;
    std::unique_ptr<oztt::Mem> y;
    std::vector<oztt::PlanePack> packs;
    uint64_t uses = 0;
    std::mutex mu;
};

namespace oztt {
namespace {

std::mutex g_resident_mu;  // one product at a time per process (the planes caches are not shared)

constexpr uint64_t kPacksKept = 2;

// Runs f on a private stream of the operand's device and waits for it.
template <class F>
void on_device(int device, F&& f) {
    open_device(device);
    cudaStream_t st;
    OZTT_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    struct Guard {
        cudaStream_t s;
        ~Guard() {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
    } guard{st};
    f(st);
    OZTT_CUDA(cudaStreamSynchronize(st));
}

// The residue planes of `r` for plan p (cached; the least recently used pack is replaced when two are kept).
PlanePack& planes_for(oztt_resident& r, const oztt_ii_plan& p, cudaStream_t st) {
    const std::vector<int32_t> mods(p.moduli, p.moduli + p.S);
    ++r.uses;
    for (PlanePack& pk : r.packs)
        if (pk.moduli == mods && pk.shift == p.shift) {
            pk.last_use = r.uses;
            return pk;
        }
    if (r.packs.size() >= kPacksKept) {
        auto old = std::min_element(r.packs.begin(), r.packs.end(),
                                    [](const PlanePack& a, const PlanePack& b) { return a.last_use < b.last_use; });
        r.packs.erase(old);
    }
    r.packs.emplace_back();
    PlanePack& pk = r.packs.back();
    pk.moduli = mods;
    pk.shift = p.shift;
    pk.last_use = r.uses;
    const uint64_t S = (uint64_t)p.S;
    const bool is_a = r.role == OZTT_ROLE_A;
    // A: rows m, planes [S][mp][kp]; B: columns n, planes [S][np][kp] (transposed)
    const uint64_t outer = is_a ? r.rows : r.cols, inner = is_a ? r.cols : r.rows;
    const uint64_t op = round_up(outer, is_a ? 128 : 256), kp = round_up(inner, 128);
    pk.delta = std::make_unique<Mem>(op * 4);
    pk.planes = std::make_unique<Mem>(S * op * kp);
    Mem words(16), colmax(is_a ? 8 : r.cols * 8);
    OZTT_CUDA(cudaMemsetAsync(words.p, 0, 16, st));
    OZTT_CUDA(cudaMemsetAsync(pk.delta->p, 0, op * 4, st));
    if (is_a) {
        launch_scale_rows(r.x->as<double>(), r.rows, r.cols, r.cols, p.shift, pk.delta->as<int32_t>(), nullptr,
                          words.as<uint32_t>(), st);
        launch_split_rows(r.x->as<double>(), r.rows, r.cols, r.cols, pk.delta->as<int32_t>(), p,
                          pk.planes->as<int8_t>(), op, kp, st);
    } else {
        launch_scale_cols(r.x->as<double>(), r.rows, r.cols, r.cols, p.shift, pk.delta->as<int32_t>(), nullptr,
                          words.as<uint32_t>(), colmax.as<unsigned long long>(), st);
        launch_split_cols(r.x->as<double>(), r.rows, r.cols, r.cols, pk.delta->as<int32_t>(), p,
                          pk.planes->as<int8_t>(), op, kp, st);
    }
    uint32_t flags = 0;
    OZTT_CUDA(cudaMemcpyAsync(&flags, words.p, 4, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaStreamSynchronize(st));
    if (flags) {
        r.packs.pop_back();
        check_flags(flags, 0);
    }
    return pk;
}

}  // namespace
}  // namespace oztt

using oztt::Error;
using oztt::guarded;

extern "C" {

int oztt_resident_create(int device_id, int32_t role, const double* x, uint64_t rows, uint64_t cols,
                         int32_t x_on_device, oztt_resident** out, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!x || !out) throw Error(OZTT_EINVAL, "resident_create: null argument");
        *out = nullptr;
        if (role != OZTT_ROLE_A && role != OZTT_ROLE_B) throw Error(OZTT_EINVAL, "resident_create: unknown role");
        if (!rows || !cols) throw Error(OZTT_EINVAL, "matrix dimensions are zero or overflow the address space");
        if (rows > 0x7FFFFFFFull - 64 || cols > 0x7FFFFFFFull - 64)
            throw Error(OZTT_EINVAL, "matrix dimension exceeds the supported device index range");
        auto r = std::make_unique<oztt_resident>();
        r->device = device_id;
        r->role = role;
        r->rows = rows;
        r->cols = cols;
        const bool is_a = role == OZTT_ROLE_A;
        const uint64_t count = is_a ? rows : cols;  // rows of A, columns of B
        oztt::on_device(device_id, [&](cudaStream_t st) {
            r->x = std::make_unique<oztt::Mem>(rows * cols * 8);
            OZTT_CUDA(cudaMemcpyAsync(r->x->p, x, rows * cols * 8,
                                      x_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
            oztt::Mem mx(count * 8);
            oztt::launch_stats_absmax(r->x->as<double>(), rows, cols, is_a ? 0 : 1, mx.as<double>(), st);
            r->maxima.resize(count);
            OZTT_CUDA(cudaMemcpyAsync(r->maxima.data(), mx.p, count * 8, cudaMemcpyDeviceToHost, st));
            OZTT_CUDA(cudaStreamSynchronize(st));
            // the values, as the front end checks them (src/context.cpp:37-62), for this operand
            const auto patterns = reinterpret_cast<const uint64_t*>(r->maxima.data());
            const char* name = is_a ? "A contains NaN or infinity" : "B contains NaN or infinity";
            for (uint64_t i = 0; i < count; ++i)
                if (patterns[i] >= 0x7FF0000000000000ull) throw Error(OZTT_EINVAL, name);
            for (uint64_t i = 0; i < count; ++i) {
                const double v = r->maxima[i];
                if (v != 0 && (v < 0x1p-126 || v > 0x1.fep127))
                    throw Error(OZTT_EINVAL,
                                "each nonzero row maximum of A and column maximum of B must be in [2^-126, max_BF16]");
            }
            double top = 0;
            for (double v : r->maxima) top = std::max(top, v);
            r->rg = oztt::pow2_scale_of(top);
            oztt::Mem s2(count * 8);
            oztt::launch_stats_sumsq(r->x->as<double>(), rows, cols, is_a ? 0 : 1, r->rg, s2.as<double>(), st);
            r->sumsq.resize(count);
            OZTT_CUDA(cudaMemcpyAsync(r->sumsq.data(), s2.p, count * 8, cudaMemcpyDeviceToHost, st));
            if (!is_a) {
                // y_l = B g_l with the vectors of the padded width the planner uses
                const uint32_t N = (uint32_t)oztt::round_up(cols, 64);
                const std::vector<double> g = oztt::policy_vectors_host(N);
                oztt::Mem dg(g.size() * 8);
                OZTT_CUDA(cudaMemcpyAsync(dg.p, g.data(), g.size() * 8, cudaMemcpyHostToDevice, st));
                r->y = std::make_unique<oztt::Mem>(8 * rows * 8);
                oztt::launch_stats_sketch(r->x->as<double>(), rows, cols, r->rg, dg.as<double>(), N, r->y->as<double>(),
                                          rows, st);
                OZTT_CUDA(cudaStreamSynchronize(st));
            }
        });
        *out = r.release();
    });
}

int oztt_resident_destroy(oztt_resident* r) {
    if (!r) return OZTT_OK;
    std::lock_guard<std::mutex> lock(oztt::g_resident_mu);
    cudaSetDevice(r->device);
    delete r;
    return OZTT_OK;
}

int oztt_resident_gemm(oztt_resident* a, oztt_resident* b, double* c, int32_t c_on_device, const oztt_options* opt,
                       oztt_info* info, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !c || !opt) throw Error(OZTT_EINVAL, "resident_gemm: null argument");
        if (a->role != OZTT_ROLE_A || b->role != OZTT_ROLE_B)
            throw Error(OZTT_EINVAL, "resident_gemm: the operands must be a left (A) and a right (B) operand");
        if (a->device != b->device) throw Error(OZTT_EINVAL, "resident_gemm: the operands live on different devices");
        if (a->cols != b->rows) throw Error(OZTT_EINVAL, "matrix span sizes do not match m, n, k");
        if (opt->scheme != OZTT_SCHEME_II || opt->format != OZTT_FMT_INT8)
            throw Error(OZTT_EINVAL, "resident operands are multiplied by Scheme II with INT8 products only");
        if (opt->slices != 0) throw Error(OZTT_EINVAL, "slices applies only to Ozaki I");
        if (opt->max_moduli > 24) throw Error(OZTT_EINVAL, "max_moduli exceeds the supported bound of 24");
        if (opt->reconstruction < OZTT_RECON_AUTO || opt->reconstruction > OZTT_RECON_TWO)
            throw Error(OZTT_EINVAL, "unknown reconstruction mode");
        std::lock_guard<std::mutex> lock(oztt::g_resident_mu);
        const uint64_t m = a->rows, k = a->cols, n = b->cols;
        oztt::on_device(a->device, [&](cudaStream_t st) {
            // s_l = A y_l, then the five statistics in the reference's order
            oztt::Mem s(8 * m * 8);
            oztt::launch_stats_sketch(a->x->as<double>(), m, k, a->rg, b->y->as<double>(), k, s.as<double>(), m, st);
            std::vector<double> hs(8 * m);
            OZTT_CUDA(cudaMemcpyAsync(hs.data(), s.p, hs.size() * 8, cudaMemcpyDeviceToHost, st));
            OZTT_CUDA(cudaStreamSynchronize(st));
            const oztt::PolicyStats ps = oztt::combine_policy_stats(a->maxima.data(), m, b->maxima.data(), n,
                                                                    a->sumsq.data(), b->sumsq.data(), hs.data(), m,
                                                                    a->rg, b->rg);
            oztt_ii_plan p{};
            std::string msg;
            const int rc = oztt::plan_ii_int8_with([&](uint32_t, uint32_t) { return ps; }, m, n, k, opt->max_moduli,
                                                   opt->reconstruction, 0, p, msg);
            if (rc != OZTT_OK) throw Error(rc, msg);
            oztt::check_plan(p);
            oztt::PlanePack& pa = oztt::planes_for(*a, p, st);
            oztt::PlanePack& pb = oztt::planes_for(*b, p, st);
            const uint64_t S = (uint64_t)p.S;
            const uint64_t mp = oztt::round_up(m, 128), np = oztt::round_up(n, 256), kp = oztt::round_up(k, 128);
            const uint64_t bands = std::min<uint64_t>(8, std::max<uint64_t>(1, mp / 2048));
            const uint64_t bm = oztt::round_up((mp + bands - 1) / bands, 128);
            oztt::DevBuf kpl(st, S * bm * np), words(st, 16);
            std::unique_ptr<oztt::DevBuf> dc;
            double* cd = c;
            if (!c_on_device) {
                dc = std::make_unique<oztt::DevBuf>(st, m * n * 8);
                cd = dc->as<double>();
            }
            OZTT_CUDA(cudaMemsetAsync(words.p, 0, 16, st));
            int* gemm_err = words.as<int>() + 1;
            for (uint64_t r0 = 0; r0 < mp; r0 += bm) {
                const uint64_t rows_p = std::min(bm, mp - r0);
                oztt::launch_residue_gemm(pa.planes->as<int8_t>() + r0 * kp, pb.planes->as<int8_t>(), rows_p, np, kp,
                                          p, 1, kpl.p, gemm_err, st, mp);
                if (r0 >= m) continue;
                const uint64_t rows = std::min(m, r0 + rows_p) - r0;
                oztt::launch_recon(kpl.as<uint8_t>(), rows_p, np, pa.delta->as<int32_t>() + r0, pb.delta->as<int32_t>(),
                                   p, cd + r0 * n, rows, n, n, st);
            }
            int host_words[2] = {0, 0};
            OZTT_CUDA(cudaMemcpyAsync(host_words, words.p, 8, cudaMemcpyDeviceToHost, st));
            OZTT_CUDA(cudaStreamSynchronize(st));
            oztt::check_flags((uint32_t)host_words[0], host_words[1]);
            if (!c_on_device) {
                OZTT_CUDA(cudaMemcpyAsync(c, cd, m * n * 8, cudaMemcpyDeviceToHost, st));
                OZTT_CUDA(cudaStreamSynchronize(st));
            }
            if (info) {
                *info = oztt_info{};
                info->scheme = OZTT_SCHEME_II;
                info->format = OZTT_FMT_INT8;
                info->moduli = (uint32_t)p.S;
                info->integer_bits = (uint32_t)p.b;
                info->reconstruction_passes = p.two_pass ? 2u : 1u;
                info->padded_m = oztt::round_up(m, 64);
                info->padded_n = oztt::round_up(n, 64);
                info->padded_k = oztt::round_up(k, 32);
            }
        });
    });
}

}  // extern "C"
