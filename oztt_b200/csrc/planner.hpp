// SPDX-License-Identifier: Apache-2.0
// Host planners: Scheme II INT8 (planner.cpp) and Scheme I INT8 (planner1.cpp).
#pragma once
#include <algorithm>
#include <cstdint>
#include <functional>
#include <string>
#include <thread>
#include <vector>

#include "oztt_cuda.h"

namespace oztt {

// The host threads this process may run on: the CPUs of its affinity mask (a container's share of
// the machine), else hardware_concurrency. Defined in planner.cpp.
unsigned host_threads();

// Runs f(begin, end) over [0, n) on up to host_threads() threads.
template <class F>
void parallel_ranges(uint64_t n, F&& f) {
    const unsigned hw = host_threads();
    const uint64_t nt = std::min<uint64_t>(hw, std::max<uint64_t>(1, n / 64));
    if (nt <= 1) {
        f(0, n);
        return;
    }
    std::vector<std::thread> th;
    th.reserve(nt);
    for (uint64_t t = 0; t < nt; ++t) {
        const uint64_t b = n * t / nt, e = n * (t + 1) / nt;
        th.emplace_back([&f, b, e] { f(b, e); });
    }
    for (auto& x : th) x.join();
}

// Power of two by which a matrix is divided before sums of squares are formed: 2^e for the exponent e
// of its largest magnitude, clamped to [-1000, 1000] (oz_pow2_scale, src/backend/common/norm_estimate.hpp:20-28).
double pow2_normalizer(const double* v, uint64_t rows, uint64_t cols, uint64_t ld);
// Low-biased Hutchinson estimate of ||(rgA A)(rgB B)||_F^2 for row-major a (m x k), b (k x n) with random
// vectors of the padded length N (estimate_product_norm, src/backend/common/norm_estimate.hpp:48-73).
double product_norm_estimate(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                             double rgA, double rgB);

struct ModuliChoice {
    bool ok = false, acc_ok = true;
    int b = 0, m_cap = 0, ncand = 0, acc_fail_m = 0;
    std::vector<int> m;
    double logM = 0;
};

struct PolicyStats {
    bool measured = false;
    double TA = 0, TB = 0, nA = 0, nB = 0, nC = 0;
};

// Moduli and width for the INT8 route (inner dimension K, limit, width cap).
ModuliChoice choose_moduli_int8(uint32_t K, int num_moduli, int b_cap);
// Input statistics of the precision policy for row-major a (m x k) and b (k x n); N and K are the
// padded planning dimensions (the random vectors have the padded length).
PolicyStats measure_policy_stats(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                                 uint32_t K);
int policy_width_cap(const PolicyStats& st);
// Bounds of the five statistics: TA, TB known exactly, nA, nB and nC in [lo, hi] (the reference's values,
// which come from sequential sums in its own rounding, lie inside).
struct PolicyBounds {
    PolicyStats lo, hi;  // lo: nA, nB and nC at their lower bounds; hi: at their upper bounds
    bool usable = false;
};
// The Scheme II INT8 plan when the bounds decide it: the width cap (and, for Automatic, the number of
// passes) is the same everywhere in the bounds, so it is the reference's decision; decided = false (and
// nothing planned) otherwise. Returns an OZTT_* code.
int plan_ii_int8_certified(const PolicyBounds& bounds, uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli,
                           int32_t reconstruction, oztt_ii_plan& p, std::string& err, bool& decided);
double one_pass_error_log2(const std::vector<int>& mods, int b, const PolicyStats& st);
void fill_crt_constants(const std::vector<int>& mods, oztt_ii_plan& p);
// The whole plan; returns an OZTT_* code and a message.
int plan_ii_int8(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli,
                 int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan& p, std::string& err);

// The same with the input statistics from `stats(N, K)` (padded N and K), e.g. measured on the device
// (device_policy_stats in stats.cu); called only when the policy needs them.
int plan_ii_int8_with(const std::function<PolicyStats(uint32_t, uint32_t)>& stats, uint64_t m, uint64_t n, uint64_t k,
                      uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan& p,
                      std::string& err);

// Whether the Scheme II INT8 plan for these dimensions and this limit succeeds whatever the statistics:
// every width cap the statistics can set (53 .. 100 bits) finds its moduli. A call that writes C before its
// statistics are complete relies on it: its plan cannot fail afterwards.
bool plan_ii_int8_never_fails(uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli);

// The magnitude patterns (sign bit cleared) of the largest element of each row of row-major a (m x k) and of
// each column of row-major b (k x n), on the host's threads: what the front end's value checks read.
void value_maxima(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint64_t* row_max,
                  uint64_t* col_max);

// Scheme II digit formats: FP8, BF16, FP16, TF32 (planner_digit.cpp); format is an OZTT_FMT_* value.
int plan_digit_with(int32_t format, const std::function<PolicyStats(uint32_t, uint32_t)>& stats, uint64_t m,
                    uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits,
                    oztt_digit_plan& p, std::string& err);
int plan_digit(int32_t format, const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
               uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_digit_plan& p, std::string& err);

// Scheme I format constants (ozaki1/param.hpp:47-70, ozaki1/format.hpp:32-97): radix, digit bound,
// normalization target 2^nshift, BF16 rounding of the maxima (1 up, 0 truncate), exact accumulator bits,
// Int32 partial products. BF16, FP16 and TF32 share radix 64 and digits +-32 (only their transport
// formats differ on the reference's device).
struct I1Format {
    int32_t format;  // OZTT_FMT_*
    double radix, dmax;
    int32_t nshift;
    uint32_t ceil_mode, acc_bits;
    bool int32_partial;
};
inline constexpr I1Format kI1Int8{OZTT_FMT_INT8, 254.0, 127.0, -1, 1u, 31u, true};
inline constexpr I1Format kI1Fp8{OZTT_FMT_FP8, 32.0, 16.0, -1, 0u, 24u, false};
inline constexpr I1Format kI1Bf16{OZTT_FMT_BF16, 64.0, 32.0, -1, 0u, 24u, false};
inline constexpr I1Format kI1Fp16{OZTT_FMT_FP16, 64.0, 32.0, -1, 0u, 24u, false};
inline constexpr I1Format kI1Tf32{OZTT_FMT_TF32, 64.0, 32.0, -1, 0u, 24u, false};
// The constants of a built format (INT8, FP8, BF16, FP16, TF32), or null.
inline const I1Format* i1_format(int32_t format) {
    switch (format) {
    case OZTT_FMT_INT8: return &kI1Int8;
    case OZTT_FMT_FP8: return &kI1Fp8;
    case OZTT_FMT_BF16: return &kI1Bf16;
    case OZTT_FMT_FP16: return &kI1Fp16;
    case OZTT_FMT_TF32: return &kI1Tf32;
    default: return nullptr;
    }
}
// Scheme I slice selection in parts, so that the per-element statistics can be measured on the device
// (plan1_dev.cu) and the rest done here with the same arithmetic:
//   I1Normalization  the global scales rg, per row of A / column of B the device exponent e, the scaled
//                    divisor s = rg 2^(e - nshift) (0: not counted) and the squared norm sum (x rg)^2;
//   I1Terms          model (1)'s per-k sums: S[i][k], R[q][k] (slice and residual contributions of A and
//                    of B, q = 1..pmax, index i*k + c) and the column norms N[k].
struct I1Normalization {
    double rgA = 1.0, rgB = 1.0;
    std::vector<int> eA, eB;
    std::vector<double> sA, sB, nrA, nrB;
};
struct I1Terms {
    std::vector<double> SA, RA, SB, RB, NA, NB;
};
// The largest slice count the search considers (ceil(160 / log2 radix) + 1).
int i1_pmax(const I1Format& f);
// The normalization from the magnitude patterns of the row and column maxima and the squared norms.
I1Normalization i1_normalization(double rgA, double rgB, const uint64_t* row_max, const uint64_t* col_max,
                                 const double* nrA, const double* nrB, uint64_t m, uint64_t n, const I1Format& f);
// Model (2) in parts, for an evaluation of its sums elsewhere (the device): the sampled rows of A and
// columns of B with their weights (the largest norms, then a seeded uniform draw), ||C||_F^2's
// denominator from the sample's C (Ch + Cl, the compensated products of the pairs) and nC, the error for
// one q from the chunk partial sums part[ch][s][u] of the dropped terms (nch chunks of the padded K), and
// the search over q with model (1)'s terms.
struct I1SamplePick {
    std::vector<uint32_t> rows, cols;
    std::vector<double> wr, wc;
};
constexpr uint32_t kI1Chunks = 64;
I1SamplePick i1_pick(const I1Normalization& nm);
double i1_sample_norm2(const I1SamplePick& sp, const std::vector<double>& Ch, double nC);
double i1_model2_finish(const double* part, uint32_t nch, const I1SamplePick& sp, const std::vector<double>& Ch,
                        const std::vector<double>& Cl, const I1Normalization& nm, double norm2);
int i1_select_with(const I1Terms& terms, uint64_t m, uint64_t n, uint64_t k, uint32_t M, uint32_t N, uint32_t K,
                   const I1Format& f, double nC, const std::function<double(int)>& model2);
// Model (1)'s error for q = 0..pmax (entries below 2 unused): from the given terms, or measured on the
// host from a and b (with the given normalization, or the host's own).
std::vector<double> i1_model1_errors(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                                     const I1Format& f, const I1Terms* terms, const I1Normalization* nm);
// Scheme I (planner1.cpp): the slice count oz_fp64_p selects for row-major a (m x k), b (k x n) with padded
// planning dimensions M, N, K; and the whole plan (slices > 0 fixes p).
int select_slices(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t M, uint32_t N,
                  uint32_t K, const I1Format& f);
int plan_i(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t slices, const I1Format& f,
           oztt_i_plan& p, std::string& err);
// Context::gemm's Scheme I call from host buffers with the transfers overlapped (scheme1.cu): the streamed
// upload with the statistics, check(row_max, col_max) as for Scheme II, the slice count (slices 0) from
// the measured statistics, the banded pipeline with the read-back overlapped.
int run_i_streamed(int device_id, int32_t format, const double* a, const double* b, double* c, uint64_t m,
                   uint64_t n, uint64_t k, uint32_t slices,
                   const std::function<void(const uint64_t*, const uint64_t*)>& check, oztt_i_plan& plan,
                   std::string& err);
// Context::gemm's Scheme I call under an evaluation Scope (plan1_dev.cu): one upload, the slice count from
// statistics measured on the device, the pipeline on the resident operands.
int run_i_uploaded(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                   uint32_t slices, const I1Format& f, oztt_i_plan& p, std::string& err);
// The same with the slice count from select(M, N, K) when slices is 0 (e.g. measured on the device).
int plan_i_with(const std::function<int(uint32_t, uint32_t, uint32_t)>& select, uint64_t m, uint64_t n, uint64_t k,
                uint32_t slices, const I1Format& f, oztt_i_plan& p, std::string& err);
int select_slices_int8(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t M, uint32_t N,
                       uint32_t K);
int plan_i_int8(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t slices,
                oztt_i_plan& p, std::string& err);

// Scheme II INT8 from host buffers with the transfers overlapped (ii_int8.cu): A and B are uploaded in
// chunks while the device measures the policy statistics; check(row_max, col_max) receives the
// magnitude patterns (sign bit cleared) of the maxima of A's m rows and B's n columns once the upload
// ends, and an exception from it ends the call (as its error code) before the plan and before C is
// written; then the pipeline runs in row bands with each band of C read back during the next.
int run_ii_int8_streamed(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                         uint64_t k, uint32_t max_moduli, int32_t reconstruction,
                         const std::function<void(const uint64_t*, const uint64_t*)>& check, oztt_ii_plan& p,
                         std::string& err);
// The same for a digit format (ii_digit.cu).
int run_ii_digit_streamed(int device_id, int32_t format, const double* a, const double* b, double* c, uint64_t m,
                          uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction,
                          const std::function<void(const uint64_t*, const uint64_t*)>& check, oztt_digit_plan& p,
                          std::string& err);
// Scheme II INT8 from host buffers without overlap (whole upload, device statistics, pipeline, C back),
// the width fixed to fixed_bits when nonzero: the path of the evaluator's profiled calls.
int run_ii_int8_uploaded(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                         uint64_t k, uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan& p,
                         std::string& err);
// Host wall-clock phases of the last completed streamed call (INT8 or a digit format) in this process.
struct StreamedPhases {
    double upload_ms = 0;      // from the call to the end of the last host-to-device copy
    double stats_ms = 0;       // then until the statistics were read back
    double check_ms = 0;       // then the value checks from the maxima
    double plan_ms = 0;        // the plan
    double pipeline_ms = 0;    // scale, split, banded GEMM and reconstruction, C read back
    double total_ms = 0;
    int bands = 0;
    double first_plan_ms = 0;  // overlapped INT8 path: when the first plan (A's first part, B's first block) was made
    int replanned = 0;         // 1 if the complete statistics gave another plan and the pipeline ran again
    int exact_stats = 0;       // 1 if the bounds left the decision open and the exact sums were computed
    int early_readback = 0;    // 1 if C's bands were read back as they finished, before the plan was confirmed
    // device timeline of that path, ms from the first copy: A's first part done against all of B, the last
    // reconstruction, the end of the last read-back of C, the last band's bounded statistics
    double gpu_prefix_ms = 0, gpu_compute_ms = 0, gpu_readback_ms = 0, gpu_bounds_ms = 0;
    double host_checked_ms = 0;  // that path: when the host's maxima of A and B were ready (ms from the call)
};
StreamedPhases last_streamed_phases();

}  // namespace oztt
