// SPDX-License-Identifier: Apache-2.0
//
// Scheme II with digit formats (FP8 e4m3, BF16, FP16, TF32) on one B200, and the C-ABI entry points of
// its stages.
//
// The reference's digit backends (the ozaki2 backend compiled with OZ_FMT_FP8 / _BF16 / _FP16 / _FP32:
// src/ozaki2.cpp:439-478 with the digit stages of src/backend/ozaki2/stages.hpp) scale, split every residue
// into one to three small digits (kernels/modslice_digit.cpp), multiply the digit planes with FP32
// accumulation (concatenating products of equal weight along K), compose the products of each modulus
// into its residue (kernels/compose.cpp; a one-digit modulus skips it and the reconstruction reduces its
// product, RAWMASK) and reconstruct (kernels/recon_crt.cpp, IN_RESIDUE=1). Here one call is six launches
// on one stream:
//     scale_rows(A) -> scale_cols(B) -> digit_split_rows(A) -> digit_split_cols(B)
//     -> digit_gemm (every output of every modulus, composition fused into the epilogue) -> recon (uint16)
// Digit planes [nplane][mp][kp] / [nplane][np][kp] int8 (every digit of every format is an integer in
// [-32, 32]), CRT digits [S][mp][np] uint16. The four formats differ only in their plans (moduli, splitting,
// concatenation): on the reference's device they also differ in the transport type of the digits, which
// carries the same integers.
//
// The digit products are integers the reference's planner keeps below 2^24, so its FP32 sums are exact;
// the s32 tensor-core sums here are exact as well, and so the composed residue classes are the
// reference's. The composition itself is done in exact integer arithmetic (the reference's binary32
// sequence gives the same class, it only picks a representative), and the reconstruction is the exact
// CRT of this library (recon.cu).
#include <algorithm>
#include <functional>
#include <string>
#include <vector>

#include "oztt_common.cuh"
#include "planner.hpp"
#include "runtime.cuh"

namespace oztt {

void launch_scale_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, int32_t shift, int32_t* delta,
                       uint16_t* bfmax, uint32_t* flags, cudaStream_t st);
void launch_scale_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift, int32_t* delta,
                       uint16_t* bfmax, uint32_t* flags, unsigned long long* colmax, cudaStream_t st);
void launch_digit_split_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta,
                             const oztt_digit_plan& fp, int8_t* planes, uint64_t mp, uint64_t kp, cudaStream_t st);
void launch_digit_split_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta,
                             const oztt_digit_plan& fp, int8_t* planes, uint64_t np, uint64_t kp, cudaStream_t st);
void launch_digit_gemm(const int8_t* ap, const int8_t* bp, uint64_t mp, uint64_t np, uint64_t kp,
                       const oztt_digit_plan& fp, int mode, void* out, int* err_word, cudaStream_t st,
                       uint64_t a_plane_rows = 0);
void launch_recon_u16(const uint16_t* kp, uint64_t mp, uint64_t np, const int32_t* dA, const int32_t* dB,
                      const oztt_ii_plan& p, double* c, uint64_t m, uint64_t n, uint64_t ldc, cudaStream_t st);
PolicyStats device_policy_stats(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                                cudaStream_t st);

// Consistency of a digit plan (its own fields only; the GEMM launcher checks the output table).
void check_digit_plan(const oztt_digit_plan& fp) {
    const oztt_ii_plan& p = fp.base;
    if (p.S < 1 || p.S > OZTT_MAXS) throw Error(OZTT_EINVAL, "plan: the number of moduli must be 1..24");
    if (p.nd < 3 || p.nd > 5) throw Error(OZTT_EINVAL, "plan: the number of digits must be 3..5");
    if (fp.nplane < 1 || fp.nplane > 3 * OZTT_MAXS) throw Error(OZTT_EINVAL, "plan: bad number of digit planes");
    for (int s = 0; s < p.S; ++s) {
        const int m = p.moduli[s], mode = fp.mode[s];
        if (m < 2 || m > 4096) throw Error(OZTT_EINVAL, "plan: digit-format moduli must be in 2..4096");
        if (mode != OZTT_SPLIT_SQ && mode != OZTT_SPLIT_KAR && mode != OZTT_SPLIT_WIDE && mode != OZTT_SPLIT_SQS &&
            mode != OZTT_SPLIT_ONE)
            throw Error(OZTT_EINVAL, "plan: unknown splitting method");
        const int npl = mode == OZTT_SPLIT_KAR ? 3 : (mode == OZTT_SPLIT_ONE ? 1 : 2);
        const bool q_ok = mode == OZTT_SPLIT_ONE ? fp.q[s] == 1 : (fp.q[s] >= 2 && fp.q[s] <= 65);
        if (fp.npl[s] != npl || fp.poff[s] < 0 || fp.poff[s] + npl > fp.nplane || !q_ok)
            throw Error(OZTT_EINVAL, "plan: bad digit layout of modulus " + std::to_string(s));
    }
}

// The device pipeline on device buffers (row-major, lda = k, ldb = n, ldc = n). stage_ms (optional, 6
// entries): scale rows, scale cols, digit split rows, digit split cols, digit GEMM, reconstruction.
void run_ii_digit_device(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                       const oztt_digit_plan& fp, cudaStream_t st, double* stage_ms = nullptr) {
    check_digit_plan(fp);
    const oztt_ii_plan& p = fp.base;
    const uint64_t S = (uint64_t)p.S, NP = (uint64_t)fp.nplane;
    const uint64_t mp = round_up(m, 128), np = round_up(n, 256), kp = round_up(k, 128);
    DevBuf dA(st, mp * 4), dB(st, np * 4), colmax(st, n * 8), words(st, 16);
    DevBuf da(st, NP * mp * kp), db(st, NP * np * kp), kd(st, S * mp * np * 2);
    OZTT_CUDA(cudaMemsetAsync(words.p, 0, 16, st));
    uint32_t* flags = words.as<uint32_t>();
    int* gemm_err = words.as<int>() + 1;
    // the stages as the evaluator sees them (the composition is fused into the GEMM epilogue)
    Pipeline pl;
    pl.add(kScale, kHead, 0, [&] { launch_scale_rows(a, m, k, k, p.shift, dA.as<int32_t>(), nullptr, flags, st); });
    pl.add(kScale, kHead, 1, [&] {
        launch_scale_cols(b, k, n, n, p.shift, dB.as<int32_t>(), nullptr, flags, colmax.as<unsigned long long>(), st);
    });
    pl.add(kSlice, kHead, 2,
           [&] { launch_digit_split_rows(a, m, k, k, dA.as<int32_t>(), fp, da.as<int8_t>(), mp, kp, st); });
    pl.add(kSlice, kHead, 3,
           [&] { launch_digit_split_cols(b, k, n, n, dB.as<int32_t>(), fp, db.as<int8_t>(), np, kp, st); });
    pl.add(kGemm, kGemmStep, 4,
           [&] { launch_digit_gemm(da.as<int8_t>(), db.as<int8_t>(), mp, np, kp, fp, 1, kd.p, gemm_err, st); });
    // under an evaluation Scope a two-pass plan's reconstruction is timed as two launches (row halves)
    const uint64_t halves = (evaluation_active() && p.two_pass && m > 1) ? 2 : 1;
    for (uint64_t h = 0; h < halves; ++h) {
        const uint64_t r0 = m * h / halves, rows = m * (h + 1) / halves - r0;
        pl.add(kRecon, kReconStep, 5, [&, r0, rows] {
            launch_recon_u16(kd.as<uint16_t>() + r0 * np, mp, np, dA.as<int32_t>() + r0, dB.as<int32_t>(), p,
                             c + r0 * n, rows, n, n, st);
        }, true);
    }
    pl.writes(dA.p, mp * 4);
    pl.writes(dB.p, np * 4);
    pl.writes(da.p, NP * mp * kp);
    pl.writes(db.p, NP * np * kp);
    pl.writes(kd.p, S * mp * np * 2);
    pl.writes(c, m * n * 8);
    pl.out = c;
    pl.out_bytes = m * n * 8;
    pl.partial_products = (unsigned)fp.nprod;
    if (!run_profiled(pl, st)) pl.run(st, stage_ms, 6);
    uint32_t host_words[2] = {0, 0};
    OZTT_CUDA(cudaMemcpyAsync(host_words, words.p, 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaStreamSynchronize(st));
    check_flags(host_words[0], (int)host_words[1]);
}

// Plan from device-resident operands (the precision policy's statistics measured on the device).
int plan_digit_device(int32_t format, const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                      uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_digit_plan& p,
                      std::string& err, cudaStream_t st) {
    return plan_digit_with(
        format, [&](uint32_t N, uint32_t) { return device_policy_stats(a, b, m, n, k, N, st); }, m, n, k, max_moduli,
        reconstruction, fixed_bits, p, err);
}

static void with_stream(int device_id, const std::function<void(cudaStream_t)>& f) {
    open_device(device_id);
    cudaStream_t st;
    OZTT_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    struct StreamGuard {
        cudaStream_t s;
        ~StreamGuard() {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
    } guard{st};
    f(st);
}

// The whole call as Context::gemm makes it: A and B to the device, the plan from device statistics (the
// width fixed to fixed_bits when nonzero), the pipeline, C back. Returns OZTT_OK, or an error code with
// its message (C is then untouched).
int run_ii_digit_planned(int device_id, int32_t format, const double* a, const double* b, double* c, uint64_t m,
                         uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits,
                         oztt_digit_plan& p, std::string& err) {
    char buf[1024];
    int inner = OZTT_OK;
    const int rc = guarded(buf, sizeof buf, [&] {
        with_stream(device_id, [&](cudaStream_t st) {
            DevBuf da(st, m * k * 8), db(st, k * n * 8);
            OZTT_CUDA(cudaMemcpyAsync(da.p, a, m * k * 8, cudaMemcpyHostToDevice, st));
            OZTT_CUDA(cudaMemcpyAsync(db.p, b, k * n * 8, cudaMemcpyHostToDevice, st));
            inner = plan_digit_device(format, da.as<double>(), db.as<double>(), m, n, k, max_moduli, reconstruction,
                                      fixed_bits, p, err, st);
            if (inner != OZTT_OK) return;
            DevBuf dc(st, m * n * 8);
            run_ii_digit_device(da.as<double>(), db.as<double>(), dc.as<double>(), m, n, k, p, st);
            OZTT_CUDA(cudaMemcpyAsync(c, dc.p, m * n * 8, cudaMemcpyDeviceToHost, st));
            OZTT_CUDA(cudaStreamSynchronize(st));
        });
    });
    if (rc != OZTT_OK) err = buf;
    return rc != OZTT_OK ? rc : inner;
}

// Context::gemm's path for a digit format (StreamedCall, streamed.cu): the upload with the statistics
// measured on the way, the caller's value checks from the measured maxima, the format's plan, scale and
// digit split, then the digit GEMM (the composition in its epilogue) and the reconstruction in bands of
// about 2048 rows (up to 8), each band of C read back while the next is computed.
static int run_ii_digit_streamed_impl(int device_id, int32_t format, const double* a, const double* b, double* c,
                                      uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli,
                                      int32_t reconstruction,
                                      const std::function<void(const uint64_t*, const uint64_t*)>& check,
                                      oztt_digit_plan& fp, std::string& err) {
    StreamedCall call(device_id, a, b, m, n, k);
    StreamedPhases& ph = call.phases();
    cudaStream_t st = call.work();
    std::vector<uint64_t> row_max, col_max;
    const PolicyStats ps = call.upload(row_max, col_max);
    double t = call.ms_since_start();
    check(row_max.data(), col_max.data());
    ph.check_ms = call.ms_since_start() - t;
    t = call.ms_since_start();
    const int rc = plan_digit_with(format, [&](uint32_t, uint32_t) { return ps; }, m, n, k, max_moduli,
                                   reconstruction, 0, fp, err);
    if (rc != OZTT_OK) return rc;
    ph.plan_ms = call.ms_since_start() - t;
    t = call.ms_since_start();
    check_digit_plan(fp);
    const oztt_ii_plan& p = fp.base;
    const uint64_t S = (uint64_t)p.S, NP = (uint64_t)fp.nplane;
    const uint64_t mp = round_up(m, 128), np = round_up(n, 256), kp = round_up(k, 128);
    const uint64_t bands = std::min<uint64_t>(8, std::max<uint64_t>(1, mp / 2048));
    const uint64_t bm = round_up((mp + bands - 1) / bands, 128);
    const double *da = call.a_dev(), *db = call.b_dev();
    double* dc = call.c_dev();
    DevBuf dA(st, mp * 4), dB(st, np * 4), colmax(st, n * 8), words(st, 16);
    DevBuf pa(st, NP * mp * kp), pb(st, NP * np * kp), kd(st, S * bm * np * 2);
    OZTT_CUDA(cudaMemsetAsync(words.p, 0, 16, st));
    uint32_t* flags = words.as<uint32_t>();
    int* gemm_err = words.as<int>() + 1;
    launch_scale_rows(da, m, k, k, p.shift, dA.as<int32_t>(), nullptr, flags, st);
    launch_scale_cols(db, k, n, n, p.shift, dB.as<int32_t>(), nullptr, flags, colmax.as<unsigned long long>(), st);
    launch_digit_split_rows(da, m, k, k, dA.as<int32_t>(), fp, pa.as<int8_t>(), mp, kp, st);
    launch_digit_split_cols(db, k, n, n, dB.as<int32_t>(), fp, pb.as<int8_t>(), np, kp, st);
    for (uint64_t r0 = 0; r0 < mp; r0 += bm) {
        const uint64_t rows_p = std::min(bm, mp - r0);
        launch_digit_gemm(pa.as<int8_t>() + r0 * kp, pb.as<int8_t>(), rows_p, np, kp, fp, 1, kd.p, gemm_err, st, mp);
        if (r0 >= m) continue;
        const uint64_t rows = std::min(m, r0 + rows_p) - r0;
        launch_recon_u16(kd.as<uint16_t>(), rows_p, np, dA.as<int32_t>() + r0, dB.as<int32_t>(), p, dc + r0 * n, rows,
                         n, n, st);
        call.band_done(r0, rows);
    }
    call.read_back(c);
    uint32_t host_words[2] = {0, 0};
    OZTT_CUDA(cudaMemcpyAsync(host_words, words.p, 8, cudaMemcpyDeviceToHost, st));
    call.finish(t);
    check_flags(host_words[0], (int)host_words[1]);
    return OZTT_OK;
}

int run_ii_digit_streamed(int device_id, int32_t format, const double* a, const double* b, double* c, uint64_t m,
                          uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction,
                          const std::function<void(const uint64_t*, const uint64_t*)>& check, oztt_digit_plan& p,
                          std::string& err) {
    char buf[1024];
    int inner = OZTT_OK;
    const int rc = guarded(buf, sizeof buf, [&] {
        inner = run_ii_digit_streamed_impl(device_id, format, a, b, c, m, n, k, max_moduli, reconstruction, check, p,
                                           err);
    });
    if (rc != OZTT_OK) err = buf;
    return rc != OZTT_OK ? rc : inner;
}

}  // namespace oztt

using oztt::Error;
using oztt::guarded;

extern "C" {

int oztt_ii_digit_plan_device(int device_id, int32_t format, const double* a, const double* b, uint64_t m,
                              uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits,
                              oztt_digit_plan* plan, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !plan) throw Error(OZTT_EINVAL, "null argument");
        oztt::open_device(device_id);
        std::string msg;
        const int rc = oztt::plan_digit_device(format, a, b, m, n, k, max_moduli, reconstruction, fixed_bits, *plan,
                                               msg,
                                             reinterpret_cast<cudaStream_t>(stream));
        if (rc != OZTT_OK) throw Error(rc, msg);
    });
}

int oztt_ii_digit_run(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                    const oztt_digit_plan* plan, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !c || !plan) throw Error(OZTT_EINVAL, "null argument");
        if (!m || !n || !k) throw Error(OZTT_EINVAL, "matrix dimensions are zero");
        oztt::with_stream(device_id, [&](cudaStream_t st) {
            oztt::DevBuf da(st, m * k * 8), db(st, k * n * 8), dc(st, m * n * 8);
            OZTT_CUDA(cudaMemcpyAsync(da.p, a, m * k * 8, cudaMemcpyHostToDevice, st));
            OZTT_CUDA(cudaMemcpyAsync(db.p, b, k * n * 8, cudaMemcpyHostToDevice, st));
            oztt::run_ii_digit_device(da.as<double>(), db.as<double>(), dc.as<double>(), m, n, k, *plan, st);
            OZTT_CUDA(cudaMemcpyAsync(c, dc.p, m * n * 8, cudaMemcpyDeviceToHost, st));
            OZTT_CUDA(cudaStreamSynchronize(st));
        });
    });
}

int oztt_ii_digit_run_device(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                           uint64_t k, const oztt_digit_plan* plan, void* stream, double* stage_ms, char* err,
                           size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !c || !plan) throw Error(OZTT_EINVAL, "null argument");
        if (!m || !n || !k) throw Error(OZTT_EINVAL, "matrix dimensions are zero");
        oztt::open_device(device_id);
        oztt::run_ii_digit_device(a, b, c, m, n, k, *plan, reinterpret_cast<cudaStream_t>(stream), stage_ms);
    });
}

int oztt_ii_digit_split_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta,
                           const oztt_digit_plan* plan, int8_t* planes, uint64_t mp, uint64_t kp, void* stream, char* err,
                           size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !delta || !plan || !planes || lda < k || mp < m || kp < k)
            throw Error(OZTT_EINVAL, "digit_split_rows: bad arguments");
        oztt::check_digit_plan(*plan);
        oztt::launch_digit_split_rows(a, m, k, lda, delta, *plan, planes, mp, kp,
                                      reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_ii_digit_split_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta,
                           const oztt_digit_plan* plan, int8_t* planes, uint64_t np, uint64_t kp, void* stream, char* err,
                           size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!b || !delta || !plan || !planes || ldb < n || np < n || kp < k)
            throw Error(OZTT_EINVAL, "digit_split_cols: bad arguments");
        oztt::check_digit_plan(*plan);
        oztt::launch_digit_split_cols(b, k, n, ldb, delta, *plan, planes, np, kp,
                                      reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_ii_digit_gemm(const int8_t* a_planes, const int8_t* b_planes, uint64_t mp, uint64_t np, uint64_t kp,
                           const oztt_digit_plan* plan, int32_t mode, void* out, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a_planes || !b_planes || !plan || !out) throw Error(OZTT_EINVAL, "digit_gemm: null argument");
        oztt::check_digit_plan(*plan);
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        oztt::DevBuf word(st, 16);
        OZTT_CUDA(cudaMemsetAsync(word.p, 0, 16, st));
        oztt::launch_digit_gemm(a_planes, b_planes, mp, np, kp, *plan, mode, out, word.as<int>(), st);
        int host_err = 0;
        OZTT_CUDA(cudaMemcpyAsync(&host_err, word.p, 4, cudaMemcpyDeviceToHost, st));
        OZTT_CUDA(cudaStreamSynchronize(st));
        oztt::check_flags(0, host_err);
    });
}

int oztt_ii_digit_recon(const uint16_t* k_digits, uint64_t mp, uint64_t np, const int32_t* delta_a,
                      const int32_t* delta_b, const oztt_digit_plan* plan, double* c, uint64_t m, uint64_t n,
                      uint64_t ldc, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!k_digits || !delta_a || !delta_b || !plan || !c || ldc < n)
            throw Error(OZTT_EINVAL, "digit_recon: bad arguments");
        oztt::check_digit_plan(*plan);
        oztt::launch_recon_u16(k_digits, mp, np, delta_a, delta_b, plan->base, c, m, n, ldc,
                               reinterpret_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"
