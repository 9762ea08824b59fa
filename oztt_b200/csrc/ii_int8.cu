// SPDX-License-Identifier: Apache-2.0
//
// Scheme II INT8 pipeline on one B200 and the C-ABI entry points of its stages.
//
// The reference's backend (ozaki2_int8::run, src/ozaki2.cpp:439-478) plans, uploads FP64 tiles,
// scales, slices, runs one GEMM workload per modulus and output panel, reconstructs in one or two
// passes and reads back. Here one call is six kernel launches on one CUDA stream:
//     scale_rows(A) -> scale_cols(B) -> split_rows(A) -> split_cols(B) -> residue_gemm (all S moduli)
//     -> recon
// with the intermediate planes in HBM ([S][mp][kp] and [S][np][kp] int8 residues, [S][mp][np] uint8
// CRT digits) taken from the stream-ordered allocator and released at the end of the call (the pool
// keeps them for the next call). The range flags of the scaling stage and the wait-timeout word of
// the GEMM are read back after C, as the reference reads its flags after C (src/ozaki2.cpp:469-472).
#include <atomic>
#include <algorithm>
#include <chrono>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

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
void launch_transpose_scale(const double* b, uint64_t k, uint64_t n, uint64_t ldb, double* bt, int32_t shift,
                            int32_t* delta, uint32_t* flags, unsigned long long* colmax, cudaStream_t st);
void launch_residue_gemm(const int8_t* ap, const int8_t* bp, uint64_t mp, uint64_t np, uint64_t kp,
                         const oztt_ii_plan& p, int mode, void* out, int* err_word, cudaStream_t st,
                         uint64_t a_plane_rows = 0, uint64_t b_plane_rows = 0);
void launch_recon(const uint8_t* kp, uint64_t mp, uint64_t np, const int32_t* dA, const int32_t* dB,
                  const oztt_ii_plan& p, double* c, uint64_t m, uint64_t n, uint64_t ldc, cudaStream_t st);

// Selects the device, checks that it is a Blackwell data-centre GPU (compute capability 10.x, the
// sm_100a code in this library) and keeps the stream-ordered pool's memory between calls.
void open_device(int device_id) {
    if (device_id < 0) throw Error(OZTT_EINVAL, "device_id must be nonnegative");
    int count = 0;
    OZTT_CUDA(cudaGetDeviceCount(&count));
    if (device_id >= count) throw Error(OZTT_ERUNTIME, "CUDA device " + std::to_string(device_id) + " does not exist");
    OZTT_CUDA(cudaSetDevice(device_id));
    int major = 0, minor = 0;
    OZTT_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_id));
    OZTT_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device_id));
    if (major != 10 || minor != 0)
        throw Error(OZTT_ERUNTIME, "ozTTgemm for B200 runs on compute capability 10.0 (sm_100a) devices only");
    static std::mutex mu;
    static std::vector<int> configured;
    std::lock_guard<std::mutex> lock(mu);
    if (std::find(configured.begin(), configured.end(), device_id) == configured.end()) {
        cudaMemPool_t pool;
        OZTT_CUDA(cudaDeviceGetDefaultMemPool(&pool, device_id));
        uint64_t keep = UINT64_MAX;
        OZTT_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
        configured.push_back(device_id);
    }
}

void check_plan(const oztt_ii_plan& p) {
    if (p.S < 1 || p.S > OZTT_MAXS) throw Error(OZTT_EINVAL, "plan: the number of moduli must be 1..24");
    if (p.nd < 3 || p.nd > 5) throw Error(OZTT_EINVAL, "plan: the number of digits must be 3..5");
    for (int s = 0; s < p.S; ++s)
        if (p.moduli[s] < 3 || p.moduli[s] > 255) throw Error(OZTT_EINVAL, "plan: INT8 moduli must be in 3..255");
}

void check_flags(uint32_t flags, int gemm_err) {
    if (gemm_err)
        throw Error(OZTT_ERUNTIME, "the residue GEMM kernel gave up waiting (code " + std::to_string(gemm_err) +
                                       "); the result was not written");
    if (flags) {
        std::string why;
        if (flags & 1u) why += " a row or column maximum above the largest BF16;";
        if (flags & 2u) why += " a nonzero row or column maximum below 2^-126;";
        if (flags & 4u) why += " an Inf or NaN element;";
        throw Error(OZTT_ERUNTIME, "the scaling stage flagged inputs outside the supported range:" + why);
    }
}


// The device pipeline on device buffers (row-major, lda = k, ldb = n, ldc = n).
// stage_ms (optional, 6 entries): device time of scale rows, scale cols, split rows, split cols, residue
// GEMM and reconstruction, from CUDA events recorded on `st` between the launches. Under an evaluation
// Scope the launches run through the evaluator's phase timing and whole-pass check instead
// (run_profiled); a two-pass plan's reconstruction is then timed as two launches, one per half of the
// rows, so that the evaluator sees one reconstruction interval per pass.
void run_ii_int8_device(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                        const oztt_ii_plan& p, cudaStream_t st, double* stage_ms = nullptr) {
    check_plan(p);
    const uint64_t S = (uint64_t)p.S;
    const uint64_t mp = round_up(m, 128), np = round_up(n, 256), kp = round_up(k, 128);
    DevBuf dA(st, mp * 4), dB(st, np * 4), words(st, 16), bt(st, n * k * 8), colmax(st, n * 8);
    DevBuf ra(st, S * mp * kp), rb(st, S * np * kp), kpl(st, S * mp * np);
    OZTT_CUDA(cudaMemsetAsync(words.p, 0, 16, st));
    uint32_t* flags = words.as<uint32_t>();
    int* gemm_err = words.as<int>() + 1;
    Pipeline pl;
    pl.add(kScale, kHead, 0, [&] { launch_scale_rows(a, m, k, k, p.shift, dA.as<int32_t>(), nullptr, flags, st); });
    // B transposed once (an HBM-bound copy that also takes its column maxima), then split by rows: its columns
    // are B^T's rows, with the same maxima, exponent deltas, flags and residue planes [S][np][kp] as the column
    // kernels give
    pl.add(kScale, kHead, 1, [&] {
        launch_transpose_scale(b, k, n, n, bt.as<double>(), p.shift, dB.as<int32_t>(), flags,
                               colmax.as<unsigned long long>(), st);
    });
    pl.add(kSlice, kHead, 2, [&] { launch_split_rows(a, m, k, k, dA.as<int32_t>(), p, ra.as<int8_t>(), mp, kp, st); });
    pl.add(kSlice, kHead, 3,
           [&] { launch_split_rows(bt.as<double>(), n, k, k, dB.as<int32_t>(), p, rb.as<int8_t>(), np, kp, st); });
    pl.add(kGemm, kGemmStep, 4,
           [&] { launch_residue_gemm(ra.as<int8_t>(), rb.as<int8_t>(), mp, np, kp, p, 1, kpl.p, gemm_err, st); });
    const uint64_t halves = (evaluation_active() && p.two_pass && m > 1) ? 2 : 1;
    for (uint64_t h = 0; h < halves; ++h) {
        const uint64_t r0 = m * h / halves, rows = m * (h + 1) / halves - r0;
        pl.add(kRecon, kReconStep, 5, [&, r0, rows] {
            launch_recon(kpl.as<uint8_t>() + r0 * np, mp, np, dA.as<int32_t>() + r0, dB.as<int32_t>(), p, c + r0 * n,
                         rows, n, n, st);
        }, true);
    }
    pl.writes(dA.p, mp * 4);
    pl.writes(dB.p, np * 4);
    pl.writes(bt.p, n * k * 8);
    pl.writes(colmax.p, n * 8);
    pl.writes(ra.p, S * mp * kp);
    pl.writes(rb.p, S * np * kp);
    pl.writes(kpl.p, S * mp * np);
    pl.writes(c, m * n * 8);
    pl.out = c;
    pl.out_bytes = m * n * 8;
    pl.partial_products = (unsigned)S;
    if (!run_profiled(pl, st)) pl.run(st, stage_ms, 6);
    uint32_t host_words[2] = {0, 0};
    OZTT_CUDA(cudaMemcpyAsync(host_words, words.p, 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaStreamSynchronize(st));
    check_flags(host_words[0], (int)host_words[1]);
}

void run_ii_int8_host(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                      const oztt_ii_plan& p) {
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
    {
        DevBuf da(st, m * k * 8), db(st, k * n * 8), dc(st, m * n * 8);
        OZTT_CUDA(cudaMemcpyAsync(da.p, a, m * k * 8, cudaMemcpyHostToDevice, st));
        OZTT_CUDA(cudaMemcpyAsync(db.p, b, k * n * 8, cudaMemcpyHostToDevice, st));
        run_ii_int8_device(da.as<double>(), db.as<double>(), dc.as<double>(), m, n, k, p, st);
        OZTT_CUDA(cudaMemcpyAsync(c, dc.p, m * n * 8, cudaMemcpyDeviceToHost, st));
        OZTT_CUDA(cudaStreamSynchronize(st));
    }
}

PolicyStats device_policy_stats(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                                cudaStream_t st);

// Plan from device-resident operands: the input statistics are measured on the device
// (device_policy_stats, bit-identical to the host measurement), the decisions made on the host.
int plan_ii_int8_device(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli,
                        int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan& p, std::string& err,
                        cudaStream_t st) {
    return plan_ii_int8_with([&](uint32_t N, uint32_t) { return device_policy_stats(a, b, m, n, k, N, st); }, m, n,
                             k, max_moduli, reconstruction, fixed_bits, p, err);
}

// The call from host buffers without overlap, as the evaluator's profiled calls make it: A and B to the
// device, the plan from device statistics (the width fixed to fixed_bits when nonzero), the pipeline
// (under the evaluation Scope), C back. Returns OZTT_OK, or an error code with its message.
int run_ii_int8_uploaded(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                         uint64_t k, uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan& p,
                         std::string& err) {
    char buf[1024];
    int inner = OZTT_OK;
    const int rc = guarded(buf, sizeof buf, [&] {
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
        DevBuf da(st, m * k * 8), db(st, k * n * 8);
        OZTT_CUDA(cudaMemcpyAsync(da.p, a, m * k * 8, cudaMemcpyHostToDevice, st));
        OZTT_CUDA(cudaMemcpyAsync(db.p, b, k * n * 8, cudaMemcpyHostToDevice, st));
        inner = plan_ii_int8_device(da.as<double>(), db.as<double>(), m, n, k, max_moduli, reconstruction, fixed_bits,
                                    p, err, st);
        if (inner != OZTT_OK) return;
        DevBuf dc(st, m * n * 8);
        run_ii_int8_device(da.as<double>(), db.as<double>(), dc.as<double>(), m, n, k, p, st);
        OZTT_CUDA(cudaMemcpyAsync(c, dc.p, m * n * 8, cudaMemcpyDeviceToHost, st));
        OZTT_CUDA(cudaStreamSynchronize(st));
    });
    if (rc != OZTT_OK) err = buf;
    return rc != OZTT_OK ? rc : inner;
}

// ---- the call from host buffers, transfers overlapped ----------------------------------------------
//
// Context::gemm's path for INT8 Scheme II (StreamedCall, streamed.cu): the upload with the statistics
// measured on the way, the caller's value checks from the measured maxima, the plan, then scale and
// split, and the residue GEMM and the reconstruction in bands of about 2048 rows (up to 8), each band of
// C read back while the next is computed. The range flags and the GEMM's wait-timeout word are read
// after C, as the reference reads its flags after C (src/ozaki2.cpp:469-472).
namespace {

int run_ii_int8_streamed_impl(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                              uint64_t k, uint32_t max_moduli, int32_t reconstruction,
                              const std::function<void(const uint64_t*, const uint64_t*)>& check,
                              oztt_ii_plan& p, std::string& err) {
    StreamedCall call(device_id, a, b, m, n, k);
    StreamedPhases& ph = call.phases();
    cudaStream_t st = call.work();
    std::vector<uint64_t> row_max, col_max;
    const PolicyStats ps = call.upload(row_max, col_max);
    // every input value checked before the plan and before C is written
    double t = call.ms_since_start();
    check(row_max.data(), col_max.data());
    ph.check_ms = call.ms_since_start() - t;
    t = call.ms_since_start();
    const int rc = plan_ii_int8_with([&](uint32_t, uint32_t) { return ps; }, m, n, k, max_moduli, reconstruction, 0, p,
                                     err);
    if (rc != OZTT_OK) return rc;
    ph.plan_ms = call.ms_since_start() - t;
    t = call.ms_since_start();
    check_plan(p);
    const uint64_t S = (uint64_t)p.S;
    const uint64_t mp = round_up(m, 128), np = round_up(n, 256), kp = round_up(k, 128);
    const uint64_t bands = std::min<uint64_t>(8, std::max<uint64_t>(1, mp / 2048));
    const uint64_t bm = round_up((mp + bands - 1) / bands, 128);
    const double *da = call.a_dev(), *db = call.b_dev();
    double* dc = call.c_dev();
    DevBuf dA(st, mp * 4), dB(st, np * 4), colmax(st, n * 8), words(st, 16);
    DevBuf ra(st, S * mp * kp), rb(st, S * np * kp), kpl(st, S * bm * np);
    OZTT_CUDA(cudaMemsetAsync(words.p, 0, 16, st));
    uint32_t* flags = words.as<uint32_t>();
    int* gemm_err = words.as<int>() + 1;
    launch_scale_rows(da, m, k, k, p.shift, dA.as<int32_t>(), nullptr, flags, st);
    launch_scale_cols(db, k, n, n, p.shift, dB.as<int32_t>(), nullptr, flags, colmax.as<unsigned long long>(), st);
    launch_split_rows(da, m, k, k, dA.as<int32_t>(), p, ra.as<int8_t>(), mp, kp, st);
    launch_split_cols(db, k, n, n, dB.as<int32_t>(), p, rb.as<int8_t>(), np, kp, st);
    for (uint64_t r0 = 0; r0 < mp; r0 += bm) {
        const uint64_t rows_p = std::min(bm, mp - r0);
        launch_residue_gemm(ra.as<int8_t>() + r0 * kp, rb.as<int8_t>(), rows_p, np, kp, p, 1, kpl.p, gemm_err, st, mp);
        if (r0 >= m) continue;
        const uint64_t rows = std::min(m, r0 + rows_p) - r0;
        launch_recon(kpl.as<uint8_t>(), rows_p, np, dA.as<int32_t>() + r0, dB.as<int32_t>(), p, dc + r0 * n, rows, n,
                     n, st);
        call.band_done(r0, rows);
    }
    call.read_back(c);
    uint32_t host_words[2] = {0, 0};
    OZTT_CUDA(cudaMemcpyAsync(host_words, words.p, 8, cudaMemcpyDeviceToHost, st));
    call.finish(t);
    check_flags(host_words[0], (int)host_words[1]);
    return OZTT_OK;
}

// ---- the call from host buffers, computing while the operands upload ------------------------------------------
//
// The magnitude patterns of A's row maxima and B's column maxima (the front end's value checks) for A's rows
// from r_begin on and all of B, measured by the host's threads from the caller's buffers while the operands
// upload: known long before A has landed. (The first r_begin rows' maxima come from the device, which measures
// them for the first plan.)
class HostMaxima {
public:
    HostMaxima(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint64_t r_begin)
        : row_max(m), col_max(n, 0), th_([this, a, b, m, n, k, r_begin] {
              value_maxima(a + r_begin * k, b, m - r_begin, n, k, row_max.data() + r_begin, col_max.data());
          }) {}
    ~HostMaxima() { wait(); }
    void wait() {
        if (th_.joinable()) th_.join();
    }
    std::vector<uint64_t> row_max, col_max;

private:
    std::thread th_;  // after the vectors it fills
};

bool overlaps(const void* p, uint64_t pbytes, const void* q, uint64_t qbytes) {
    const uintptr_t p0 = reinterpret_cast<uintptr_t>(p), q0 = reinterpret_cast<uintptr_t>(q);
    return p0 < q0 + qbytes && q0 < p0 + pbytes;
}

// Context::gemm from host buffers, computing while the operands upload. The upload order is B's first block
// of columns (of eight), A's first half (bands of 1024 rows), B's next four blocks, the rest of A, then B's
// last three blocks. The precision decision depends on the statistics of the whole A and B, so the pipeline
// starts on a first plan made from an estimate: A's first half and B's first block, each standing for its
// matrix (the decision depends on the size-free ratio (TA nB + TB nA) / 12 nC, which such parts estimate
// closely), measured as they land. On that plan A's first half is split once and multiplied by each of B's
// first five blocks (the first one at once, the others as they land); each later band of A is split and
// multiplied by those five blocks as it lands; each of B's last blocks by the whole A. The value checks
// need the maxima of every row of A and column of B: the device measures A's first half for the first plan,
// the host's threads measure the rest of A and all of B from the caller's buffers meanwhile. Once every value
// is checked, the pieces of C (a block of rows against a block of columns) are read back as they finish --
// when that cannot change the outcome of the call: no plan for these dimensions can fail, and C does not
// overlap A or B. When A has landed, the reference's plan is decided from bounds of its statistics
// measured as the blocks and bands landed (only a decision that lies within the bounds needs the exact
// long-double sums). If it equals the first plan, C is its result; otherwise the pipeline runs again with it
// and C is read back again. An invalid input is reported before anything is written to C, as the front end
// requires.
int run_ii_int8_overlapped(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                           uint64_t k, uint32_t max_moduli, int32_t reconstruction,
                           const std::function<void(const uint64_t*, const uint64_t*)>& check, oztt_ii_plan& p,
                           std::string& err) {
    StreamedCall call(device_id, a, b, m, n, k);
    StreamedPhases& ph = call.phases();
    cudaStream_t st = call.work();
    const uint64_t mp = round_up(m, 128), np = round_up(n, 256), kp = round_up(k, 128);
    const uint64_t bm = 1024;
    // The upload order: B's first block, A's first half (whole bands), B's next blocks up to 5/8 of B, the
    // rest of A, B's last blocks. The first plan waits for A's first half; then each piece that lands brings
    // its products with everything already there, and the order keeps that work close to the rate at which
    // the pieces arrive: the first half of A against each block of B (about 0.8 of a block's upload time at
    // 16384^3), each later band against 5/8 of B (0.9 of a band's), each last block against the whole A
    // (1.5 of a block's, the excess left for the end), so that the device is idle little after the first
    // plan and the last work is short. (9/16 of A first and all of B before the rest of A measured the same
    // per call; this order leaves the pass over A that needs all of B until after the last upload, where one
    // launch over all rows keeps every SM busy.)
    const uint64_t pre = std::min(round_up(m / 2, bm), m);
    const uint64_t pre_bands = (pre + bm - 1) / bm;
    const uint64_t nb = round_up((n + 7) / 8, 256);  // B's blocks of columns
    const uint64_t nblocks = (n + nb - 1) / nb;
    const uint64_t mid_blocks = nblocks / 2;         // B's blocks after the first one, before the rest of A
    HostMaxima host(a, b, m, n, k, pre);
    std::vector<cudaEvent_t> b_landed;
    const std::vector<cudaEvent_t> landed = call.upload_prefix_first(pre, bm, nb, mid_blocks, m - pre, b_landed);
    // the first plan, from A's first part and B's first block
    bool estimated = false;
    std::vector<uint64_t> pre_max;
    const PolicyStats first = call.prefix_estimate(estimated, &pre_max);
    oztt_ii_plan p0{};
    std::string err0;
    const int rc0 = estimated ? plan_ii_int8_with([&](uint32_t, uint32_t) { return first; }, m, n, k, max_moduli,
                                                  reconstruction, 0, p0, err0)
                              : OZTT_ERUNTIME;
    ph.first_plan_ms = call.ms_since_start();
    const double *da = call.a_dev(), *db = call.b_dev();
    double* dc = call.c_dev();
    DevBuf dA(st, mp * 4), dB(st, np * 4), colmax(st, n * 8), words(st, 16);
    OZTT_CUDA(cudaMemsetAsync(words.p, 0, 16, st));
    uint32_t* flags = words.as<uint32_t>();
    int* gemm_err = words.as<int>() + 1;
    std::unique_ptr<DevBuf> rb, ra, kpl;
    const auto buffers = [&](const oztt_ii_plan& q, uint64_t a_rows) {
        const uint64_t S = (uint64_t)q.S;
        rb = std::make_unique<DevBuf>(st, S * np * kp);
        ra = std::make_unique<DevBuf>(st, S * a_rows * kp);
        kpl = std::make_unique<DevBuf>(st, S * std::max(a_rows * std::min(nb, np), bm * np));
    };
    // one band of A's rows (at most h) against the whole B (B's planes complete)
    const auto band = [&](const oztt_ii_plan& q, uint64_t r0, uint64_t h = 1024) {
        const uint64_t rows_p = std::min(h, mp - r0), rows = std::min(m, r0 + rows_p) - r0;
        launch_scale_rows(da + r0 * k, rows, k, k, q.shift, dA.as<int32_t>() + r0, nullptr, flags, st);
        launch_split_rows(da + r0 * k, rows, k, k, dA.as<int32_t>() + r0, q, ra->as<int8_t>(), rows_p, kp, st);
        launch_residue_gemm(ra->as<int8_t>(), rb->as<int8_t>(), rows_p, np, kp, q, 1, kpl->p, gemm_err, st, 0);
        launch_recon(kpl->as<uint8_t>(), rows_p, np, dA.as<int32_t>() + r0, dB.as<int32_t>(), q, dc + r0 * n, rows, n,
                     n, st);
        call.band_done(r0, rows);
    };
    // on the first plan, following the upload: every piece that lands is split and multiplied by everything
    // already split (A's planes kept whole, [S][mp][kp]): A's first half, then each block of B against the
    // rows there, each band of A against the columns there
    const auto following = [&](const oztt_ii_plan& q) {
        buffers(q, mp);
        uint64_t rows_done = 0, cols_done = 0;
        // rows [r0, r0 + rows) of A (a multiple of 128 rows unless they end A): split into the whole planes
        const auto a_rows = [&](uint64_t r0, uint64_t rows_p) {
            const uint64_t rows = std::min(m, r0 + rows_p) - r0;
            launch_scale_rows(da + r0 * k, rows, k, k, q.shift, dA.as<int32_t>() + r0, nullptr, flags, st);
            launch_split_rows(da + r0 * k, rows, k, k, dA.as<int32_t>() + r0, q, ra->as<int8_t>() + r0 * kp, rows_p,
                              kp, st, mp);
            return rows;
        };
        // the product of rows [r0, r0 + rows) with columns [c0, c0 + cols), both split, and its read-back
        const auto tile = [&](uint64_t r0, uint64_t rows, uint64_t c0, uint64_t cols) {
            const uint64_t rows_p = std::min(round_up(rows, 128), mp - r0);
            const uint64_t cols_p = std::min(round_up(cols, 256), np - c0);
            launch_residue_gemm(ra->as<int8_t>() + r0 * kp, rb->as<int8_t>() + c0 * kp, rows_p, cols_p, kp, q, 1,
                                kpl->p, gemm_err, st, mp, np);
            launch_recon(kpl->as<uint8_t>(), rows_p, cols_p, dA.as<int32_t>() + r0, dB.as<int32_t>() + c0, q,
                         dc + r0 * n + c0, rows, cols, n, st);
            call.tile_done(r0, rows, c0, cols);  // read back as soon as it is written (2-D copy)
        };
        // block j of B against the rows there; chunk: rows per product once all of A is there, so that the
        // read-back of one part overlaps the product of the next
        // (a block of 2048 columns: the column kernels cost about what a transpose and the row split would)
        const auto b_block = [&](uint64_t j, uint64_t chunk) {
            const uint64_t c0 = j * nb, cols_p = std::min(nb, np - c0), cols = std::min(n, c0 + cols_p) - c0;
            OZTT_CUDA(cudaStreamWaitEvent(st, b_landed.at(j), 0));
            launch_scale_cols(db + c0, k, cols, n, q.shift, dB.as<int32_t>() + c0, nullptr, flags,
                              colmax.as<unsigned long long>() + c0, st);
            launch_split_cols(db + c0, k, cols, n, dB.as<int32_t>() + c0, q, rb->as<int8_t>() + c0 * kp, cols_p, kp,
                              st, np);
            for (uint64_t r0 = 0; r0 < rows_done; r0 += chunk) tile(r0, std::min(chunk, rows_done - r0), c0, cols);
            cols_done = c0 + cols;
        };
        // band i of A (h rows from r0) against the columns there
        const auto a_band = [&](uint64_t i, uint64_t r0, uint64_t h) {
            OZTT_CUDA(cudaStreamWaitEvent(st, landed[i], 0));
            const uint64_t rows = a_rows(r0, std::min(h, mp - r0));
            if (cols_done) tile(r0, rows, 0, cols_done);
            rows_done = r0 + rows;
        };
        OZTT_CUDA(cudaStreamWaitEvent(st, landed[pre_bands - 1], 0));
        rows_done = a_rows(0, std::min(round_up(pre, 128), mp));
        uint64_t j = 0;
        for (; j <= mid_blocks && j < nblocks; ++j) b_block(j, rows_done);
        call.timeline(st, 0);
        for (uint64_t i = pre_bands, r0 = pre; r0 < m; ++i, r0 += bm) a_band(i, r0, bm);
        for (; j < nblocks; ++j) b_block(j, j + 1 < nblocks ? 4 * bm : 2 * bm);
        call.timeline(st, 1);
    };
    // after everything has landed: the whole pipeline on a plan
    const auto whole = [&](const oztt_ii_plan& q) {
        OZTT_CUDA(cudaStreamWaitEvent(st, landed.back(), 0));
        OZTT_CUDA(cudaStreamWaitEvent(st, b_landed.back(), 0));
        buffers(q, bm);
        launch_scale_cols(db, k, n, n, q.shift, dB.as<int32_t>(), nullptr, flags, colmax.as<unsigned long long>(), st);
        launch_split_cols(db, k, n, n, dB.as<int32_t>(), q, rb->as<int8_t>(), np, kp, st);
        for (uint64_t r0 = 0; r0 < m; r0 += bm) band(q, r0);
        call.timeline(st, 1);
    };
    if (rc0 == OZTT_OK) {
        check_plan(p0);
        following(p0);
    }
    // every value checked (from the host's maxima); then C is read back as its bands finish when writing it
    // before the plan is confirmed cannot change the outcome of the call
    host.wait();
    if (pre_max.size() == pre)
        std::copy(pre_max.begin(), pre_max.end(), host.row_max.begin());
    else  // (no device measurement of the first part: the host measures it too)
        value_maxima(a, b, pre, 0, k, host.row_max.data(), nullptr);
    ph.host_checked_ms = call.ms_since_start();
    double t = call.ms_since_start();
    check(host.row_max.data(), host.col_max.data());
    ph.check_ms = call.ms_since_start() - t;
    const bool early = rc0 == OZTT_OK && plan_ii_int8_never_fails(m, n, k, max_moduli) &&
                       !overlaps(c, m * n * 8, a, m * k * 8) && !overlaps(c, m * n * 8, b, k * n * 8);
    if (early) call.read_back(c);
    ph.early_readback = early ? 1 : 0;
    // the reference's plan: decided by the bounds, or from the exact sums
    const PolicyBounds bounds = call.certified_bounds();
    t = call.ms_since_start();
    bool decided = false;
    int rc = plan_ii_int8_certified(bounds, m, n, k, max_moduli, reconstruction, p, err, decided);
    if (rc == OZTT_OK && !decided) {
        const PolicyStats ps = call.exact_stats();
        rc = plan_ii_int8_with([&](uint32_t, uint32_t) { return ps; }, m, n, k, max_moduli, reconstruction, 0, p, err);
    }
    if (rc != OZTT_OK) return rc;
    ph.plan_ms = call.ms_since_start() - t;
    const bool same = rc0 == OZTT_OK && p0.S == p.S && p0.b == p.b && p0.nd == p.nd && p0.shift == p.shift &&
                      std::equal(p0.moduli, p0.moduli + p0.S, p.moduli);
    ph.replanned = same ? 0 : 1;
    if (!same) {  // the first plan was not the reference's: again, with the reference's plan
        call.discard_bands();
        check_plan(p);
        whole(p);
        call.read_back(c);
    } else if (!early) {
        call.read_back(c);
    }
    uint32_t host_words[2] = {0, 0};
    OZTT_CUDA(cudaMemcpyAsync(host_words, words.p, 8, cudaMemcpyDeviceToHost, st));
    call.finish(ph.first_plan_ms);
    check_flags(host_words[0], (int)host_words[1]);
    return OZTT_OK;
}

}  // namespace

int run_ii_int8_streamed(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                         uint64_t k, uint32_t max_moduli, int32_t reconstruction,
                         const std::function<void(const uint64_t*, const uint64_t*)>& check, oztt_ii_plan& p,
                         std::string& err) {
    char buf[1024];
    int inner = OZTT_OK;
    const int rc = guarded(buf, sizeof buf, [&] {
        // calls of 4096 rows and more compute while their operands upload (a first plan estimated from A's first
        // half and B's first block, confirmed by the complete statistics); smaller calls upload everything first
        if (round_up(m, 128) >= 4096)
            inner = run_ii_int8_overlapped(device_id, a, b, c, m, n, k, max_moduli, reconstruction, check, p, err);
        else
            inner = run_ii_int8_streamed_impl(device_id, a, b, c, m, n, k, max_moduli, reconstruction, check, p, err);
    });
    if (rc != OZTT_OK) err = buf;
    return rc != OZTT_OK ? rc : inner;
}

void open_device_checked(int device_id) { open_device(device_id); }

namespace {
std::atomic<int> g_options[3];  // indexed by OZTT_OPT_*; zero-initialised (the defaults)
}

int option_value(int option) { return option > 0 && option < 3 ? g_options[option].load() : 0; }

}  // namespace oztt

using oztt::Error;
using oztt::guarded;

extern "C" {

int oztt_set_option(int32_t option, int32_t value, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (option != OZTT_OPT_GEMM_CTA_PAIRS && option != OZTT_OPT_RECON_INT)
            throw Error(OZTT_EINVAL, "unknown option " + std::to_string(option));
        if (value != 0 && value != 1) throw Error(OZTT_EINVAL, "option values are 0 or 1");
        oztt::g_options[option].store(value);
    });
}

int oztt_get_option(int32_t option, int32_t* value) {
    if (!value || (option != OZTT_OPT_GEMM_CTA_PAIRS && option != OZTT_OPT_RECON_INT)) return OZTT_EINVAL;
    *value = oztt::option_value(option);
    return OZTT_OK;
}

int oztt_ii_int8_run(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                     const oztt_ii_plan* plan, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !c || !plan) throw Error(OZTT_EINVAL, "null argument");
        if (!m || !n || !k) throw Error(OZTT_EINVAL, "matrix dimensions are zero");
        oztt::run_ii_int8_host(device_id, a, b, c, m, n, k, *plan);
    });
}

int oztt_ii_int8_plan_device(int device_id, const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                             uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan* plan,
                             void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !plan) throw Error(OZTT_EINVAL, "null argument");
        oztt::open_device(device_id);
        std::string msg;
        const int rc = oztt::plan_ii_int8_device(a, b, m, n, k, max_moduli, reconstruction, fixed_bits, *plan, msg,
                                                 reinterpret_cast<cudaStream_t>(stream));
        if (rc != OZTT_OK) throw Error(rc, msg);
    });
}

int oztt_ii_int8_run_device(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                            uint64_t k, const oztt_ii_plan* plan, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !c || !plan) throw Error(OZTT_EINVAL, "null argument");
        if (!m || !n || !k) throw Error(OZTT_EINVAL, "matrix dimensions are zero");
        oztt::open_device(device_id);
        oztt::run_ii_int8_device(a, b, c, m, n, k, *plan, reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_ii_int8_run_device_timed(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                                  uint64_t k, const oztt_ii_plan* plan, void* stream, double* stage_ms, char* err,
                                  size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !b || !c || !plan || !stage_ms) throw Error(OZTT_EINVAL, "null argument");
        if (!m || !n || !k) throw Error(OZTT_EINVAL, "matrix dimensions are zero");
        oztt::open_device(device_id);
        oztt::run_ii_int8_device(a, b, c, m, n, k, *plan, reinterpret_cast<cudaStream_t>(stream), stage_ms);
    });
}

void oztt_ii_padded_dims(uint64_t m, uint64_t n, uint64_t k, uint64_t* mp, uint64_t* np, uint64_t* kp) {
    if (mp) *mp = oztt::round_up(m, 128);
    if (np) *np = oztt::round_up(n, 256);
    if (kp) *kp = oztt::round_up(k, 128);
}

int oztt_ii_scale_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, int32_t shift, int32_t* delta,
                       uint16_t* bf16max, uint32_t* flags, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !delta || !flags || lda < k) throw Error(OZTT_EINVAL, "scale_rows: bad arguments");
        oztt::launch_scale_rows(a, m, k, lda, shift, delta, bf16max, flags, reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_ii_scale_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift, int32_t* delta,
                       uint16_t* bf16max, uint32_t* flags, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!b || !delta || !flags || ldb < n) throw Error(OZTT_EINVAL, "scale_cols: bad arguments");
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        oztt::DevBuf colmax(st, n * 8);
        oztt::launch_scale_cols(b, k, n, ldb, shift, delta, bf16max, flags, colmax.as<unsigned long long>(), st);
    });
}

int oztt_ii_split_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta,
                       const oztt_ii_plan* plan, int8_t* planes, uint64_t mp, uint64_t kp, void* stream, char* err,
                       size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a || !delta || !plan || !planes || lda < k || mp < m || kp < k)
            throw Error(OZTT_EINVAL, "split_rows: bad arguments");
        oztt::check_plan(*plan);
        oztt::launch_split_rows(a, m, k, lda, delta, *plan, planes, mp, kp, reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_ii_split_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta,
                       const oztt_ii_plan* plan, int8_t* planes, uint64_t np, uint64_t kp, void* stream, char* err,
                       size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!b || !delta || !plan || !planes || ldb < n || np < n || kp < k)
            throw Error(OZTT_EINVAL, "split_cols: bad arguments");
        oztt::check_plan(*plan);
        oztt::launch_split_cols(b, k, n, ldb, delta, *plan, planes, np, kp, reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_ii_residue_gemm(const int8_t* a_planes, const int8_t* b_planes, uint64_t mp, uint64_t np, uint64_t kp,
                         const oztt_ii_plan* plan, int32_t mode, void* out, void* stream, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!a_planes || !b_planes || !plan || !out) throw Error(OZTT_EINVAL, "residue_gemm: null argument");
        oztt::check_plan(*plan);
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        oztt::DevBuf word(st, 16);
        OZTT_CUDA(cudaMemsetAsync(word.p, 0, 16, st));
        oztt::launch_residue_gemm(a_planes, b_planes, mp, np, kp, *plan, mode, out, word.as<int>(), st);
        int host_err = 0;
        OZTT_CUDA(cudaMemcpyAsync(&host_err, word.p, 4, cudaMemcpyDeviceToHost, st));
        OZTT_CUDA(cudaStreamSynchronize(st));
        oztt::check_flags(0, host_err);
    });
}

int oztt_ii_recon(const uint8_t* k_planes, uint64_t mp, uint64_t np, const int32_t* delta_a, const int32_t* delta_b,
                  const oztt_ii_plan* plan, double* c, uint64_t m, uint64_t n, uint64_t ldc, void* stream, char* err,
                  size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!k_planes || !delta_a || !delta_b || !plan || !c || ldc < n) throw Error(OZTT_EINVAL, "recon: bad arguments");
        oztt::check_plan(*plan);
        oztt::launch_recon(k_planes, mp, np, delta_a, delta_b, *plan, c, m, n, ldc,
                           reinterpret_cast<cudaStream_t>(stream));
    });
}

int oztt_device_info(int device_id, int32_t* sm_count, int32_t* cc_major, int32_t* cc_minor) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device_id) != cudaSuccess) return OZTT_ERUNTIME;
    if (sm_count) *sm_count = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMajor, device_id) != cudaSuccess) return OZTT_ERUNTIME;
    if (cc_major) *cc_major = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMinor, device_id) != cudaSuccess) return OZTT_ERUNTIME;
    if (cc_minor) *cc_minor = v;
    return OZTT_OK;
}

}  // extern "C"
