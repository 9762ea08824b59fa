// SPDX-License-Identifier: Apache-2.0
//
// Context::gemm from host buffers with the transfers overlapped (StreamedCall, runtime.cuh), shared by
// the INT8 and digit-format Scheme II paths.
//
//   copy-up stream   B, then A, in blocks of columns of about 64 MiB (2-D copies of all rows); for the
//                    INT8 path that computes while its operands land (upload_prefix_first): B's first
//                    block of columns, A's first part in bands of rows, then further blocks of B and bands
//                    of A
//   work stream      the precision-policy statistics of each piece as it lands (PolicyStatsRun), then
//                    the caller's pipeline, which marks each finished band of rows of C
//   copy-down stream each finished band of C read back while the next is computed
//
// The statistics left after the upload are those of the last block of A, so the plan can be made as
// soon as the upload ends; the values are checked from the measured maxima before that.
#include <chrono>
#include <cmath>
#include <mutex>

#include "oztt_common.cuh"
#include "planner.hpp"
#include "runtime.cuh"

namespace oztt {

void launch_stats_absmax(const double* x, uint64_t rows, uint64_t cols, int mode, double* out, cudaStream_t st);
void launch_stats_sumsq(const double* x, uint64_t rows, uint64_t cols, int mode, double rg, double* out,
                        cudaStream_t st);
void launch_stats_sketch(const double* x, uint64_t rows, uint64_t cols, double rg, const double* v, uint64_t vstride,
                         double* out, uint64_t ostride, cudaStream_t st);
PolicyStats combine_policy_stats(const double* row_max, uint64_t m, const double* col_max, uint64_t n,
                                 const double* row_sumsq, const double* col_sumsq, const double* s, uint64_t sstride,
                                 double rgA, double rgB);
void launch_band_certify(const double* x, uint64_t rows, uint64_t k, const double* y, const double* ew, double* out,
                         uint32_t* flags, cudaStream_t st);
void launch_bcert_block(const double* b, uint64_t k, uint64_t w, uint64_t ldb, const double* g, uint64_t gstride,
                        double* acc, uint32_t* flags, cudaStream_t st);
void launch_bcert_finish(const unsigned long long* col_max, uint64_t n, const double* acc, uint64_t k, double c1,
                         double* rgB, double* y, double* ew, cudaStream_t st);
void launch_col_absmax(const double* b, uint64_t k, uint64_t w, uint64_t ldb, unsigned long long* out,
                       cudaStream_t st);
double bcert_error_factor(uint64_t n);
void bounded_nb(const double* acc, uint64_t k, uint64_t n, double rgB, double& lo, double& hi);
std::vector<double> policy_vectors_host(uint32_t N);
PolicyBounds certified_policy_bounds(const double* cert, uint64_t m, uint64_t k, const double* col_max, uint64_t n,
                                     double nB_lo, double nB_hi, double rgB);
constexpr uint64_t kCertWidth = 19;   // doubles per row of A written by launch_band_certify
constexpr uint64_t kBCertWidth = 17;  // doubles per row of B accumulated by launch_bcert_block

namespace {
StreamedPhases g_last_phases;
std::mutex g_phases_mu;
constexpr uint64_t kUploadChunkBytes = 64ull << 20;

// One pinned staging buffer kept for the process (pinning a few MiB per call costs about a millisecond);
// a call that finds it in use pins its own.
struct PinnedStage {
    std::mutex mu;
    double* p = nullptr;
    uint64_t bytes = 0;
    bool busy = false;
} g_stage;

double* acquire_stage(uint64_t bytes, bool& shared) {
    {
        std::lock_guard<std::mutex> lock(g_stage.mu);
        if (!g_stage.busy) {
            if (g_stage.bytes < bytes) {
                if (g_stage.p) OZTT_CUDA(cudaFreeHost(g_stage.p));
                g_stage.p = nullptr;
                g_stage.bytes = 0;
                OZTT_CUDA(cudaHostAlloc((void**)&g_stage.p, bytes, cudaHostAllocPortable));
                g_stage.bytes = bytes;
            }
            g_stage.busy = true;
            shared = true;
            return g_stage.p;
        }
    }
    double* p = nullptr;
    OZTT_CUDA(cudaHostAlloc((void**)&p, bytes, cudaHostAllocPortable));
    shared = false;
    return p;
}

void release_stage(double* p, bool shared) {
    if (!p) return;
    if (shared) {
        std::lock_guard<std::mutex> lock(g_stage.mu);
        g_stage.busy = false;
    } else {
        cudaFreeHost(p);
    }
}
}  // namespace

StreamedPhases last_streamed_phases() {
    std::lock_guard<std::mutex> lock(g_phases_mu);
    return g_last_phases;
}

StreamedCall::StreamedCall(int device_id, const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k)
    : a_(a), b_(b), m_(m), n_(n), k_(k), t0_(std::chrono::steady_clock::now()) {
    open_device(device_id);
    for (cudaStream_t* s : {&work_, &up_, &down_}) OZTT_CUDA(cudaStreamCreateWithFlags(s, cudaStreamNonBlocking));
    da_ = std::make_unique<DevBuf>(work_, m * k * 8);
    db_ = std::make_unique<DevBuf>(work_, k * n * 8);
}

StreamedCall::~StreamedCall() {
    for (cudaStream_t s : {up_, down_, stat_, cert_, est_, work_})
        if (s) cudaStreamSynchronize(s);
    // the buffers go back to the pool on the work stream, after everything that used them
    stats_.reset();
    est_run_.reset();
    cert_buf_.reset();
    bparts_.reset();
    cert_flags_.reset();
    dc_.reset();
    da_.reset();
    db_.reset();
    release_stage(stage_, stage_shared_);
    for (cudaEvent_t e : events_) cudaEventDestroy(e);
    for (cudaEvent_t e : {tl_start_, tl_[0], tl_[1], tl_[2], tl_[3]})
        if (e) cudaEventDestroy(e);
    for (cudaStream_t s : {up_, down_, stat_, cert_, est_, work_})
        if (s) {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
}

double StreamedCall::ms_since_start() const {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0_).count();
}

cudaEvent_t StreamedCall::mark(cudaStream_t s) {
    cudaEvent_t e;
    OZTT_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    events_.push_back(e);
    OZTT_CUDA(cudaEventRecord(e, s));
    return e;
}

cudaEvent_t StreamedCall::order(cudaStream_t from, cudaStream_t to) {
    cudaEvent_t e = mark(from);
    OZTT_CUDA(cudaStreamWaitEvent(to, e, 0));
    return e;
}

PolicyStats StreamedCall::upload(std::vector<uint64_t>& row_max, std::vector<uint64_t>& col_max,
                                 std::vector<double>* row_sumsq, std::vector<double>* col_sumsq, double* rg) {
    const uint64_t m = m_, n = n_, k = k_;
    const uint32_t N = (uint32_t)round_up(n, 64);  // the planners' padded width
    stats_ = std::make_unique<PolicyStatsRun>(m, n, k, N, work_);
    order(work_, up_);  // the allocations before the first copy
    double* db = db_->as<double>();
    double* da = da_->as<double>();
    // both operands in blocks of columns (2-D copies of all rows; blocks of at least 512 columns keep them
    // at full speed), B first
    const uint64_t cols_b = std::min<uint64_t>(n, std::max<uint64_t>(512, kUploadChunkBytes / (8 * k)));
    for (uint64_t c0 = 0; c0 < n; c0 += cols_b) {
        const uint64_t w = std::min(cols_b, n - c0);
        OZTT_CUDA(cudaMemcpy2DAsync(db + c0, n * 8, b_ + c0, n * 8, w * 8, k, cudaMemcpyHostToDevice, up_));
        order(up_, work_);
        stats_->b_cols(db, c0, c0 + w);
    }
    stats_->b_done(db);
    const uint64_t cols_a = std::min<uint64_t>(k, std::max<uint64_t>(512, kUploadChunkBytes / (8 * m)));
    cudaEvent_t uploaded = nullptr;
    for (uint64_t c0 = 0; c0 < k; c0 += cols_a) {
        const uint64_t w = std::min(cols_a, k - c0);
        OZTT_CUDA(cudaMemcpy2DAsync(da + c0, k * 8, a_ + c0, k * 8, w * 8, m, cudaMemcpyHostToDevice, up_));
        uploaded = order(up_, work_);
        stats_->a_cols(da, c0, c0 + w);
    }
    stats_->a_done(da);
    OZTT_CUDA(cudaEventSynchronize(uploaded));
    phases_.upload_ms = ms_since_start();
    const PolicyStats ps = stats_->collect(&row_max, &col_max, row_sumsq, col_sumsq, rg);
    phases_.stats_ms = ms_since_start() - phases_.upload_ms;
    return ps;
}

std::vector<cudaEvent_t> StreamedCall::upload_prefix_first(uint64_t pre_rows, uint64_t band_rows, uint64_t block_cols,
                                                           uint64_t mid_blocks, uint64_t mid_rows,
                                                           std::vector<cudaEvent_t>& b_landed) {
    const uint64_t N = round_up(n_, 64);  // the planners' padded width
    double* da = da_->as<double>();
    double* db = db_->as<double>();
    int lo = 0, hi = 0;
    OZTT_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
    OZTT_CUDA(cudaStreamCreateWithPriority(&cert_, cudaStreamNonBlocking, hi));
    OZTT_CUDA(cudaStreamCreateWithPriority(&est_, cudaStreamNonBlocking, hi));
    order(work_, cert_);  // the operand buffers before the measurement buffers
    cert_buf_ = std::make_unique<DevBuf>(cert_, m_ * kCertWidth * 8);
    bparts_ = std::make_unique<DevBuf>(cert_, (k_ * kBCertWidth + n_ + 1 + 8 * k_ + k_ + 8 * N) * 8);
    cert_flags_ = std::make_unique<DevBuf>(cert_, 16);
    // the probe vectors (1 MiB) first, while the copy engine is idle; then A's first part at once
    const std::vector<double> g = policy_vectors_host((uint32_t)N);
    OZTT_CUDA(cudaMemcpyAsync(b_probe(), g.data(), g.size() * 8, cudaMemcpyHostToDevice, cert_));
    OZTT_CUDA(cudaStreamSynchronize(cert_));  // the probe vectors leave the host vector
    g_ready_ = mark(cert_);
    order(work_, up_);
    OZTT_CUDA(cudaEventCreate(&tl_start_));
    OZTT_CUDA(cudaEventRecord(tl_start_, up_));
    est_run_ = std::make_unique<PrefixEstimate>(pre_rows, k_, std::min(block_cols, n_), est_);
    OZTT_CUDA(cudaStreamWaitEvent(est_, g_ready_, 0));
    OZTT_CUDA(cudaMemsetAsync(cert_flags_->p, 0, 16, cert_));
    OZTT_CUDA(cudaMemsetAsync(bparts_->p, 0, (k_ * kBCertWidth + n_) * 8, cert_));  // accumulators, maxima
    order(cert_, up_);
    // B's blocks, each measured as it lands (its columns' maxima exactly, its rows' partial sketch sums
    // bounded); the first block also for the first plan's estimate
    b_landed.clear();
    const auto b_block = [&](uint64_t c0) {
        const uint64_t w = std::min(block_cols, n_ - c0);
        OZTT_CUDA(cudaMemcpy2DAsync(db + c0, n_ * 8, b_ + c0, n_ * 8, w * 8, k_, cudaMemcpyHostToDevice, up_));
        b_landed.push_back(order(up_, cert_));
        launch_col_absmax(db + c0, k_, w, n_, b_colmax() + c0, cert_);
        launch_bcert_block(db + c0, k_, w, n_, b_probe() + c0, N, b_acc(), cert_flags_->as<uint32_t>() + 1, cert_);
    };
    b_block(0);
    OZTT_CUDA(cudaStreamWaitEvent(est_, b_landed[0], 0));
    est_run_->b_block(db, n_, b_probe(), N);
    // A's first part, each band measured for the estimate as it lands
    std::vector<cudaEvent_t> landed;
    const auto a_band = [&](uint64_t r0) {
        const uint64_t rows = std::min(band_rows, m_ - r0);
        OZTT_CUDA(cudaMemcpyAsync(da + r0 * k_, a_ + r0 * k_, rows * k_ * 8, cudaMemcpyHostToDevice, up_));
        landed.push_back(mark(up_));
        return rows;
    };
    for (uint64_t r0 = 0; r0 < pre_rows; r0 += band_rows) {
        const uint64_t rows = a_band(r0);
        OZTT_CUDA(cudaStreamWaitEvent(est_, landed.back(), 0));
        est_run_->a_band(da, r0, std::min(rows, pre_rows - r0));
    }
    // B's next blocks, A's next bands, B's other blocks, the rest of A
    const uint64_t mid_end = std::min(m_, pre_rows + mid_rows);
    uint64_t c0 = block_cols;
    for (uint64_t j = 0; j < mid_blocks && c0 < n_; ++j, c0 += block_cols) b_block(c0);
    uint64_t r0 = pre_rows;
    for (; r0 < mid_end; r0 += band_rows) a_band(r0);
    for (; c0 < n_; c0 += block_cols) b_block(c0);
    launch_bcert_finish(b_colmax(), n_, b_acc(), k_, bcert_error_factor(n_), b_rg(), b_y(), b_ew(), cert_);
    // A's rows that landed before B's last block (r0 steps by whole bands, past m after a short last one)
    const uint64_t early_rows = std::min(r0, m_), early_bands = landed.size();
    for (; r0 < m_; r0 += band_rows) a_band(r0);
    // the bands' bounded statistics need B's sketch: those that landed before B's last block in one pass (all
    // the rows at once keep every SM busy), each later one after it lands
    if (early_rows) {
        OZTT_CUDA(cudaStreamWaitEvent(cert_, landed[early_bands - 1], 0));
        launch_band_certify(da, early_rows, k_, b_y(), b_ew(), cert_buf_->as<double>(), cert_flags_->as<uint32_t>(),
                            cert_);
    }
    for (uint64_t r0 = early_rows, i = early_bands; r0 < m_; r0 += band_rows, ++i) {
        const uint64_t rows = std::min(band_rows, m_ - r0);
        OZTT_CUDA(cudaStreamWaitEvent(cert_, landed[i], 0));
        launch_band_certify(da + r0 * k_, rows, k_, b_y(), b_ew(), cert_buf_->as<double>() + r0 * kCertWidth,
                            cert_flags_->as<uint32_t>(), cert_);
    }
    timeline(cert_, 3);
    // the measurements come back to the host as soon as they are written, ahead of C's read-back in the
    // copy engine (pinned memory, so that the copies are queued now and the host does not wait for them)
    const uint64_t words = m_ * kCertWidth + k_ * kBCertWidth + n_ + 2;
    stage_ = acquire_stage(words * 8, stage_shared_);
    OZTT_CUDA(cudaMemcpyAsync(stage_, cert_buf_->p, m_ * kCertWidth * 8, cudaMemcpyDeviceToHost, cert_));
    OZTT_CUDA(cudaMemcpyAsync(stage_ + m_ * kCertWidth, b_acc(), (k_ * kBCertWidth + n_ + 1) * 8,
                              cudaMemcpyDeviceToHost, cert_));  // accumulators, column maxima, scale
    OZTT_CUDA(cudaMemcpyAsync(stage_ + words - 1, cert_flags_->p, 8, cudaMemcpyDeviceToHost, cert_));
    a_last_ = landed.back();
    b_last_ = b_landed.back();
    return landed;
}

PolicyStats StreamedCall::prefix_estimate(bool& ok, std::vector<uint64_t>* row_max) {
    return est_run_->finish(ok, row_max);
}

PolicyBounds StreamedCall::certified_bounds() {
    OZTT_CUDA(cudaEventSynchronize(a_last_));
    phases_.upload_ms = ms_since_start();
    OZTT_CUDA(cudaStreamSynchronize(cert_));  // the measurements, copied to stage_ as they were written
    const double* cert = stage_;
    const double* acc = stage_ + m_ * kCertWidth;
    const double* col_max = acc + k_ * kBCertWidth;  // magnitude patterns, which order like the magnitudes
    const double rgB = col_max[n_];
    uint32_t flags[2];
    std::memcpy(flags, col_max + n_ + 1, 8);
    double nb_lo = 0, nb_hi = 0;
    bounded_nb(acc, k_, n_, rgB, nb_lo, nb_hi);
    PolicyBounds pb = certified_policy_bounds(cert, m_, k_, col_max, n_, nb_lo, nb_hi, rgB);
    if (flags[0] || flags[1]) pb.usable = false;  // elements below 2^-383: the bounds do not hold
    phases_.stats_ms = ms_since_start() - phases_.upload_ms;
    return pb;
}

PolicyStats StreamedCall::exact_stats() {
    // the reference's sequential sums over the whole A and B, for the rare call whose bounds leave a
    // decision open
    const double* da = da_->as<double>();
    const double* db = db_->as<double>();
    if (!stat_) OZTT_CUDA(cudaStreamCreateWithFlags(&stat_, cudaStreamNonBlocking));
    OZTT_CUDA(cudaStreamWaitEvent(stat_, a_last_, 0));
    OZTT_CUDA(cudaStreamWaitEvent(stat_, b_last_, 0));
    stats_ = std::make_unique<PolicyStatsRun>(m_, n_, k_, (uint32_t)round_up(n_, 64), stat_);
    stats_->b_cols(db, 0, n_);
    stats_->b_done(db);
    stats_->a_cols(da, 0, k_);
    stats_->a_done(da);
    const PolicyStats ps = stats_->collect();
    phases_.exact_stats = 1;
    return ps;
}

double* StreamedCall::c_dev() {
    if (!dc_) dc_ = std::make_unique<DevBuf>(work_, m_ * n_ * 8);
    return dc_->as<double>();
}

void StreamedCall::band_done(uint64_t r0, uint64_t rows) { bands_.push_back({r0, rows, 0, n_, mark(work_)}); }

void StreamedCall::tile_done(uint64_t r0, uint64_t rows, uint64_t c0, uint64_t cols) {
    bands_.push_back({r0, rows, c0, cols, mark(work_)});
}

void StreamedCall::timeline(cudaStream_t s, int slot) {
    if (!tl_start_ || slot < 0 || slot > 3) return;
    if (!tl_[slot]) OZTT_CUDA(cudaEventCreate(&tl_[slot]));
    OZTT_CUDA(cudaEventRecord(tl_[slot], s));
}

void StreamedCall::read_back(double* c) {
    // all bands are queued before the first read-back is issued: a read-back into pageable memory
    // returns only when it is done, and the GPU keeps computing meanwhile
    const double* dc = c_dev();
    for (const Band& band : bands_) {
        OZTT_CUDA(cudaStreamWaitEvent(down_, band.done, 0));
        if (band.c0 == 0 && band.cols == n_)
            OZTT_CUDA(cudaMemcpyAsync(c + band.r0 * n_, dc + band.r0 * n_, band.rows * n_ * 8,
                                      cudaMemcpyDeviceToHost, down_));
        else
            OZTT_CUDA(cudaMemcpy2DAsync(c + band.r0 * n_ + band.c0, n_ * 8, dc + band.r0 * n_ + band.c0, n_ * 8,
                                        band.cols * 8, band.rows, cudaMemcpyDeviceToHost, down_));
    }
    timeline(down_, 2);
    order(down_, work_);
}

void StreamedCall::finish(double pipeline_start_ms) {
    OZTT_CUDA(cudaStreamSynchronize(work_));
    phases_.total_ms = ms_since_start();
    double* gpu[4] = {&phases_.gpu_prefix_ms, &phases_.gpu_compute_ms, &phases_.gpu_readback_ms,
                      &phases_.gpu_bounds_ms};
    for (int i = 0; i < 4; ++i) {
        float ms = 0;
        if (tl_start_ && tl_[i] && cudaEventElapsedTime(&ms, tl_start_, tl_[i]) == cudaSuccess) *gpu[i] = ms;
    }
    phases_.pipeline_ms = phases_.total_ms - pipeline_start_ms;
    phases_.bands = (int)bands_.size();
    std::lock_guard<std::mutex> lock(g_phases_mu);
    g_last_phases = phases_;
}

}  // namespace oztt
