// SPDX-License-Identifier: Apache-2.0
// Host-side helpers shared by the pipelines: device selection, stream-ordered scratch buffers and
// the read-back checks of the range flags and the GEMM wait-timeout word.
#pragma once
#include <algorithm>
#include <chrono>
#include <functional>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "oztt_common.cuh"
#include "planner.hpp"

namespace oztt {

// Selects the device, checks that it is a B200-class GPU (compute capability 10.0) and keeps the
// stream-ordered pool's memory between calls.
void open_device(int device_id);
// Throws runtime_error for a GEMM wait timeout or for range flags of the scaling stage.
void check_flags(uint32_t flags, int gemm_err);

// Stream-ordered device buffer, released on the stream when it goes out of scope.
struct DevBuf {
    void* p = nullptr;
    cudaStream_t st;
    explicit DevBuf(cudaStream_t s) : st(s) {}
    DevBuf(cudaStream_t s, size_t bytes) : st(s) { alloc(bytes); }
    ~DevBuf() {
        if (p) cudaFreeAsync(p, st);
    }
    void alloc(size_t bytes) {
        const cudaError_t e = cudaMallocAsync(&p, std::max<size_t>(bytes, 256), st);
        if (e != cudaSuccess) {
            cudaGetLastError();
            p = nullptr;
            throw Error(OZTT_ERUNTIME, "device memory allocation of " + std::to_string(bytes) +
                                           " bytes failed: " + cudaGetErrorString(e));
        }
    }
    template <class T>
    T* as() const {
        return reinterpret_cast<T*>(p);
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
};

// One device pipeline as an ordered list of launches on one stream. Each launch belongs to a stage of
// the evaluator hooks (include/evaluation_hooks.hpp: kScale .. kRecon), is a kind of device step
// (kHead .. kComposeStep) and fills one slot of the caller's per-stage timings; consecutive launches
// of one stage form one timed phase unless a launch opens a new one.
enum EvStage { kScale = 0, kSlice = 1, kGemm = 2, kCompose = 3, kRecon = 4 };
enum EvStep { kHead = 0, kGemmStep = 1, kReconStep = 2, kComposeStep = 3 };

struct Pipeline {
    struct Launch {
        int stage, step, slot, phase;
        std::function<void()> issue;
    };
    std::vector<Launch> launches;
    std::vector<std::pair<void*, size_t>> written;  // buffers the pass writes (whole-pass sentinel fill)
    void* out = nullptr;                            // the output the whole-pass check compares
    size_t out_bytes = 0;
    unsigned partial_products = 0;                  // products the GEMM stage forms
    void add(int stage, int step, int slot, std::function<void()> issue, bool new_phase = false) {
        const bool next = launches.empty() || new_phase || launches.back().stage != stage;
        const int phase = launches.empty() ? 0 : launches.back().phase + (next ? 1 : 0);
        launches.push_back({stage, step, slot, phase, std::move(issue)});
    }
    void writes(void* p, size_t bytes) { written.push_back({p, bytes}); }
    // Issues every launch in order; stage_ms (optional, `slots` entries) receives the device time of
    // each slot from CUDA events recorded between them.
    void run(cudaStream_t st, double* stage_ms = nullptr, int slots = 0) const;
};

// Under an evaluation Scope open on this thread (evaluation_hooks.hpp): runs the pipeline with the
// evaluator's phase timing and, when asked, its whole-pass check and timing, and reports the GEMM's
// partial products and grid; returns false, running nothing, when no Scope is open.
bool run_profiled(const Pipeline& pl, cudaStream_t st);
// The scaled-integer width of Ozaki II that the open Scope fixes (0: none, or no Scope).
unsigned evaluation_fixed_bits();
// True while a Scope is open on this thread.
bool evaluation_active();

struct PolicyStats;

// The input statistics of the Scheme II precision policy measured on the device in stages: B's blocks,
// then B's own stages, then A's blocks, then A's; collect() reads back (synchronising the stream) and
// finishes the reductions on the host in the reference's order. The result is bit-identical to the host
// measurement for the padded planning width N. Operands come in blocks of columns (all rows), B first and then A, so that every row's and column's
// sequential sums advance as each block lands and only the last block's share is left when the upload
// ends. The caller orders each block's arrival before st ahead of the block's call.
class PolicyStatsRun {
public:
    PolicyStatsRun(uint64_t m, uint64_t n, uint64_t k, uint32_t N, cudaStream_t st);
    ~PolicyStatsRun();
    // maxima, sums of squares and sketch over columns c0 .. c1-1 of B (b: the whole row-major B; blocks in
    // column order)
    void b_cols(const double* b, uint64_t c0, uint64_t c1);
    void b_done(const double* b);  // B's scale, then its sums and y = B g scaled
    // the same for columns c0 .. c1-1 of all rows of A (a: the whole row-major A), after b_done
    void a_cols(const double* a, uint64_t c0, uint64_t c1);
    // or for rows r0 .. r1-1 of A, whole rows (bands in any order, together covering every row), after b_done
    void a_rows(const double* a, uint64_t r0, uint64_t r1);
    void a_done(const double* a);
    // row_max / col_max, when given, receive the magnitude patterns of A's row and B's column maxima;
    // row_sumsq / col_sumsq the scaled squared norms of A's rows and B's columns; rg the scales of A and B
    PolicyStats collect(std::vector<uint64_t>* row_max = nullptr, std::vector<uint64_t>* col_max = nullptr,
                        std::vector<double>* row_sumsq = nullptr, std::vector<double>* col_sumsq = nullptr,
                        double* rg = nullptr);

private:
    struct Bufs;
    uint64_t m_, n_, k_;
    uint32_t N_;
    cudaStream_t st_;
    cudaStream_t cols_st_ = nullptr;  // B's per-column stages, rejoined into st by b_done
    cudaEvent_t landed_ = nullptr, cols_done_ = nullptr;
    int sms_ = 148;
    std::unique_ptr<Bufs> bufs_;
    std::shared_ptr<const std::vector<double>> g_;
};

// The first plan's estimate of the policy statistics from A's first rows_a rows and B's first cols_b columns,
// in steps that follow the upload on stream st (stats.cu).
class PrefixEstimate {
public:
    PrefixEstimate(uint64_t rows_a, uint64_t k, uint64_t cols_b, cudaStream_t st);
    // B's first block (rows ldb apart) with the probe vectors g (8 rows gstride apart), once it has landed
    void b_block(const double* b, uint64_t ldb, const double* g, uint64_t gstride);
    // rows r0 .. r0+rows-1 of A (the whole row-major A), after b_block, once they have landed
    void a_band(const double* a, uint64_t r0, uint64_t rows);
    // waits for the steps; ok is false when no estimate could be made; row_max receives the magnitude
    // patterns of the maxima of A's rows_a rows
    PolicyStats finish(bool& ok, std::vector<uint64_t>* row_max);

private:
    uint64_t rows_a_, k_, cols_b_;
    cudaStream_t st_;
    DevBuf cmax_, y_, sq_, cert_, flags_;
};

class StreamedCall {
public:
    StreamedCall(int device_id, const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k);
    ~StreamedCall();
    // B, then A, in blocks of columns, with the statistics measured as they land;
    // returns them, with the magnitude patterns of A's row maxima and B's column maxima (and, when asked,
    // the scaled squared norms of A's rows and B's columns and the two scales).
    PolicyStats upload(std::vector<uint64_t>& row_max, std::vector<uint64_t>& col_max,
                       std::vector<double>* row_sumsq = nullptr, std::vector<double>* col_sumsq = nullptr,
                       double* rg = nullptr);
    const double* a_dev() const { return da_->as<double>(); }
    const double* b_dev() const { return db_->as<double>(); }
    double* c_dev();
    cudaStream_t work() const { return work_; }
    // rows [r0, r0 + rows) of the device C are complete once the work issued so far has run
    void band_done(uint64_t r0, uint64_t rows);
    // the same for the tile of rows [r0, r0 + rows) and columns [c0, c0 + cols)
    void tile_done(uint64_t r0, uint64_t rows, uint64_t c0, uint64_t cols);
    // issues the read-back of every completed band into c, in order
    void read_back(double* c);
    // waits for everything (the read-back included) and records the phases of the call, the pipeline
    // counted from pipeline_start_ms (ms_since_start when it was issued)
    void finish(double pipeline_start_ms);
    // The upload of the INT8 path that computes while its operands land: B's first block of block_cols
    // columns, A's first pre_rows rows in bands of band_rows, B's next mid_blocks blocks, A's next mid_rows
    // rows, B's other blocks, then the rest of A in bands (B's first block first, so that the first plan's
    // estimate follows A's bands as they land). Each block of B is measured as it lands and each band of A
    // once B has landed (one fast pass each that bounds the reference's statistics, on a high-priority
    // stream, so that it runs between the GEMM's launches). Returns the events that mark each band's arrival
    // and fills b_landed with those of B's blocks.
    std::vector<cudaEvent_t> upload_prefix_first(uint64_t pre_rows, uint64_t band_rows, uint64_t block_cols,
                                                 uint64_t mid_blocks, uint64_t mid_rows,
                                                 std::vector<cudaEvent_t>& b_landed);
    // After upload_prefix_first: the estimate of the statistics from A's first pre_rows rows and B's first
    // block (PrefixEstimate, measured as they landed); waits for it. ok is false when no estimate could be
    // made; row_max receives the magnitude patterns of those rows' maxima.
    PolicyStats prefix_estimate(bool& ok, std::vector<uint64_t>* row_max);
    // After upload_prefix_first: bounds of the statistics that contain the reference's values. Waits for
    // every band's measurements.
    PolicyBounds certified_bounds();
    // The reference's exact statistics of the whole A and B (its sequential long-double sums), for the rare
    // call whose bounds leave a decision open.
    PolicyStats exact_stats();
    // forgets the bands marked so far (their C is recomputed)
    void discard_bands() { bands_.clear(); }
    // The device timeline of the computing-while-uploading path: slot 0 when A's first part has met every
    // block of B, slot 1 when the last band's reconstruction has run (marked on stream s), slot 2 when the
    // last read-back of C has ended, slot 3 when the bounded statistics of the last band are written;
    // finish() reports them in milliseconds from the call's first copy.
    void timeline(cudaStream_t s, int slot);
    StreamedPhases& phases() { return phases_; }
    double ms_since_start() const;
    StreamedCall(const StreamedCall&) = delete;
    StreamedCall& operator=(const StreamedCall&) = delete;

private:
    cudaEvent_t mark(cudaStream_t s);
    cudaEvent_t order(cudaStream_t from, cudaStream_t to);
    struct Band {
        uint64_t r0, rows, c0, cols;  // a tile of C: rows r0.., columns c0.. (cols = n: whole rows)
        cudaEvent_t done;
    };
    const double *a_, *b_;
    uint64_t m_, n_, k_;
    std::chrono::steady_clock::time_point t0_;
    cudaStream_t work_ = nullptr, up_ = nullptr, down_ = nullptr, stat_ = nullptr, cert_ = nullptr, est_ = nullptr;
    cudaEvent_t a_last_ = nullptr, b_last_ = nullptr, g_ready_ = nullptr;
    std::unique_ptr<DevBuf> cert_buf_, cert_flags_;
    // B's bounded measurements (upload_prefix_first): per row of B 17 accumulators, the column maxima (n
    // patterns), the scale, the scaled sketch (8 x k), its error bounds (k), the probe vectors (8 x N)
    std::unique_ptr<DevBuf> bparts_;
    std::unique_ptr<PrefixEstimate> est_run_;
    double* stage_ = nullptr;  // pinned: the measurements of A's bands and B, copied back as they are written
    bool stage_shared_ = false;
    double* b_acc() const { return bparts_->as<double>(); }
    unsigned long long* b_colmax() const { return reinterpret_cast<unsigned long long*>(b_acc() + k_ * 17); }
    double* b_rg() const { return b_acc() + k_ * 17 + n_; }
    double* b_y() const { return b_rg() + 1; }
    double* b_ew() const { return b_y() + 8 * k_; }
    double* b_probe() const { return b_ew() + k_; }
    std::vector<cudaEvent_t> events_;
    cudaEvent_t tl_start_ = nullptr, tl_[4] = {nullptr, nullptr, nullptr, nullptr};
    std::vector<Band> bands_;
    std::unique_ptr<DevBuf> da_, db_, dc_;
    std::unique_ptr<PolicyStatsRun> stats_;
    StreamedPhases phases_;
};

}  // namespace oztt
