// TEST INFRASTRUCTURE — the CPU baseline of bench.py, never part of the product.
//
// Compiles the reference's own host FP64 GEMM, paper_eval::reference_gemm (compensated Dot2,
// OpenMP, evaluation/numerics.hpp:58-93), in place from the reference tree, and times it on a sample
// of rows of C. Built by oracle/Makefile (target ref) with the reference evaluator's flags
// (-O3, no contraction, OpenMP) for the x86-64-v3 ISA.
#include <omp.h>

#include <cstdint>
#include <vector>

#include "evaluation/numerics.hpp"

namespace {
std::vector<double> g_a, g_b, g_hi, g_lo;
uint32_t g_rows = 0, g_n = 0, g_k = 0;
}  // namespace

extern "C" {

// Keeps copies of the first `rows` rows of A (rows x k) and of B (k x n) for ozr_dot2_run.
int ozr_dot2_prepare(const double* a, const double* b, uint32_t rows, uint32_t n, uint32_t k) {
    g_a.assign(a, a + (size_t)rows * k);
    g_b.assign(b, b + (size_t)k * n);
    g_rows = rows;
    g_n = n;
    g_k = k;
    return 0;
}

// Seconds of one reference_gemm over the prepared rows on `threads` OpenMP threads.
double ozr_dot2_run(int threads) {
    if (threads > 0) omp_set_num_threads(threads);
    const double t0 = omp_get_wtime();
    paper_eval::reference_gemm(g_a, g_b, g_rows, g_k, g_n, g_hi, g_lo);
    return omp_get_wtime() - t0;
}

// The prepared result (hi + lo as the reference's accuracy() combines them), for checking.
const double* ozr_dot2_hi() { return g_hi.data(); }
const double* ozr_dot2_lo() { return g_lo.data(); }

void ozr_dot2_release() {
    std::vector<double>().swap(g_a);
    std::vector<double>().swap(g_b);
    std::vector<double>().swap(g_hi);
    std::vector<double>().swap(g_lo);
}
}
