// SPDX-License-Identifier: Apache-2.0
// Scheme II INT8 planner (host side); see planner.cpp.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "oztt_cuda.h"

namespace oztt {

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
double one_pass_error_log2(const std::vector<int>& mods, int b, const PolicyStats& st);
void fill_crt_constants(const std::vector<int>& mods, oztt_ii_plan& p);
// The whole plan; returns an OZTT_* code and a message.
int plan_ii_int8(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli,
                 int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan& p, std::string& err);

}  // namespace oztt
