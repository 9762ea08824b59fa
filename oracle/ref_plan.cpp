// TEST INFRASTRUCTURE — checker only, never shipped.
//
// Compiles the reference's own Scheme II planner headers in place (src/backend/ozaki2/
// auto_precision.hpp, which includes moduli.hpp, split.hpp, awe.hpp, format.hpp and
// common/norm_estimate.hpp) with the tt-metal name stub in ref_shim/, and exposes them through
// a C ABI so the tests can compare the project's planner and the oracle's restatement with the
// reference's decisions. The glue below restates the few lines of choose_moduli_and_width
// (src/backend/ozaki2/plan.hpp:258-306), whose header cannot be included without TT-Metalium.
// Built by oracle/Makefile (target ref) into oracle/_ref/; see that file for the command.
#include "oz2_oracle.h"

#include <cstring>
#include <vector>

#include "ozaki2/auto_precision.hpp"

namespace rp = ozTTgemm::detail::ozaki2_x;

namespace {
void fill(const rp::Ozaki2Moduli& mo, ozo_plan* out) {
    out->ok = mo.ok;
    out->acc_ok = mo.acc_ok;
    out->S = mo.s;
    out->b = mo.b;
    out->m_cap = mo.m_cap;
    out->ncand = mo.ncand;
    for (int i = 0; i < mo.s && i < OZO_MAXS; ++i) {
        out->m[i] = mo.m[i];
        out->yi[i] = mo.yi[i];
        out->rinv[i] = mo.rinv[i];
        out->c[0][i] = mo.c0[i];
        out->c[1][i] = mo.c1[i];
        out->c[2][i] = mo.c2[i];
        out->c[3][i] = mo.c3[i];
        out->m16[i] = mo.m16[i];
        for (int t = 0; t < OZ2_NRP0; ++t) out->rp0[i][t] = mo.rp0[i][t];
        for (int t = 0; t < OZ2_NRP1; ++t) out->rp1[i][t] = mo.rp1[i][t];
        for (int t = 0; t < OZ2_NRP2; ++t) out->rp2[i][t] = mo.rp2[i][t];
    }
    auto packed = [&](auto& src, int nrp) {
        std::vector<float> v((size_t)mo.s * nrp);
        for (int i = 0; i < mo.s; ++i)
            for (int t = 0; t < nrp; ++t) v[(size_t)i * nrp + t] = src[i][t];
        return v;
    };
    const auto p0 = packed(mo.rp0, OZ2_NRP0), p1 = packed(mo.rp1, OZ2_NRP1), p2 = packed(mo.rp2, OZ2_NRP2);
    out->nsmall0 = (int)rp::oz2_choose_small_tail(p0.data(), OZ2_NRP0, mo.m.data(), (uint32_t)mo.s);
    out->nsmall1 = (int)rp::oz2_choose_small_tail(p1.data(), OZ2_NRP1, mo.m.data(), (uint32_t)mo.s);
    out->nsmall2 = (int)rp::oz2_choose_small_tail(p2.data(), OZ2_NRP2, mo.m.data(), (uint32_t)mo.s);
    const rp::OzScale64 w = rp::oz_split_scale_ld(mo.KMl);
    out->W_hi = w.hi;
    out->W_lo = w.lo;
    out->qw = w.q;
    out->nd = (mo.b > 4 * OZ2_DIGIT_BITS) ? 5 : ((mo.b > 3 * OZ2_DIGIT_BITS) ? 4 : 3);
    out->shift = mo.b - (out->nd - 1) * OZ2_DIGIT_BITS;
    double l = 0;
    for (int mm : mo.m) l += std::log2((double)mm);
    out->logM = l;
}
}  // namespace

extern "C" {

int ozr_choose_moduli(uint32_t M, uint32_t N, uint32_t K, int num_moduli, int b_cap, ozo_plan* out) {
    std::memset(out, 0, sizeof(*out));
    fill(rp::ozaki2_choose_moduli(M, N, K, num_moduli, b_cap), out);
    out->b_cap = b_cap;
    out->S_req = num_moduli;
    return 0;
}

// choose_moduli_and_width for padded row-major A (M x K) and B (K x N). Returns 1 where the
// reference throws (oz2_report_moduli_failure, oz2_check_width).
int ozr_plan(const double* a, const double* b, uint32_t M, uint32_t N, uint32_t K, uint32_t max_moduli, int passes,
             int fixed_bits, ozo_plan* out) {
    std::memset(out, 0, sizeof(*out));
    const std::vector<double> A(a, a + (size_t)M * K), B(b, b + (size_t)K * N);
    const bool b_fixed = fixed_bits > 0;
    rp::Oz2PrecisionPolicy pol;
    int b_cap = rp::OZ2_B_DEFAULT;
    if (b_fixed)
        b_cap = fixed_bits;
    else {
        pol = rp::choose_precision_policy(A, B, M, N, K);
        b_cap = pol.b_cap;
    }
    const uint32_t S_req = max_moduli ? max_moduli : (b_fixed ? rp::OZ2_PARAM.def_s : (uint32_t)OZ2_MAXS);
    if (b_fixed && passes == 0) rp::oz2_measure_stats(A, B, M, N, K, pol);
    const rp::Ozaki2Moduli mo = rp::ozaki2_choose_moduli(M, N, K, (int)S_req, b_cap);
    fill(mo, out);
    out->b_cap = b_cap;
    out->S_req = (int)S_req;
    out->TA = pol.st.TA;
    out->TB = pol.st.TB;
    out->nA = pol.st.nA;
    out->nB = pol.st.nB;
    out->nC = pol.nC;
    if (!mo.ok) return 1;
    if (!b_fixed && mo.b < rp::OZ2_TARGET_BITS) return 1;
    const double r1 = rp::oz2_recon1_log2(mo, mo.b, pol);
    out->recon1_log2 = r1;
    out->two_pass = passes != 0 ? (passes == 2) : !(r1 <= rp::OZ2_RECON1_THR_LOG2);
    return 0;
}

}  // extern "C"
