// TEST INFRASTRUCTURE — checker only, never shipped.
//
// Compiles the reference's Scheme II planner headers in place for one digit format (-DOZ_FMT_FP8,
// -DOZ_FMT_BF16, -DOZ_FMT_FP16 or -DOZ_FMT_FP32: the route of src/backend/ozaki2/split.hpp, the moduli
// selection of moduli.hpp with the stage-time model of awe.hpp, the precision policy of
// auto_precision.hpp) with the TT-Metalium name stub of ref_shim/, and fills the project's plan
// structure (include/oztt_cuda.h) from its decisions, so that tests can compare the product's digit
// planner field by field. The glue restates the few lines of choose_moduli_and_width
// (src/backend/ozaki2/plan.hpp:258-306), whose header cannot be included without TT-Metalium.
#include <cstring>
#include <vector>

#include "oztt_cuda.h"
#include "ozaki2/auto_precision.hpp"

namespace rp = ozTTgemm::detail::OZTTGEMM_BACKEND_NS;

#if defined(OZ_FMT_FP8)
constexpr int32_t kFormat = OZTT_FMT_FP8;
#elif defined(OZ_FMT_BF16)
constexpr int32_t kFormat = OZTT_FMT_BF16;
#elif defined(OZ_FMT_FP16)
constexpr int32_t kFormat = OZTT_FMT_FP16;
#else
constexpr int32_t kFormat = OZTT_FMT_TF32;
#endif

namespace {
void fill(const rp::Ozaki2Moduli& mo, oztt_digit_plan* out) {
    oztt_ii_plan& b = out->base;
    out->format = kFormat;
    b.S = mo.s;
    b.b = mo.b;
    out->nplane = mo.nplane;
    out->nprod = mo.nprod;
    out->nout = mo.nout;
    out->fold_first = mo.fold_first ? 1 : 0;
    int o = 0;
    for (int i = 0; i < mo.s && i < OZTT_MAXS; ++i) {
        b.moduli[i] = mo.m[i];
        b.yi[i] = mo.yi[i];
        b.rinv[i] = mo.rinv[i];
        b.c[0][i] = mo.c0[i];
        b.c[1][i] = mo.c1[i];
        b.c[2][i] = mo.c2[i];
        b.c[3][i] = mo.c3[i];
        out->q[i] = mo.q[i];
        out->mode[i] = mo.mode[i];
        out->poff[i] = mo.poff[i];
        const int np = rp::oz2_digit_planes(mo.m[i], rp::OZ2_PARAM.digit_bound, rp::OZ2_PARAM.nd());
        out->npl[i] = np;
        out->oout[i] = o;
        rp::Oz2ProductGroup gr[OZ2_MAXPROD];
        const uint32_t ng =
            rp::oz2_product_groups(mo.m[i], gr, rp::OZ2_PARAM.digit_bound, rp::OZ2_PARAM.nd(), mo.maxg_m[i]);
        for (uint32_t j = 0; j < ng && o < OZTT_MAXOUT; ++j, ++o) {
            out->out_a[o] = mo.poff[i] + gr[j].a0;
            out->out_b[o] = mo.poff[i] + (np - 1 - gr[j].b0);
            out->out_g[o] = gr[j].g;
            out->out_mod[o] = i;
            out->coeff[o] = (int32_t)gr[j].coeff_lo;
        }
    }
    out->oout[mo.s] = o;
}
}  // namespace

extern "C" {

// The moduli selection alone for output dimensions M x N (the stage-time model's DRAM estimate reads
// them); returns ok (and acc_ok in *acc).
int ozr_digit_choose(uint32_t M, uint32_t N, uint32_t K, int num_moduli, int b_cap, oztt_digit_plan* out, int* acc) {
    std::memset(out, 0, sizeof(*out));
    const rp::Ozaki2Moduli mo = rp::ozaki2_choose_moduli(M, N, K, num_moduli, b_cap);
    fill(mo, out);
    *acc = mo.acc_ok ? 1 : 0;
    return mo.ok ? 1 : 0;
}

// choose_moduli_and_width for padded row-major A (M x K) and B (K x N) with the format's route. Returns 1
// where the reference throws.
int ozr_digit_plan(const double* a, const double* b, uint32_t M, uint32_t N, uint32_t K, uint32_t max_moduli,
                int passes, int fixed_bits, oztt_digit_plan* out) {
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
    oztt_ii_plan& p = out->base;
    p.M = M;
    p.N = N;
    p.K = K;
    p.b_cap = b_cap;
    p.S_req = (int32_t)S_req;
    p.TA = pol.st.TA;
    p.TB = pol.st.TB;
    p.nA = pol.st.nA;
    p.nB = pol.st.nB;
    p.nC = pol.nC;
    if (!mo.ok) return 1;
    if (!b_fixed && mo.b < rp::OZ2_TARGET_BITS) return 1;
    p.recon1_log2 = rp::oz2_recon1_log2(mo, mo.b, pol);
    p.two_pass = passes != 0 ? (passes == 2) : !(p.recon1_log2 <= rp::OZ2_RECON1_THR_LOG2);
    p.nd = (mo.b > 4 * OZ2_DIGIT_BITS) ? 5 : ((mo.b > 3 * OZ2_DIGIT_BITS) ? 4 : 3);
    p.shift = mo.b - (p.nd - 1) * OZ2_DIGIT_BITS;
    return 0;
}

}  // extern "C"
