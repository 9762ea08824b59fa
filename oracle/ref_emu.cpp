// TEST INFRASTRUCTURE — checker only, never shipped.
//
// Composes the reference's own host-side device emulation, compiled in place from the
// reference's experiments tree, into the Scheme II INT8 pipeline:
//   scale      common/kernels/scale_bits.h (oz_absf64_to_bf16<1>, oz_bf16_scale_exp)
//   slice      checks/sfpu_tf_emu.hpp (Dst, load_f64, tfMulP2, ModRound) driven in the order of the
//              device kernel ozaki2/kernels/oz2_digits.h (digit loop and residue chain)
//   GEMM       exact 64-bit integer dot products, written back as sign-magnitude int32 words
//   recon      tools/oz_sim.h (make_recon_kernels, crt_element, crt_pack) and
//              common/kernels/f64_tf.h (assemble_frac_f64, a128_add_limbs, a128_frac_to_f64)
// with the moduli constants from the experiments planner (ozaki2/ozaki2_moduli.h,
// ozaki2_choose_moduli_route with OZ2_ROUTE_INT8). Only the element order, the integer GEMM and
// the loops are written here. Built by oracle/Makefile (target ref) into oracle/_ref/.
#include "oz2_oracle.h"

#include <cstring>
#include <vector>

#include "common/kernels/scale_bits.h"
#include "oz_sim.h"

namespace {
uint64_t bits64(double x) {
    uint64_t u;
    std::memcpy(&u, &x, 8);
    return u;
}
// Residues of one element: load_f64 + digit loop + residue chain (oz2_digits.h order).
void element_residues(const Ozaki2Moduli& mo, int nd, double x, int32_t d, int8_t* out, size_t stride) {
    using sfpu_emu::Dst;
    Dst D;
    sfpu_emu::load_f64(D, x, d);
    float dig[5];
    for (int i = 0; i < nd; ++i) {
        if (i > 0) sfpu_emu::tfMulP2(D, 1048576.0f);
        D.Cpy(0, 7);
        D.Rnd(7);
        dig[i] = D.r[7];
        D.Sub(0, 7, 0);
    }
    for (int s = 0; s < mo.s; ++s) {
        Dst R;
        const float m = (float)mo.m[s], ri = mo.rinv[s];
        R.r[2] = dig[nd - 1];
        R.r[7] = dig[nd - 2];
        R.r[1] = dig[nd - 3];
        R.r[0] = nd >= 4 ? dig[nd - 4] : 0.f;
        R.r[3] = nd >= 5 ? dig[nd - 5] : 0.f;
        sfpu_emu::ModRound(R, 7, 4, m, ri);
        R.MulS(7, mo.c0[s]);
        R.Add(2, 7, 2);
        sfpu_emu::ModRound(R, 1, 4, m, ri);
        R.MulS(1, mo.c1[s]);
        R.Add(2, 1, 2);
        if (nd >= 4) {
            sfpu_emu::ModRound(R, 2, 4, m, ri);
            if (nd >= 5) {
                sfpu_emu::ModRound(R, 3, 4, m, ri);
                R.MulS(3, mo.c3[s]);
                R.Add(2, 3, 2);
                sfpu_emu::ModRound(R, 2, 4, m, ri);
            }
            sfpu_emu::ModRound(R, 0, 4, m, ri);
            R.MulS(0, mo.c2[s]);
            R.Add(2, 0, 2);
        }
        sfpu_emu::ModRound(R, 2, 4, m, ri);
        out[(size_t)s * stride] = (int8_t)(int)R.r[2];
    }
}
}  // namespace

extern "C" {

// Whole pipeline for A (m x k) and B (k x n), both already padded by the caller (m, n multiples
// of 64, k of 32), with a fixed width b (the evaluator's fixed_bits) and num_moduli as the limit.
// C receives the reference-faithful FP64 result. Returns the number of moduli, or -1.
int ozr_emulate_int8(const double* a, const double* b, double* c, uint32_t m, uint32_t n, uint32_t k, int b_fixed,
                     int num_moduli, int two_pass, int32_t* moduli_out) {
    const Ozaki2Moduli mo = ozaki2_choose_moduli_route(k, OZ2_ROUTE_INT8, b_fixed, num_moduli);
    if (!mo.ok) return -1;
    const int nd = (mo.b > 80) ? 5 : ((mo.b > 60) ? 4 : 3);
    const int32_t shift = mo.b - 20 * (nd - 1);
    for (int s = 0; s < mo.s; ++s) moduli_out[s] = mo.m[s];
    // Scaling: maxima on the 63-bit patterns, BF16 rounded up, e = ceil(log2), delta = shift - e.
    std::vector<int32_t> dA(m), dB(n);
    uint32_t bad = 0;
    for (uint32_t i = 0; i < m; ++i) {
        uint64_t mx = 0;
        for (uint32_t l = 0; l < k; ++l) mx = std::max<uint64_t>(mx, bits64(a[(size_t)i * k + l]) & 0x7FFFFFFFFFFFFFFFull);
        dA[i] = shift - oz_bf16_scale_exp(oz_absf64_to_bf16<1>((uint32_t)(mx >> 32), (uint32_t)mx), bad);
    }
    for (uint32_t j = 0; j < n; ++j) {
        uint64_t mx = 0;
        for (uint32_t l = 0; l < k; ++l) mx = std::max<uint64_t>(mx, bits64(b[(size_t)l * n + j]) & 0x7FFFFFFFFFFFFFFFull);
        dB[j] = shift - oz_bf16_scale_exp(oz_absf64_to_bf16<1>((uint32_t)(mx >> 32), (uint32_t)mx), bad);
    }
    if (bad) return -1;
    const size_t S = (size_t)mo.s;
    std::vector<int8_t> ra(S * m * k), rb(S * n * k);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)m; ++i)
        for (uint32_t l = 0; l < k; ++l)
            element_residues(mo, nd, a[(size_t)i * k + l], dA[i], ra.data() + (size_t)i * k + l, (size_t)m * k);
#pragma omp parallel for schedule(static)
    for (int64_t l = 0; l < (int64_t)k; ++l)
        for (uint32_t j = 0; j < n; ++j)
            element_residues(mo, nd, b[(size_t)l * n + j], dB[j], rb.data() + (size_t)j * k + l, (size_t)n * k);
    const oz_sim::ReconKernels kern = oz_sim::make_recon_kernels(mo, false);
    const OzScale64 w = oz_split_scale_ld(mo.KMl);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)m; ++i)
        for (uint32_t j = 0; j < n; ++j) {
            uint32_t raw[OZ2_MAXS];
            for (size_t s = 0; s < S; ++s) {
                const int8_t* ar = ra.data() + (s * m + (size_t)i) * k;
                const int8_t* br = rb.data() + (s * n + j) * k;
                int64_t acc = 0;
                for (uint32_t l = 0; l < k; ++l) acc += (int32_t)ar[l] * (int32_t)br[l];
                raw[s] = (acc < 0 ? 0x80000000u : 0u) | (uint32_t)(acc < 0 ? -acc : acc);
            }
            const int32_t g = 2 * shift - (dA[i] + dB[j]);
            uint64_t u;
            if (!two_pass) {
                sfpu_emu::Dst D;
                uint32_t limb[3];
                oz_sim::crt_element(D, kern.one, nullptr, raw);
                oz_sim::crt_pack(D, kern.one, limb);
                u = assemble_frac_f64(limb, 3u, g, w.hi, w.lo, w.q);
            } else {
                sfpu_emu::Dst D1, D2;
                uint32_t l1[3], l2[3];
                oz_sim::crt_element(D1, kern.first, nullptr, raw);
                oz_sim::crt_pack(D1, kern.first, l1);
                oz_sim::crt_element(D2, kern.second, nullptr, raw);
                oz_sim::crt_pack(D2, kern.second, l2);
                A128 acc{{0, 0, 0, 0}};
                a128_add_limbs(acc, l1, 3u);
                a128_add_limbs(acc, l2, 3u);
                u = a128_frac_to_f64(acc, g, w.hi, w.lo, w.q);
            }
            std::memcpy(&c[(size_t)i * n + j], &u, 8);
        }
    return mo.s;
}

}  // extern "C"
