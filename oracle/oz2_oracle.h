// TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT.
//
// CPU oracle for the Ozaki-II INT8 path of mukunoki/ozTT (library ozTTgemm). Only tests/,
// __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg may load it, and only as
// the checker. Every function restates one piece of the reference algorithm in this project's
// own code; the file:line in each comment names the reference source it follows (paths are
// relative to the reference project root).
//
// Pinning: the composed pipeline (ozo_ii_int8_emulate) reproduces the reference device's
// published output hash fe063f5214e93e2e and relative Frobenius error 4.68753276457e-17 for
// n=128, seed 7, uniform(-1,1), b=54, one pass (tools/validated/quick.csv:13); the planner is
// cross-checked against the reference's own planner compiled in place (oracle/Makefile, target
// ref) over a case table (tests/golden/plan_cases.json).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "oztt_cuda.h"  // the plain C struct oztt_digit_plan (digit layout of one FP8 plan)

#ifdef __cplusplus
extern "C" {
#endif

#define OZO_MAXS 24
#define OZO_MAXRP 5

// Plan of one Scheme II INT8 call: what choose_moduli_and_width (src/backend/ozaki2/plan.hpp:258-306)
// and ozaki2_choose_moduli (src/backend/ozaki2/moduli.hpp:719-769) decide.
typedef struct ozo_plan {
    int32_t ok;          // a usable set was found (Ozaki2Moduli::ok)
    int32_t acc_ok;      // accumulation conditions hold (Ozaki2Moduli::acc_ok)
    int32_t S;           // number of moduli
    int32_t b;           // integer width
    int32_t nd;          // radix-2^20 digits of A' (3..5)
    int32_t shift;       // b - 20*(nd-1) (oz2_shift, plan.hpp:81)
    int32_t two_pass;    // reconstruction passes - 1
    int32_t b_cap;       // cap passed to the selection
    int32_t m_cap;       // modulus cap
    int32_t ncand;       // candidates before trimming
    int32_t S_req;       // limit on the number of moduli
    int32_t m[OZO_MAXS];
    int32_t yi[OZO_MAXS];
    float rinv[OZO_MAXS];
    float c[4][OZO_MAXS];   // 2^20, 2^40, 2^60, 2^80 mod m
    float m16[OZO_MAXS];    // 2^16 mod m
    float rp0[OZO_MAXS][OZO_MAXRP];
    float rp1[OZO_MAXS][OZO_MAXRP];
    float rp2[OZO_MAXS][OZO_MAXRP];
    int32_t nsmall0, nsmall1, nsmall2;  // trailing fragments added with tfAddSmall, per pass
    uint32_t W_hi, W_lo;    // 64-bit significand of KM = M*2^-2b (long double)
    int32_t qw;             // exponent of KM
    double logM;            // log2 of the product of the moduli
    // statistics of the precision policy (auto_precision.hpp:24-80)
    double TA, TB, nA, nB, nC;
    double recon1_log2;     // oz2_recon1_log2 (auto_precision.hpp:133-138)
} ozo_plan;

// Reference input generator (evaluation/numerics.hpp:19-38) with the seed as a parameter:
// A (m x k) then B (k x n), row-major; phi < 0: uniform(-1,1), else (u-1/2)*exp(phi*z).
int ozo_gen_inputs(double* a, double* b, uint64_t m, uint64_t n, uint64_t k, double phi, uint32_t seed);

// The pattern generator of tests/correctness.cpp:174-212 (mt19937_64(42)); mode as Pattern there.
int ozo_gen_pattern(double* a, double* b, uint64_t m, uint64_t n, uint64_t k, int mode);

// Scheme II INT8 plan. a, b: zero-padded row-major matrices of the padded dimensions M x K and
// K x N (M, N multiples of 64, K of 32). fixed_bits > 0 fixes the width like the evaluator's
// fixed_bits; passes: 0 Automatic, 1 OnePass, 2 TwoPass. Returns 0, or 1 with a message when
// the reference would throw std::runtime_error (the plan is filled either way).
int ozo_plan_ii_int8(const double* a, const double* b, uint32_t M, uint32_t N, uint32_t K, uint32_t max_moduli,
                     int passes, int fixed_bits, ozo_plan* out, char* err, size_t errlen);

// Moduli selection alone (ozaki2_choose_moduli) for K, a limit and a width cap.
int ozo_choose_moduli_int8(uint32_t K, int num_moduli, int b_cap, ozo_plan* out);

// Scaling stage: maxima of the rows of A (rows x cols, row-major, ld) or of the columns of B
// (col_mode=1) as BF16 rounded up (scale_f64_reader.cpp:129-198, scale_bits.h:33-44), then the
// exponent deltas d = shift - e (expdelta.cpp:44-91). flags: OR of 1 (above BF16), 2 (below
// 2^-126), 4 (Inf/NaN).
int ozo_scale(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, int32_t shift,
              uint16_t* bf16_max, int32_t* delta, uint32_t* flags);

// Slicing stage: the S residues of every element (digits.h:80-179, slice_tf_core.h:67-75,
// f64_tf.h:141-168). A mode (col_mode=0): x is rows x cols row-major with a delta per row,
// output planes [S][rows][cols]. B mode (col_mode=1): x is rows(=K) x cols(=N), delta per column,
// output planes [S][cols][rows] (transposed, K contiguous). Residues are int8 values.
int ozo_split(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, const int32_t* delta,
              const ozo_plan* plan, int8_t* planes);

// Digits of one element (for unit tests): the nd digits d_{nd-1}..d_0 as made.
int ozo_digits(double x, int32_t delta, int nd, float* digits);

// Exact integer GEMM per modulus: C[s][i][j] = sum_k A[s][i][k] * B[s][j][k] (int32, checked).
int ozo_gemm_i32(const int8_t* ap, const int8_t* bp, uint64_t S, uint64_t M, uint64_t N, uint64_t K, int32_t* c);

// Reference reconstruction (recon_crt.cpp:219-338 with recon_crt_proc.h and recon_elem.h): C
// (M x N, ld) from the S int32 planes [S][M][N] as the device computes it in FP32 triple-float.
int ozo_recon_faithful(const int32_t* cs, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                       const ozo_plan* plan, double* c, uint64_t ldc);

// Exact CRT reconstruction: the arithmetic of the B200 reconstruction kernel restated on the CPU
// (not the reference's; its link to the reference is the tolerance test against
// ozo_recon_faithful). C' from the residues exactly, one round-to-nearest-even conversion,
// exact power-of-two scale, results below 2^-1022 flushed to +-0.
int ozo_recon_exact(const int32_t* cs, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                    const ozo_plan* plan, double* c, uint64_t ldc);

// Whole emulated pipeline for unpadded m x k, k x n (row-major): pads like context.cpp:103-117,
// plans, scales, slices, multiplies and reconstructs. recon: 0 faithful, 1 exact. Returns 0, or 1
// with a message when the plan is rejected. info_out (optional) receives the plan.
int ozo_ii_int8_emulate(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                        uint32_t max_moduli, int passes, int fixed_bits, int recon, ozo_plan* info_out, char* err,
                        size_t errlen);

// Dot2 reference GEMM (evaluation/numerics.hpp:58-93): C = hi + lo.
int ozo_dot2_gemm(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, double* hi, double* lo);
// Relative Frobenius error and effective bits (evaluation/numerics.hpp:98-129).
int ozo_accuracy(const double* c, const double* hi, const double* lo, uint64_t count, double* rel_fro, double* ebits);
// Output hash of the bit patterns (evaluation/numerics.hpp:46-57).
uint64_t ozo_output_hash(const double* c, uint64_t count);
// Maximum element-wise relative error against a binary128 reference, over the rows listed (all
// rows if rows == NULL) and all columns. Elements whose reference is 0 count as absolute errors.
int ozo_maxrel_f128(const double* a, const double* b, const double* c, uint64_t m, uint64_t n, uint64_t k,
                    const uint64_t* rows, uint64_t nrows, double* maxrel);
// The same for nc results at once, each given only on the listed rows: cs[t] points at nrows x n values
// (row r of cs[t] is row rows[r] of that result); maxrel[t] receives its error. One binary128 product per
// row serves all of them.
int ozo_maxrel_f128_rows(const double* a, const double* b, const double* const* cs, int nc, uint64_t m, uint64_t n,
                         uint64_t k, const uint64_t* rows, uint64_t nrows, double* maxrel);

// Time the Dot2 reference GEMM on `threads` OpenMP threads for the first `rows` rows of C
// (m x n x k problem); returns seconds.
double ozo_time_dot2_rows(const double* a, const double* b, uint64_t rows, uint64_t n, uint64_t k, int threads);

// ---- Scheme I INT8 (src/ozaki1.cpp:192-282) -------------------------------------------------------
// Scaling with the scheme I target 2^-1 (OZ1_NSHIFT, ozaki1/format.hpp): delta = -1 - e; then p
// radix-254 slices per element (slice_tf_body.h with tfMulR, sfpu_tf_proc.h:108-133), digits clamped
// to +-127. planes: A [p][rows][cols], B (col_mode=1) [p][cols][rows].
int ozo_i_slice(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, const int32_t* delta, int p,
                int8_t* planes);
// Diagonal products P_d = sum_{i+j=d} A_i B_j^T, d = 0..p-1 (the concatenated GEMMs of
// issue_panel_diagonals), int32 [p][M][N].
int ozo_i_gemm(const int8_t* ap, const int8_t* bp, int p, uint64_t M, uint64_t N, uint64_t K, int32_t* pd);
// Reference reconstruction: triple-float Horner S = sum_d 254^(L-d) P_d (recon_tf_i32in.cpp) and the
// FP64 assembly times 254^-(L+2) 2^-(dA+dB) (recon_f64_writer.cpp, assemble_tf_f64 of f64_tf.h).
int ozo_i_recon_faithful(const int32_t* pd, int p, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                         double* c, uint64_t ldc);
// The B200 reconstruction restated: S exactly (multiword), top 64 bits times the 64-bit significand
// of 254^-(L+2), one round-to-nearest-even, subnormal results flushed to +-0.
int ozo_i_recon_exact(const int32_t* pd, int p, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                      double* c, uint64_t ldc);
// Whole scheme I INT8 pipeline with p slices (p > 0) for unpadded inputs (padded like the reference).
int ozo_i_emulate(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k, int p, int exact);

// The same stages for a scheme I format (format: the OZTT_FMT_* value, 5 INT8, 4 FP8, 0 BF16, 1 FP16,
// 2 TF32). FP8 (ozaki1/param.hpp:50, format.hpp): radix 32 multiplied by tfMulP2 (sfpu_tf.h:121-134),
// digits clamped to +-16; BF16, FP16, TF32 (param.hpp:55-65): radix 64, digits +-32; the FP formats
// truncate the row/column maxima to BF16 (CEIL mode 0).
int ozo_scale_mode(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, int32_t shift, int ceil,
                   uint16_t* bf16_max, int32_t* delta, uint32_t* flags);
int ozo_i_slice_fmt(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, const int32_t* delta,
                    int p, int format, int8_t* planes);
// The reference's deferred reconstruction (the FP formats' Int32 accumulation of the pair loop,
// ozaki1/plan.hpp:141-226): recon_tf_i32in.cpp with two's complement input, the first recon_nsmall(K)
// diagonals converted whole, the radix multiplication of the format; then recon_f64_writer.cpp.
int ozo_i_recon_faithful_deferred(const int32_t* pd, int p, int format, uint64_t K, uint64_t M, uint64_t N,
                                  const int32_t* dA, const int32_t* dB, double* c, uint64_t ldc);
int ozo_i_recon_exact_fmt(const int32_t* pd, int p, int format, uint64_t M, uint64_t N, const int32_t* dA,
                          const int32_t* dB, double* c, uint64_t ldc);
int ozo_i_emulate_fmt(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k, int p,
                      int format, int exact);

// ---- Scheme II with digit formats: FP8 (e4m3), BF16, FP16, TF32 (src/backend/ozaki2/kernels/
// modslice_digit.cpp, compose.cpp, sparse_fix.h; the digit layout comes from an oztt_digit_plan) -----------
// CRT constants of a moduli set with integer width b (crt_constants of the INT8 path; nothing in them
// depends on the route): yi, rinv, 2^20k mod m, the reciprocal fragments, W, qw, nd, shift.
int ozo_crt_plan(const int32_t* m, int S, int b, int two_pass, ozo_plan* out);
// Digit planes of every element: the residue r of A' modulo m (the INT8 path's oz2_residue) split per
// modulus as modslice_digit.cpp:193-226 does (the residue itself for a one-digit modulus, rounding to
// nearest for squares and wide moduli, the sparse-digit fix of sparse_fix.h for SQS, radix-16 Karatsuba
// with rounding up for KAR); plane poff[i]+0 = l (or the residue), +1 = h, +2 = s. A: [nplane][rows][cols];
// B (col_mode=1): [nplane][cols][rows]. Returns 1 if a digit is not an integer of the format's digit set
// (e4m3's for FP8, |x| <= 32 otherwise), else 0.
int ozo_digit_split(const double* x, uint64_t rows, uint64_t cols, uint64_t ld, int col_mode, const int32_t* delta,
                  const ozo_plan* crt, const oztt_digit_plan* fp, int8_t* planes);
// GEMM outputs P_o = sum_{t < out_g[o]} A_(out_a[o]+t) B_(out_b[o]-t)^T, int32 [nout][M][N]. Returns 1 if
// some |P_o| exceeds 2^24 (the sums would not be exact in the reference's FP32 accumulation).
int ozo_digit_gemm(const int8_t* ap, const int8_t* bp, const oztt_digit_plan* fp, uint64_t M, uint64_t N, uint64_t K,
                 int32_t* out);
// Composition (compose.cpp:118-146) in the reference's binary32 operations: per modulus the sum of its
// outputs times their coefficients, reduced first (fold_first) or split at 2^12, then ModRound; for a
// one-digit modulus the ModRound of its product that the reconstruction applies (RAWMASK); the residues
// r [S][M][N] as floats.
int ozo_digit_compose(const int32_t* P, const oztt_digit_plan* fp, const ozo_plan* crt, uint64_t M, uint64_t N, float* r);
// Reference reconstruction from residues given as binary32 values (recon_crt.cpp with IN_RESIDUE=1).
int ozo_recon_faithful_residue(const float* r, uint64_t M, uint64_t N, const int32_t* dA, const int32_t* dB,
                               const ozo_plan* plan, double* c, uint64_t ldc);
// Whole digit-format pipeline for unpadded m x k, k x n with the plan fp (made for the same inputs): pads like
// context.cpp:103-117, scales with the plan's shift, splits, multiplies, composes and reconstructs
// (exact: 0 the reference's triple-float reconstruction, 1 the exact one). Returns 0, or 1 with a
// message (out-of-range maxima, a digit outside the format's set, a GEMM output above 2^24).
int ozo_digit_emulate(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                    const oztt_digit_plan* fp, int exact, char* err, size_t errlen);

#ifdef __cplusplus
}
#endif
