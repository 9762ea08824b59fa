/* SPDX-License-Identifier: Apache-2.0
 *
 * C ABI of the B200 Ozaki backend (liboztt.so). Plain pointers and sizes only; every entry point
 * returns OZTT_OK or an error code and writes a message into err[errlen] (NUL-terminated, may be
 * NULL). The C++ public API (ozTTgemm/ozTTgemm.hpp) turns the codes into the reference's exception
 * types: OZTT_EINVAL -> std::invalid_argument, OZTT_ERUNTIME -> std::runtime_error,
 * OZTT_ENOMEM -> std::bad_alloc.
 *
 * Layering, with the reference interface each entry point stands in for (paths relative to the
 * reference project root):
 *   oztt_gemm                 Context::gemm (src/context.cpp:182-186): validation, planning, GPU run
 *   oztt_is_available         ozTTgemm::is_available / format_name (src/dispatch.cpp:18-50)
 *   oztt_ii_digit_*           the same stages for the digit formats of scheme II (FP8, BF16, FP16, TF32)
 *   oztt_ii_int8_plan         choose_moduli_and_width (src/backend/ozaki2/plan.hpp:258-306) for INT8
 *   oztt_ii_int8_run          ozaki2_int8::run (src/ozaki2.cpp:439-478) on host buffers: the backend
 *                             seam Backend = Output(*)(Device&, const Problem&)
 *                             (src/backend_interface.hpp:34)
 *   oztt_ii_int8_run_device   the same pipeline on device-resident operands (the whole-pass replay
 *                             of src/evaluation_hooks.hpp:175-214 times this part)
 *   oztt_ii_scale_rows/cols   scale_f64_reader.cpp:129-198 + expdelta.cpp:44-91 (row maxima of A,
 *                             column maxima of B, exponent deltas, range flags)
 *   oztt_ii_split_rows/cols   slice_f64_reader.cpp + ozaki2/kernels/modslice_int8.cpp (residues)
 *   oztt_ii_residue_gemm      run_int8_gemms (src/ozaki2.cpp:333-348) with bmm_int32_spill.cpp
 *   oztt_ii_recon             recon_crt.cpp + recon_reader.cpp/recon_writer.cpp (CRT to FP64)
 */
#ifndef OZTT_CUDA_H
#define OZTT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OZTT_OK 0
#define OZTT_EINVAL 1   /* invalid argument (std::invalid_argument) */
#define OZTT_ERUNTIME 2 /* configuration cannot be executed, or a CUDA failure (std::runtime_error) */
#define OZTT_ENOMEM 3   /* host memory exhausted (std::bad_alloc) */

#define OZTT_MAXS 24

/* Values of the public enums (ozTTgemm::Scheme, Format, Reconstruction), in declaration order. */
enum { OZTT_SCHEME_I = 0, OZTT_SCHEME_II = 1 };
enum {
    OZTT_FMT_BF16 = 0,
    OZTT_FMT_FP16 = 1,
    OZTT_FMT_TF32 = 2,
    OZTT_FMT_BFP8 = 3,
    OZTT_FMT_FP8 = 4,
    OZTT_FMT_INT8 = 5,
    OZTT_FMT_BFP4 = 6,
    OZTT_FMT_BFP2 = 7
};
enum { OZTT_RECON_AUTO = 0, OZTT_RECON_ONE = 1, OZTT_RECON_TWO = 2 };

typedef struct oztt_options {
    int32_t scheme;
    int32_t format;
    uint32_t slices;
    uint32_t max_moduli;
    int32_t reconstruction;
} oztt_options;

typedef struct oztt_info {
    int32_t scheme;
    int32_t format;
    uint32_t slices;
    uint32_t moduli;
    uint32_t integer_bits;
    uint32_t reconstruction_passes;
    uint64_t padded_m, padded_n, padded_k;
} oztt_info;

/* Plan of one Scheme II INT8 call (the decisions of choose_moduli_and_width and the constants of
 * oz2_crt_constants, src/backend/ozaki2/moduli.hpp:615-703, that the kernels need). */
typedef struct oztt_ii_plan {
    uint32_t M, N, K;      /* planning dimensions: m, n rounded up to 64, k to 32 */
    int32_t S;             /* number of moduli */
    int32_t b;             /* integer width */
    int32_t nd;            /* radix-2^20 digits of A' (3, 4 or 5) */
    int32_t shift;         /* b - 20*(nd-1) */
    int32_t two_pass;      /* 1 if the reference would run two reconstruction passes */
    int32_t b_cap;         /* width cap passed to the moduli selection */
    int32_t S_req;         /* limit on the number of moduli */
    int32_t moduli[OZTT_MAXS];
    int32_t yi[OZTT_MAXS];         /* (M/m_i)^-1 mod m_i */
    float rinv[OZTT_MAXS];         /* fl32(1/m_i) */
    float c[4][OZTT_MAXS];         /* 2^20, 2^40, 2^60, 2^80 mod m_i */
    double TA, TB, nA, nB, nC;     /* input statistics of the precision policy (0 when not measured) */
    double recon1_log2;            /* estimated log2 error of one reconstruction pass */
} oztt_ii_plan;

/* ---- Scheme II with digit formats: FP8 (e4m3), BF16, FP16, TF32 ------------------------------------
 * (the routes OZ2_ROUTE_FP8, OZ2_ROUTE_BF16A, OZ2_ROUTE_FP16A, OZ2_ROUTE_D32 of src/backend/ozaki2/split.hpp)
 * Residues are split into one to three small digits per modulus (|digit| <= 16, or the sparse e4m3 set up
 * to 32, for FP8; <= 32 for the others); the products of digit planes are grouped by weight (concatenated
 * along K) into GEMM outputs, which the composition combines into the residue of C modulo m. Splitting
 * methods (OZ2_SPLIT_* of split.hpp): */
#define OZTT_SPLIT_SQ 0   /* square m = q^2, digits by rounding to nearest, 3 products */
#define OZTT_SPLIT_KAR 1  /* radix-16 Karatsuba (l, h, s = h + l), 3 products */
#define OZTT_SPLIT_WIDE 2 /* two digits of radix ~sqrt(m), 4 products */
#define OZTT_SPLIT_SQS 4  /* square of odd q with the sparse e4m3 digits (|x| <= 16, or even and <= 32) */
#define OZTT_SPLIT_ONE 5  /* one digit: the residue itself (|r| <= 32; BF16 and FP16), 1 product */
#define OZTT_MAXOUT 96    /* GEMM outputs: at most 4 per modulus */

typedef struct oztt_digit_plan {
    oztt_ii_plan base; /* moduli, width, digits of A', passes, CRT constants, statistics */
    int32_t format;    /* OZTT_FMT_FP8, _BF16, _FP16 or _TF32 */
    int32_t nplane;    /* digit planes per operand */
    int32_t nprod;     /* digit products */
    int32_t nout;      /* GEMM outputs after concatenation */
    int32_t fold_first;
    int32_t q[OZTT_MAXS], mode[OZTT_MAXS], poff[OZTT_MAXS], npl[OZTT_MAXS];
    int32_t oout[OZTT_MAXS + 1]; /* outputs of modulus i: oout[i] .. oout[i+1]-1 */
    /* output o = sum_{t < out_g[o]} A digit plane (out_a[o] + t) x B digit plane (out_b[o] - t), with the
     * composition coefficient coeff[o] (mod the modulus out_mod[o]) */
    int32_t out_a[OZTT_MAXOUT], out_b[OZTT_MAXOUT], out_g[OZTT_MAXOUT], out_mod[OZTT_MAXOUT], coeff[OZTT_MAXOUT];
} oztt_digit_plan;

/* Scheme II plan of a digit format (choose_moduli_and_width with the format's route,
 * src/backend/ozaki2/plan.hpp:258-306 and moduli.hpp:700-770; for BF16 and FP16 the moduli set of the
 * stage-time model search, awe.hpp); arguments as oztt_ii_int8_plan (with a fixed width the default limit
 * is the route's: 14 moduli for FP8, 11 for TF32, 24 for BF16 and FP16). */
int oztt_ii_digit_plan(int32_t format, const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                       uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_digit_plan* plan,
                       char* err, size_t errlen);
/* The same plan from DEVICE operands a (m x k) and b (k x n) on `stream`: the precision policy's statistics
 * are measured on the GPU (as oztt_ii_int8_plan_device). */
int oztt_ii_digit_plan_device(int device_id, int32_t format, const double* a, const double* b, uint64_t m,
                              uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits,
                              oztt_digit_plan* plan, void* stream, char* err, size_t errlen);

/* Whole digit-format pipeline with a given plan on HOST buffers (row-major, C = A B): upload, scale, digit
 * split, digit products with the composition fused, reconstruction, download. Replaces the digit backends'
 * run (src/ozaki2.cpp:439-478 compiled with OZ_FMT_FP8 / _BF16 / _FP16 / _FP32). */
int oztt_ii_digit_run(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                      const oztt_digit_plan* plan, char* err, size_t errlen);
/* The same on DEVICE buffers, stream-ordered on `stream`; stage_ms (NULL or 6 doubles) receives the device
 * time of scale rows, scale cols, split rows, split cols, digit GEMM and reconstruction. */
int oztt_ii_digit_run_device(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                             uint64_t k, const oztt_digit_plan* plan, void* stream, double* stage_ms, char* err,
                             size_t errlen);

/* Digit-format stages (device buffers, stream-ordered). Digit split (kernels/modslice_digit.cpp with
 * sparse_fix.h): the residues of A (m x k, lda) split into the digits of each modulus, written as int8
 * values to planes [nplane][mp][kp] (plane poff[s] + 0 = l, + 1 = h, + 2 = s; a one-digit modulus has its
 * residue in plane poff[s]); B (k x n, ldb) transposed into [nplane][np][kp]. delta as from
 * oztt_ii_scale_rows / _cols with the plan's shift. */
int oztt_ii_digit_split_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta,
                             const oztt_digit_plan* plan, int8_t* planes, uint64_t mp, uint64_t kp, void* stream,
                             char* err, size_t errlen);
int oztt_ii_digit_split_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta,
                             const oztt_digit_plan* plan, int8_t* planes, uint64_t np, uint64_t kp, void* stream,
                             char* err, size_t errlen);
/* Digit products (the reference's GEMM stage on digit planes with compose.cpp): mode 0 writes every GEMM
 * output P_o as int32 [nout][mp][np]; mode 1 composes in the epilogue and writes the CRT digits
 * k_s = (sum_o coeff_o P_o) y_s mod m_s as uint16 [S][mp][np]. mp, np, kp multiples of 128, 256, 128. */
int oztt_ii_digit_gemm(const int8_t* a_planes, const int8_t* b_planes, uint64_t mp, uint64_t np, uint64_t kp,
                       const oztt_digit_plan* plan, int32_t mode, void* out, void* stream, char* err, size_t errlen);
/* Reconstruction from uint16 CRT digits [S][mp][np] (as oztt_ii_recon). */
int oztt_ii_digit_recon(const uint16_t* k_digits, uint64_t mp, uint64_t np, const int32_t* delta_a,
                        const int32_t* delta_b, const oztt_digit_plan* plan, double* c, uint64_t m, uint64_t n,
                        uint64_t ldc, void* stream, char* err, size_t errlen);

/* Plan of one Scheme I call (src/ozaki1.cpp:192-210): the number of slices p, the last diagonal L = p-1
 * kept, and the format's slicing (src/backend/ozaki1/param.hpp:47-70): INT8 radix 254, digits +-127; FP8
 * radix 32, digits +-16; BF16, FP16, TF32 radix 64, digits +-32; all normalised to 2^-1. */
typedef struct oztt_i_plan {
    uint32_t M, N, K;  /* planning dimensions: m, n rounded up to 64, k to 32 */
    int32_t p;         /* number of slices (Info::slices) */
    int32_t auto_p;    /* 1 if p was chosen from the input (oz_fp64_p), 0 if requested */
    int32_t format;    /* OZTT_FMT_INT8, _FP8, _BF16, _FP16 or _TF32 */
    int32_t radix;     /* 254, 32 or 64 */
    int32_t dmax;      /* 127, 16 or 32 */
} oztt_i_plan;

/* ---- whole calls ---------------------------------------------------------------------------- */

/* Context::gemm on host row-major buffers (a: m*k, b: k*n, c: m*n; the *_len are the span sizes).
 * Validates exactly like the reference front end, plans, runs on CUDA device device_id, writes C
 * and info. c may overlap a or b. */
int oztt_gemm(int device_id, const double* a, uint64_t a_len, const double* b, uint64_t b_len, double* c,
              uint64_t c_len, uint64_t m, uint64_t n, uint64_t k, const oztt_options* opt, oztt_info* info, char* err,
              size_t errlen);

/* ozTTgemm::is_available / format_name (src/dispatch.cpp:18-50) for an OZTT_FMT_* value: 1 for the formats
 * this build provides (INT8, FP8), 0 otherwise; the name, or "unknown". */
int oztt_is_available(int32_t format);
const char* oztt_format_name(int32_t format);

/* Scheme II INT8 plan for row-major a (m x k) and b (k x n) on the host. reconstruction is an
 * OZTT_RECON_* value; fixed_bits > 0 fixes the width (the reference evaluator's fixed_bits), 0 lets
 * the library choose it from the input. */
int oztt_ii_int8_plan(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli,
                      int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan* plan, char* err, size_t errlen);

/* The Scheme II INT8 pipeline for host buffers (copies in, runs, copies C back). */
int oztt_ii_int8_run(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                     const oztt_ii_plan* plan, char* err, size_t errlen);

/* The pipeline on device buffers (row-major, lda = k, ldb = n, ldc = n) on a cudaStream_t (NULL:
 * the legacy default stream). Scratch comes from the stream-ordered allocator and is released
 * before return. Synchronises the stream before returning. */
int oztt_ii_int8_run_device(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                            uint64_t k, const oztt_ii_plan* plan, void* stream, char* err, size_t errlen);

/* The same, also returning the device time of each stage in stage_ms[6] (scale rows, scale columns,
 * split rows, split columns, residue GEMM, reconstruction), from CUDA events on `stream`. */
int oztt_ii_int8_run_device_timed(int device_id, const double* a, const double* b, double* c, uint64_t m,
                                  uint64_t n, uint64_t k, const oztt_ii_plan* plan, void* stream, double* stage_ms,
                                  char* err, size_t errlen);

/* Host wall-clock phases (ms) of the last INT8 Scheme II call made through oztt_gemm / Context::gemm in
 * this process, out[0..count-1] of (16 values):
 *   0 upload (to the end of the last host-to-device copy), 1 statistics read-back after it, 2 value checks,
 *   3 plan, 4 pipeline with the read-back of C, 5 total, 6 the number of pieces of C read back (row bands,
 *   or tiles);
 * and for calls of at least 4096 rows, which compute while their operands upload:
 *   7 when the first plan was made, 8 1 if the complete statistics gave another plan, 9 1 if the bounds of
 *   the statistics left a decision open so that the exact sums were computed, 10 1 if C was read back as
 *   its pieces finished (before the plan was confirmed); the device timeline in ms from the first copy:
 *   11 A's first part (half of its rows) done against B's first blocks, 12 the last reconstruction, 13 the end of the
 *   read-back of C, 14 the last band's bounded statistics; 15 when the host's value checks were ready
 *   (ms from the call).
 * Zeros before the first such call. */
int oztt_ii_int8_last_phases(double* out, int32_t count);

/* Scheme I INT8 plan (plan_issue and the slice count of src/backend/ozaki1/plan.hpp:128-250 and
 * auto_precision.hpp:506): slices > 0 fixes p, 0 chooses it from the input. OZTT_ERUNTIME when the
 * reference would throw (K blocking needed, Horner exponent budget exceeded). */
int oztt_i_int8_plan(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t slices,
                     oztt_i_plan* plan, char* err, size_t errlen);
/* Scheme I plan of any built format (the same with the format's constants: for FP8, BF16, FP16 and TF32
 * K blocking is allowed and the pair loop folds the FP32 partial products into Int32,
 * ozaki1/plan.hpp:141-226). */
int oztt_i_format_plan(int32_t format, const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                       uint32_t slices, oztt_i_plan* plan, char* err, size_t errlen);
/* Scheme I plan of a built format for operands on the device (row-major a_dev: m x k, b_dev: k x n), the
 * slice count (slices = 0) selected from statistics measured there (oz_fp64_p,
 * src/backend/ozaki1/auto_precision.hpp:65-526). Bit-identical to oztt_i_format_plan on the same finite
 * values. Synchronises `stream`. */
int oztt_i_format_plan_device(int32_t format, const double* a_dev, const double* b_dev, uint64_t m, uint64_t n,
                              uint64_t k, uint32_t slices, oztt_i_plan* plan, void* stream, char* err,
                              size_t errlen);
/* The Scheme I slice selection's model (1) errors (out[q] for q = 2..count-1) and the estimate of
 * ||C||_F^2 (out[0]), measured on the host from a, b (a_dev NULL) or on the device from a_dev, b_dev:
 * for checking the two against each other. */
int oztt_i_model1_errors(int32_t format, const double* a, const double* b, const double* a_dev, const double* b_dev,
                         uint64_t m, uint64_t n, uint64_t k, double* out, int32_t count, void* stream, char* err,
                         size_t errlen);
/* Scheme II INT8 plan for operands already on the device (a: m x k, b: k x n, row-major): the input
 * statistics of the precision policy are measured by kernels on `stream` (bit-identical to the host
 * measurement of oztt_ii_int8_plan), the decisions made on the host. Synchronises `stream`. */
int oztt_ii_int8_plan_device(int device_id, const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                             uint32_t max_moduli, int32_t reconstruction, int32_t fixed_bits, oztt_ii_plan* plan,
                             void* stream, char* err, size_t errlen);
/* The statistics stages of the Scheme II precision policy (estimate_product_norm and oz2_measure_stats,
 * src/backend/common/norm_estimate.hpp:20-73, src/backend/ozaki2/auto_precision.hpp:24-80), for callers
 * whose A and B are split into panels over several devices: each device measures its panels, the
 * caller combines them (all-reduce) and plans once with oztt_ii_int8_plan_from_stats.
 *   absmax  exact max |x| per row (mode 0) or per column (mode 1) of a row-major rows x cols matrix,
 *           written as doubles to device memory;
 *   sumsq   sum of (x*rg)^2 per row (mode 0) or column (mode 1), in index order, one rounding per step;
 *   sketch  out[l*ostride + r] = (double) sum_j (long double)(x[r][j]*rg) * v[l*vstride + j], l = 0..7,
 *           j ascending, in 64-bit-significand arithmetic (the reference's long double). */
int oztt_stats_absmax(const double* x, uint64_t rows, uint64_t cols, int32_t mode, double* out, void* stream,
                      char* err, size_t errlen);
int oztt_stats_sumsq(const double* x, uint64_t rows, uint64_t cols, int32_t mode, double rg, double* out,
                     void* stream, char* err, size_t errlen);
int oztt_stats_sketch(const double* x, uint64_t rows, uint64_t cols, double rg, const double* v, uint64_t vstride,
                      double* out, uint64_t ostride, void* stream, char* err, size_t errlen);
/* The sketch y_l = B g_l over a stretch of columns, for B split into column panels over several devices
 * (no counterpart in the reference, which is single-device; it continues the sums of estimate_product_norm,
 * src/backend/common/norm_estimate.hpp:48-73, across panels): state holds 8 x rows extended-precision sums
 * of 16 bytes each (state[l*rows + r]); x is rows x cols with rows ldx apart, v the vectors' entries for
 * these columns (8 rows, vstride apart). carry = 0 starts the sums, 1 continues them from state (e.g. a
 * state received from the device holding the earlier columns). The terms are (x*rg) * v in the
 * reference's long-double arithmetic, columns ascending. */
int oztt_stats_sketch_chain(const double* x, uint64_t rows, uint64_t cols, uint64_t ldx, double rg, const double* v,
                            uint64_t vstride, void* state, int32_t carry, void* stream, char* err, size_t errlen);
/* out[i] = the extended sum state[i] rounded to double, i < count (the end of a chain). */
int oztt_stats_sketch_round(const void* state, uint64_t count, double* out, void* stream, char* err, size_t errlen);
/* The five statistics (TA, TB, nA, nB, nC into out5) from the per-row and per-column measurements of the
 * whole problem, summed on the host in the reference's order (choose_precision_policy and
 * estimate_product_norm, src/backend/ozaki2/auto_precision.hpp:24-80, common/norm_estimate.hpp:48-73):
 * row_max / col_max the |maxima| of A's m rows and B's n columns, row_sumsq / col_sumsq their sums of
 * (x*rg)^2, sketch_s the 8 x m sketches s_l = A y_l; rgA, rgB the power-of-two scales. Host memory. */
int oztt_policy_stats_combine(const double* row_max, uint64_t m, const double* col_max, uint64_t n,
                              const double* row_sumsq, const double* col_sumsq, const double* sketch_s, double rgA,
                              double rgB, double* out5, char* err, size_t errlen);
/* The 8 x N Gaussian vectors of the norm estimate (mt19937 seeded 12345, the reference's draw order). */
void oztt_policy_vectors(uint32_t N, double* out);
/* Scheme II INT8 plan from the five input statistics of the precision policy (TA, TB: sums of squared
 * power-of-two row/column scales; nA, nB: squared Frobenius norms; nC: the low-biased estimate of
 * ||AB||_F^2, all after the power-of-two normalisation) for an m x k by k x n problem. */
int oztt_ii_int8_plan_from_stats(uint64_t m, uint64_t n, uint64_t k, uint32_t max_moduli, int32_t reconstruction,
                                 int32_t fixed_bits, double TA, double TB, double nA, double nB, double nC,
                                 oztt_ii_plan* plan, char* err, size_t errlen);
/* The Scheme I pipeline on host buffers (ozaki1_int8::run and its FP8 counterpart, src/ozaki1.cpp:192-282),
 * in the plan's format. */
int oztt_i_int8_run(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                    const oztt_i_plan* plan, char* err, size_t errlen);
/* The same on device buffers (lda = k, ldb = n, ldc = n); synchronises `stream`. stage_ms (NULL or 5
 * entries) receives the device time of scale rows, scale columns, slicing, diagonal GEMMs and
 * reconstruction. */
int oztt_i_int8_run_device(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n,
                           uint64_t k, const oztt_i_plan* plan, void* stream, double* stage_ms, char* err,
                           size_t errlen);

/* ---- stages (device pointers; asynchronous on `stream`) -------------------------------------- */

/* Tile-padded dimensions of the residue planes: mp = m rounded up to 128, np = n rounded up to 256,
 * kp = k rounded up to 128. */
void oztt_ii_padded_dims(uint64_t m, uint64_t n, uint64_t k, uint64_t* mp, uint64_t* np, uint64_t* kp);

/* Row maxima of a (m x k, lda): BF16 of max|a_ij| rounded up (bf16max, may be NULL), delta[i] =
 * shift - ceil(log2 bf16max) (0 exponent for a zero row), flags |= 1 (above BF16), 2 (below
 * 2^-126), 4 (Inf/NaN). flags must be zeroed by the caller; delta has m entries. */
int oztt_ii_scale_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, int32_t shift, int32_t* delta,
                       uint16_t* bf16max, uint32_t* flags, void* stream, char* err, size_t errlen);
/* Column maxima of b (k x n, ldb); delta has n entries. Uses n*8 bytes of stream-ordered scratch. */
int oztt_ii_scale_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift, int32_t* delta,
                       uint16_t* bf16max, uint32_t* flags, void* stream, char* err, size_t errlen);

/* Largest n accepted by oztt_ii_scale_cols_noalloc (2 MiB of column scratch per device). */
#define OZTT_NOALLOC_MAX_COLS 262144u
/* No counterpart in the reference: oztt_ii_scale_cols without any device allocation, for callers that
 * cannot let a library allocate device memory (all memory owned by their own allocator or reserved up
 * front, or latency-critical paths where an allocation may synchronise or fail). Its scratch is a
 * fixed static device array that every GPU loading the library keeps until exit; n is limited to
 * OZTT_NOALLOC_MAX_COLS (larger n: OZTT_EINVAL). The first call on a device looks up the array's
 * address with that device current; make it before any stream capture (after a cudaDeviceReset the next
 * call looks it up again, so make that one before any capture too). Calls on one device share the
 * array (each clears the part it uses first); calls that overlap on the GPU race. */
int oztt_ii_scale_cols_noalloc(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift, int32_t* delta,
                               uint16_t* bf16max, uint32_t* flags, void* stream, char* err, size_t errlen);

/* Residues of a (m x k, lda) with delta per row: planes [S][mp][kp] int8, zero in the padding. */
int oztt_ii_split_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta,
                       const oztt_ii_plan* plan, int8_t* planes, uint64_t mp, uint64_t kp, void* stream, char* err,
                       size_t errlen);
/* Residues of b (k x n, ldb) with delta per column, transposed: planes [S][np][kp] int8. */
int oztt_ii_split_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta,
                       const oztt_ii_plan* plan, int8_t* planes, uint64_t np, uint64_t kp, void* stream, char* err,
                       size_t errlen);

/* Per-modulus products of the planes on the tensor cores (tcgen05 kind::i8, s32 in TMEM).
 * mode 0: out is int32 [S][mp][np], C_s = A_s * B_s^T exactly.
 * mode 1: out is uint8 [S][mp][np], k_s = (C_s mod m_s) * y_s mod m_s in [0, m_s). */
int oztt_ii_residue_gemm(const int8_t* a_planes, const int8_t* b_planes, uint64_t mp, uint64_t np, uint64_t kp,
                         const oztt_ii_plan* plan, int32_t mode, void* out, void* stream, char* err, size_t errlen);

/* Exact CRT reconstruction from the uint8 planes k_s [S][mp][np]: C[i][j] (i < m, j < n, ldc) =
 * C'_ij * 2^(2*shift - delta_a[i] - delta_b[j] - 2b), rounded once to nearest even; results below
 * 2^-1022 are returned as signed zero. */
int oztt_ii_recon(const uint8_t* k_planes, uint64_t mp, uint64_t np, const int32_t* delta_a, const int32_t* delta_b,
                  const oztt_ii_plan* plan, double* c, uint64_t m, uint64_t n, uint64_t ldc, void* stream, char* err,
                  size_t errlen);

/* ---- evaluation utilities (the reference evaluator's input generator and output hash) ----------- */

/* Seeded inputs of evaluation/numerics.hpp:19-38 with the seed as a parameter: std::mt19937(seed); A
 * (m x k) then B (k x n), row-major; phi < 0: uniform(-1, 1); else (u - 1/2) * exp(phi * z) with
 * u ~ U[0,1) then z ~ N(0,1) per element. Host memory. */
void oztt_eval_inputs(double* a, double* b, uint64_t m, uint64_t n, uint64_t k, double phi, uint32_t seed);
/* Hash of the output bit patterns (evaluation/numerics.hpp:46-57). */
uint64_t oztt_eval_output_hash(const double* c, uint64_t count);

/* Scheme I scaling (scale_f64_reader.cpp + expdelta.cpp with OZ1_NSHIFT = -1): delta = -1 - ceil(log2 u)
 * of the BF16 u of each row maximum of A (rows) / column maximum of B (cols), rounded up for INT8 and
 * truncated for FP8 (OZ1_CEIL_MODE, ozaki1/format.hpp:79-97); flags as oztt_ii_scale_rows. */
int oztt_i_scale_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, int32_t format, int32_t* delta,
                      uint32_t* flags, void* stream, char* err, size_t errlen);
int oztt_i_scale_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t format, int32_t* delta,
                      uint32_t* flags, void* stream, char* err, size_t errlen);
/* Scheme I slices (slice_tf_sm8.cpp / slice_tf_num.cpp): p digits of x * 2^delta per element in the
 * format's radix (INT8: 254, digits in [-127, 127]; FP8: 32, digits in [-16, 16], each an integer e4m3
 * holds, stored as int8); rows: A (m x k) -> [p][mp][kp]; cols: B (k x n) -> [p][np][kp] (transposed). */
int oztt_i_slice_rows(const double* a, uint64_t m, uint64_t k, uint64_t lda, const int32_t* delta, int32_t p,
                      int32_t format, int8_t* planes, uint64_t mp, uint64_t kp, void* stream, char* err,
                      size_t errlen);
int oztt_i_slice_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, const int32_t* delta, int32_t p,
                      int32_t format, int8_t* planes, uint64_t np, uint64_t kp, void* stream, char* err,
                      size_t errlen);
/* Diagonal products P_d = sum_{i=0..d} A_i B_{d-i}^T (int32 [p][mp][np]) on the tensor cores: the
 * concatenated per-diagonal GEMMs of issue_panel_diagonals (src/backend/ozaki1/stages.hpp). */
int oztt_i_diag_gemm(const int8_t* a_planes, const int8_t* b_planes, uint64_t mp, uint64_t np, uint64_t kp, int32_t p,
                     int32_t* out, void* stream, char* err, size_t errlen);
/* Scheme I reconstruction (recon_tf_i32in.cpp + recon_f64_writer.cpp): C = sum_d r^(p-1-d) P_d *
 * r^-(p+1) * 2^-(dA_i + dB_j) with the format's radix r, the sum exact, one rounding. */
int oztt_i_recon(const int32_t* diag, uint64_t mp, uint64_t np, const int32_t* delta_a, const int32_t* delta_b,
                 int32_t p, int32_t format, double* c, uint64_t m, uint64_t n, uint64_t ldc, void* stream, char* err,
                 size_t errlen);

/* ---- resident operands ----------------------------------------------------------------------------
 * No counterpart in the reference: it rebuilds its buffers and programs on every call and keeps no operand
 * on the device (README.md:81-85), as Context::gemm does here. For callers that multiply by the same matrix
 * many times, a resident operand is uploaded once and keeps in HBM what the Scheme II INT8 pipeline derives
 * from it alone: its precision-policy measurements (row or column maxima, scale, sums of squares, and for B
 * the sketch y = B g of estimate_product_norm) and the exponent deltas and residue planes of the last two
 * plans it was used with. A product of two resident operands makes the plan Context::gemm makes for the same
 * values (byte for byte) and returns the same C, bit for bit; with an unchanged plan it starts at the
 * residue GEMM. Scheme II with INT8 products only. Products on one process are serialised. */
#define OZTT_ROLE_A 0 /* left operand, m x k */
#define OZTT_ROLE_B 1 /* right operand, k x n */
typedef struct oztt_resident oztt_resident;
/* Uploads x (rows x cols, row-major; host memory, or device memory of device_id when x_on_device) as a
 * left (OZTT_ROLE_A) or right (OZTT_ROLE_B) operand and measures it. The values are checked as the front
 * end checks them (finiteness, the range of the nonzero row maxima of A / column maxima of B), with the
 * same messages. */
int oztt_resident_create(int device_id, int32_t role, const double* x, uint64_t rows, uint64_t cols,
                         int32_t x_on_device, oztt_resident** out, char* err, size_t errlen);
/* Frees the operand's device memory. NULL is allowed. */
int oztt_resident_destroy(oztt_resident* r);
/* C = A B for resident A (m x k) and B (k x n) on one device; c is m x n row-major, in host memory or (when
 * c_on_device) device memory of that device. opt must name Scheme II and INT8 (max_moduli and
 * reconstruction as in oztt_gemm); info (may be NULL) receives what Context::gemm reports. */
int oztt_resident_gemm(oztt_resident* a, oztt_resident* b, double* c, int32_t c_on_device, const oztt_options* opt,
                       oztt_info* info, char* err, size_t errlen);

/* ---- kernel variants ------------------------------------------------------------------------------
 * No counterpart in the reference (it has one kernel per stage and reads no environment). Process-wide
 * switches between kernels that give identical results; the defaults (0) are the faster ones on a B200
 * under its 1 kW power cap. A change applies to launches issued after it returns.
 *   OZTT_OPT_GEMM_CTA_PAIRS  1: the INT8 residue GEMMs and Scheme I diagonal GEMMs on CTA pairs
 *                            (tcgen05 cta_group::2, M = 256 per pair); 0: one CTA per tile.
 *   OZTT_OPT_RECON_INT       1: the Scheme II INT8 reconstruction on the integer pipe (32-bit words);
 *                            0: the FP64-pipe kernel (moduli in pairs, 32-bit FP64 limbs). */
#define OZTT_OPT_GEMM_CTA_PAIRS 1
#define OZTT_OPT_RECON_INT 2
/* Sets an option to 0 or 1 (OZTT_EINVAL for an unknown option or value). */
int oztt_set_option(int32_t option, int32_t value, char* err, size_t errlen);
/* Reads an option's current value into *value. */
int oztt_get_option(int32_t option, int32_t* value);

/* Number of SMs and compute capability of a device (0 on success). */
int oztt_device_info(int device_id, int32_t* sm_count, int32_t* cc_major, int32_t* cc_minor);

#ifdef __cplusplus
}
#endif

#endif /* OZTT_CUDA_H */
