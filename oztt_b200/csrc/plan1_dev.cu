// SPDX-License-Identifier: Apache-2.0
//
// Scheme I slice selection with its per-element statistics measured on the device.
//
// The reference selects p from the whole input (oz_fp64_p, src/backend/ozaki1/auto_precision.hpp:65-526):
// a normalization (global scales, per-row/column exponents and norms), model (1) -- every element of A
// and B expanded slice by slice, its slice and residual contributions summed per k in row (column)
// order -- the Hutchinson estimate of ||C||_F^2, and model (2) on 64 sampled rows and columns. On the
// host, model (1) costs seconds at 8192^3. Here the normalization and ||C||_F^2 come from the policy
// statistics kernels (PolicyStatsRun, stats.cu), model (1)'s per-k sums and model (2)'s sample sums from
// the kernels below, and the host finishes with the same code as the host planner (planner1.cpp:
// combining the terms, picking the sample, the rounding simulation, the search). The result is
// bit-identical to the host planner's.
//
// terms_kernel sums per column c of A (rows in ascending order) and per row r of B (columns in ascending
// order), as the host sums them, both operands in one launch. Each element x (scaled by 2^(nshift - e) of its row or column)
// is expanded as the reference's device slicer does -- u = radix t (FMA-exact product, TwoSum), digit
// d = clamp(rint(fl32(u_hi)), +-dmax), t = u - d in two doubles -- until its residual is zero, adding
// (s d w)^2 to S[i] and (s t w)^2 to R[i+1] with w = radix^-(i+1) formed by repeated division. Every
// operation is an explicitly rounded intrinsic in the host's order (no contraction), so each sum is the
// host's to the bit.
#include <algorithm>
#include <vector>

#include "oztt_common.cuh"
#include "planner.hpp"
#include "runtime.cuh"

namespace oztt {

namespace {

__device__ __forceinline__ void two_sum_d(double a, double b, double& s, double& e) {
    s = __dadd_rn(a, b);
    const double bb = __dsub_rn(s, a);
    e = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
}

// w_i = radix^-(i+1) formed by repeated division, w_0 = 1/radix, w_(i+1) = w_i / radix, exactly as the
// host planner forms it in its loops; passed to the kernels by value.
constexpr int kMaxSteps = 40;
struct Weights {
    double w[kMaxSteps];
};

Weights weights_of(double radix) {
    Weights t;
    double x = 1.0;
    for (int i = 0; i < kMaxSteps; ++i) t.w[i] = x = x / radix;
    return t;
}

// 2^e for |e| <= 1022.
__device__ __forceinline__ double pow2d(int e) { return __longlong_as_double((long long)(1023 + e) << 52); }

// One step of the expansion t = th + tl: u = radix t, digit d = clamp(rint(fl32(u_hi)), +-dmax), t = u - d.
__device__ __forceinline__ double expand_step(double& th, double& tl, double radix, double dmax) {
    const double ph = __dmul_rn(radix, th);
    const double pe = __fma_rn(radix, th, -ph);
    double uh, ul;
    two_sum_d(ph, __dadd_rn(pe, __dmul_rn(radix, tl)), uh, ul);
    const double dg = fmin(dmax, fmax(-dmax, rint((double)__double2float_rn(uh))));
    two_sum_d(__dsub_rn(uh, dg), ul, th, tl);
    return dg;
}

// The sums of one side (A or B) of model (1): `chains` sequential sums (a column of A over its rows, a row
// of B over its columns) of `len` elements each; element e of chain q sits at x + q*chain_stride +
// e*elem_stride.
struct TermsSide {
    const double* x;
    uint64_t chains, len, chain_stride, elem_stride;
    const double* s;    // divisor of element e's row of A (column of B); 0: not counted
    const int32_t* sh;  // its exponent shift nshift - e
    double rg;
    double *S, *R, *N;  // S[i][q], R[r][q], N[q]
};

// A block owns kChains adjacent chains. It takes their elements kSpan at a time: every thread expands one
// element (the expansions are independent of one another and of the sums), kGroup steps at a time, and
// leaves the group's per-step contributions in shared memory; then the owners of the group's sums -- one
// thread per (chain, sum) -- add the kSpan contributions in element order, so each sum receives its terms
// in the host's order. A step after an element's residual reached exactly zero contributes +0, which
// leaves a sum unchanged (the sums are never -0), as the host adds nothing; once every element of the
// block is exhausted the remaining groups are skipped. Holding one group at a time keeps the shared
// memory per thread small, so that more warps hide the latency of the dependent FP64 chains. For A
// (element stride = a row) the kChains adjacent columns make a warp's loads cover whole 32-byte sectors;
// for B (element stride 1) a warp reads runs of kSpan consecutive elements of a row.
// Groups of 5 steps stop a block within 5 steps of its longest expansion. Measured at 8192^2 per operand
// (INT8 / BF16 digits, ms per launch) with the padded layout below and the owners' loads issued 8 at a
// time, 4 chains of 32 elements: groups of 2 15.2 / 8.9, of 3 11.3 / 6.1, of 4 10.9 / 5.9, of 5 10.1 / 6.0;
// 8 chains of 16 elements (shorter serial sums, A's loads two sectors wide) with groups of 5: 9.97 / 5.77.
// With an unpadded layout and one load per add, groups of 3 took 20.9 / 11.0 and groups of 8 24.9 / 17.1.
constexpr int kChains = 8, kSpan = 16, kTermsThreads = kChains * kSpan, kGroup = 5;
// contributions of one group: [2 kGroup + 1][kRowStride] (S steps, R steps, N)
constexpr int kGroupRows = 2 * kGroup + 1;
// Layout of the contributions: thread t writes slot t + (t / kSpan) (one pad per kSpan slots) of every
// row, rows kRowStride apart. kRowStride = 4 (mod 16) and B's chains kSpan + 1 slots apart (A's chains
// adjacent) give owner (row i, chain q) the 8-byte bank 4 i + q + const (mod 16): at most 3 of a warp's
// owners share a bank, so a load takes at most 3 wavefronts (2 is the minimum for 32 doubles; unpadded,
// the owners of B's chains all read one bank).
constexpr int kChainPad = 1, kSlots = kTermsThreads + kTermsThreads / kSpan * kChainPad;
constexpr int kRowStride = kSlots + ((4 - kSlots) % 16 + 16) % 16;
static_assert(kRowStride % 16 == 4 && kSpan % kChains == 0 && kChains * kGroupRows <= kTermsThreads, "layout");
static_assert(kTermsThreads - 1 + (kTermsThreads - 1) / kSpan * kChainPad < kRowStride, "slots fit a row");

template <int PMAX>
__global__ void __launch_bounds__(kTermsThreads) terms_kernel(TermsSide A, TermsSide B, uint32_t a_blocks,
                                                              double radix, double dmax, const Weights wt) {
    __shared__ double contrib[kGroupRows * kRowStride];
    constexpr int NG = (PMAX + kGroup - 1) / kGroup;
    const bool side_b = blockIdx.x >= a_blocks;
    const TermsSide& sd = side_b ? B : A;
    const uint64_t q0 = (uint64_t)(blockIdx.x - (side_b ? a_blocks : 0)) * kChains;
    const int t = threadIdx.x;
    // the element slot of this thread: chain fastest for A (adjacent columns), element fastest for B
    const int cq = side_b ? t / kSpan : t % kChains, ce = side_b ? t % kSpan : t / kChains;
    const uint64_t q = q0 + cq;
    // the sum this thread owns in every group (kChains * kGroupRows <= kTermsThreads): chain oq, row oi of
    // the group's contributions; the S and R sums of all groups and N stay in registers
    const int oq = t / kGroupRows, oi = t % kGroupRows;
    const bool owner = t < kChains * kGroupRows;
    double accS[NG], accR[NG], accN = 0.0;
#pragma unroll
    for (int g = 0; g < NG; ++g) accS[g] = accR[g] = 0.0;
    double* col = contrib + t + t / kSpan * kChainPad;
    for (uint64_t e0 = 0; e0 < sd.len; e0 += kSpan) {
        const uint64_t e = e0 + ce;
        double th = 0.0, tl = 0.0, sc = 0.0, vr2 = 0.0;
        bool live = false;
        if (q < sd.chains && e < sd.len) {
            const double v = __ldg(sd.x + q * sd.chain_stride + e * sd.elem_stride);
            const double vr = __dmul_rn(v, sd.rg);
            vr2 = __dmul_rn(vr, vr);
            const double se = __ldg(sd.s + e);
            if (v != 0.0 && se > 0.0) {
                live = true;
                th = __dmul_rn(v, pow2d(__ldg(sd.sh + e)));
                sc = se;
            }
        }
        const int n_el = sd.len - e0 < (uint64_t)kSpan ? (int)(sd.len - e0) : kSpan;
        // first element's slot of the owned chain; element el is el slots further on B's side and
        // kChains el + el / (kSpan / kChains) further on A's side (chains interleaved, one pad per kSpan)
        const int slot = side_b ? oq * (kSpan + kChainPad) : oq;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            // the block stops at the first group in which no element is still being expanded
            if (!__syncthreads_or(live) && g > 0) break;
#pragma unroll
            for (int j = 0; j < kGroup; ++j) {
                const int i = g * kGroup + j;
                double cs = 0.0, cr = 0.0;
                if (i < PMAX && live) {
                    const double w = wt.w[i];
                    const double dg = expand_step(th, tl, radix, dmax);
                    const double c = __dmul_rn(__dmul_rn(sc, dg), w);
                    cs = __dmul_rn(c, c);
                    const double r = __dmul_rn(__dmul_rn(sc, __dadd_rn(th, tl)), w);
                    cr = __dmul_rn(r, r);
                    live = th != 0.0;
                }
                col[j * kRowStride] = cs;
                col[(kGroup + j) * kRowStride] = cr;
            }
            col[2 * kGroup * kRowStride] = vr2;
            __syncthreads();
            if (owner) {
                const double* src = contrib + oi * kRowStride + slot;
                double a = oi < kGroup ? accS[g] : (oi < 2 * kGroup ? accR[g] : accN);
                const bool skip = oi == 2 * kGroup && g > 0;  // N is summed once, with group 0
                if (!skip && n_el == kSpan) {
#pragma unroll 8
                    for (int el = 0; el < kSpan; ++el) a = __dadd_rn(a, src[side_b ? el : el * kChains + el / (kSpan / kChains)]);
                } else if (!skip) {
                    for (int el = 0; el < n_el; ++el) a = __dadd_rn(a, src[side_b ? el : el * kChains + el / (kSpan / kChains)]);
                }
                if (oi < kGroup)
                    accS[g] = a;
                else if (oi < 2 * kGroup)
                    accR[g] = a;
                else
                    accN = a;
            }
        }
        __syncthreads();
    }
    // S[i][q] (i < PMAX) and R[i + 1][q] for i = g kGroup + (oi mod kGroup); N[q]; R[0][q] = 0. Groups the
    // block skipped left their sums at +0.
    if (owner) {
        const uint64_t qq = q0 + oq;
        if (qq < sd.chains) {
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                if (oi < kGroup) {
                    const int i = g * kGroup + oi;
                    if (i < PMAX) sd.S[(uint64_t)i * sd.chains + qq] = accS[g];
                } else if (oi < 2 * kGroup) {
                    const int i = g * kGroup + oi - kGroup;
                    if (i < PMAX) sd.R[(uint64_t)(i + 1) * sd.chains + qq] = accR[g];
                }
            }
            if (oi == 2 * kGroup) sd.N[qq] = accN;
        }
    }
    if (t < kChains && q0 + t < sd.chains) sd.R[q0 + t] = 0.0;
}

template <int PMAX>
void launch_terms(const TermsSide& A, const TermsSide& B, const I1Format& f, cudaStream_t st) {
    const uint32_t a_blocks = (uint32_t)((A.chains + kChains - 1) / kChains);
    const uint32_t b_blocks = (uint32_t)((B.chains + kChains - 1) / kChains);
    terms_kernel<PMAX><<<a_blocks + b_blocks, kTermsThreads, 0, st>>>(A, B, a_blocks, f.radix, f.dmax,
                                                                     weights_of(f.radix));
    OZTT_CUDA(cudaGetLastError());
}

void launch_terms_any(int pmax, const TermsSide& A, const TermsSide& B, const I1Format& f, cudaStream_t st) {
    switch (pmax) {
    case 22: launch_terms<22>(A, B, f, st); break;
    case 28: launch_terms<28>(A, B, f, st); break;
    case 33: launch_terms<33>(A, B, f, st); break;
    default: throw Error(OZTT_EINVAL, "scheme I: no device slice-selection kernel for this radix");
    }
}

// ---- model (2) on the sampled rows and columns ----------------------------------------------------
// XA[s][c] = a[rows[s]][c] and YB[u][c] = b[c][cols[u]], the sampled values unscaled.
__global__ void __launch_bounds__(256) gather_kernel(const double* __restrict__ a, const double* __restrict__ b,
                                                     uint64_t n, uint64_t k, const uint32_t* __restrict__ rows,
                                                     const uint32_t* __restrict__ cols, uint32_t na, uint32_t nb,
                                                     double* __restrict__ XA, double* __restrict__ YB) {
    const uint64_t total = (uint64_t)(na + nb) * k;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t s = t / k, c = t % k;
        if (s < na)
            XA[s * k + c] = __ldg(a + (uint64_t)rows[s] * k + c);
        else
            YB[(s - na) * k + c] = __ldg(b + c * n + cols[s - na]);
    }
}

// C of each sampled pair (s, u), scaled: the compensated dot product of the host planner (TwoProduct by
// FMA, TwoSum on the high word, the low parts summed plainly), c ascending.
__global__ void __launch_bounds__(128) sample_c_kernel(const double* __restrict__ XA, const double* __restrict__ YB,
                                                       uint32_t na, uint32_t nb, uint64_t k, double rgA, double rgB,
                                                       double* __restrict__ Ch, double* __restrict__ Cl) {
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)na * nb) return;
    const uint64_t s = t / nb, u = t % nb;
    const double* x = XA + s * k;
    const double* y = YB + u * k;
    double hi = 0.0, lo = 0.0;
    for (uint64_t c = 0; c < k; ++c) {
        const double xv = __dmul_rn(__ldg(x + c), rgA), yv = __dmul_rn(__ldg(y + c), rgB);
        const double pr = __dmul_rn(xv, yv), pe = __fma_rn(xv, yv, -pr);
        double v, ve;
        two_sum_d(hi, pr, v, ve);
        hi = v;
        lo = __dadd_rn(lo, __dadd_rn(pe, ve));
    }
    two_sum_d(hi, lo, Ch[t], Cl[t]);
}

// One chunk's sum of the terms q slices drop, for one pair: thread (ch, s, u), c over the chunk
// [K ch / 64, min(K (ch + 1) / 64, k)) of the padded K. X (row s) and Y (column u) are the sampled values
// scaled by 2^shx[s], 2^shy[u] and expanded q steps as in the host planner: digits D_i w_i (i < q) and
// the residual of X after q steps, residuals of Y after r = 1..q steps;
// e = RX Y + sum_i D_i RY_(q-i), summed in c order.
template <int PMAX>
__global__ void __launch_bounds__(128) sample_err_kernel(const double* __restrict__ XA, const double* __restrict__ YB,
                                                         uint32_t na, uint32_t nb, uint64_t k, uint64_t K,
                                                         const int32_t* __restrict__ shx,
                                                         const int32_t* __restrict__ shy, int q, double radix,
                                                         double dmax, const Weights wt,
                                                         double* __restrict__ part) {
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t pairs = (uint64_t)na * nb;
    if (t >= pairs * kI1Chunks) return;
    const uint64_t ch = t / pairs, su = t % pairs, s = su / nb, u = su % nb;
    const uint64_t k0 = K * ch / kI1Chunks, k1 = min(K * (ch + 1) / kI1Chunks, k);
    const double px = pow2d(shx[s]), py = pow2d(shy[u]);
    double acc = 0.0;
    for (uint64_t c = k0; c < k1; ++c) {
        double D[PMAX], RY[PMAX + 1];
        double th = __dmul_rn(__ldg(XA + s * k + c), px), tl = 0.0;
#pragma unroll
        for (int i = 0; i < PMAX; ++i) {
            if (i < q) {
                const double dg = expand_step(th, tl, radix, dmax);
                D[i] = __dmul_rn(dg, wt.w[i]);
            }
        }
        const double rx = __dmul_rn(__dadd_rn(th, tl), wt.w[q - 1]);
        const double yk = __dmul_rn(__ldg(YB + u * k + c), py);
        th = yk;
        tl = 0.0;
#pragma unroll
        for (int r = 1; r <= PMAX; ++r) {
            if (r <= q) {
                (void)expand_step(th, tl, radix, dmax);
                RY[r] = __dmul_rn(__dadd_rn(th, tl), wt.w[r - 1]);
            }
        }
        double e = __dmul_rn(rx, yk);
#pragma unroll
        for (int i = 0; i < PMAX; ++i)
            if (i < q) e = __dadd_rn(e, __dmul_rn(D[i], RY[q - i]));
        acc = __dadd_rn(acc, e);
    }
    part[t] = acc;
}

template <int PMAX>
void launch_sample_err(const double* XA, const double* YB, uint32_t na, uint32_t nb, uint64_t k, uint64_t K,
                       const int32_t* shx, const int32_t* shy, int q, const I1Format& f, double* part,
                       cudaStream_t st) {
    const uint64_t threads = (uint64_t)na * nb * kI1Chunks;
    sample_err_kernel<PMAX><<<(unsigned)((threads + 127) / 128), 128, 0, st>>>(XA, YB, na, nb, k, K, shx, shy, q,
                                                                               f.radix, f.dmax, weights_of(f.radix),
                                                                               part);
    OZTT_CUDA(cudaGetLastError());
}

}  // namespace

// Model (2) with its sums on the device: the sample picked on the host from the normalization, the
// sampled rows and columns gathered from a_dev, b_dev, C of the pairs and each q's chunk sums computed
// there, the host finishing with the host planner's code.
class DeviceSample {
public:
    DeviceSample(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t K, const I1Format& f,
                 const I1Normalization& nm, double nC, cudaStream_t st)
        : k_(k), K_(K), f_(f), nm_(nm), st_(st), sp_(i1_pick(nm)), na_((uint32_t)sp_.rows.size()),
          nb_((uint32_t)sp_.cols.size()), XA_(st, (uint64_t)std::max(na_, 1u) * k * 8),
          YB_(st, (uint64_t)std::max(nb_, 1u) * k * 8), shx_(st, std::max(na_, 1u) * 4), shy_(st, std::max(nb_, 1u) * 4),
          part_(st, (uint64_t)std::max(na_ * nb_, 1u) * kI1Chunks * 8) {
        (void)m;
        if (!na_ || !nb_) return;
        DevBuf rows(st, na_ * 4), cols(st, nb_ * 4);
        std::vector<int32_t> shx(na_), shy(nb_);
        for (uint32_t s = 0; s < na_; ++s) shx[s] = f.nshift - nm.eA[sp_.rows[s]];
        for (uint32_t u = 0; u < nb_; ++u) shy[u] = f.nshift - nm.eB[sp_.cols[u]];
        OZTT_CUDA(cudaMemcpyAsync(rows.p, sp_.rows.data(), na_ * 4, cudaMemcpyHostToDevice, st));
        OZTT_CUDA(cudaMemcpyAsync(cols.p, sp_.cols.data(), nb_ * 4, cudaMemcpyHostToDevice, st));
        OZTT_CUDA(cudaMemcpyAsync(shx_.p, shx.data(), na_ * 4, cudaMemcpyHostToDevice, st));
        OZTT_CUDA(cudaMemcpyAsync(shy_.p, shy.data(), nb_ * 4, cudaMemcpyHostToDevice, st));
        const uint64_t total = (uint64_t)(na_ + nb_) * k;
        gather_kernel<<<(unsigned)std::min<uint64_t>((total + 255) / 256, 4096), 256, 0, st>>>(
            a, b, n, k, rows.as<uint32_t>(), cols.as<uint32_t>(), na_, nb_, XA_.as<double>(), YB_.as<double>());
        OZTT_CUDA(cudaGetLastError());
        DevBuf ch(st, (uint64_t)na_ * nb_ * 8), cl(st, (uint64_t)na_ * nb_ * 8);
        sample_c_kernel<<<(unsigned)(((uint64_t)na_ * nb_ + 127) / 128), 128, 0, st>>>(
            XA_.as<double>(), YB_.as<double>(), na_, nb_, k, nm.rgA, nm.rgB, ch.as<double>(), cl.as<double>());
        OZTT_CUDA(cudaGetLastError());
        Ch_.resize((size_t)na_ * nb_);
        Cl_.resize((size_t)na_ * nb_);
        OZTT_CUDA(cudaMemcpyAsync(Ch_.data(), ch.p, Ch_.size() * 8, cudaMemcpyDeviceToHost, st));
        OZTT_CUDA(cudaMemcpyAsync(Cl_.data(), cl.p, Cl_.size() * 8, cudaMemcpyDeviceToHost, st));
        OZTT_CUDA(cudaStreamSynchronize(st));
        norm2_ = i1_sample_norm2(sp_, Ch_, nC);
    }
    // model (2)'s error for q slices
    double err2(int q) {
        if (!na_ || !nb_) return 0.0;
        const int pmax = i1_pmax(f_);
        if (q < 1 || q > pmax) throw Error(OZTT_EINVAL, "scheme I: slice count outside the search range");
        const int32_t *shx = shx_.as<int32_t>(), *shy = shy_.as<int32_t>();
        double* part = part_.as<double>();
        switch (pmax) {
        case 22: launch_sample_err<22>(XA_.as<double>(), YB_.as<double>(), na_, nb_, k_, K_, shx, shy, q, f_, part, st_); break;
        case 28: launch_sample_err<28>(XA_.as<double>(), YB_.as<double>(), na_, nb_, k_, K_, shx, shy, q, f_, part, st_); break;
        case 33: launch_sample_err<33>(XA_.as<double>(), YB_.as<double>(), na_, nb_, k_, K_, shx, shy, q, f_, part, st_); break;
        default: throw Error(OZTT_EINVAL, "scheme I: no device slice-selection kernel for this radix");
        }
        std::vector<double> host((size_t)na_ * nb_ * kI1Chunks);
        OZTT_CUDA(cudaMemcpyAsync(host.data(), part, host.size() * 8, cudaMemcpyDeviceToHost, st_));
        OZTT_CUDA(cudaStreamSynchronize(st_));
        return i1_model2_finish(host.data(), kI1Chunks, sp_, Ch_, Cl_, nm_, norm2_);
    }

private:
    uint64_t k_;
    uint32_t K_;
    I1Format f_;
    const I1Normalization& nm_;
    cudaStream_t st_;
    I1SamplePick sp_;
    uint32_t na_, nb_;
    DevBuf XA_, YB_, shx_, shy_, part_;
    std::vector<double> Ch_, Cl_;
    double norm2_ = 0;
};

I1Terms measure_i1_terms(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                         const I1Normalization& nm, const I1Format& f, cudaStream_t st);

// The normalization and model (1)'s terms of device-resident a (m x k) and b (k x n), with nC; the stream
// is synchronised.
void measure_i1_device(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                       const I1Format& f, cudaStream_t st, I1Normalization& nm, I1Terms& terms, double& nC) {
    std::vector<uint64_t> row_max, col_max;
    std::vector<double> nrA, nrB;
    double rg[2] = {1.0, 1.0};
    {
        PolicyStatsRun run(m, n, k, N, st);
        run.b_cols(b, 0, n);
        run.b_done(b);
        run.a_cols(a, 0, k);
        run.a_done(a);
        nC = run.collect(&row_max, &col_max, &nrA, &nrB, rg).nC;
    }
    nm = i1_normalization(rg[0], rg[1], row_max.data(), col_max.data(), nrA.data(), nrB.data(), m, n, f);
    terms = measure_i1_terms(a, b, m, n, k, nm, f, st);
}

// Model (1)'s per-k sums of device-resident a, b with a given normalization; the stream is synchronised.
I1Terms measure_i1_terms(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k,
                         const I1Normalization& nm, const I1Format& f, cudaStream_t st) {
    const int pmax = i1_pmax(f);
    const uint64_t P1 = (uint64_t)pmax + 1;
    I1Terms terms;
    // per row of A / column of B: the divisor and the shift nshift - e (0 where the row is not counted)
    std::vector<int32_t> shA(m, 0), shB(n, 0);
    for (uint64_t i = 0; i < m; ++i)
        if (nm.sA[i] > 0) shA[i] = f.nshift - nm.eA[i];
    for (uint64_t j = 0; j < n; ++j)
        if (nm.sB[j] > 0) shB[j] = f.nshift - nm.eB[j];
    DevBuf dsA(st, m * 8), dsB(st, n * 8), dshA(st, m * 4), dshB(st, n * 4);
    DevBuf SA(st, P1 * k * 8), RA(st, P1 * k * 8), SB(st, P1 * k * 8), RB(st, P1 * k * 8), NA(st, k * 8),
        NB(st, k * 8);
    OZTT_CUDA(cudaMemcpyAsync(dsA.p, nm.sA.data(), m * 8, cudaMemcpyHostToDevice, st));
    OZTT_CUDA(cudaMemcpyAsync(dsB.p, nm.sB.data(), n * 8, cudaMemcpyHostToDevice, st));
    OZTT_CUDA(cudaMemcpyAsync(dshA.p, shA.data(), m * 4, cudaMemcpyHostToDevice, st));
    OZTT_CUDA(cudaMemcpyAsync(dshB.p, shB.data(), n * 4, cudaMemcpyHostToDevice, st));
    OZTT_CUDA(cudaMemsetAsync(SA.p, 0, P1 * k * 8, st));  // row pmax of S stays zero
    OZTT_CUDA(cudaMemsetAsync(SB.p, 0, P1 * k * 8, st));
    // A: thread c walks rows i (elements i*k + c); B: thread r walks columns j (elements r*n + j); one launch
    const TermsSide sa{a, k, m, 1, k, dsA.as<double>(), dshA.as<int32_t>(), nm.rgA, SA.as<double>(), RA.as<double>(),
                       NA.as<double>()};
    const TermsSide sb{b, k, n, n, 1, dsB.as<double>(), dshB.as<int32_t>(), nm.rgB, SB.as<double>(), RB.as<double>(),
                       NB.as<double>()};
    launch_terms_any(pmax, sa, sb, f, st);
    terms.SA.resize(P1 * k);
    terms.RA.resize(P1 * k);
    terms.SB.resize(P1 * k);
    terms.RB.resize(P1 * k);
    terms.NA.resize(k);
    terms.NB.resize(k);
    OZTT_CUDA(cudaMemcpyAsync(terms.SA.data(), SA.p, P1 * k * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaMemcpyAsync(terms.RA.data(), RA.p, P1 * k * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaMemcpyAsync(terms.SB.data(), SB.p, P1 * k * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaMemcpyAsync(terms.RB.data(), RB.p, P1 * k * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaMemcpyAsync(terms.NA.data(), NA.p, k * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaMemcpyAsync(terms.NB.data(), NB.p, k * 8, cudaMemcpyDeviceToHost, st));
    OZTT_CUDA(cudaStreamSynchronize(st));
    return terms;
}

// The same with the normalization and nC already measured (the streamed upload measures them on the way).
int plan_i_measured(const double* a_dev, const double* b_dev, uint64_t m, uint64_t n, uint64_t k, uint32_t slices,
                    const I1Format& f, const I1Normalization& nm, double nC, oztt_i_plan& p, std::string& err,
                    cudaStream_t st) {
    return plan_i_with(
        [&](uint32_t M, uint32_t N, uint32_t K) {
            (void)N;
            const I1Terms terms = measure_i1_terms(a_dev, b_dev, m, n, k, nm, f, st);
            DeviceSample sample(a_dev, b_dev, m, n, k, K, f, nm, nC, st);
            return i1_select_with(terms, m, n, k, M, N, K, f, nC, [&](int q) { return sample.err2(q); });
        },
        m, n, k, slices, f, p, err);
}

// The Scheme I plan with the slice count selected from statistics measured on the device (a_dev, b_dev),
// both models' sums included; the host planner's plan.
int plan_i_device(const double* a_dev, const double* b_dev, uint64_t m, uint64_t n, uint64_t k, uint32_t slices,
                  const I1Format& f, oztt_i_plan& p, std::string& err, cudaStream_t st) {
    return plan_i_with(
        [&](uint32_t M, uint32_t N, uint32_t K) {
            I1Normalization nm;
            I1Terms terms;
            double nC = 0;
            measure_i1_device(a_dev, b_dev, m, n, k, N, f, st, nm, terms, nC);
            DeviceSample sample(a_dev, b_dev, m, n, k, K, f, nm, nC, st);
            return i1_select_with(terms, m, n, k, M, N, K, f, nC, [&](int q) { return sample.err2(q); });
        },
        m, n, k, slices, f, p, err);
}

}  // namespace oztt

namespace oztt {

void run_i_device(const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                  const oztt_i_plan& plan, cudaStream_t st, double* stage_ms);
double product_norm_estimate(const double* a, const double* b, uint64_t m, uint64_t n, uint64_t k, uint32_t N,
                             double rgA, double rgB);

// Context::gemm's Scheme I call: A and B to the device once, the slice count selected from statistics
// measured there (slices 0), the feasibility checks, the pipeline on the resident operands, C back.
int run_i_uploaded(int device_id, const double* a, const double* b, double* c, uint64_t m, uint64_t n, uint64_t k,
                   uint32_t slices, const I1Format& f, oztt_i_plan& p, std::string& err) {
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
        inner = plan_i_device(da.as<double>(), db.as<double>(), m, n, k, slices, f, p, err, st);
        if (inner != OZTT_OK) return;
        DevBuf dc(st, m * n * 8);
        run_i_device(da.as<double>(), db.as<double>(), dc.as<double>(), m, n, k, p, st, nullptr);
        OZTT_CUDA(cudaMemcpyAsync(c, dc.p, m * n * 8, cudaMemcpyDeviceToHost, st));
        OZTT_CUDA(cudaStreamSynchronize(st));
    });
    if (rc != OZTT_OK) err = buf;
    return rc != OZTT_OK ? rc : inner;
}

}  // namespace oztt

using oztt::Error;
using oztt::guarded;

extern "C" {

int oztt_i_format_plan_device(int32_t format, const double* a_dev, const double* b_dev, uint64_t m, uint64_t n,
                              uint64_t k, uint32_t slices, oztt_i_plan* plan, void* stream, char* err,
                              size_t errlen) {
    return guarded(err, errlen, [&] {
        const oztt::I1Format* f = oztt::i1_format(format);
        if (!f) throw Error(OZTT_EINVAL, "format is unknown or was not built");
        if (!plan || (slices == 0 && (!a_dev || !b_dev))) throw Error(OZTT_EINVAL, "null argument");
        std::string msg;
        const int rc = oztt::plan_i_device(a_dev, b_dev, m, n, k, slices, *f, *plan, msg,
                                           reinterpret_cast<cudaStream_t>(stream));
        if (rc != OZTT_OK) throw Error(rc, msg);
    });
}

int oztt_i_model1_errors(int32_t format, const double* a, const double* b, const double* a_dev, const double* b_dev,
                         uint64_t m, uint64_t n, uint64_t k, double* out, int32_t count, void* stream, char* err,
                         size_t errlen) {
    return guarded(err, errlen, [&] {
        const oztt::I1Format* f = oztt::i1_format(format);
        if (!f) throw Error(OZTT_EINVAL, "format is unknown or was not built");
        if (!out || count < 1 || !m || !n || !k || (!a_dev && (!a || !b)) || (a_dev && !b_dev))
            throw Error(OZTT_EINVAL, "model1_errors: bad arguments");
        const uint32_t N = (uint32_t)((n + 63) / 64 * 64);
        std::vector<double> e2;
        double nC = 0;
        if (a_dev) {
            oztt::I1Normalization nm;
            oztt::I1Terms terms;
            oztt::measure_i1_device(a_dev, b_dev, m, n, k, N, *f, reinterpret_cast<cudaStream_t>(stream), nm, terms,
                                    nC);
            e2 = oztt::i1_model1_errors(nullptr, nullptr, m, n, k, *f, &terms, nullptr);
        } else {
            e2 = oztt::i1_model1_errors(a, b, m, n, k, *f, nullptr, nullptr);
            double rgA = 1.0 / oztt::pow2_normalizer(a, m, k, k), rgB = 1.0 / oztt::pow2_normalizer(b, k, n, n);
            nC = oztt::product_norm_estimate(a, b, m, n, k, N, rgA, rgB);
        }
        for (int32_t i = 0; i < count; ++i) out[i] = i == 0 ? nC : (i < (int32_t)e2.size() ? e2[i] : 0.0);
    });
}

}  // extern "C"
