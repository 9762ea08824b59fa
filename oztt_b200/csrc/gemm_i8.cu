// SPDX-License-Identifier: Apache-2.0
//
// Per-modulus residue products on the 5th-generation tensor cores (sm_100a):
//     C_s = A_s * B_s^T,  A_s [mp x kp] int8, B_s [np x kp] int8 (both K-major), s = 0..S-1,
// exactly, in s32 accumulators in tensor memory, with the modular reduction fused into the epilogue.
// Replaces the reference's GEMM stage (run_int8_gemms, src/ozaki2.cpp:333-348, one Metalium
// workload per modulus and output panel; kernels/bmm_int32_spill.cpp) by one persistent launch for
// all S moduli.
//
// Structure (one CTA per SM, 192 threads):
//   warp 0      TMA producer: 128x128 A and 256x128 B int8 boxes (128-byte swizzle) into a 4-stage
//               shared-memory ring; completion is counted in bytes on the stage's mbarrier.
//   warp 1      MMA issuer: one thread issues tcgen05.mma.cta_group::1.kind::i8 (M=128, N=256, K=32;
//               4 per stage) into one of two 256-column TMEM accumulators and releases each stage
//               with tcgen05.commit; allocates and frees the 512 TMEM columns.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator rows (warp w reads lanes 32*(w%4)..+31),
//               then either the raw int32 C_s (mode 0, for bit-exact checks) or the CRT digit
//               k_s = (C_s mod m_s) * y_s mod m_s as uint8 (mode 1), stored to HBM; the accumulator
//               is handed back to the MMA warp while the next tile accumulates in the other one.
// Tiles are scheduled persistently: tile t -> (modulus s, tile row, tile column) with the rows of
// each modulus taken in groups of 16 so that the CTAs running at one time share A and B panels in
// L2. TMA loads never use cluster multicast.
//
// Every mbarrier wait is bounded (2 s of global time). On a timeout the CTA records an error code,
// all roles leave their loops, the producer waits (bounded) for the loads it issued, the MMA thread
// waits (bounded) for its last commit, and the TMEM is freed before the kernel returns; the host
// reports the code as a runtime error.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "oztt_common.cuh"

namespace oztt {
namespace gemm {

constexpr uint32_t BM = 128, BN = 256, BK = 128, UK = 32;
constexpr uint32_t STAGES = 4;
constexpr uint32_t A_BYTES = BM * BK;
constexpr uint32_t B_BYTES = BN * BK;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t ACC_COLS = BN;
constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
constexpr uint32_t NUM_THREADS = 192;
constexpr uint32_t GROUP_M = 16;
constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 256 + 1024;
constexpr uint64_t TIMEOUT_NS = 2000000000ull;

// Instruction descriptor of kind::i8: s32 accumulator, signed A and B, both K-major, N=256, M=128.
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((BN >> 3) << 17) | ((BM >> 4) << 24);

enum ErrCode : int { ERR_WAIT_PRODUCER = 1, ERR_WAIT_MMA_FULL = 2, ERR_WAIT_MMA_EMPTY = 4, ERR_WAIT_EPILOGUE = 8 };

struct EpiConst {
    uint32_t S;
    uint32_t m[OZTT_MAXS], y[OZTT_MAXS], magic[OZTT_MAXS], shift[OZTT_MAXS];
    // FP8 digit products (modes 3 and 4): the outputs of modulus s are oout[s] .. oout[s+1]-1; output u
    // sums the products of A digit plane out_a[u] + t and B digit plane out_b[u] - t over t < out_g[u]
    // (the concatenation along K); weight[u] = (composition coefficient * y_s) mod m_s.
    uint16_t oout[OZTT_MAXS + 1];
    uint8_t out_a[OZTT_MAXOUT], out_b[OZTT_MAXOUT], out_g[OZTT_MAXOUT];
    uint16_t weight[OZTT_MAXOUT];
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase of `parity` to complete. Gives up when another role raised the abort flag or
// after limit_ns (then records `code` and raises the flag). Returns true when the phase completed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code, uint64_t limit_ns = TIMEOUT_NS) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > limit_ns) {
                atomicOr(err, code);
                *abort_flag = 1;
                return false;
            }
        }
    }
}
// Bounded wait used on the abort path only (ignores the abort flag).
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_timer_ns() - t0 > limit_ns) return;
}

__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint32_t dst, uint64_t* bar, int32_t c0,
                                            int32_t c1, int32_t c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// Shared-memory matrix descriptor: K-major operand in 128-byte-swizzled 8-row atoms (1024 bytes
// apart), descriptor version 1.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// floor(a / m) for a < 2^31 with a precomputed (magic, shift) pair (round-up reciprocal method).
__device__ __forceinline__ uint32_t udiv_small(uint32_t a, uint32_t magic, uint32_t shift) {
    return (__umulhi(a, magic) + a) >> shift;
}

__device__ __forceinline__ void decode_tile(uint32_t tile, uint32_t tiles_m, uint32_t tiles_n, uint32_t& s,
                                            uint32_t& tm, uint32_t& tn) {
    const uint32_t per_s = tiles_m * tiles_n;
    s = tile / per_s;
    const uint32_t r = tile - s * per_s;
    const uint32_t span = GROUP_M * tiles_n;
    const uint32_t g = r / span;
    const uint32_t first = g * GROUP_M;
    const uint32_t gsz = min(tiles_m - first, GROUP_M);
    const uint32_t rr = r - g * span;
    tm = first + rr % gsz;
    tn = rr / gsz;
}

// Work of one output tile: the output plane, the tile row and column, and the number of 128-wide
// K blocks. Modes 0 and 1 (scheme II): plane = modulus s, num_kb blocks of A_s and B_s. Mode 2
// (scheme I): plane = diagonal d, taken from the largest down so that the longest tiles start first,
// over the concatenation of the d+1 slice pairs (A_i, B_{d-i}): (d+1)*num_kb blocks.
template <int MODE>
__device__ __forceinline__ void tile_work(uint32_t tile, uint32_t planes, uint32_t tiles_m, uint32_t tiles_n,
                                          uint32_t num_kb, uint32_t& plane, uint32_t& tm, uint32_t& tn,
                                          uint32_t& kb_total) {
    uint32_t s;
    decode_tile(tile, tiles_m, tiles_n, s, tm, tn);
    if constexpr (MODE == 2) {
        plane = planes - 1u - s;
        kb_total = (plane + 1u) * num_kb;
    } else {
        plane = s;
        kb_total = num_kb;
    }
}
// Coordinates (K offset, slice/modulus plane) of K block kb of a tile for A and for B.
template <int MODE>
__device__ __forceinline__ void kblock_coords(uint32_t kb, uint32_t plane, uint32_t num_kb, int32_t& k_el,
                                              int32_t& pa, int32_t& pb) {
    if constexpr (MODE == 2) {
        const uint32_t i = kb / num_kb;
        k_el = (int32_t)((kb - i * num_kb) * BK);
        pa = (int32_t)i;
        pb = (int32_t)(plane - i);
    } else {
        k_el = (int32_t)(kb * BK);
        pa = pb = (int32_t)plane;
    }
}

// Accumulator units of a tile: one for modes 0-2; for the digit modes 3 and 4 one per GEMM output of
// the tile's modulus, each accumulated in its own TMEM buffer.
template <int MODE>
__device__ __forceinline__ void tile_units(uint32_t plane, const EpiConst& ec, uint32_t& u0, uint32_t& u1) {
    if constexpr (MODE >= 3) {
        u0 = ec.oout[plane];
        u1 = ec.oout[plane + 1];
    } else {
        u0 = 0;
        u1 = 1;
    }
}
// The operand planes of unit u: g pairs (A plane a0 + t, B plane b0 - t), each over all K blocks.
template <int MODE>
__device__ __forceinline__ void unit_operands(uint32_t plane, uint32_t u, const EpiConst& ec, uint32_t& a0,
                                              uint32_t& b0, uint32_t& g) {
    if constexpr (MODE >= 3) {
        a0 = ec.out_a[u];
        b0 = ec.out_b[u];
        g = ec.out_g[u];
    } else if constexpr (MODE == 2) {
        a0 = 0;
        b0 = plane;
        g = plane + 1;
    } else {
        a0 = b0 = plane;
        g = 1;
    }
}

template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    residue_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        void* __restrict__ out, uint32_t tiles_m, uint32_t tiles_n, uint32_t num_kb, uint64_t mp,
                        uint64_t np, const EpiConst ec, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty_bar = full_bar + STAGES;
    uint64_t* tfull_bar = empty_bar + STAGES;
    uint64_t* tempty_bar = tfull_bar + 2;
    uint64_t* drain_bar = tempty_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t num_tiles = ec.S * tiles_m * tiles_n;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < STAGES; ++s) {
            mbar_init(full_bar + s, 1);
            mbar_init(empty_bar + s, 1);
        }
        for (uint32_t a = 0; a < 2; ++a) {
            mbar_init(tfull_bar + a, 1);
            mbar_init(tempty_bar + a, 128);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
            uint32_t stage = 0, phase = 0;
            uint32_t filled = 0, last_phase = 0;  // per-stage bit masks of the last fill
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                uint32_t plane, tm, tn, kb_total, u0, u1;
                tile_work<MODE>(tile, ec.S, tiles_m, tiles_n, num_kb, plane, tm, tn, kb_total);
                tile_units<MODE>(plane, ec, u0, u1);
                for (uint32_t u = u0; ok && u < u1; ++u) {
                    uint32_t a0, b0, g;
                    unit_operands<MODE>(plane, u, ec, a0, b0, g);
                    for (uint32_t t = 0; ok && t < g; ++t)
                        for (uint32_t kb = 0; kb < num_kb; ++kb) {
                            if (!mbar_wait(empty_bar + stage, phase ^ 1u, abort_flag, err, ERR_WAIT_PRODUCER)) {
                                ok = false;
                                break;
                            }
                            const int32_t k_el = (int32_t)(kb * BK);
                            mbar_expect_tx(full_bar + stage, STAGE_BYTES);
                            const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
                            tma_load_3d(&tmA, sa, full_bar + stage, k_el, (int32_t)(tm * BM), (int32_t)(a0 + t));
                            tma_load_3d(&tmB, sa + A_BYTES, full_bar + stage, k_el, (int32_t)(tn * BN),
                                        (int32_t)(b0 - t));
                            filled |= 1u << stage;
                            last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
                            if (++stage == STAGES) {
                                stage = 0;
                                phase ^= 1u;
                            }
                        }
                }
            }
            if (!ok)  // let every load this thread issued land before the CTA may exit
                for (uint32_t st = 0; st < STAGES; ++st)
                    if (filled & (1u << st)) mbar_wait_drain(full_bar + st, (last_phase >> st) & 1u, 200000000ull);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                uint32_t plane, tm, tn, kb_total, u0, u1;
                tile_work<MODE>(tile, ec.S, tiles_m, tiles_n, num_kb, plane, tm, tn, kb_total);
                tile_units<MODE>(plane, ec, u0, u1);
                for (uint32_t u = u0; ok && u < u1; ++u) {
                    uint32_t a0, b0, g;
                    unit_operands<MODE>(plane, u, ec, a0, b0, g);
                    if (!mbar_wait(tempty_bar + acc, acc_phase ^ 1u, abort_flag, err, ERR_WAIT_MMA_EMPTY)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
                    for (uint32_t t = 0; ok && t < g; ++t)
                        for (uint32_t kb = 0; kb < num_kb; ++kb) {
                            if (!mbar_wait(full_bar + stage, phase, abort_flag, err, ERR_WAIT_MMA_FULL)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + A_BYTES;
#pragma unroll
                            for (uint32_t k = 0; k < BK / UK; ++k)
                                umma_i8(d_tmem, sdesc_sw128(sa + k * UK), sdesc_sw128(sb + k * UK),
                                        (t | kb | k) != 0u);
                            umma_commit(empty_bar + stage);
                            if (++stage == STAGES) {
                                stage = 0;
                                phase ^= 1u;
                            }
                        }
                    if (!ok) break;
                    umma_commit(tfull_bar + acc);
                    acc ^= 1u;
                    if (acc == 0) acc_phase ^= 1u;
                }
            }
            // Every MMA this thread issued completes before the columns are freed.
            umma_commit(drain_bar);
            mbar_wait_drain(drain_bar, 0, 1000000000ull);
        }
    } else {
        const uint32_t quarter = warp & 3u;
        uint32_t acc = 0, acc_phase = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
            uint32_t s, tm, tn, kb_total, u0, u1;
            tile_work<MODE>(tile, ec.S, tiles_m, tiles_n, num_kb, s, tm, tn, kb_total);
            tile_units<MODE>(s, ec, u0, u1);
            for (uint32_t u = u0; u < u1; ++u) {
                if (!mbar_wait(tfull_bar + acc, acc_phase, abort_flag, err, ERR_WAIT_EPILOGUE)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t row = (uint64_t)tm * BM + quarter * 32u + lane;
                const uint32_t tbase = tmem_base + ((quarter * 32u) << 16) + acc * ACC_COLS;
                const uint32_t m = ec.m[s % OZTT_MAXS], y = ec.y[s % OZTT_MAXS], mg = ec.magic[s % OZTT_MAXS],
                               sh = ec.shift[s % OZTT_MAXS];
                const uint32_t out_plane = MODE == 4 ? u : s;
#pragma unroll 1
                for (uint32_t c = 0; c < BN; c += 32) {
                    uint32_t v[32];
                    tmem_ld32(tbase + c, v);
                    const uint64_t off = ((uint64_t)out_plane * mp + row) * np + (uint64_t)tn * BN + c;
                    if constexpr (MODE == 0 || MODE == 2 || MODE == 4) {
                        uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<int32_t*>(out) + off);
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            o[q] = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    } else if constexpr (MODE == 1) {
                        uint32_t w[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q) w[q] = 0;
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const int32_t cv = (int32_t)v[e];
                            const uint32_t a = cv < 0 ? (uint32_t)(-cv) : (uint32_t)cv;
                            uint32_t r = a - udiv_small(a, mg, sh) * m;
                            if (cv < 0 && r) r = m - r;
                            const uint32_t t = r * y;
                            const uint32_t kk = t - udiv_small(t, mg, sh) * m;
                            w[e >> 2] |= kk << (8 * (e & 3));
                        }
                        uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(out) + off);
                        o[0] = make_uint4(w[0], w[1], w[2], w[3]);
                        o[1] = make_uint4(w[4], w[5], w[6], w[7]);
                    } else {
                        // Composition into the CRT digit k_s = sum_u weight_u (P_u mod m) mod m, uint16: the
                        // first output of the modulus writes its term, the later ones add to what this same
                        // thread wrote for the previous output (a plain load of its own store).
                        const uint32_t wgt = ec.weight[u];
                        uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + off);
                        uint32_t w[16];
                        if (u == u0) {
#pragma unroll
                            for (int q = 0; q < 16; ++q) w[q] = 0;
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const uint4 pv = o[q];
                                w[4 * q] = pv.x;
                                w[4 * q + 1] = pv.y;
                                w[4 * q + 2] = pv.z;
                                w[4 * q + 3] = pv.w;
                            }
                        }
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const int32_t cv = (int32_t)v[e];
                            const uint32_t a = cv < 0 ? (uint32_t)(-cv) : (uint32_t)cv;
                            uint32_t r = a - udiv_small(a, mg, sh) * m;
                            if (cv < 0 && r) r = m - r;
                            const uint32_t t = r * wgt;
                            uint32_t kk = t - udiv_small(t, mg, sh) * m + ((w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
                            if (kk >= m) kk -= m;
                            w[e >> 1] = (w[e >> 1] & (0xFFFF0000u >> (16 * (e & 1)))) | (kk << (16 * (e & 1)));
                        }
#pragma unroll
                        for (int q = 0; q < 4; ++q) o[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
                    }
                }
                tc_fence_before();
                mbar_arrive(tempty_bar + acc);
                acc ^= 1u;
                if (acc == 0) acc_phase ^= 1u;
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
    }
}

// ---- CTA pairs: tcgen05.mma.cta_group::2 -------------------------------------------------------
// The same work with two CTAs (one per SM of a cluster pair) sharing each MMA: M = 256 rows of A
// (128 in each CTA's shared memory) against N = 256 rows of B (128 in each CTA), so that each SM
// stages 32 KB per 128-deep K block instead of 48 KB for the same 128 x 256 output per SM. The leader
// CTA (rank 0) issues the MMAs; both CTAs load their halves with TMA (no multicast), completing bytes
// on the leader's stage barrier; the leader's tcgen05.commit releases the stage in both CTAs and hands
// each CTA its 128 x 256 accumulator half; the epilogue warps of both CTAs report a drained
// accumulator to the leader. Six stages of 32 KB per CTA.
namespace pair {

constexpr uint32_t BM = 128, BN = 256, BNH = 128, BK = 128, UK = 32;
constexpr uint32_t STAGES = 6;
constexpr uint32_t A_BYTES = BM * BK;
constexpr uint32_t B_BYTES = BNH * BK;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t ACC_COLS = BN;
constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
constexpr uint32_t NUM_THREADS = 192;
constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 256 + 1024;
// kind::i8, s32 accumulator, signed A and B, K-major, N = 256, M = 256 (the pair).
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((BN >> 3) << 17) | ((256u >> 4) << 24);
constexpr uint64_t PEER_DRAIN_NS = 5000000ull;

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory, completing its bytes on a barrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_3d_pair(const CUtensorMap* map, uint32_t dst, uint32_t bar_cluster,
                                                 int32_t c0, int32_t c1, int32_t c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
        "%5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
        : "memory");
}
// Arrives once on the barrier at `bar_cluster` (either CTA) when all MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}

}  // namespace pair

template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::NUM_THREADS, 1)
    residue_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             void* __restrict__ out, uint32_t tiles_m2, uint32_t tiles_n, uint32_t num_kb, uint64_t mp,
                             uint64_t np, const EpiConst ec, int* err) {
    // the pair's tile constants (they shadow the single-CTA ones of namespace gemm)
    constexpr uint32_t BM = pair::BM, BN = pair::BN, BNH = pair::BNH, BK = pair::BK, UK = pair::UK;
    constexpr uint32_t STAGES = pair::STAGES, A_BYTES = pair::A_BYTES, STAGE_BYTES = pair::STAGE_BYTES;
    constexpr uint32_t ACC_COLS = pair::ACC_COLS, TMEM_COLS = pair::TMEM_COLS;
    using pair::arrive_remote;
    using pair::cluster_rank;
    using pair::cluster_sync;
    using pair::map_to;
    using pair::tma_load_3d_pair;
    using pair::umma_commit_pair;
    using pair::umma_i8_pair;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty_bar = full_bar + STAGES;
    uint64_t* tfull_bar = empty_bar + STAGES;
    uint64_t* tempty_bar = tfull_bar + 2;
    uint64_t* drain_bar = tempty_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const uint32_t first_tile = blockIdx.x >> 1, tile_step = gridDim.x >> 1;
    const uint32_t num_tiles = ec.S * tiles_m2 * tiles_n;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < STAGES; ++s) {
            mbar_init(full_bar + s, 1);
            mbar_init(empty_bar + s, 1);
        }
        for (uint32_t a = 0; a < 2; ++a) {
            mbar_init(tfull_bar + a, 1);
            mbar_init(tempty_bar + a, 8);  // 4 epilogue warps in each CTA of the pair
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's barriers are initialised before anything is signalled across the pair
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
            uint32_t stage = 0, phase = 0;
            uint32_t filled = 0, last_phase = 0;
            bool ok = true, issued = false;
            for (uint32_t tile = first_tile; ok && tile < num_tiles; tile += tile_step) {
                uint32_t plane, tm2, tn, kb_total;
                tile_work<MODE>(tile, ec.S, tiles_m2, tiles_n, num_kb, plane, tm2, tn, kb_total);
                for (uint32_t kb = 0; kb < kb_total; ++kb) {
                    if (!mbar_wait(empty_bar + stage, phase ^ 1u, abort_flag, err, ERR_WAIT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    int32_t k_el, pa, pb;
                    kblock_coords<MODE>(kb, plane, num_kb, k_el, pa, pb);
                    if (rank == 0) mbar_expect_tx(full_bar + stage, 2 * STAGE_BYTES);
                    const uint32_t full_leader = map_to(smem_u32(full_bar + stage), 0);
                    const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
                    tma_load_3d_pair(&tmA, sa, full_leader, k_el, (int32_t)(tm2 * 2 * BM + rank * BM), pa);
                    tma_load_3d_pair(&tmB, sa + A_BYTES, full_leader, k_el, (int32_t)(tn * BN + rank * BNH), pb);
                    issued = true;
                    filled |= 1u << stage;
                    last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {  // let the loads this thread issued land before the CTA may exit
                if (rank == 0) {
                    for (uint32_t st = 0; st < STAGES; ++st)
                        if (filled & (1u << st)) mbar_wait_drain(full_bar + st, (last_phase >> st) & 1u, 200000000ull);
                } else if (issued) {  // the peer's loads complete on the leader's barriers: wait a fixed time
                    const uint64_t t0 = global_timer_ns();
                    while (global_timer_ns() - t0 < pair::PEER_DRAIN_NS) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (uint32_t tile = first_tile; ok && tile < num_tiles; tile += tile_step) {
                uint32_t plane, tm2, tn, kb_total;
                tile_work<MODE>(tile, ec.S, tiles_m2, tiles_n, num_kb, plane, tm2, tn, kb_total);
                if (!mbar_wait(tempty_bar + acc, acc_phase ^ 1u, abort_flag, err, ERR_WAIT_MMA_EMPTY)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
                for (uint32_t kb = 0; kb < kb_total; ++kb) {
                    if (!mbar_wait(full_bar + stage, phase, abort_flag, err, ERR_WAIT_MMA_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + A_BYTES;
#pragma unroll
                    for (uint32_t k = 0; k < BK / UK; ++k)
                        umma_i8_pair(d_tmem, sdesc_sw128(sa + k * UK), sdesc_sw128(sb + k * UK), (kb | k) != 0u);
                    const uint32_t eb = smem_u32(empty_bar + stage);
                    umma_commit_pair(eb);
                    umma_commit_pair(map_to(eb, 1));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                const uint32_t tb = smem_u32(tfull_bar + acc);
                umma_commit_pair(tb);
                umma_commit_pair(map_to(tb, 1));
                acc ^= 1u;
                if (acc == 0) acc_phase ^= 1u;
            }
            // Every MMA this thread issued completes before the columns of either CTA are freed.
            umma_commit_pair(smem_u32(drain_bar));
            mbar_wait_drain(drain_bar, 0, 1000000000ull);
        }
    } else {
        const uint32_t quarter = warp & 3u;
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t tile = first_tile; tile < num_tiles; tile += tile_step) {
            uint32_t s, tm2, tn, kb_total;
            tile_work<MODE>(tile, ec.S, tiles_m2, tiles_n, num_kb, s, tm2, tn, kb_total);
            if (!mbar_wait(tfull_bar + acc, acc_phase, abort_flag, err, ERR_WAIT_EPILOGUE)) break;
            tc_fence_after();
            const uint64_t row = (uint64_t)tm2 * 2 * BM + rank * BM + quarter * 32u + lane;
            const uint32_t tbase = tmem_base + ((quarter * 32u) << 16) + acc * ACC_COLS;
            const uint32_t m = ec.m[s % OZTT_MAXS], y = ec.y[s % OZTT_MAXS], mg = ec.magic[s % OZTT_MAXS],
                           sh = ec.shift[s % OZTT_MAXS];
#pragma unroll 1
            for (uint32_t c = 0; c < BN; c += 32) {
                uint32_t v[32];
                tmem_ld32(tbase + c, v);
                if (row >= mp) continue;  // rows of the last pair tile beyond the planes (zero-filled loads)
                const uint64_t off = ((uint64_t)s * mp + row) * np + (uint64_t)tn * BN + c;
                if constexpr (MODE == 0 || MODE == 2) {
                    uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<int32_t*>(out) + off);
#pragma unroll
                    for (int q = 0; q < 8; ++q) o[q] = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                } else {
                    uint32_t w[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) w[q] = 0;
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const int32_t cv = (int32_t)v[e];
                        const uint32_t a = cv < 0 ? (uint32_t)(-cv) : (uint32_t)cv;
                        uint32_t r = a - udiv_small(a, mg, sh) * m;
                        if (cv < 0 && r) r = m - r;
                        const uint32_t t = r * y;
                        const uint32_t kk = t - udiv_small(t, mg, sh) * m;
                        w[e >> 2] |= kk << (8 * (e & 3));
                    }
                    uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(out) + off);
                    o[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    o[1] = make_uint4(w[4], w[5], w[6], w[7]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_remote(map_to(smem_u32(tempty_bar + acc), 0));
            acc ^= 1u;
            if (acc == 0) acc_phase ^= 1u;
        }
    }
    __syncthreads();
    cluster_sync();  // no CTA frees its tensor memory or exits while the pair may still use it
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
    }
}

// Test of the bounded wait: one CTA waits, through the GEMM's own mbar_wait, on an mbarrier that nothing
// arrives at, with no TMA load or MMA issued, and gives up after limit_ns; the code the GEMM's epilogue
// would record lands in *err_word. A second thread then waits (bounded) on the same barrier with the abort
// flag raised, as the GEMM's other roles do, and must leave at once.
__global__ void __launch_bounds__(64) wait_probe_kernel(int* err_word, uint64_t limit_ns, int* left_on_abort) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, err_word, ERR_WAIT_EPILOGUE, limit_ns);
    __syncthreads();
    if (threadIdx.x == 32) {
        const bool done = mbar_wait(&bar, 0, &abort_flag, err_word, ERR_WAIT_PRODUCER, limit_ns);
        if (!done && abort_flag) atomicAdd(left_on_abort, 1);
    }
}

// ---- host side -------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (!fn) throw Error(OZTT_ERUNTIME, "cuTensorMapEncodeTiled is not available from the CUDA driver");
    return fn;
}

// 3-D map over S planes of rows x kp int8 (K innermost), box BK x box_rows x 1, 128-byte swizzle. The
// planes lie plane_rows x pitch apart (plane_rows >= rows; a band of rows of taller planes), or rows x pitch;
// rows lie pitch apart (pitch >= kp; a window of kp columns of wider rows), or kp.
static CUtensorMap make_plane_map(const int8_t* base, uint64_t rows, uint64_t kp, uint64_t S, uint32_t box_rows,
                                  uint64_t plane_rows = 0, uint64_t pitch = 0) {
    CUtensorMap map;
    const uint64_t rp = pitch ? pitch : kp;
    const cuuint64_t dims[3] = {kp, rows, S};
    const cuuint64_t strides[2] = {rp, (plane_rows ? plane_rows : rows) * rp};
    const cuuint32_t box[3] = {BK, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(base), dims, strides,
                                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(OZTT_ERUNTIME, "cuTensorMapEncodeTiled failed for a residue plane map");
    return map;
}

// (magic, shift) with floor(a/d) = (umulhi(a, magic) + a) >> shift for all a < 2^31.
static void udiv_magic(uint32_t d, uint32_t& magic, uint32_t& shift) {
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    magic = (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1);
    shift = l;
}

}  // namespace gemm

namespace {

// The single-CTA kernel is the default; oztt_set_option(OZTT_OPT_GEMM_CTA_PAIRS, 1) selects the CTA-pair
// kernel for modes 0-2. Both give identical results. Measured on B200 at 16384^3 (S = 17, 20 steps): the
// pair kernel needs about 9 % fewer SM cycles for the residue GEMM, but it draws more power per cycle,
// and under the 1 kW cap the SM clock settles near 1130 MHz instead of 1500 MHz, so it takes 64 ms
// instead of 53 ms. In short runs that stay below the cap (Scheme I at 8192^3) it is the faster of the
// two. Read once per launch, so the tensor maps and the kernel of one launch always agree.
bool use_pairs() { return option_value(OZTT_OPT_GEMM_CTA_PAIRS) == 1; }

// Launches mode MODE of the GEMM over `planes` planes of tiles (a plane = a modulus or a diagonal), on
// CTA pairs when `pairs` (modes 0-2 only; the tensor maps must have been made for the same choice).
template <int MODE>
void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, void* out, uint64_t mp, uint64_t np, uint64_t kp,
                 uint32_t planes, const gemm::EpiConst& ec, int* err_word, cudaStream_t st, bool pairs = false) {
    using namespace gemm;
    int dev = 0, sms = 148;
    OZTT_CUDA(cudaGetDevice(&dev));
    OZTT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const uint32_t tiles_n = (uint32_t)(np / BN), num_kb = (uint32_t)(kp / BK);
    if (MODE < 3 && pairs) {
        // the CTA-pair kernel covers modes 0-2
        const uint32_t tiles_m2 = (uint32_t)((mp / 128 + 1) / 2);
        const uint64_t num_tiles = (uint64_t)planes * tiles_m2 * tiles_n;
        OZTT_CUDA(cudaFuncSetAttribute(residue_gemm_pair_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)pair::SMEM_BYTES));
        // one resident pair per two SMs, as many pairs as the GPCs can hold at once (persistent)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(sms & ~1), 1, 1);
        cfg.blockDim = dim3(pair::NUM_THREADS, 1, 1);
        cfg.dynamicSmemBytes = pair::SMEM_BYTES;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        OZTT_CUDA(cudaOccupancyMaxActiveClusters(&clusters, residue_gemm_pair_kernel<MODE>, &cfg));
        if (clusters < 1) throw Error(OZTT_ERUNTIME, "residue_gemm: no CTA pair fits on this device");
        const unsigned grid = 2u * (unsigned)std::min<uint64_t>(num_tiles, (uint64_t)clusters);
        if constexpr (MODE < 3)
            residue_gemm_pair_kernel<MODE><<<grid, pair::NUM_THREADS, pair::SMEM_BYTES, st>>>(
                ta, tb, out, tiles_m2, tiles_n, num_kb, mp, np, ec, err_word);
    } else {
        const uint32_t tiles_m = (uint32_t)(mp / BM);
        const uint64_t num_tiles = (uint64_t)planes * tiles_m * tiles_n;
        OZTT_CUDA(cudaFuncSetAttribute(residue_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)SMEM_BYTES));
        const unsigned grid = (unsigned)std::min<uint64_t>(num_tiles, (uint64_t)sms);
        residue_gemm_kernel<MODE><<<grid, NUM_THREADS, SMEM_BYTES, st>>>(ta, tb, out, tiles_m, tiles_n, num_kb, mp, np,
                                                                        ec, err_word);
    }
    OZTT_CUDA(cudaGetLastError());
}

}  // namespace

// a_plane_rows: when nonzero, ap points at row r0 of A planes that are a_plane_rows tall, and the
// GEMM covers the band of mp rows from there (output planes [S][mp][np] of the band). b_plane_rows: the
// same for B, whose planes hold a block of np of their b_plane_rows columns (output [S][mp][np] of the block).
void launch_residue_gemm(const int8_t* ap, const int8_t* bp, uint64_t mp, uint64_t np, uint64_t kp,
                         const oztt_ii_plan& p, int mode, void* out, int* err_word, cudaStream_t st,
                         uint64_t a_plane_rows, uint64_t b_plane_rows) {
    using namespace gemm;
    if (mp % BM || np % BN || kp % BK || mp == 0 || np == 0 || kp == 0)
        throw Error(OZTT_EINVAL, "residue_gemm: mp, np, kp must be positive multiples of 128, 256 and 128");
    if (a_plane_rows && a_plane_rows < mp) throw Error(OZTT_EINVAL, "residue_gemm: band taller than its planes");
    if (b_plane_rows && b_plane_rows < np) throw Error(OZTT_EINVAL, "residue_gemm: block wider than its planes");
    if (p.S < 1 || p.S > OZTT_MAXS) throw Error(OZTT_EINVAL, "residue_gemm: bad number of moduli");
    if ((reinterpret_cast<uintptr_t>(ap) | reinterpret_cast<uintptr_t>(bp)) & 15)
        throw Error(OZTT_EINVAL, "residue_gemm: planes must be 16-byte aligned");
    if (mode != 0 && mode != 1) throw Error(OZTT_EINVAL, "residue_gemm: mode must be 0 or 1");
    if (mp / BM * (np / BN) * (uint64_t)p.S >= (1ull << 31) || kp / BK >= (1ull << 31))
        throw Error(OZTT_EINVAL, "residue_gemm: problem too large");
    EpiConst ec{};
    ec.S = (uint32_t)p.S;
    for (int s = 0; s < p.S; ++s) {
        ec.m[s] = (uint32_t)p.moduli[s];
        ec.y[s] = (uint32_t)p.yi[s];
        udiv_magic(ec.m[s], ec.magic[s], ec.shift[s]);
    }
    const bool pairs = use_pairs();
    const CUtensorMap ta = make_plane_map(ap, mp, kp, (uint64_t)p.S, pairs ? pair::BM : BM, a_plane_rows);
    const CUtensorMap tb = make_plane_map(bp, np, kp, (uint64_t)p.S, pairs ? pair::BNH : BN, b_plane_rows);
    if (mode == 0)
        launch_gemm<0>(ta, tb, out, mp, np, kp, (uint32_t)p.S, ec, err_word, st, pairs);
    else
        launch_gemm<1>(ta, tb, out, mp, np, kp, (uint32_t)p.S, ec, err_word, st, pairs);
}

// Scheme I diagonal products P_d = sum_{i=0..d} A_i B_{d-i}^T, d = 0..p-1, int32 [p][mp][np], from
// slice planes A [p][mp][kp] and B [p][np][kp] (tcgen05 kind::i8, s32 accumulation over the
// concatenated K of (d+1)*kp).
// a_plane_rows: when nonzero, ap points at row r0 of A slice planes that are a_plane_rows tall, and the
// GEMM covers the band of mp rows from there (diagonals [p][mp][np] of the band).
// k0, kw: when kw is nonzero, the products run over the K window [k0, k0 + kw) of planes whose rows are kp
// long (a K block of a sum too long for exact 32-bit diagonal sums); k0 and kw multiples of 128.
void launch_diag_gemm(const int8_t* ap, const int8_t* bp, uint64_t mp, uint64_t np, uint64_t kp, int p,
                      int32_t* out, int* err_word, cudaStream_t st, uint64_t a_plane_rows, uint64_t k0, uint64_t kw) {
    using namespace gemm;
    if (mp % BM || np % BN || kp % BK || mp == 0 || np == 0 || kp == 0)
        throw Error(OZTT_EINVAL, "diag_gemm: mp, np, kp must be positive multiples of 128, 256 and 128");
    if (kw) {
        if (k0 % BK || kw % BK || k0 + kw > kp) throw Error(OZTT_EINVAL, "diag_gemm: bad K window");
        ap += k0;
        bp += k0;
    }
    if (a_plane_rows && a_plane_rows < mp) throw Error(OZTT_EINVAL, "diag_gemm: band taller than its planes");
    if (p < 1 || p > 64) throw Error(OZTT_EINVAL, "diag_gemm: the number of slices must be 1..64");
    if ((reinterpret_cast<uintptr_t>(ap) | reinterpret_cast<uintptr_t>(bp)) & 15)
        throw Error(OZTT_EINVAL, "diag_gemm: planes must be 16-byte aligned");
    if (mp / BM * (np / BN) * (uint64_t)p >= (1ull << 31) || (uint64_t)p * (kp / BK) >= (1ull << 31))
        throw Error(OZTT_EINVAL, "diag_gemm: problem too large");
    EpiConst ec{};
    ec.S = (uint32_t)p;
    const bool pairs = use_pairs();
    const uint64_t kext = kw ? kw : kp;
    const CUtensorMap ta = make_plane_map(ap, mp, kext, (uint64_t)p, pairs ? pair::BM : BM, a_plane_rows, kp);
    const CUtensorMap tb = make_plane_map(bp, np, kext, (uint64_t)p, pairs ? pair::BNH : BN, 0, kp);
    launch_gemm<2>(ta, tb, out, mp, np, kext, (uint32_t)p, ec, err_word, st, pairs);
}

// FP8 digit products on the tensor cores: for each GEMM output u of the plan, P_u = sum_t A_(out_a+t)
// B_(out_b-t)^T over the digit planes A [nplane][mp][kp] and B [nplane][np][kp] (int8 values of the e4m3
// digits, exact s32 sums). mode 0: P_u as int32 [nout][mp][np]; mode 1: the composition fused into the
// epilogue, the CRT digits k_s = (sum_u c_u P_u) y_s mod m_s as uint16 [S][mp][np] (compose.cpp and the
// term_k of recon_crt_proc.h, as one exact integer computation).
// a_plane_rows: when nonzero, ap points at row r0 of A digit planes that are a_plane_rows tall, and the
// GEMM covers the band of mp rows from there (outputs [S or nout][mp][np] of the band).
void launch_digit_gemm(const int8_t* ap, const int8_t* bp, uint64_t mp, uint64_t np, uint64_t kp,
                       const oztt_digit_plan& fp, int mode, void* out, int* err_word, cudaStream_t st,
                       uint64_t a_plane_rows) {
    using namespace gemm;
    if (mp % BM || np % BN || kp % BK || mp == 0 || np == 0 || kp == 0)
        throw Error(OZTT_EINVAL, "digit_gemm: mp, np, kp must be positive multiples of 128, 256 and 128");
    if (a_plane_rows && a_plane_rows < mp) throw Error(OZTT_EINVAL, "digit_gemm: band taller than its planes");
    const int S = fp.base.S;
    if (S < 1 || S > OZTT_MAXS) throw Error(OZTT_EINVAL, "digit_gemm: bad number of moduli");
    if (fp.nout < 1 || fp.nout > OZTT_MAXOUT || fp.nplane < 1 || fp.nplane > 255 || fp.oout[0] != 0 ||
        fp.oout[S] != fp.nout)
        throw Error(OZTT_EINVAL, "digit_gemm: bad digit plan");
    if ((reinterpret_cast<uintptr_t>(ap) | reinterpret_cast<uintptr_t>(bp)) & 15)
        throw Error(OZTT_EINVAL, "digit_gemm: planes must be 16-byte aligned");
    if (mode != 0 && mode != 1) throw Error(OZTT_EINVAL, "digit_gemm: mode must be 0 or 1");
    EpiConst ec{};
    ec.S = (uint32_t)S;
    int max_g = 1;
    for (int s = 0; s < S; ++s) {
        const int m = fp.base.moduli[s];
        if (m < 3 || m > 4096) throw Error(OZTT_EINVAL, "digit_gemm: moduli must be in 3..4096");
        ec.m[s] = (uint32_t)m;
        ec.y[s] = (uint32_t)fp.base.yi[s];
        udiv_magic(ec.m[s], ec.magic[s], ec.shift[s]);
        if (fp.oout[s + 1] < fp.oout[s]) throw Error(OZTT_EINVAL, "digit_gemm: bad output ranges");
        ec.oout[s] = (uint16_t)fp.oout[s];
        for (int u = fp.oout[s]; u < fp.oout[s + 1]; ++u) {
            const int g = fp.out_g[u];
            if (fp.out_mod[u] != s || g < 1 || fp.out_a[u] < 0 || fp.out_a[u] + g > fp.nplane ||
                fp.out_b[u] - g + 1 < 0 || fp.out_b[u] >= fp.nplane)
                throw Error(OZTT_EINVAL, "digit_gemm: output " + std::to_string(u) + " names planes outside the plan");
            max_g = std::max(max_g, g);
            ec.out_a[u] = (uint8_t)fp.out_a[u];
            ec.out_b[u] = (uint8_t)fp.out_b[u];
            ec.out_g[u] = (uint8_t)g;
            const int64_t c = ((int64_t)fp.coeff[u] % m + m) % m;
            ec.weight[u] = (uint16_t)(c * fp.base.yi[s] % m);
        }
    }
    ec.oout[S] = (uint16_t)fp.nout;
    // |P_u| <= kp * g * 32^2 must stay below 2^31 (s32 accumulators, the epilogue's division)
    if ((uint64_t)kp * (uint64_t)max_g * 1024ull >= (1ull << 31))
        throw Error(OZTT_EINVAL, "digit_gemm: K too large for exact 32-bit digit sums");
    if (mp / BM * (np / BN) * (uint64_t)S >= (1ull << 31)) throw Error(OZTT_EINVAL, "digit_gemm: problem too large");
    const CUtensorMap ta = make_plane_map(ap, mp, kp, (uint64_t)fp.nplane, BM, a_plane_rows);
    const CUtensorMap tb = make_plane_map(bp, np, kp, (uint64_t)fp.nplane, BN);
    if (mode == 0)
        launch_gemm<4>(ta, tb, out, mp, np, kp, (uint32_t)S, ec, err_word, st);
    else
        launch_gemm<3>(ta, tb, out, mp, np, kp, (uint32_t)S, ec, err_word, st);
}

// Runs wait_probe_kernel with a limit of limit_ns and reports its outcome as the GEMM pipelines do: the
// recorded code becomes a runtime error through check_flags.
void check_flags(uint32_t flags, int gemm_err);

}  // namespace oztt

extern "C" int oztt_test_gemm_wait_timeout(uint64_t limit_ns, int32_t* code_out, void* stream, char* err,
                                           size_t errlen) {
    return oztt::guarded(err, errlen, [&] {
        if (limit_ns == 0 || limit_ns > 1000000000ull) throw oztt::Error(OZTT_EINVAL, "limit must be in (0, 1 s]");
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        int* words = nullptr;
        OZTT_CUDA(cudaMallocAsync(&words, 2 * sizeof(int), st));
        OZTT_CUDA(cudaMemsetAsync(words, 0, 2 * sizeof(int), st));
        oztt::gemm::wait_probe_kernel<<<1, 64, 0, st>>>(words, limit_ns, words + 1);
        OZTT_CUDA(cudaGetLastError());
        int host[2] = {0, 0};
        OZTT_CUDA(cudaMemcpyAsync(host, words, sizeof host, cudaMemcpyDeviceToHost, st));
        OZTT_CUDA(cudaFreeAsync(words, st));
        OZTT_CUDA(cudaStreamSynchronize(st));
        if (code_out) {
            code_out[0] = host[0];
            code_out[1] = host[1];
        }
        oztt::check_flags(0, host[0]);
    });
}

namespace oztt {

// Host model of the epilogue's division, for the CPU tests of the C ABI.
extern "C" uint32_t oztt_test_udiv_small(uint32_t a, uint32_t d) {
    uint32_t mg, sh;
    gemm::udiv_magic(d, mg, sh);
    const uint32_t hi = (uint32_t)(((uint64_t)a * mg) >> 32);
    return (uint32_t)(hi + a) >> sh;
}

}  // namespace oztt
