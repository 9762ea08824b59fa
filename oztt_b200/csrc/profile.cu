// SPDX-License-Identifier: Apache-2.0
//
// The device pipelines under the evaluator hooks (include/evaluation_hooks.hpp), and their plain run.
//
// A pipeline is the ordered list of launches of one call (Pipeline, runtime.cuh). Plainly it is issued
// once, back to back on one stream. Under an evaluation Scope, as the reference's backends do with
// their programs (src/ozaki2.cpp:63-65, 147-200, 391-455; src/ozaki1.cpp:113-210):
//   * each phase (consecutive launches of one stage) goes through evaluation::execute: issued and
//     waited for once, offered to the warm-up policy, then issued `repeats` times and timed; every
//     launch writes its outputs from its inputs only, so repeating a phase leaves the same bits;
//   * with `whole` set, evaluation::whole fills every buffer the pass writes with the sentinel, issues
//     the complete list once without waiting between launches (noting each launch's step kind against
//     the counts the list implies), compares the output with the phase-timed bits and times the
//     uninterrupted pass;
//   * partial_products and the GEMM grid (`cores`: the SMs it occupies) are reported; `bandwidth` has no
//     B200 counterpart and stays zero.
#include <evaluation_hooks.hpp>

#include "oztt_common.cuh"
#include "runtime.cuh"

namespace oztt {

namespace ev = ozTTgemm::detail::evaluation;
static_assert(kScale == ev::Scale && kSlice == ev::Slice && kGemm == ev::Gemm && kCompose == ev::Compose &&
                  kRecon == ev::Recon,
              "pipeline stages follow the evaluator's");
static_assert(kHead == ev::Head && kGemmStep == ev::GemmStep && kReconStep == ev::ReconStep &&
                  kComposeStep == ev::ComposeStep,
              "pipeline steps follow the evaluator's");

namespace {

__global__ void fill_words_kernel(uint32_t* __restrict__ p, uint64_t count, uint32_t value) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x)
        p[i] = value;
}

}  // namespace

void Pipeline::run(cudaStream_t st, double* stage_ms, int slots) const {
    if (!stage_ms || slots <= 0) {
        for (const Launch& l : launches) l.issue();
        return;
    }
    std::vector<cudaEvent_t> ev((size_t)slots + 1, nullptr);
    struct Events {
        std::vector<cudaEvent_t>& e;
        ~Events() {
            for (cudaEvent_t x : e)
                if (x) cudaEventDestroy(x);
        }
    } guard{ev};
    for (auto& e : ev) OZTT_CUDA(cudaEventCreate(&e));
    int slot = 0;
    OZTT_CUDA(cudaEventRecord(ev[0], st));
    for (const Launch& l : launches) {
        while (slot < l.slot && slot < slots) OZTT_CUDA(cudaEventRecord(ev[++slot], st));
        l.issue();
    }
    while (slot < slots) OZTT_CUDA(cudaEventRecord(ev[++slot], st));
    OZTT_CUDA(cudaStreamSynchronize(st));
    for (int i = 0; i < slots; ++i) {
        float ms = 0;
        OZTT_CUDA(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
        stage_ms[i] = ms;
    }
}

bool evaluation_active() { return ev::active != nullptr; }

unsigned evaluation_fixed_bits() { return ev::active ? ev::active->fixed_bits : 0u; }

bool run_profiled(const Pipeline& pl, cudaStream_t st) {
    if (!ev::active) return false;
    const auto sync = [&] { OZTT_CUDA(cudaStreamSynchronize(st)); };
    int dev = 0, sms = 0;
    OZTT_CUDA(cudaGetDevice(&dev));
    OZTT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    ev::active->partial_products = pl.partial_products;
    ev::active->bandwidth = 0;
    ev::active->cores = (unsigned)sms;
    // phase timing
    for (size_t i = 0; i < pl.launches.size();) {
        size_t j = i;
        while (j < pl.launches.size() && pl.launches[j].phase == pl.launches[i].phase) ++j;
        ev::execute(
            static_cast<ev::Stage>(pl.launches[i].stage),
            [&] {
                for (size_t q = i; q < j; ++q) pl.launches[q].issue();
            },
            sync);
        i = j;
    }
    // whole pass
    ev::Counts expected;
    for (const auto& l : pl.launches) ++expected[l.step];
    const size_t words = pl.out_bytes / 4;
    ev::whole(
        [&] {
            for (const auto& w : pl.written) {
                const uint64_t count = w.second / 4;
                if (!count) continue;
                fill_words_kernel<<<(unsigned)std::min<uint64_t>((count + 255) / 256, 4096), 256, 0, st>>>(
                    static_cast<uint32_t*>(w.first), count, ev::SENTINEL);
                OZTT_CUDA(cudaGetLastError());
            }
            sync();
        },
        [&](std::vector<std::uint32_t>& v) {
            v.resize(words);
            if (words) OZTT_CUDA(cudaMemcpyAsync(v.data(), pl.out, words * 4, cudaMemcpyDeviceToHost, st));
            sync();
        },
        sync,
        [&](auto&& note) {
            for (const auto& l : pl.launches) {
                l.issue();
                note(l.step);
            }
        },
        expected);
    return true;
}

}  // namespace oztt
