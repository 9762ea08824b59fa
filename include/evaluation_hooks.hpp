// SPDX-License-Identifier: Apache-2.0
//
// Evaluator hooks of ozTTgemm for B200: the private interface through which the paper evaluator
// (evaluation/evaluate.cpp) and the acceptance test (tests/correctness.cpp) of the reference profile a
// GEMM call. It keeps the reference's names and meanings (src/evaluation_hooks.hpp:28-220), so those
// programs build unchanged against this library; the code is this project's.
//
// An ordinary call runs each device step once. While a Scope is open on the calling thread, the
// library instead
//   * times each stage (scale, slice, gemm, compose, recon): issued once, offered to the caller's
//     warm-up policy, then issued `repeats` times and synchronised; the mean goes to seconds[stage] and
//     each timed interval to the `interval` callback;
//   * with `whole` set, checks and times the whole pass: every buffer the pass writes is filled with
//     SENTINEL, the complete sequence of device steps is issued once without synchronisation between
//     them (counted per kind against the counts the configuration implies), the output must come back
//     bit-identical to the phase-timed one, and the uninterrupted pass is then timed over `repeats`;
//   * reports the number of partial products of the GEMM stage and its launch geometry.
// On B200 the composition of the digit formats is fused into the GEMM epilogue, so Compose stays zero;
// `bandwidth` is zero (the reference's DRAM-bank setting has no counterpart) and `cores` is the number
// of SMs the GEMM grid occupies.
#pragma once
#include <array>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string_view>
#include <utility>
#include <vector>

namespace ozTTgemm::detail::evaluation {

enum Stage { Scale, Slice, Gemm, Compose, Recon, Count };

inline const char* name(Stage stage) {
    switch (stage) {
    case Scale: return "scale";
    case Slice: return "slice";
    case Gemm: return "gemm";
    case Compose: return "compose";
    case Recon: return "recon";
    default: return "unknown";
    }
}

// Kinds of device steps of the whole pass: the scaling and slicing launches (Head), a GEMM launch, a
// reconstruction launch and a composition launch.
enum Step { Head, GemmStep, ReconStep, ComposeStep, StepCount };

struct Counts {
    std::array<unsigned long long, StepCount> n{};
    unsigned long long& operator[](int kind) { return n[kind]; }
    unsigned long long operator[](int kind) const { return n[kind]; }
    bool operator==(const Counts& other) const { return n == other.n; }
};

// Written into every buffer the whole pass writes before it is replayed: a NaN in FP32/BF16 and a huge
// finite FP64 value, so that a buffer the pass failed to write changes the output.
constexpr std::uint32_t SENTINEL = 0x7FC07FC0u;

// Seconds on a monotonic clock.
inline double now() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// A device step kept for a later replay (its kind and the closure that issues it).
struct RecordedStep {
    Step kind;
    std::function<void()> issue;
};

// What a profiled call is asked to do, and what it reports. Opening a Scope resets the results, so one
// Settings can serve several Scopes in turn.
struct Settings {
    // requests
    unsigned repeats = 3;
    unsigned fixed_bits = 0;  // Ozaki II scaled-integer width forced to this value; 0: chosen from the input
    std::function<void(std::string_view, const std::function<void()>&)> warmup;
    std::function<void(Stage, double, double)> interval;
    bool whole = true;
    // results
    unsigned partial_products = 0, bandwidth = 0, cores = 0;
    std::array<double, Count> seconds{};
    bool recording = false;
    double whole_seconds = NAN;
    bool whole_checked = false;
    Counts whole_expected, whole_ran;
    std::vector<RecordedStep> steps;  // released by the end of every profiled call

    void reset_results() {
        partial_products = bandwidth = cores = 0;
        seconds.fill(0);
        recording = false;
        whole_seconds = NAN;
        whole_checked = false;
        whole_expected = whole_ran = Counts{};
        steps.clear();
    }
};

// The Settings of the Scope open on this thread, if any.
inline thread_local Settings* active = nullptr;

class Scope {
public:
    explicit Scope(Settings& settings) : settings_(settings), outer_(active) {
        if (settings.repeats == 0) throw std::invalid_argument("evaluation repeats must be positive");
        settings.reset_results();
        active = &settings;
    }
    ~Scope() {
        settings_.steps.clear();
        active = outer_;
    }
    Scope(const Scope&) = delete;
    Scope& operator=(const Scope&) = delete;

private:
    Settings& settings_;
    Settings* outer_;
};

inline bool recording_whole() { return active != nullptr && active->whole; }

// Keeps a device step for the whole pass (no effect unless a whole pass is requested).
inline void record(Step kind, std::function<void()> issue) {
    if (recording_whole()) active->steps.push_back({kind, std::move(issue)});
}

// Adds one timed interval of `repeats` issues of a stage.
inline void record(Stage stage, double begin, double end) {
    active->seconds[stage] += (end - begin) / active->repeats;
    if (active->interval) active->interval(stage, begin, end);
}

// Times one issue of a stage while a sweep is being recorded; otherwise just issues it.
template <class F>
void phase(Stage stage, F&& issue) {
    if (!active || !active->recording) {
        issue();
        return;
    }
    const double begin = now();
    issue();
    record(stage, begin, now());
}

// Issues a stage and waits for it; under a Scope, then offers it to the warm-up policy and times
// `repeats` issues followed by one wait.
template <class F, class S>
void execute(Stage stage, F&& issue, S&& sync) {
    issue();
    sync();
    if (!active) return;
    Settings& s = *active;
    if (s.warmup)
        s.warmup(stage == Compose ? "gemm" : name(stage), [&] {
            for (unsigned i = 0; i < s.repeats; ++i) issue();
            sync();
        });
    const double begin = now();
    for (unsigned i = 0; i < s.repeats; ++i) issue();
    sync();
    record(stage, begin, now());
}
template <class F>
void execute(Stage stage, F&& issue) {
    execute(stage, std::forward<F>(issue), [] {});
}

// A loop of stages timed as a whole with phase(): issued once, warmed, then `repeats` times recorded.
template <class F>
void sweep(F&& issue) {
    issue();
    if (!active) return;
    Settings& s = *active;
    if (s.warmup) s.warmup("sweep", issue);
    s.recording = true;
    struct Off {
        Settings& s;
        ~Off() { s.recording = false; }
    } off{s};
    for (unsigned i = 0; i < s.repeats; ++i) issue();
}

// Checks and times the whole pass. fill() writes SENTINEL into every buffer the pass writes (not the
// inputs), read_out(words) reads the whole output, sync() waits for the device, run_once(note) issues
// the complete pass calling note(kind) for each step, and `expected` holds the step counts the
// configuration implies. The output is left holding the replayed result.
template <class Fill, class ReadOut, class Sync, class RunOnce>
void whole(Fill&& fill, ReadOut&& read_out, Sync&& sync, RunOnce&& run_once, const Counts& expected) {
    if (!recording_whole()) return;
    Settings& s = *active;
    struct Release {
        std::vector<RecordedStep>& steps;
        ~Release() { steps.clear(); }
    } release{s.steps};
    std::vector<std::uint32_t> phased, seen;
    read_out(phased);
    fill();
    read_out(seen);
    bool filled = !seen.empty();
    for (std::uint32_t w : seen) filled = filled && w == SENTINEL;
    Counts ran;
    run_once([&](int kind) { ++ran[kind]; });
    sync();
    read_out(seen);
    const bool replayed = filled && seen == phased;
    const auto pass = [&] { run_once([](int) {}); };
    if (s.warmup)
        s.warmup("whole", [&] {
            pass();
            sync();
        });
    const double begin = now();
    for (unsigned i = 0; i < s.repeats; ++i) pass();
    sync();
    s.whole_seconds = (now() - begin) / s.repeats;
    read_out(seen);
    s.whole_expected = expected;
    s.whole_ran = ran;
    s.whole_checked = replayed && ran == expected && seen == phased;
}

// Issues the kept steps in order, calling note(kind) for each.
template <class Note>
void replay(Note&& note) {
    for (const RecordedStep& step : active->steps) {
        step.issue();
        note(step.kind);
    }
}

}  // namespace ozTTgemm::detail::evaluation
