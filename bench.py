#!/usr/bin/env python
"""Benchmark: Ozaki-II INT8 effective FP64 TFLOPS on B200 (the metric of BASELINE.json).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl oztt|reference]
    python bench.py --scheme I [--slices 0,4,8,12] [--format FP8]
                                   (Scheme I INT8 or FP8, 8192^3, phi=1: one line per p)
    python bench.py --format FP8|BF16|FP16|TF32 [--moduli 12,16,20,24] [--passes 1,2]
                                   (Scheme II digit formats, 8192 x 8192 x 16384, phi=4: one line per setting)

One step is one pass of the Scheme II INT8 pipeline (scale -> split -> residue GEMM on the tensor
cores -> exact CRT reconstruction) over one m x n x k problem with FP64 operands already resident in
HBM. The workload at N=1 is the metric point m=n=k=16384, phi=0.5, seed 0 of the reference
evaluator's generator (evaluation/numerics.hpp:19-38, synthetic data). With N>1 ranks (one process
per GPU, torchrun) it is config 5, m = n = 32768, k = 16384, as strong scaling: rank 0 generates the
whole A and B (the evaluator's stream), the panels are placed over NVLink (timed separately), and rank
(p, q) of a P x Q grid computes output tile C_pq from its resident A row panel and B column panel; the
same problem on one GPU is timed in the same run (config5_1gpu).

Printed (rank 0, one JSON line): value = 2*m*n*k / (max over ranks of the device time of one step),
e2e = the same metric through the public API from pinned host buffers, the copies in and out included
(N=1: ozTTgemm::Context::gemm via the C ABI, computing while the operands upload and reading C back as its
pieces finish; N>1: oztt_b200.distributed.gemm_tiled from each rank's host panels), the roofline of the
residue GEMM
(int8 tensor ops per launch / its CUDA-event duration against the measured sustained int8 rate), the
effective rate the selected moduli allow at that rate (moduli_roofline), the ratio to the B200 FP64 peak, the
reference's host FP64 GEMM (Dot2, compiled from the reference sources in oracle/_ref) timed on a sample
of rows as the CPU baseline, cuBLAS DGEMM and cuBLASLt's int8 GEMM on the same GPU for comparison, and the
maximum relative error of sampled rows against a binary128 reference, beside the reference device's own
result on the same rows.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

DEFAULT_SIZE = 16384
FP64_PEAK_TFLOPS = 40.0
METRIC = "Ozaki-II INT8 effective FP64 TFLOPS at m=n=k=16384; max rel err vs binary128"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["oztt", "reference"], default="oztt")
    ap.add_argument("--size", type=int, default=None, help="per-GPU tile side m = n = k")
    ap.add_argument("--phi", type=float, default=None)
    ap.add_argument("--scheme", choices=["II", "I"], default="II",
                    help="I: the Scheme I INT8 workload (default 8192^3, phi=1.0), one JSON line per slice count")
    ap.add_argument("--slices", default="0", help="Scheme I: comma-separated slice counts, 0 = selected from the input")
    ap.add_argument("--format", choices=["INT8", "FP8", "BF16", "FP16", "TF32"], default="INT8",
                    help="format of the low-precision products (both schemes)")
    ap.add_argument("--moduli", default="12,16,20,24", help="digit formats: comma-separated max_moduli settings")
    ap.add_argument("--passes", default="1,2", help="digit formats: reconstruction passes (1 OnePass, 2 TwoPass)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-accuracy", action="store_true")
    args = ap.parse_args()
    if args.size is None:
        args.size = DEFAULT_SIZE if args.scheme == "II" and args.format == "INT8" else 8192
    if args.phi is None:
        args.phi = 1.0 if args.scheme == "I" else (0.5 if args.format == "INT8" else 4.0)
    return args


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "bf16_tflops": d.get("bf16_tflops", 1590.0),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", 1400.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock and throttle-reason samples (200 ms) during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="oztt_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return float("nan")

        sm = [num(r[1]) for r in rows]
        smax = max(num(r[2]) for r in rows)
        loaded = [s for s in sm if s > 0.5 * smax] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": smax, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(num(r[3]) for r in rows)}


# ---- CPU baseline: the reference's host FP64 GEMM (Dot2) -------------------------------------------
def cpu_dot2_library():
    ref = ROOT / "oracle" / "_ref" / "libozref_dot2.so"
    if ref.exists():
        lib = ctypes.CDLL(str(ref))
        lib.ozr_dot2_prepare.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_uint32] * 3
        lib.ozr_dot2_run.restype = ctypes.c_double
        lib.ozr_dot2_run.argtypes = [ctypes.c_int]
        return lib, "reference"
    return None, "port"


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def gemm_traffic(m: int, n: int, k: int, S: int) -> float:
    """DRAM bytes per launch of the residue GEMM: the ncu capture at 4096^3 (S = 16) scaled by the
    units the launch processes (every residue plane is read from HBM once and every digit plane written
    once, so the traffic grows with S*(mk + nk + mn))."""
    captured = 537.35e6 + 246.64e6
    return captured * (S * (m * k + n * k + m * n)) / (16 * 3 * 4096.0 ** 2)


def calibrate_rows(run, threads: int, n: int, target_s: float) -> tuple[int, float]:
    """Grows the row sample (a multiple of the thread count, at most n) until one run takes at least
    half of target_s; returns the rows and the time of the last run. The first run warms the thread
    pool and the copies up and is not used."""
    rows = max(threads, 8)
    run(rows)
    t = run(rows)
    while t < 0.5 * target_s and rows < n:
        grow = min(8.0, target_s / max(t, 1e-3))
        rows = min(n, max(rows + threads, int(rows * grow) // threads * threads))
        t = run(rows)
    return rows, t


def time_cpu_dot2(a: np.ndarray, b: np.ndarray, n: int, k: int, target_s: float) -> dict:
    """Times the reference's Dot2 GEMM on the first rows of C, sized to about target_s seconds."""
    threads = cpu_threads()
    lib, kind = cpu_dot2_library()
    if lib is None:  # the oracle's restatement of the same routine
        sys.path.insert(0, str(ROOT / "tests"))
        from oracle_lib import Oracle  # noqa: E402

        orc = Oracle()

        def run(rows):
            return orc.lib.ozo_time_dot2_rows(a.ctypes.data, b.ctypes.data, rows, n, k, threads)
    else:
        def run(rows):
            lib.ozr_dot2_prepare(a.ctypes.data, b.ctypes.data, rows, n, k)
            return lib.ozr_dot2_run(threads)
    rows, t = calibrate_rows(run, threads, n, target_s)
    flops = 2.0 * rows * n * k
    return {"value": flops / t / 1e12, "unit": "TFLOPS", "cores": threads, "kind": kind,
            "sample": f"Dot2 reference_gemm (evaluation/numerics.hpp) on the first {rows} rows of C "
                      f"({rows}x{n}x{k}), {t:.2f} s"}


def headline_dims(args, world: int = 1) -> tuple[int, int, int]:
    """m, n, k of the headline workload: the metric point size^3 on one GPU; config 5, m = n = 2 size and
    k = size (32768 x 32768 x 16384), on several."""
    return (args.size, args.size, args.size) if world == 1 else (2 * args.size, 2 * args.size, args.size)


def headline_config(args, world: int = 1) -> dict:
    """The workload of the headline line; both arms (this library and --impl reference) print this same
    object, so their numbers are quoted on one configuration."""
    m, n, k = headline_dims(args, world)
    if world == 1:
        return {"workload": f"Scheme II INT8, {m}x{n}x{k}, phi={args.phi}, seed {args.seed}, auto precision",
                "l2": "inputs (2.1 GB each) larger than the 126 MB L2; no flush"}
    P = Q = int(math.isqrt(world))  # the grid of oztt_b200.distributed.grid_shape (this arm maps no product code)
    while world % Q:
        Q -= 1
    P = world // Q
    return {"workload": f"Scheme II INT8, {m}x{n}x{k} (config 5) in {P}x{Q} output tiles over {world} GPUs, "
                        f"phi={args.phi}, seed {args.seed}, auto precision",
            "l2": "panels (1 GB and more per GPU) larger than the 126 MB L2; no flush"}


def run_reference(args) -> None:
    """--impl reference: the reference's own CPU FP64 GEMM (paper_eval::reference_gemm, Dot2 with OpenMP,
    compiled from the reference sources into oracle/_ref) on the box's host cores, per step a bounded row
    sample of the same workload; rank 0 only. The inputs come from the oracle's restatement of the
    evaluator's generator (oracle/liboz2oracle.so), so this process maps no library of the product."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    m, n, k = headline_dims(args, world)
    sys.path.insert(0, str(ROOT / "tests"))
    from oracle_lib import Oracle  # noqa: E402  (generator and, without oracle/_ref, the Dot2 port)

    orc = Oracle()
    a, b = orc.gen_inputs(m, n, k, args.phi, args.seed)
    threads = cpu_threads()
    lib, kind = cpu_dot2_library()
    if lib is None:
        def run(rows):
            return orc.lib.ozo_time_dot2_rows(a.ctypes.data, b.ctypes.data, rows, n, k, threads)
    else:
        def run(rows):
            lib.ozr_dot2_prepare(a.ctypes.data, b.ctypes.data, rows, n, k)
            return lib.ozr_dot2_run(threads)
    rows, _ = calibrate_rows(run, threads, n, 10.0)  # each step about 10 s of CPU work
    times = []
    for _ in range(args.warmup):
        run(rows)
    for _ in range(args.steps):
        times.append(run(rows))
    t = statistics.median(times)
    value = 2.0 * rows * n * k / t / 1e12
    sample = (f"Dot2 reference_gemm (evaluation/numerics.hpp:58-93) on the first {rows} rows of C per step "
              f"({rows}x{n}x{k}, {2.0 * rows * n * k:.3g} FP64 flops), median of {args.steps} steps")
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": "TFLOPS", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "weak" if world == 1 else "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": headline_config(args, world),
            "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def time_int8_cublaslt(m: int, n: int, k: int, gpu_index: int, seconds: float = 1.5) -> dict:
    """cuBLASLt's int8 GEMM (torch._int_mm, int8 x int8 -> int32, A row-major times B column-major) on one
    modulus-sized product m x n x k, run back to back for about `seconds` like the residue GEMM inside the
    timed steps, with the SM clock sampled meanwhile: the library's int8 rate on this GPU, the bar for
    the residue GEMM."""
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    a8 = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda", generator=g)
    b8 = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g).t()
    for _ in range(3):
        c32 = torch._int_mm(a8, b8)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    c32 = torch._int_mm(a8, b8)
    e1.record()
    torch.cuda.synchronize()
    reps = max(3, int(seconds / max(e0.elapsed_time(e1) * 1e-3, 1e-4)))
    with ClockSampler(gpu_index) as clocks:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            c32 = torch._int_mm(a8, b8)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del a8, b8, c32
    clk = clocks.summary()
    return {"tops": 2.0 * m * n * k / (ms * 1e-3) / 1e12, "ms": ms, "reps": reps, "sm_mhz": clk.get("sm_mhz"),
            "reasons": clk.get("reasons"), "shape": f"{m}x{n}x{k} int8 -> int32 (torch._int_mm, cuBLASLt)"}


def reference_faithful_rows(oz, orc, A, B, m: int, n: int, k: int, plan, rows: np.ndarray) -> np.ndarray:
    """The reference device's result on the listed rows of C, for the accuracy comparison: this library's
    scaling, residues and exact int32 residue products (bit-identical to the reference's, pinned by the
    published device hashes) on the GPU, then the oracle's restatement of the reference's triple-float CRT
    reconstruction (recon_crt_proc.h, f64_tf.h) on the host. Checker only; outside the timed steps."""
    import torch

    r = len(rows)
    st = torch.cuda.current_stream().cuda_stream
    idx = torch.as_tensor(rows.astype(np.int64), device=A.device)
    Ar = A.view(m, k).index_select(0, idx).contiguous()
    mp, np_, kp = oz.padded_dims(r, n, k)
    S = plan.S
    dA = torch.zeros(mp, dtype=torch.int32, device="cuda")
    dB = torch.zeros(np_, dtype=torch.int32, device="cuda")
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    oz.call("oztt_ii_scale_rows", Ar.data_ptr(), r, k, k, plan.shift, dA.data_ptr(), None, flags.data_ptr(), st)
    oz.call("oztt_ii_scale_cols", B.data_ptr(), k, n, n, plan.shift, dB.data_ptr(), None, flags[1:].data_ptr(), st)
    ra = torch.zeros(S * mp * kp, dtype=torch.int8, device="cuda")
    rb = torch.zeros(S * np_ * kp, dtype=torch.int8, device="cuda")
    oz.call("oztt_ii_split_rows", Ar.data_ptr(), r, k, k, dA.data_ptr(), plan, ra.data_ptr(), mp, kp, st)
    oz.call("oztt_ii_split_cols", B.data_ptr(), k, n, n, dB.data_ptr(), plan, rb.data_ptr(), np_, kp, st)
    cs = torch.empty(S * mp * np_, dtype=torch.int32, device="cuda")
    oz.call("oztt_ii_residue_gemm", ra.data_ptr(), rb.data_ptr(), mp, np_, kp, plan, 0, cs.data_ptr(), st)
    torch.cuda.synchronize()
    del ra, rb
    host = np.ascontiguousarray(cs.view(S, mp, np_)[:, :r, :n].cpu().numpy()).reshape(-1)
    del cs
    oplan = orc.crt_plan(plan.moduli_list, plan.b, plan.two_pass)
    return orc.recon(host, r, n, dA[:r].cpu().numpy(), dB[:n].cpu().numpy(), oplan, exact=False)


# ---- Scheme I INT8 (a separate workload, one GPU) -------------------------------------------------------
def run_scheme_i(args) -> None:
    """One step = one pass of the Scheme I INT8 pipeline (scale -> slice -> diagonal products on the
    tensor cores -> exact Horner reconstruction) with the operands resident in HBM."""
    import torch

    import oztt_b200 as oz

    m = n = k = args.size
    a, b = oz.eval_inputs(m, n, k, args.phi, args.seed)
    A = torch.from_numpy(a).cuda()
    B = torch.from_numpy(b).cuda()
    C = torch.empty(m * n, dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    peaks = measured_peaks()
    fmt = getattr(oz.Format, args.format)
    for req in [int(x) for x in args.slices.split(",")]:
        # the slice count as Context::gemm selects it, from statistics measured on the device (the host
        # planner is timed beside it)
        t_plan = time.perf_counter()
        plan = oz.i_plan_device(A.data_ptr(), B.data_ptr(), m, n, k, slices=req, fmt=fmt, stream=stream)
        t_plan = time.perf_counter() - t_plan
        t_host = time.perf_counter()
        host_plan = oz.i_int8_plan(a, b, m, n, k, slices=req, fmt=fmt)
        t_host = time.perf_counter() - t_host
        assert host_plan.p == plan.p, "device and host slice selection disagree"
        p = plan.p

        def step():
            return oz.i_int8_run_device(A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, plan, stream, 0,
                                        timed=True)

        for _ in range(max(args.warmup, 0)):
            step()
        stage_sum = [0.0] * 5
        with ClockSampler(0) as clocks:
            torch.cuda.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            for _ in range(args.steps):
                stage_sum = [x + y for x, y in zip(stage_sum, step())]
            ev1.record()
            torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / args.steps
        st = [x / args.steps for x in stage_sum]
        pairs = p * (p + 1) // 2
        gemm_ops = 2.0 * m * n * k * pairs
        gemm_tops = gemm_ops / (st[3] * 1e-3) / 1e12
        int8_peak = 2.0 * peaks["bf16_tflops_sustained"]
        line = {"metric": f"Ozaki-I {args.format} effective FP64 TFLOPS at m=n=k={m}",
                "value": 2.0 * m * n * k / (ms * 1e-3) / 1e12,
                "unit": "TFLOPS", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f64 (int8-held slice products, s32 accumulate)",
                "data": f"synthetic: evaluation/numerics.hpp generator, phi={args.phi}, mt19937 seed {args.seed}",
                "config": {"workload": f"Scheme I {args.format} {m}x{n}x{k}", "slices": p, "radix": plan.radix,
                           "slices_selected_from_input": bool(plan.auto_p), "slice_pair_products": pairs,
                           "planning_s": round(t_plan, 3), "planning": "device-measured statistics",
                           "planning_s_host_planner": round(t_host, 3),
                           "l2": "inputs larger than the 126 MB L2; no flush"},
                "stage_ms": {"scale_rows": st[0], "scale_cols": st[1], "slice": st[2], "diag_gemm": st[3],
                             "recon": st[4]},
                "roofline": {"bound": "tensor", "kernel": "residue_gemm_kernel<2> (tcgen05 kind::i8, diagonals)",
                             "achieved": gemm_tops, "peak": int8_peak, "unit": "TOP/s (int8)",
                             "frac": gemm_tops / int8_peak,
                             "peak_source": f"2 x bf16_tflops_sustained of MEASURED_PEAKS.json ({peaks['source']}): "
                                            "the diagonal GEMM runs inside steps of tens of ms, back to back",
                             "algorithmic": f"2*m*n*k*p(p+1)/2 = {gemm_ops:.4g} int8 ops per launch"},
                "gpu_launches": 7 * args.steps, "clocks": clocks.summary()}
        if args.e2e_steps > 0:
            # the same request through the public API from pinned host buffers (the slice count selected
            # on the device when not fixed)
            ha = torch.from_numpy(a).pin_memory().numpy()
            hb = torch.from_numpy(b).pin_memory().numpy()
            hc = torch.empty(m * n, dtype=torch.float64).pin_memory().numpy()
            ctx = oz.Context(oz.DeviceOptions(device_id=0))
            opt = oz.Options(scheme=oz.Scheme.I, format=fmt, slices=req)
            ctx.gemm(ha, hb, hc, m, n, k, opt)  # warm-up
            times = []
            for _ in range(args.e2e_steps):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                ctx.gemm(ha, hb, hc, m, n, k, opt)
                times.append(time.perf_counter() - t0)
            e2e_s = statistics.median(times)
            phases = oz.ii_int8_last_phases()
            line["e2e"] = {"value": 2.0 * m * n * k / e2e_s / 1e12, "unit": "TFLOPS", "s_per_step": e2e_s,
                           "h2d_bytes_per_step": 8 * (m * k + k * n), "d2h_bytes_per_step": 8 * m * n,
                           "phases_ms_last_call": {key: round(v, 2) if isinstance(v, float) else v
                                                   for key, v in phases.items()},
                           "path": "ozTTgemm::Context::gemm via oztt_gemm"}
            del ha, hb, hc
        print(json.dumps(line), flush=True)


def run_digit(args) -> None:
    """One step = one pass of the Scheme II pipeline of a digit format (FP8, BF16, FP16, TF32: scale -> digit
    split -> digit products on the tensor cores with the composition in the epilogue -> exact CRT
    reconstruction) with the operands resident in HBM, for each max_moduli and reconstruction setting of the
    configuration; a setting the planner rejects prints its message instead of a number."""
    import torch

    import oztt_b200 as oz

    m = n = args.size
    k = 2 * args.size
    a, b = oz.eval_inputs(m, n, k, args.phi, args.seed)
    A = torch.from_numpy(a).cuda()
    B = torch.from_numpy(b).cuda()
    C = torch.empty(m * n, dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    peaks = measured_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops_sustained"]
    fmt = getattr(oz.Format, args.format)
    workload = f"Scheme II {args.format} digits {m}x{n}x{k}, phi={args.phi}"
    for S_req in [int(x) for x in args.moduli.split(",")]:
        for passes in [int(x) for x in args.passes.split(",")]:
            base = {"metric": f"Ozaki-II {args.format} effective FP64 TFLOPS at m=n={m}, k={k}", "unit": "TFLOPS",
                    "n_gpus": 1, "config": {"workload": workload, "max_moduli": S_req, "reconstruction_passes": passes}}
            t_plan = time.perf_counter()
            try:
                plan = oz.digit_plan_device(A.data_ptr(), B.data_ptr(), m, n, k, max_moduli=S_req,
                                            reconstruction=passes, stream=stream, fmt=fmt)
            except (RuntimeError, ValueError) as exc:
                print(json.dumps({**base, "value": None, "rejected": str(exc)}), flush=True)
                continue
            t_plan = time.perf_counter() - t_plan

            def step():
                return oz.digit_run_device(A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, plan, stream, 0,
                                         timed=True)

            for _ in range(max(args.warmup, 0)):
                step()
            stage_sum = [0.0] * 6
            with ClockSampler(0) as clocks:
                torch.cuda.synchronize()
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record()
                for _ in range(args.steps):
                    stage_sum = [x + y for x, y in zip(stage_sum, step())]
                ev1.record()
                torch.cuda.synchronize()
            ms = ev0.elapsed_time(ev1) / args.steps
            st = [x / args.steps for x in stage_sum]
            mp, np_, kp = -(-m // 128) * 128, -(-n // 256) * 256, -(-k // 128) * 128
            gemm_ops = 2.0 * mp * np_ * kp * plan.nprod
            gemm_tops = gemm_ops / (st[4] * 1e-3) / 1e12
            line = {**base, "value": 2.0 * m * n * k / (ms * 1e-3) / 1e12, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": f"f64 (int8-held {args.format} digit products, s32 accumulate)",
                    "data": f"synthetic: evaluation/numerics.hpp generator, phi={args.phi}, mt19937 seed {args.seed}",
                    "config": {**base["config"], "moduli": plan.base.S, "integer_bits": plan.base.b,
                               "passes_planned": 2 if plan.base.two_pass else 1, "digit_planes": plan.nplane,
                               "digit_products": plan.nprod, "gemm_outputs": plan.nout,
                               "planning_s": round(t_plan, 3), "planning": "device-measured statistics",
                               "l2": "inputs larger than the 126 MB L2; no flush"},
                    "stage_ms": {"scale_rows": st[0], "scale_cols": st[1], "split_rows": st[2], "split_cols": st[3],
                                 "digit_gemm": st[4], "recon": st[5]},
                    "roofline": {"bound": "tensor", "kernel": "residue_gemm_kernel<3> (tcgen05 kind::i8, digit outputs, "
                                                              "composition in the epilogue)",
                                 "achieved": gemm_tops, "peak": int8_peak, "unit": "TOP/s (int8)",
                                 "frac": gemm_tops / int8_peak,
                                 "peak_source": f"2 x bf16_tflops_sustained of MEASURED_PEAKS.json ({peaks['source']})",
                                 "algorithmic": f"2*mp*np*kp*nprod = {gemm_ops:.4g} int8 ops per launch"},
                    "gpu_launches": 7 * args.steps, "clocks": clocks.summary()}
            if args.e2e_steps > 0:
                # the same setting through the public API from pinned host buffers (streamed upload with the
                # statistics, banded pipeline with the read-back overlapped)
                ha = torch.from_numpy(a).pin_memory().numpy()
                hb = torch.from_numpy(b).pin_memory().numpy()
                hc = torch.empty(m * n, dtype=torch.float64).pin_memory().numpy()
                ctx = oz.Context(oz.DeviceOptions(device_id=0))
                opt = oz.Options(format=fmt, max_moduli=S_req, reconstruction=passes)
                ctx.gemm(ha, hb, hc, m, n, k, opt)  # warm-up
                times = []
                for _ in range(args.e2e_steps):
                    torch.cuda.synchronize()
                    t0 = time.perf_counter()
                    ctx.gemm(ha, hb, hc, m, n, k, opt)
                    times.append(time.perf_counter() - t0)
                e2e_s = statistics.median(times)
                phases = oz.ii_int8_last_phases()
                line["e2e"] = {"value": 2.0 * m * n * k / e2e_s / 1e12, "unit": "TFLOPS", "s_per_step": e2e_s,
                               "h2d_bytes_per_step": 8 * (m * k + k * n), "d2h_bytes_per_step": 8 * m * n,
                               "phases_ms_last_call": {key: round(v, 2) if isinstance(v, float) else v
                                                       for key, v in phases.items()},
                               "path": "ozTTgemm::Context::gemm via oztt_gemm (streamed upload and statistics, "
                                       "banded pipeline, overlapped read-back)"}
                del ha, hb, hc
            if not args.no_accuracy:
                sys.path.insert(0, str(ROOT / "tests"))
                try:
                    from oracle_lib import Oracle  # checker only

                    rows = np.linspace(0, m - 1, 4).astype(np.uint64)
                    line["max_rel_err"] = Oracle().maxrel_f128(a, b, C.cpu().numpy(), m, n, k, rows=rows)
                    line["accuracy_sample"] = "4 rows of C (all columns) vs a binary128 reference"
                except Exception as exc:  # noqa: BLE001
                    line["accuracy_error"] = str(exc)
            print(json.dumps(line), flush=True)


# ---- the GPU arm --------------------------------------------------------------------------------------
def run_single(args) -> None:
    """N = 1: the metric point m = n = k = 16384 on one GPU."""
    import torch

    import oztt_b200 as oz

    rank, world, local = 0, 1, int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    m = n = k = args.size
    # the evaluator's stream: all of A, then all of B
    a, b = oz.eval_inputs(m, n, k, args.phi, args.seed)
    A = torch.from_numpy(a).cuda()
    B = torch.from_numpy(b).cuda()
    t_plan = time.perf_counter()
    # as Context::gemm plans: the policy statistics measured on the device
    plan = oz.ii_int8_plan_device(A.data_ptr(), B.data_ptr(), m, n, k, stream=torch.cuda.current_stream().cuda_stream)
    t_plan = time.perf_counter() - t_plan
    C = torch.empty(m * n, dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def step():
        return oz.ii_int8_run_device_timed(A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, plan, stream, local)

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()
    stage_sum = [0.0] * 6
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(args.steps):
            st = step()
            stage_sum = [x + y for x, y in zip(stage_sum, st)]
        ev1.record()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    stage_ms = [x / args.steps for x in stage_sum]
    flops = 2.0 * m * n * k * world
    value = flops / (ms * 1e-3) / 1e12
    clk = clocks.summary()

    # ---- roofline of the residue GEMM (dominant kernel) --------------------------------------------
    peaks = measured_peaks()
    S = plan.S
    gemm_ops = 2.0 * m * n * k * S  # int8 multiply-adds of all moduli in one launch (x2 ops)
    gemm_tops = gemm_ops / (stage_ms[4] * 1e-3) / 1e12
    # B200 dense int8 = 2 x dense bf16. The GEMM is timed inside back-to-back steps (a long run under
    # the power cap), so the sustained figure is its denominator; the burst one is reported beside it.
    int8_peak = 2.0 * peaks["bf16_tflops_sustained"]
    int8_burst = 2.0 * peaks["bf16_tflops"]
    # HBM-bound stages against the measured copy bandwidth
    split_bytes = 8.0 * (m * k + k * n) + S * (m * k + k * n)
    recon_bytes = S * m * n + 8.0 * m * n
    result = {"metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
              "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
              "vs_baseline": None, "dtype": "f64 (int8 residue products, s32 accumulate)",
              "data": "synthetic: evaluation/numerics.hpp generator (u-0.5)*exp(phi*z), mt19937 seed "
                      f"{args.seed}",
              "config": headline_config(args, world),
              "plan": {"moduli": S, "moduli_set": plan.moduli_list, "integer_bits": plan.b,
                       "reconstruction_passes": 2 if plan.two_pass else 1, "planning_s": round(t_plan, 3),
                       "planning": "device-measured statistics"},
              "moduli_roofline": {
                  "tflops": int8_peak * world / S, "frac": value / (int8_peak * world / S),
                  "meaning": "whole-job effective FP64 TFLOPS the sustained int8 tensor rate of the N GPUs "
                             "allows with S moduli (2mnk FP64 flops cost 2mnk*S int8 ops); frac = value / that"},
              "vs_fp64_peak": {"fp64_peak_tflops": FP64_PEAK_TFLOPS * world,
                               "ratio": value / (FP64_PEAK_TFLOPS * world),
                               "source": "B200 nominal dense FP64 (vector and tensor core), NVIDIA datasheet, "
                                         "times the N GPUs"},
              "stage_ms": {"scale_rows": stage_ms[0], "scale_cols": stage_ms[1], "split_rows": stage_ms[2],
                           "split_cols": stage_ms[3], "residue_gemm": stage_ms[4], "recon": stage_ms[5]},
              "stages": "scale_cols = B transposed on the device and its rows scaled; split_cols = B^T's rows split",
              "roofline": {"bound": "tensor", "kernel": "residue_gemm_kernel<1> (tcgen05 kind::i8)",
                           "achieved": gemm_tops, "peak": int8_peak, "unit": "TOP/s (int8)",
                           "frac": gemm_tops / int8_peak, "frac_of_burst": gemm_tops / int8_burst,
                           "peak_source": f"2 x bf16_tflops_sustained of MEASURED_PEAKS.json ({peaks['source']}); "
                                          f"burst 2 x bf16_tflops = {int8_burst:.1f}",
                           "traffic": gemm_traffic(m, n, k, S),
                           "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of residue_gemm_kernel<1> "
                                             "captured by ncu at 4096^3 with S = 16 (537.35 MB + 246.64 MB), scaled "
                                             "by S*(mk + nk + mn) to this launch",
                           "algorithmic": f"2*m*n*k*S = {gemm_ops:.4g} int8 ops per launch"},
              "hbm_stages": {
                  "split_GBps": (split_bytes / ((stage_ms[2] + stage_ms[3]) * 1e-3)) / 1e9,
                  "recon_GBps": (recon_bytes / (stage_ms[5] * 1e-3)) / 1e9,
                  "peak_GBps": peaks["hbm_gbs"]},
              "gpu_launches": 7 * args.steps,
              "clocks": clk}

    # ---- cuBLAS DGEMM on the same GPU, and the accuracy of both on sampled rows ----------------------
    if rank == 0:
        A2, B2 = A.view(m, k), B.view(k, n)
        for _ in range(2):
            D = A2 @ B2
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            D = A2 @ B2
        e1.record()
        torch.cuda.synchronize()
        dms = e0.elapsed_time(e1) / 3
        result["cublas_dgemm"] = {"ms": dms, "tflops": 2.0 * m * n * k / (dms * 1e-3) / 1e12}
        result["vs_cublas_dgemm"] = (2.0 * m * n * k / (ms * 1e-3) / 1e12) / result["cublas_dgemm"]["tflops"]
        if not args.no_accuracy:
            sys.path.insert(0, str(ROOT / "tests"))
            try:
                from oracle_lib import Oracle  # checker only

                orc = Oracle()
                rows = np.linspace(0, m - 1, 8).astype(np.int64)
                idx = torch.as_tensor(rows, device="cuda")
                c_oz = C.view(m, n).index_select(0, idx).cpu().numpy()
                c_dg = D.index_select(0, idx).cpu().numpy()
                del D
                c_ref = reference_faithful_rows(oz, orc, A, B, m, n, k, plan, rows)
                e_oz, e_dg, e_ref = orc.maxrel_f128_rows(a, b, [c_oz, c_dg, c_ref], m, n, k, rows)
                result["max_rel_err"] = e_oz
                result["cublas_dgemm"]["max_rel_err"] = e_dg
                result["max_rel_err_reference"] = e_ref
                result["max_rel_err_ratio_to_reference"] = e_oz / e_ref if e_ref > 0 else None
                result["accuracy_sample"] = (
                    "8 rows of C (all columns) vs a binary128 reference; max_rel_err_reference is the reference "
                    "device's result on the same rows (its integer stages are this library's, bit-identical; its "
                    "triple-float CRT reconstruction restated on the host)")
            except Exception as exc:  # noqa: BLE001
                result["max_rel_err"] = None
                result["accuracy_error"] = str(exc)
        if "D" in locals():
            del D
        torch.cuda.empty_cache()
        # cuBLASLt's int8 GEMM on one modulus's product, back to back for about the length of the timed
        # steps: the library rate the residue GEMM (all S moduli per launch) is compared with, clock for clock
        lt = time_int8_cublaslt(m, n, k, local, seconds=max(1.0, ms * args.steps * 1e-3))
        result["int8_cublaslt_tops"] = lt["tops"]
        result["int8_cublaslt"] = lt
        result["roofline"]["vs_int8_cublaslt"] = {
            "residue_gemm_tops": gemm_tops, "residue_gemm_sm_mhz": clk.get("sm_mhz"),
            "cublaslt_tops": lt["tops"], "cublaslt_sm_mhz": lt["sm_mhz"],
            "ratio": gemm_tops / lt["tops"],
            "ratio_per_clock": (gemm_tops / clk["sm_mhz"]) / (lt["tops"] / lt["sm_mhz"])
            if clk.get("sm_mhz") and lt.get("sm_mhz") else None}

    # ---- end to end through the public API --------------------------------------------------------
    if args.e2e_steps > 0:
        ha = torch.from_numpy(a).pin_memory().numpy()
        hb = torch.from_numpy(b).pin_memory().numpy()
        hc = torch.empty(m * n, dtype=torch.float64).pin_memory().numpy()
        ctx = oz.Context(oz.DeviceOptions(device_id=local))
        opt = oz.Options(format=oz.Format.INT8)
        ctx.gemm(ha, hb, hc, m, n, k, opt)  # warm-up
        times = []
        for _ in range(args.e2e_steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            ctx.gemm(ha, hb, hc, m, n, k, opt)
            times.append(time.perf_counter() - t0)
        e2e_s = statistics.median(times)
        phases = oz.ii_int8_last_phases()
        result["e2e"] = {"value": flops / e2e_s / 1e12, "unit": "TFLOPS", "s_per_step": e2e_s,
                         "phases_ms_last_call": {key: round(v, 2) if isinstance(v, float) else v
                                                 for key, v in phases.items()},
                         "h2d_bytes_per_step": 8 * (m * k + k * n), "d2h_bytes_per_step": 8 * m * n,
                         "path": "ozTTgemm::Context::gemm via oztt_gemm: pinned H2D in the order B's first column block, A's "
                                 "first half of rows, B's next four column blocks, the rest of A, B's last three blocks; the "
                                 "pipeline on a first plan estimated from A's first half and B's first block (each piece "
                                 "times everything already there as it lands); the host's value checks meanwhile, then "
                                 "each piece of C read back as it finishes; the reference's plan from bounds of the "
                                 "statistics measured as the operands landed (pipeline run again if it differs)"}
    # ---- CPU baseline (rank 0 at N=1) ------------------------------------------------------------------
    if not args.no_cpu_baseline:
        result["cpu_baseline"] = time_cpu_dot2(a, b, n, k, target_s=12.0)
    print(json.dumps(result), flush=True)


def run_tiled(args) -> None:
    """N > 1 (torchrun, one process per GPU): config 5, m = n = 2 * size, k = size (32768 x 32768 x 16384),
    strong scaling over a P x Q grid of output tiles. Rank 0 generates the whole A and B (the evaluator's
    stream) in its HBM; the panels are placed over NVLink (timed as placement_ms); every rank makes the
    reference's plan from the tiled statistics; a step is every rank's pipeline on its resident panels,
    timed with CUDA events, the maximum over ranks. The same problem on rank 0's GPU alone, under the same
    plan, is timed in the same run (config5_1gpu), and the gathered C is checked against it."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import oztt_b200 as oz
    from oztt_b200.distributed import DeviceStats, Grid, GridComm, gather_tiles, gemm_tiled, place_panels, \
        plan_ii_int8_tiled

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    comm = GridComm(Grid.of(rank, world))
    g = comm.grid
    m = n = 2 * args.size
    k = args.size
    stream = torch.cuda.current_stream().cuda_stream

    def max_over_ranks(values):
        t = torch.tensor(values, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(x) for x in t]

    a0 = b0 = None
    if rank == 0:
        a, b = oz.eval_inputs(m, n, k, args.phi, args.seed)
        a0, b0 = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        del a, b
    torch.cuda.synchronize()
    dist.barrier()
    # placement of the panels from rank 0 over NVLink: median of three
    times = []
    for _ in range(3):
        torch.cuda.synchronize()
        dist.barrier()
        t0 = time.perf_counter()
        a_p, b_q = place_panels(comm, a0, b0, m, n, k)
        torch.cuda.synchronize()
        times.append((time.perf_counter() - t0) * 1e3)
    place_ms = max_over_ranks([statistics.median(times)])[0]
    t0 = time.perf_counter()
    plan = plan_ii_int8_tiled(comm, a_p, b_q, m, n, k, stats=DeviceStats(stream))
    t_plan = max_over_ranks([time.perf_counter() - t0])[0]
    (r0, r1), (c0, c1) = g.row_range(m), g.col_range(n)
    mt, nt = r1 - r0, c1 - c0
    C = torch.empty(mt * nt, dtype=torch.float64, device="cuda")

    def step():
        return oz.ii_int8_run_device_timed(a_p.data_ptr(), b_q.data_ptr(), C.data_ptr(), mt, nt, k, plan, stream, local)

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    stage_sum = [0.0] * 6
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(args.steps):
            stage_sum = [x + y for x, y in zip(stage_sum, step())]
        ev1.record()
        torch.cuda.synchronize()
    dist.barrier()
    mx = max_over_ranks([ev0.elapsed_time(ev1) / args.steps] + [x / args.steps for x in stage_sum])
    ms, stage_ms = mx[0], mx[1:]
    flops = 2.0 * m * n * k
    value = flops / (ms * 1e-3) / 1e12
    clk = clocks.summary()
    # the tiles gathered to rank 0 (assembly on request); the first gather also sets up NCCL's
    # point-to-point channels and C's memory, so the second is the one reported
    gather_times = []
    for _ in range(2):
        c_all = None
        torch.cuda.synchronize()
        dist.barrier()
        t0 = time.perf_counter()
        c_all = gather_tiles(comm, C, m, n, to="rank0")
        torch.cuda.synchronize()
        gather_times.append((time.perf_counter() - t0) * 1e3)
    gather_ms, gather_first_ms = max_over_ranks([gather_times[1], gather_times[0]])
    # the same problem on rank 0's GPU alone, same plan: the strong-scaling baseline and the check
    single = None
    if rank == 0:
        c1 = torch.empty(m * n, dtype=torch.float64, device="cuda")

        def step1():
            oz.ii_int8_run_device(a0.data_ptr(), b0.data_ptr(), c1.data_ptr(), m, n, k, plan, stream, local)

        step1()
        reps = max(2, min(args.steps, 5))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            step1()
        e1.record()
        torch.cuda.synchronize()
        ms1 = e0.elapsed_time(e1) / reps
        same = bool(torch.equal(c_all.view(torch.int64), c1.view(torch.int64)))
        single = {"ms_per_step": ms1, "value": flops / (ms1 * 1e-3) / 1e12, "steps": reps,
                  "tiled_C_bit_identical": same,
                  "meaning": "the same 32768x32768x16384 problem on rank 0's GPU alone under the same plan"}
        del c1
    del c_all
    torch.cuda.empty_cache()
    dist.barrier()
    # end to end through the public multi-GPU call: each rank's panels in pinned host memory, uploaded,
    # planned (tiled statistics), computed, and its tile of C read back into pinned host memory
    e2e = None
    if args.e2e_steps > 0:
        ha = a_p.cpu().pin_memory()
        hb = b_q.cpu().pin_memory()
        hc = torch.empty(mt * nt, dtype=torch.float64).pin_memory()
        gemm_tiled(comm, ha, hb, m, n, k, source="panels", gather="host", out=hc)
        e2e_times, phases = [], {}
        for _ in range(args.e2e_steps):
            torch.cuda.synchronize()
            dist.barrier()
            t0 = time.perf_counter()
            res = gemm_tiled(comm, ha, hb, m, n, k, source="panels", gather="host", out=hc)
            e2e_times.append(time.perf_counter() - t0)
            phases = res.phases_ms
        e2e_s = max_over_ranks([statistics.median(e2e_times)])[0]
        e2e = {"value": flops / e2e_s / 1e12, "unit": "TFLOPS", "s_per_step": e2e_s,
               "h2d_bytes_per_step": 8 * world * (mt * k + k * nt),
               "d2h_bytes_per_step": 8 * m * n,
               "phases_ms_rank0_last_call": {kk: round(v, 2) for kk, v in phases.items()},
               "path": "oztt_b200.distributed.gemm_tiled(source='panels', gather='host'): every rank uploads its A row "
                       "panel and B column panel from pinned host memory, the plan from the tiled statistics "
                       "(NCCL), the tile pipeline, the tile read back into pinned host memory; max over ranks"}
        del ha, hb, hc
    peaks = measured_peaks()
    S = plan.S
    gemm_ops = 2.0 * mt * nt * k * S
    gemm_tops = gemm_ops / (stage_ms[4] * 1e-3) / 1e12
    int8_peak = 2.0 * peaks["bf16_tflops_sustained"]
    result = {"metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
              "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
              "vs_baseline": None, "dtype": "f64 (int8 residue products, s32 accumulate)",
              "data": "synthetic: evaluation/numerics.hpp generator (u-0.5)*exp(phi*z), mt19937 seed "
                      f"{args.seed}, the whole A then the whole B",
              "config": headline_config(args, world),
              "grid": {"P": g.P, "Q": g.Q, "tile": f"{mt}x{nt}x{k}"},
              "plan": {"moduli": S, "moduli_set": plan.moduli_list, "integer_bits": plan.b,
                       "reconstruction_passes": 2 if plan.two_pass else 1, "planning_s": round(t_plan, 3),
                       "planning": "tiled statistics: panel measurements gathered and summed in the reference's "
                                   "order, the sketch chained along grid row 0 (NCCL)"},
              "stage_ms": {"scale_rows": stage_ms[0], "scale_cols": stage_ms[1], "split_rows": stage_ms[2],
                           "split_cols": stage_ms[3], "residue_gemm": stage_ms[4], "recon": stage_ms[5]},
              "placement_ms": place_ms,
              "placement": "rank 0's A and B to every rank's panels: one batched group of NCCL sends from rank 0 "
                           "(each byte it does not keep, once), then NCCL broadcasts along grid rows and columns; "
                           "outside the timed steps (inputs resident in HBM)",
              "gather_ms": gather_ms, "gather_first_ms": gather_first_ms,
              "moduli_roofline": {"tflops": int8_peak * world / S, "frac": value / (int8_peak * world / S)},
              "roofline": {"bound": "tensor", "kernel": "residue_gemm_kernel<1> (tcgen05 kind::i8), per GPU",
                           "achieved": gemm_tops, "peak": int8_peak, "unit": "TOP/s (int8)",
                           "frac": gemm_tops / int8_peak,
                           "peak_source": f"2 x bf16_tflops_sustained of MEASURED_PEAKS.json ({peaks['source']})",
                           "traffic": gemm_traffic(mt, nt, k, S),
                           "algorithmic": f"2*m_p*n_q*k*S = {gemm_ops:.4g} int8 ops per launch"},
              "gpu_launches": 7 * args.steps * world, "clocks": clk}
    if single is not None:
        result["config5_1gpu"] = single
    if e2e is not None:
        result["e2e"] = e2e
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.scheme == "I":
        run_scheme_i(args)
        return
    if args.format != "INT8":
        run_digit(args)
        return
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_tiled(args)
    else:
        run_single(args)


if __name__ == "__main__":
    main()
