"""Generate tests/golden/baseline_plans.json: the reference planners' decisions on the BASELINE
configurations (test infrastructure).

The plans are made by the reference's own planner code compiled in place under oracle/_ref
(oracle/Makefile, target `ref`): the Scheme II INT8 policy and moduli selection (ref_plan.cpp:
choose_precision_policy + ozaki2_choose_moduli + oz2_recon1_log2), the Scheme II digit-format planner
(ref_plan_digit.cpp, one library per format) and the Scheme I slice-count selection (ref_plan1.cpp:
oz_fp64_p). The inputs are the evaluator's generator (evaluation/numerics.hpp:19-38) restated by the
oracle, (u - 1/2) exp(phi z) with mt19937 seed 0, padded as the reference pads (m, n to 64, k to 32):

  config 1   Scheme II INT8, 256^3, phi 0.5, auto moduli, Automatic reconstruction
  config 2   Scheme II INT8, 4096^3, phi 0.5, auto moduli, TwoPass
  config 3   Scheme I INT8, 8192^3, phi 1.0, slices auto (the fixed sweep 4..12 needs no plan)
  config 4   Scheme II FP8 and BF16, 8192 x 8192 x 16384, phi 4.0, max_moduli 12/16/20/24 x OnePass/TwoPass
  metric     Scheme II INT8, 16384^3, phi 0.5, auto moduli, Automatic reconstruction

Recorded per plan: whether the reference accepts it, the moduli, width, passes and the policy statistics
(as exact hex floats). Takes several minutes and about 20 GB of host memory; run where oracle/_ref was
built (the reference tree is needed only to build it):

    python tests/golden/make_baseline_plans.py
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parents[1]))

from oracle_lib import Oracle, RefPlan, RefPlan1, RefPlanDigit, pad, round_up  # noqa: E402
from oztt_b200 import DigitPlan  # noqa: E402  (the ctypes layout of oztt_digit_plan only; no library load)

FORMATS = {"FP8": 4, "BF16": 0}


def padded(orc: Oracle, m: int, n: int, k: int, phi: float, seed: int):
    a, b = orc.gen_inputs(m, n, k, phi, seed)
    M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
    if (M, N, K) == (m, n, k):
        return a, b, M, N, K
    return pad(a, m, k, M, K), pad(b, k, n, K, N), M, N, K


def hexs(vals) -> list[str]:
    return [float.hex(float(v)) for v in vals]


def int8_case(ref: RefPlan, orc: Oracle, name: str, size: int, phi: float, passes: int) -> dict:
    t = time.time()
    a, b, M, N, K = padded(orc, size, size, size, phi, 0)
    rc, p = ref.plan(a, b, M, N, K, 0, passes, 0)
    rec = {"name": name, "scheme": "II", "format": "INT8", "m": size, "n": size, "k": size, "phi": phi, "seed": 0,
           "max_moduli": 0, "passes": passes, "fixed_bits": 0, "rc": rc, "S": p.S, "b": p.b, "b_cap": p.b_cap,
           "two_pass": p.two_pass, "moduli": p.moduli, "stats": hexs((p.TA, p.TB, p.nA, p.nB, p.nC)),
           "recon1_log2": float.hex(p.recon1_log2)}
    print(f"{name}: S={p.S} b={p.b} two_pass={p.two_pass} ({time.time() - t:.1f} s)", flush=True)
    return rec


def digit_cases(orc: Oracle) -> list[dict]:
    m = n = 8192
    k = 16384
    a, b, M, N, K = padded(orc, m, n, k, 4.0, 0)
    out = []
    for fname, fmt in FORMATS.items():
        ref = RefPlanDigit(fmt)
        for S_req in (12, 16, 20, 24):
            for passes in (1, 2):
                t = time.time()
                rc, p = ref.plan(a, b, M, N, K, DigitPlan, S_req, passes, 0)
                base = p.base
                rec = {"name": f"config4-{fname}-S{S_req}-p{passes}", "scheme": "II", "format": fname, "m": m, "n": n,
                       "k": k, "phi": 4.0, "seed": 0, "max_moduli": S_req, "passes": passes, "fixed_bits": 0,
                       "rc": rc, "S": base.S, "b": base.b, "b_cap": base.b_cap, "two_pass": base.two_pass,
                       "moduli": [int(base.moduli[i]) for i in range(base.S)],
                       "stats": hexs((base.TA, base.TB, base.nA, base.nB, base.nC)),
                       "nplane": p.nplane, "nprod": p.nprod, "nout": p.nout}
                print(f"{rec['name']}: rc={rc} S={base.S} b={base.b} nprod={p.nprod} ({time.time() - t:.1f} s)",
                      flush=True)
                out.append(rec)
    return out


def scheme1_case(orc: Oracle) -> dict:
    t = time.time()
    a, b, M, N, K = padded(orc, 8192, 8192, 8192, 1.0, 0)
    p = RefPlan1().slices(a, b, M, N, K)
    print(f"config3: p={p} ({time.time() - t:.1f} s)", flush=True)
    return {"name": "config3-auto", "scheme": "I", "format": "INT8", "m": 8192, "n": 8192, "k": 8192, "phi": 1.0,
            "seed": 0, "slices": 0, "p": p}


def main() -> None:
    orc, ref = Oracle(), RefPlan()
    cases = [int8_case(ref, orc, "config1", 256, 0.5, 0), int8_case(ref, orc, "config2", 4096, 0.5, 2),
             scheme1_case(orc)]
    cases += digit_cases(orc)
    cases.append(int8_case(ref, orc, "metric", 16384, 0.5, 0))
    data = {"generator": "tests/golden/make_baseline_plans.py (reference planners compiled in oracle/_ref)",
            "cases": cases}
    (HERE / "baseline_plans.json").write_text(json.dumps(data, indent=1) + "\n")
    print(f"wrote {HERE / 'baseline_plans.json'}: {len(cases)} plans")


if __name__ == "__main__":
    main()
