"""Generate tests/golden/ref_cases.json from the reference's own host code (test infrastructure).

Run in the build container, where the reference tree exists and ``oracle/_ref`` has been built
(``make -C oracle ref``). It records, for a table of cases, what the reference itself decides and
computes:
  * moduli_table  ozaki2_choose_moduli of the INT8 route (src/backend/ozaki2/moduli.hpp:719-769)
                  over K, the limit on the number of moduli and the width cap;
  * plans         choose_moduli_and_width (plan.hpp:258-306) with the precision policy
                  (auto_precision.hpp) on seeded generator inputs;
  * emulations    the reference's host emulation of its device pipeline (oracle/ref_emu.cpp) on
                  seeded inputs: output hash (evaluation/numerics.hpp:46-57) of C.
plus the published device values of tools/validated/quick.csv:13. The GPU machine has no reference
tree; the tests read these fixtures there.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from oracle_lib import Oracle, RefEmu, RefPlan, pad, round_up  # noqa: E402

PUBLISHED = {
    # tools/validated/quick.csv:13 — Blackhole P150a device output, II INT8, n=128, seed 7,
    # uniform(-1,1), fixed_bits=54, one pass, 15 moduli.
    "source": "tools/validated/quick.csv:13",
    "n": 128, "phi": -1.0, "seed": 7, "fixed_bits": 54, "moduli": 15, "passes": 1,
    "output_hash": "fe063f5214e93e2e", "relative_fro": 4.68753276457e-17, "effective_bits": 54.2439488385,
}


def moduli_table(ref: RefPlan) -> list[dict]:
    out = []
    Ks = [32, 64, 96, 128, 256, 512, 1024, 2048, 3520, 4096, 7040, 8192, 14080, 16384, 32768, 65536, 131072,
          262144, 1048576, 4194304]
    for K in Ks:
        for num in (2, 8, 12, 14, 15, 16, 17, 20, 24):
            for b_cap in (30, 53, 54, 55, 56, 58, 60, 61, 64, 70, 80, 81, 90, 100):
                p = ref.choose_moduli(K, num, b_cap)
                out.append({"K": K, "num_moduli": num, "b_cap": b_cap, "ok": int(p.ok), "acc_ok": int(p.acc_ok),
                            "S": p.S, "b": p.b, "m_cap": p.m_cap, "ncand": p.ncand, "moduli": p.moduli,
                            "yi": [int(p.yi[i]) for i in range(p.S)]})
    return out


def plans(ref: RefPlan, orc: Oracle) -> list[dict]:
    out = []
    shapes = [(64, 64, 64), (3, 5, 7), (65, 67, 97), (128, 96, 160), (200, 72, 256)]
    for (m, n, k) in shapes:
        for phi in (-1.0, 0.5, 1.0, 2.0, 4.0, 8.0):
            for (max_moduli, passes, fixed_bits) in ((0, 0, 0), (0, 1, 0), (0, 2, 0), (20, 0, 0), (14, 0, 0),
                                                     (0, 0, 54), (0, 1, 54), (2, 0, 0)):
                a, b = orc.gen_inputs(m, n, k, phi, 11)
                M, N, K = round_up(m, 64), round_up(n, 64), round_up(k, 32)
                ap, bp = pad(a, m, k, M, K), pad(b, k, n, K, N)
                rc, p = ref.plan(ap, bp, M, N, K, max_moduli, passes, fixed_bits)
                out.append({"m": m, "n": n, "k": k, "phi": phi, "seed": 11, "max_moduli": max_moduli,
                            "passes": passes, "fixed_bits": fixed_bits, "rc": rc, "S": p.S, "b": p.b,
                            "two_pass": p.two_pass, "moduli": p.moduli, "b_cap": p.b_cap,
                            "stats": [float.hex(x) for x in (p.TA, p.TB, p.nA, p.nB, p.nC)]})
    return out


def emulations(emu: RefEmu, orc: Oracle) -> list[dict]:
    out = []
    cases = [(128, -1.0, 7, 54, 16, False), (64, -1.0, 3, 54, 16, True), (96, 0.5, 0, 56, 16, False),
             (96, 0.5, 0, 56, 16, True), (64, 1.0, 5, 61, 20, False), (64, 4.0, 1, 81, 24, False),
             (128, 2.0, 9, 58, 16, True)]
    for (n, phi, seed, bfix, num, two) in cases:
        a, b = orc.gen_inputs(n, n, n, phi, seed)
        N = round_up(n, 64)
        ap, bp = pad(a, n, n, N, N), pad(b, n, n, N, N)
        s, c, mods = emu.emulate(ap, bp, N, N, N, bfix, num, two)
        cc = c.reshape(N, N)[:n, :n].copy().reshape(-1)
        out.append({"n": n, "phi": phi, "seed": seed, "fixed_bits": bfix, "num_moduli": num, "two_pass": int(two),
                    "S": s, "moduli": mods, "output_hash": orc.output_hash(cc)})
    return out


def main() -> None:
    orc, ref, emu = Oracle(), RefPlan(), RefEmu()
    data = {"published": PUBLISHED, "moduli_table": moduli_table(ref), "plans": plans(ref, orc),
            "emulations": emulations(emu, orc)}
    (HERE / "ref_cases.json").write_text(json.dumps(data, separators=(",", ":")) + "\n")
    print(f"wrote {HERE / 'ref_cases.json'}: {len(data['moduli_table'])} selections, {len(data['plans'])} plans, "
          f"{len(data['emulations'])} emulations")


if __name__ == "__main__":
    main()
