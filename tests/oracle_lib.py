"""ctypes bindings of the CPU checkers (test infrastructure only).

* ``Oracle``  — oracle/liboz2oracle.so, this project's CPU restatement of the reference's Scheme II
  INT8 path (oracle/oz2_oracle.h documents every function and the reference source it follows).
* ``RefPlan`` / ``RefPlan1`` / ``RefEmu`` — oracle/_ref/*.so, the reference's own host code compiled in place
  (oracle/Makefile, target ``ref``); present only where they were built.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
ORACLE_SO = ROOT / "oracle" / "liboz2oracle.so"
REF_PLAN_SO = ROOT / "oracle" / "_ref" / "libozref_plan.so"
REF_EMU_SO = ROOT / "oracle" / "_ref" / "libozref_emu.so"
REF_PLAN1_SO = ROOT / "oracle" / "_ref" / "libozref_plan1.so"
REF_PLAN1_F8_SO = ROOT / "oracle" / "_ref" / "libozref_plan1_f8.so"

MAXS, MAXRP = 24, 5
P = ctypes.c_void_p


class OzoPlan(ctypes.Structure):
    _fields_ = [
        ("ok", ctypes.c_int32), ("acc_ok", ctypes.c_int32), ("S", ctypes.c_int32), ("b", ctypes.c_int32),
        ("nd", ctypes.c_int32), ("shift", ctypes.c_int32), ("two_pass", ctypes.c_int32), ("b_cap", ctypes.c_int32),
        ("m_cap", ctypes.c_int32), ("ncand", ctypes.c_int32), ("S_req", ctypes.c_int32),
        ("m", ctypes.c_int32 * MAXS), ("yi", ctypes.c_int32 * MAXS), ("rinv", ctypes.c_float * MAXS),
        ("c", (ctypes.c_float * MAXS) * 4), ("m16", ctypes.c_float * MAXS),
        ("rp0", (ctypes.c_float * MAXRP) * MAXS), ("rp1", (ctypes.c_float * MAXRP) * MAXS),
        ("rp2", (ctypes.c_float * MAXRP) * MAXS),
        ("nsmall0", ctypes.c_int32), ("nsmall1", ctypes.c_int32), ("nsmall2", ctypes.c_int32),
        ("W_hi", ctypes.c_uint32), ("W_lo", ctypes.c_uint32), ("qw", ctypes.c_int32), ("logM", ctypes.c_double),
        ("TA", ctypes.c_double), ("TB", ctypes.c_double), ("nA", ctypes.c_double), ("nB", ctypes.c_double),
        ("nC", ctypes.c_double), ("recon1_log2", ctypes.c_double),
    ]

    @property
    def moduli(self) -> list[int]:
        return [int(self.m[i]) for i in range(self.S)]


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Oracle:
    def __init__(self, path: Path = ORACLE_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (python -m oztt_b200.build)")
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.ozo_output_hash.restype = ctypes.c_uint64
        L.ozo_output_hash.argtypes = [P, ctypes.c_uint64]
        L.ozo_time_dot2_rows.restype = ctypes.c_double
        L.ozo_time_dot2_rows.argtypes = [P, P, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int]
        u64 = ctypes.c_uint64
        L.ozo_gen_inputs.argtypes = [P, P, u64, u64, u64, ctypes.c_double, ctypes.c_uint32]
        L.ozo_gen_pattern.argtypes = [P, P, u64, u64, u64, ctypes.c_int]
        L.ozo_plan_ii_int8.argtypes = [P, P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                       ctypes.c_int, ctypes.c_int, ctypes.POINTER(OzoPlan), ctypes.c_char_p,
                                       ctypes.c_size_t]
        L.ozo_choose_moduli_int8.argtypes = [ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.POINTER(OzoPlan)]
        L.ozo_scale.argtypes = [P, u64, u64, u64, ctypes.c_int, ctypes.c_int32, P, P, P]
        L.ozo_split.argtypes = [P, u64, u64, u64, ctypes.c_int, P, ctypes.POINTER(OzoPlan), P]
        L.ozo_digits.argtypes = [ctypes.c_double, ctypes.c_int32, ctypes.c_int, P]
        L.ozo_gemm_i32.argtypes = [P, P, u64, u64, u64, u64, P]
        L.ozo_recon_faithful.argtypes = [P, u64, u64, P, P, ctypes.POINTER(OzoPlan), P, u64]
        L.ozo_recon_exact.argtypes = [P, u64, u64, P, P, ctypes.POINTER(OzoPlan), P, u64]
        L.ozo_ii_int8_emulate.argtypes = [P, P, P, u64, u64, u64, ctypes.c_uint32, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.POINTER(OzoPlan), ctypes.c_char_p, ctypes.c_size_t]
        L.ozo_dot2_gemm.argtypes = [P, P, u64, u64, u64, P, P]
        L.ozo_accuracy.argtypes = [P, P, P, u64, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        L.ozo_maxrel_f128.argtypes = [P, P, P, u64, u64, u64, P, u64, ctypes.POINTER(ctypes.c_double)]
        L.ozo_maxrel_f128_rows.argtypes = [P, P, P, ctypes.c_int, u64, u64, u64, P, u64, P]
        L.ozo_i_slice.argtypes = [P, u64, u64, u64, ctypes.c_int, P, ctypes.c_int, P]
        L.ozo_i_gemm.argtypes = [P, P, ctypes.c_int, u64, u64, u64, P]
        L.ozo_i_recon_faithful.argtypes = [P, ctypes.c_int, u64, u64, P, P, P, u64]
        L.ozo_i_recon_exact.argtypes = [P, ctypes.c_int, u64, u64, P, P, P, u64]
        L.ozo_i_emulate.argtypes = [P, P, P, u64, u64, u64, ctypes.c_int, ctypes.c_int]
        L.ozo_scale_mode.argtypes = [P, u64, u64, u64, ctypes.c_int, ctypes.c_int32, ctypes.c_int, P, P, P]
        L.ozo_i_slice_fmt.argtypes = [P, u64, u64, u64, ctypes.c_int, P, ctypes.c_int, ctypes.c_int, P]
        L.ozo_i_recon_faithful_deferred.argtypes = [P, ctypes.c_int, ctypes.c_int, u64, u64, u64, P, P, P, u64]
        L.ozo_i_recon_exact_fmt.argtypes = [P, ctypes.c_int, ctypes.c_int, u64, u64, P, P, P, u64]
        L.ozo_i_emulate_fmt.argtypes = [P, P, P, u64, u64, u64, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.ozo_crt_plan.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(OzoPlan)]
        L.ozo_digit_split.argtypes = [P, u64, u64, u64, ctypes.c_int, P, ctypes.POINTER(OzoPlan), P, P]
        L.ozo_digit_gemm.argtypes = [P, P, P, u64, u64, u64, P]
        L.ozo_digit_compose.argtypes = [P, P, ctypes.POINTER(OzoPlan), u64, u64, P]
        L.ozo_recon_faithful_residue.argtypes = [P, u64, u64, P, P, ctypes.POINTER(OzoPlan), P, u64]
        L.ozo_digit_emulate.argtypes = [P, P, P, u64, u64, u64, P, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]

    # -- generators ---------------------------------------------------------------------------
    def gen_inputs(self, m: int, n: int, k: int, phi: float, seed: int) -> tuple[np.ndarray, np.ndarray]:
        a, b = np.empty(m * k), np.empty(k * n)
        self.lib.ozo_gen_inputs(ptr(a), ptr(b), m, n, k, phi, seed)
        return a, b

    def gen_pattern(self, m: int, n: int, k: int, mode: int) -> tuple[np.ndarray, np.ndarray]:
        a, b = np.empty(m * k), np.empty(k * n)
        self.lib.ozo_gen_pattern(ptr(a), ptr(b), m, n, k, mode)
        return a, b

    # -- planner ------------------------------------------------------------------------------
    def plan(self, ap: np.ndarray, bp: np.ndarray, M: int, N: int, K: int, max_moduli=0, passes=0,
             fixed_bits=0) -> tuple[int, OzoPlan, str]:
        p = OzoPlan()
        err = ctypes.create_string_buffer(512)
        rc = self.lib.ozo_plan_ii_int8(ptr(ap), ptr(bp), M, N, K, max_moduli, passes, fixed_bits, ctypes.byref(p),
                                       err, 512)
        return rc, p, err.value.decode()

    def choose_moduli(self, K: int, num_moduli: int, b_cap: int) -> OzoPlan:
        p = OzoPlan()
        self.lib.ozo_choose_moduli_int8(K, num_moduli, b_cap, ctypes.byref(p))
        return p

    # -- stages -------------------------------------------------------------------------------
    def scale(self, x: np.ndarray, rows: int, cols: int, col_mode: int, shift: int, ceil: int = 1):
        """ceil: 1 rounds the BF16 maxima up (scheme II, scheme I INT8), 0 truncates (scheme I FP8)."""
        nout = cols if col_mode else rows
        bf = np.zeros(nout, dtype=np.uint16)
        d = np.zeros(nout, dtype=np.int32)
        fl = np.zeros(1, dtype=np.uint32)
        self.lib.ozo_scale_mode(ptr(x), rows, cols, cols, col_mode, shift, ceil, ptr(bf), ptr(d), ptr(fl))
        return bf, d, int(fl[0])

    def split(self, x: np.ndarray, rows: int, cols: int, col_mode: int, delta: np.ndarray, plan: OzoPlan):
        out = np.zeros(plan.S * rows * cols, dtype=np.int8)
        self.lib.ozo_split(ptr(x), rows, cols, cols, col_mode, ptr(delta), ctypes.byref(plan), ptr(out))
        return out

    def digits(self, x: float, delta: int, nd: int) -> np.ndarray:
        out = np.zeros(nd, dtype=np.float32)
        self.lib.ozo_digits(x, delta, nd, ptr(out))
        return out

    def gemm_i32(self, ra: np.ndarray, rb: np.ndarray, S: int, M: int, N: int, K: int) -> np.ndarray:
        c = np.zeros(S * M * N, dtype=np.int32)
        bad = self.lib.ozo_gemm_i32(ptr(ra), ptr(rb), S, M, N, K, ptr(c))
        assert bad == 0, "int32 overflow in the oracle GEMM"
        return c

    def recon(self, cs: np.ndarray, M: int, N: int, dA: np.ndarray, dB: np.ndarray, plan: OzoPlan,
              exact: bool) -> np.ndarray:
        c = np.zeros(M * N)
        fn = self.lib.ozo_recon_exact if exact else self.lib.ozo_recon_faithful
        fn(ptr(cs), M, N, ptr(dA), ptr(dB), ctypes.byref(plan), ptr(c), N)
        return c

    def emulate(self, a, b, m, n, k, max_moduli=0, passes=0, fixed_bits=0, exact=False):
        c = np.zeros(m * n)
        p = OzoPlan()
        err = ctypes.create_string_buffer(512)
        rc = self.lib.ozo_ii_int8_emulate(ptr(a), ptr(b), ptr(c), m, n, k, max_moduli, passes, fixed_bits,
                                          1 if exact else 0, ctypes.byref(p), err, 512)
        return rc, c, p, err.value.decode()

    # -- Scheme I ------------------------------------------------------------------------------
    # fmt: the OZTT_FMT_* value, 5 INT8 (radix 254), 4 FP8 (radix 32), 0/1/2 BF16/FP16/TF32 (radix 64).
    def i_slice(self, x: np.ndarray, rows: int, cols: int, col_mode: int, delta: np.ndarray, p: int,
                fmt: int = 5) -> np.ndarray:
        out = np.zeros(p * rows * cols, dtype=np.int8)
        self.lib.ozo_i_slice_fmt(ptr(x), rows, cols, cols, col_mode, ptr(delta), p, fmt, ptr(out))
        return out

    def i_gemm(self, sa: np.ndarray, sb: np.ndarray, p: int, M: int, N: int, K: int) -> np.ndarray:
        out = np.zeros(p * M * N, dtype=np.int32)
        assert self.lib.ozo_i_gemm(ptr(sa), ptr(sb), p, M, N, K, ptr(out)) == 0, "int32 overflow in the oracle"
        return out

    def i_recon(self, pd: np.ndarray, p: int, M: int, N: int, dA: np.ndarray, dB: np.ndarray,
                exact: bool, fmt: int = 5, K: int = 0) -> np.ndarray:
        """FP8 faithful: the reference's deferred reconstruction, whose single-conversion diagonals depend
        on the padded K."""
        c = np.zeros(M * N)
        if exact:
            self.lib.ozo_i_recon_exact_fmt(ptr(pd), p, fmt, M, N, ptr(dA), ptr(dB), ptr(c), N)
        elif fmt != 5:
            self.lib.ozo_i_recon_faithful_deferred(ptr(pd), p, fmt, K, M, N, ptr(dA), ptr(dB), ptr(c), N)
        else:
            self.lib.ozo_i_recon_faithful(ptr(pd), p, M, N, ptr(dA), ptr(dB), ptr(c), N)
        return c

    def i_emulate(self, a, b, m, n, k, p, exact=False, fmt: int = 5) -> np.ndarray:
        c = np.zeros(m * n)
        self.lib.ozo_i_emulate_fmt(ptr(a), ptr(b), ptr(c), m, n, k, p, fmt, 1 if exact else 0)
        return c

    # -- Scheme II FP8 digits ---------------------------------------------------------------
    # `fp` is an oztt_digit_plan ctypes structure (the product's DigitPlan or the reference planner's).
    def crt_plan(self, moduli, b: int, two_pass: int) -> OzoPlan:
        m = np.asarray(moduli, dtype=np.int32)
        p = OzoPlan()
        assert self.lib.ozo_crt_plan(ptr(m), len(m), b, two_pass, ctypes.byref(p)) == 0
        return p

    def digit_split(self, x: np.ndarray, rows: int, cols: int, col_mode: int, delta: np.ndarray, crt: OzoPlan,
                  fp) -> tuple[int, np.ndarray]:
        out = np.zeros(fp.nplane * rows * cols, dtype=np.int8)
        bad = self.lib.ozo_digit_split(ptr(x), rows, cols, cols, col_mode, ptr(delta), ctypes.byref(crt),
                                     ctypes.byref(fp), ptr(out))
        return bad, out

    def digit_gemm(self, da: np.ndarray, db: np.ndarray, fp, M: int, N: int, K: int) -> tuple[int, np.ndarray]:
        out = np.zeros(fp.nout * M * N, dtype=np.int32)
        bad = self.lib.ozo_digit_gemm(ptr(da), ptr(db), ctypes.byref(fp), M, N, K, ptr(out))
        return bad, out

    def digit_compose(self, P_: np.ndarray, fp, crt: OzoPlan, M: int, N: int) -> np.ndarray:
        r = np.zeros(crt.S * M * N, dtype=np.float32)
        self.lib.ozo_digit_compose(ptr(P_), ctypes.byref(fp), ctypes.byref(crt), M, N, ptr(r))
        return r

    def recon_residue(self, r: np.ndarray, M: int, N: int, dA: np.ndarray, dB: np.ndarray, crt: OzoPlan) -> np.ndarray:
        c = np.zeros(M * N)
        self.lib.ozo_recon_faithful_residue(ptr(r), M, N, ptr(dA), ptr(dB), ctypes.byref(crt), ptr(c), N)
        return c

    def digit_emulate(self, a, b, m, n, k, fp, exact=False) -> tuple[int, np.ndarray, str]:
        c = np.zeros(m * n)
        err = ctypes.create_string_buffer(512)
        rc = self.lib.ozo_digit_emulate(ptr(a), ptr(b), ptr(c), m, n, k, ctypes.byref(fp), 1 if exact else 0, err, 512)
        return rc, c, err.value.decode()

    # -- metrics ------------------------------------------------------------------------------
    def output_hash(self, c: np.ndarray) -> str:
        return "%016x" % self.lib.ozo_output_hash(ptr(c), c.size)

    def dot2(self, a, b, m, n, k):
        hi, lo = np.zeros(m * n), np.zeros(m * n)
        self.lib.ozo_dot2_gemm(ptr(a), ptr(b), m, n, k, ptr(hi), ptr(lo))
        return hi, lo

    def accuracy(self, c, hi, lo) -> tuple[float, float]:
        r, e = ctypes.c_double(), ctypes.c_double()
        self.lib.ozo_accuracy(ptr(c), ptr(hi), ptr(lo), c.size, ctypes.byref(r), ctypes.byref(e))
        return r.value, e.value

    def maxrel_f128(self, a, b, c, m, n, k, rows=None) -> float:
        out = ctypes.c_double()
        if rows is None:
            self.lib.ozo_maxrel_f128(ptr(a), ptr(b), ptr(c), m, n, k, None, 0, ctypes.byref(out))
        else:
            r = np.ascontiguousarray(rows, dtype=np.uint64)
            self.lib.ozo_maxrel_f128(ptr(a), ptr(b), ptr(c), m, n, k, ptr(r), r.size, ctypes.byref(out))
        return out.value


    def maxrel_f128_rows(self, a, b, results, m, n, k, rows) -> list[float]:
        """Maximum relative errors against binary128 of several results given on the listed rows only
        (each result: len(rows) x n values, row r standing for row rows[r])."""
        r = np.ascontiguousarray(rows, dtype=np.uint64)
        cs = [np.ascontiguousarray(c, dtype=np.float64).reshape(-1) for c in results]
        for c in cs:
            assert c.size == r.size * n
        ptrs = (ctypes.c_void_p * len(cs))(*[ptr(c) for c in cs])
        out = np.zeros(len(cs))
        rc = self.lib.ozo_maxrel_f128_rows(ptr(a), ptr(b), ptrs, len(cs), m, n, k, ptr(r), r.size, ptr(out))
        assert rc == 0, "bad arguments to ozo_maxrel_f128_rows"
        return [float(x) for x in out]


class RefPlan:
    """The reference's planner headers compiled in place (oracle/ref_plan.cpp)."""

    def __init__(self, path: Path = REF_PLAN_SO):
        if not path.exists():
            raise FileNotFoundError(str(path))
        self.lib = ctypes.CDLL(str(path))
        self.lib.ozr_choose_moduli.argtypes = [ctypes.c_uint32] * 3 + [ctypes.c_int, ctypes.c_int,
                                                                      ctypes.POINTER(OzoPlan)]
        self.lib.ozr_plan.argtypes = [P, P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                      ctypes.c_int, ctypes.c_int, ctypes.POINTER(OzoPlan)]

    def choose_moduli(self, K: int, num_moduli: int, b_cap: int, M: int = 0, N: int = 0) -> OzoPlan:
        p = OzoPlan()
        self.lib.ozr_choose_moduli(M or K, N or K, K, num_moduli, b_cap, ctypes.byref(p))
        return p

    def plan(self, ap, bp, M, N, K, max_moduli=0, passes=0, fixed_bits=0) -> tuple[int, OzoPlan]:
        p = OzoPlan()
        rc = self.lib.ozr_plan(ptr(ap), ptr(bp), M, N, K, max_moduli, passes, fixed_bits, ctypes.byref(p))
        return rc, p


class RefEmu:
    """The reference's host emulation of its device kernels, composed (oracle/ref_emu.cpp)."""

    def __init__(self, path: Path = REF_EMU_SO):
        if not path.exists():
            raise FileNotFoundError(str(path))
        self.lib = ctypes.CDLL(str(path))
        self.lib.ozr_emulate_int8.argtypes = [P, P, P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int, P]

    def emulate(self, ap, bp, M, N, K, b_fixed, num_moduli=16, two_pass=False):
        c = np.zeros(M * N)
        mods = np.zeros(MAXS, dtype=np.int32)
        s = self.lib.ozr_emulate_int8(ptr(ap), ptr(bp), ptr(c), M, N, K, b_fixed, num_moduli, 1 if two_pass else 0,
                                      ptr(mods))
        return s, c, [int(x) for x in mods[:max(s, 0)]]


class RefPlanDigit:
    """The reference's Scheme II planner headers compiled for one digit format (oracle/ref_plan_digit.cpp);
    fmt is the OZTT_FMT_* value (4 FP8, 0 BF16, 1 FP16, 2 TF32)."""

    LIBS = {4: "libozref_plan_f8.so", 0: "libozref_plan_bf16.so", 1: "libozref_plan_fp16.so", 2: "libozref_plan_tf32.so"}

    def __init__(self, fmt: int = 4):
        path = ROOT / "oracle" / "_ref" / self.LIBS[fmt]
        if not path.exists():
            raise FileNotFoundError(str(path))
        self.lib = ctypes.CDLL(str(path))
        self.lib.ozr_digit_choose.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int,
                                              ctypes.c_int, P, P]
        self.lib.ozr_digit_plan.argtypes = [P, P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                            ctypes.c_int, ctypes.c_int, P]

    def choose(self, K: int, num_moduli: int, b_cap: int, plan_type, M: int = 0, N: int = 0):
        out = plan_type()
        acc = ctypes.c_int()
        ok = self.lib.ozr_digit_choose(M or K, N or K, K, num_moduli, b_cap, ctypes.byref(out), ctypes.byref(acc))
        return ok, acc.value, out

    def plan(self, ap, bp, M, N, K, plan_type, max_moduli=0, passes=0, fixed_bits=0):
        out = plan_type()
        rc = self.lib.ozr_digit_plan(ptr(ap), ptr(bp), M, N, K, max_moduli, passes, fixed_bits, ctypes.byref(out))
        return rc, out


class RefPlan1:
    """The reference's Scheme I slice-count selection compiled in place (oracle/ref_plan1.cpp); the FP8
    build when fp8 is set, the radix-64 build (BF16, FP16, TF32) when r64 is set."""

    def __init__(self, path: Path = REF_PLAN1_SO, fp8: bool = False, r64: bool = False):
        if fp8:
            path = REF_PLAN1_F8_SO
        if r64:
            path = ROOT / "oracle" / "_ref" / "libozref_plan1_r64.so"
        if not path.exists():
            raise FileNotFoundError(str(path))
        self.lib = ctypes.CDLL(str(path))
        self.lib.ozr_i_slices.argtypes = [P, P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]

    def slices(self, ap, bp, M, N, K) -> int:
        return self.lib.ozr_i_slices(ptr(ap), ptr(bp), M, N, K)


def pad(a: np.ndarray, rows: int, cols: int, prow: int, pcol: int) -> np.ndarray:
    out = np.zeros((prow, pcol))
    out[:rows, :cols] = a.reshape(rows, cols)
    return out.reshape(-1)


def round_up(v: int, q: int) -> int:
    return (v + q - 1) // q * q
