"""ozTTgemm for NVIDIA B200 — Python mirror of the reference's public interface.

The product is the C++/CUDA library ``oztt_b200/liboztt.so`` (C ABI in ``include/oztt_cuda.h``, C++
API in ``include/ozTTgemm/ozTTgemm.hpp``). This module binds its C ABI with ctypes and mirrors the
reference's C++ interface (mukunoki/ozTT ``include/ozTTgemm/ozTTgemm.hpp:25-121``) one to one:

    Scheme, Format, Reconstruction, Options, DeviceOptions, Info, is_available, format_name,
    Context.gemm / Context.multiply

with the same argument meaning and the same error behaviour: ``ValueError`` where the reference
throws ``std::invalid_argument``, ``RuntimeError`` for ``std::runtime_error``, ``MemoryError`` for
``std::bad_alloc``. The lower-level functions (``ii_int8_plan``, ``ii_int8_run``, the stage calls)
expose the backend seam and the individual kernels for tests and benchmarks.

There is no CPU fallback: every compute call goes to the CUDA kernels, and importing the module
fails if the library has not been built.
"""

from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

__all__ = [
    "Scheme", "Format", "Reconstruction", "Options", "DeviceOptions", "Info", "Context",
    "is_available", "format_name", "IIPlan", "ii_int8_plan", "ii_int8_run", "ii_int8_run_device",
    "lib", "library_path",
]

_HERE = Path(__file__).resolve().parent
library_path = _HERE / "liboztt.so"

OK, EINVAL, ERUNTIME, ENOMEM = 0, 1, 2, 3
MAXS = 24


class Scheme(enum.IntEnum):
    I = 0
    II = 1


class Format(enum.IntEnum):
    BF16 = 0
    FP16 = 1
    TF32 = 2
    BFP8 = 3
    FP8 = 4
    INT8 = 5
    BFP4 = 6
    BFP2 = 7


class Reconstruction(enum.IntEnum):
    Automatic = 0
    OnePass = 1
    TwoPass = 2


@dataclass
class Options:
    scheme: int = Scheme.II
    format: int = Format.BFP8
    slices: int = 0
    max_moduli: int = 0
    reconstruction: int = Reconstruction.Automatic


@dataclass
class DeviceOptions:
    device_id: int = 0
    kernel_directory: str = ""


@dataclass
class Info:
    scheme: Scheme = Scheme.II
    format: Format = Format.INT8
    slices: int = 0
    moduli: int = 0
    integer_bits: int = 0
    reconstruction_passes: int = 0
    padded_m: int = 0
    padded_n: int = 0
    padded_k: int = 0


class _COptions(ctypes.Structure):
    _fields_ = [("scheme", ctypes.c_int32), ("format", ctypes.c_int32), ("slices", ctypes.c_uint32),
                ("max_moduli", ctypes.c_uint32), ("reconstruction", ctypes.c_int32)]


class _CInfo(ctypes.Structure):
    _fields_ = [("scheme", ctypes.c_int32), ("format", ctypes.c_int32), ("slices", ctypes.c_uint32),
                ("moduli", ctypes.c_uint32), ("integer_bits", ctypes.c_uint32),
                ("reconstruction_passes", ctypes.c_uint32), ("padded_m", ctypes.c_uint64),
                ("padded_n", ctypes.c_uint64), ("padded_k", ctypes.c_uint64)]


class IIPlan(ctypes.Structure):
    """oztt_ii_plan: the decisions and CRT constants of one Scheme II INT8 call."""
    _fields_ = [("M", ctypes.c_uint32), ("N", ctypes.c_uint32), ("K", ctypes.c_uint32),
                ("S", ctypes.c_int32), ("b", ctypes.c_int32), ("nd", ctypes.c_int32), ("shift", ctypes.c_int32),
                ("two_pass", ctypes.c_int32), ("b_cap", ctypes.c_int32), ("S_req", ctypes.c_int32),
                ("moduli", ctypes.c_int32 * MAXS), ("yi", ctypes.c_int32 * MAXS), ("rinv", ctypes.c_float * MAXS),
                ("c", (ctypes.c_float * MAXS) * 4), ("TA", ctypes.c_double), ("TB", ctypes.c_double),
                ("nA", ctypes.c_double), ("nB", ctypes.c_double), ("nC", ctypes.c_double),
                ("recon1_log2", ctypes.c_double)]

    @property
    def moduli_list(self) -> list[int]:
        return [int(self.moduli[i]) for i in range(self.S)]


MAXOUT = 96
# Digit splitting methods of a digit plan (OZTT_SPLIT_* of include/oztt_cuda.h).
SPLIT_SQ, SPLIT_KAR, SPLIT_WIDE, SPLIT_SQS, SPLIT_ONE = 0, 1, 2, 4, 5


class DigitPlan(ctypes.Structure):
    """oztt_digit_plan: the Scheme II plan of a digit format (moduli, splitting, GEMM outputs, coefficients)."""
    _fields_ = [("base", IIPlan), ("format", ctypes.c_int32), ("nplane", ctypes.c_int32), ("nprod", ctypes.c_int32), ("nout", ctypes.c_int32),
                ("fold_first", ctypes.c_int32), ("q", ctypes.c_int32 * MAXS), ("mode", ctypes.c_int32 * MAXS),
                ("poff", ctypes.c_int32 * MAXS), ("npl", ctypes.c_int32 * MAXS), ("oout", ctypes.c_int32 * (MAXS + 1)),
                ("out_a", ctypes.c_int32 * MAXOUT), ("out_b", ctypes.c_int32 * MAXOUT),
                ("out_g", ctypes.c_int32 * MAXOUT), ("out_mod", ctypes.c_int32 * MAXOUT),
                ("coeff", ctypes.c_int32 * MAXOUT)]


class IPlan(ctypes.Structure):
    """oztt_i_plan: the slice count and the format's slicing (radix, digit bound) of one Scheme I call."""
    _fields_ = [("M", ctypes.c_uint32), ("N", ctypes.c_uint32), ("K", ctypes.c_uint32), ("p", ctypes.c_int32),
                ("auto_p", ctypes.c_int32), ("format", ctypes.c_int32), ("radix", ctypes.c_int32),
                ("dmax", ctypes.c_int32)]


_P = ctypes.c_void_p
_U64 = ctypes.c_uint64
_I32 = ctypes.c_int32
_ERR = ctypes.c_char_p
_SZ = ctypes.c_size_t

_SIGNATURES = {
    "oztt_gemm": [ctypes.c_int, _P, _U64, _P, _U64, _P, _U64, _U64, _U64, _U64, ctypes.POINTER(_COptions),
                  ctypes.POINTER(_CInfo), _ERR, _SZ],
    "oztt_ii_int8_plan": [_P, _P, _U64, _U64, _U64, ctypes.c_uint32, _I32, _I32, ctypes.POINTER(IIPlan), _ERR, _SZ],
    "oztt_ii_int8_run": [ctypes.c_int, _P, _P, _P, _U64, _U64, _U64, ctypes.POINTER(IIPlan), _ERR, _SZ],
    "oztt_ii_int8_run_device": [ctypes.c_int, _P, _P, _P, _U64, _U64, _U64, ctypes.POINTER(IIPlan), _P, _ERR, _SZ],
    "oztt_ii_int8_run_device_timed": [ctypes.c_int, _P, _P, _P, _U64, _U64, _U64, ctypes.POINTER(IIPlan), _P, _P,
                                      _ERR, _SZ],
    "oztt_eval_inputs": [_P, _P, _U64, _U64, _U64, ctypes.c_double, ctypes.c_uint32],
    "oztt_eval_output_hash": [_P, _U64],
    "oztt_ii_scale_rows": [_P, _U64, _U64, _U64, _I32, _P, _P, _P, _P, _ERR, _SZ],
    "oztt_ii_scale_cols": [_P, _U64, _U64, _U64, _I32, _P, _P, _P, _P, _ERR, _SZ],
    "oztt_ii_scale_cols_noalloc": [_P, _U64, _U64, _U64, _I32, _P, _P, _P, _P, _ERR, _SZ],
    "oztt_ii_split_rows": [_P, _U64, _U64, _U64, _P, ctypes.POINTER(IIPlan), _P, _U64, _U64, _P, _ERR, _SZ],
    "oztt_ii_split_cols": [_P, _U64, _U64, _U64, _P, ctypes.POINTER(IIPlan), _P, _U64, _U64, _P, _ERR, _SZ],
    "oztt_ii_residue_gemm": [_P, _P, _U64, _U64, _U64, ctypes.POINTER(IIPlan), _I32, _P, _P, _ERR, _SZ],
    "oztt_ii_recon": [_P, _U64, _U64, _P, _P, ctypes.POINTER(IIPlan), _P, _U64, _U64, _U64, _P, _ERR, _SZ],
    "oztt_device_info": [ctypes.c_int, ctypes.POINTER(_I32), ctypes.POINTER(_I32), ctypes.POINTER(_I32)],
    "oztt_ii_padded_dims": [_U64, _U64, _U64, ctypes.POINTER(_U64), ctypes.POINTER(_U64), ctypes.POINTER(_U64)],
    "oztt_ii_int8_plan_device": [ctypes.c_int, _P, _P, _U64, _U64, _U64, ctypes.c_uint32, _I32, _I32,
                                 ctypes.POINTER(IIPlan), _P, _ERR, _SZ],
    "oztt_stats_absmax": [_P, _U64, _U64, _I32, _P, _P, _ERR, _SZ],
    "oztt_stats_sumsq": [_P, _U64, _U64, _I32, ctypes.c_double, _P, _P, _ERR, _SZ],
    "oztt_stats_sketch": [_P, _U64, _U64, ctypes.c_double, _P, _U64, _P, _U64, _P, _ERR, _SZ],
    "oztt_policy_vectors": [ctypes.c_uint32, _P],
    "oztt_stats_sketch_chain": [_P, _U64, _U64, _U64, ctypes.c_double, _P, _U64, _P, _I32, _P, _ERR, _SZ],
    "oztt_stats_sketch_round": [_P, _U64, _P, _P, _ERR, _SZ],
    "oztt_policy_stats_combine": [_P, _U64, _P, _U64, _P, _P, _P, ctypes.c_double, ctypes.c_double, _P, _ERR, _SZ],
    "oztt_ii_int8_last_phases": [_P, _I32],
    "oztt_ii_int8_plan_from_stats": [_U64, _U64, _U64, ctypes.c_uint32, _I32, _I32, ctypes.c_double, ctypes.c_double,
                                     ctypes.c_double, ctypes.c_double, ctypes.c_double, ctypes.POINTER(IIPlan), _ERR,
                                     _SZ],
    "oztt_ii_digit_plan": [_I32, _P, _P, _U64, _U64, _U64, ctypes.c_uint32, _I32, _I32, ctypes.POINTER(DigitPlan),
                           _ERR, _SZ],
    "oztt_ii_digit_plan_device": [ctypes.c_int, _I32, _P, _P, _U64, _U64, _U64, ctypes.c_uint32, _I32, _I32,
                                  ctypes.POINTER(DigitPlan), _P, _ERR, _SZ],
    "oztt_ii_digit_run": [ctypes.c_int, _P, _P, _P, _U64, _U64, _U64, ctypes.POINTER(DigitPlan), _ERR, _SZ],
    "oztt_ii_digit_run_device": [ctypes.c_int, _P, _P, _P, _U64, _U64, _U64, ctypes.POINTER(DigitPlan), _P, _P, _ERR,
                               _SZ],
    "oztt_ii_digit_split_rows": [_P, _U64, _U64, _U64, _P, ctypes.POINTER(DigitPlan), _P, _U64, _U64, _P, _ERR, _SZ],
    "oztt_ii_digit_split_cols": [_P, _U64, _U64, _U64, _P, ctypes.POINTER(DigitPlan), _P, _U64, _U64, _P, _ERR, _SZ],
    "oztt_ii_digit_gemm": [_P, _P, _U64, _U64, _U64, ctypes.POINTER(DigitPlan), _I32, _P, _P, _ERR, _SZ],
    "oztt_ii_digit_recon": [_P, _U64, _U64, _P, _P, ctypes.POINTER(DigitPlan), _P, _U64, _U64, _U64, _P, _ERR, _SZ],
    "oztt_i_int8_plan": [_P, _P, _U64, _U64, _U64, ctypes.c_uint32, ctypes.POINTER(IPlan), _ERR, _SZ],
    "oztt_i_int8_run": [ctypes.c_int, _P, _P, _P, _U64, _U64, _U64, ctypes.POINTER(IPlan), _ERR, _SZ],
    "oztt_i_int8_run_device": [ctypes.c_int, _P, _P, _P, _U64, _U64, _U64, ctypes.POINTER(IPlan), _P, _P, _ERR, _SZ],
    "oztt_i_format_plan": [_I32, _P, _P, _U64, _U64, _U64, ctypes.c_uint32, ctypes.POINTER(IPlan), _ERR, _SZ],
    "oztt_i_format_plan_device": [_I32, _P, _P, _U64, _U64, _U64, ctypes.c_uint32, ctypes.POINTER(IPlan), _P, _ERR,
                                  _SZ],
    "oztt_i_model1_errors": [_I32, _P, _P, _P, _P, _U64, _U64, _U64, _P, _I32, _P, _ERR, _SZ],
    "oztt_i_scale_rows": [_P, _U64, _U64, _U64, _I32, _P, _P, _P, _ERR, _SZ],
    "oztt_i_scale_cols": [_P, _U64, _U64, _U64, _I32, _P, _P, _P, _ERR, _SZ],
    "oztt_i_slice_rows": [_P, _U64, _U64, _U64, _P, _I32, _I32, _P, _U64, _U64, _P, _ERR, _SZ],
    "oztt_i_slice_cols": [_P, _U64, _U64, _U64, _P, _I32, _I32, _P, _U64, _U64, _P, _ERR, _SZ],
    "oztt_i_diag_gemm": [_P, _P, _U64, _U64, _U64, _I32, _P, _P, _ERR, _SZ],
    "oztt_i_recon": [_P, _U64, _U64, _P, _P, _I32, _I32, _P, _U64, _U64, _U64, _P, _ERR, _SZ],
    "oztt_resident_create": [ctypes.c_int, _I32, _P, _U64, _U64, _I32, ctypes.POINTER(_P), _ERR, _SZ],
    "oztt_resident_destroy": [_P],
    "oztt_resident_gemm": [_P, _P, _P, _I32, ctypes.POINTER(_COptions), ctypes.POINTER(_CInfo), _ERR, _SZ],
    "oztt_set_option": [_I32, _I32, _ERR, _SZ],
    "oztt_get_option": [_I32, ctypes.POINTER(_I32)],
    "oztt_is_available": [_I32],
    "oztt_format_name": [_I32],
    "oztt_test_udiv_small": [ctypes.c_uint32, ctypes.c_uint32],
    "oztt_test_ext80_dot": [_P, _P, _U64, ctypes.c_double],
    "oztt_test_gemm_wait_timeout": [_U64, _P, _P, _ERR, _SZ],
    "oztt_test_scheme1_kblock": [_U64],
    "oztt_test_certified_plan": [_P, _U64, _U64, _U64, _P, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                 ctypes.c_uint32, _I32, ctypes.POINTER(IIPlan), ctypes.POINTER(_I32), _P, _ERR, _SZ],
    "oztt_test_bounded_nb": [_P, _U64, _U64, ctypes.c_double, _P, _ERR, _SZ],
    "oztt_test_band_certify": [_P, _U64, _U64, _P, _P, _P, _P, _P, _ERR, _SZ],
}

_RESTYPES = {"oztt_test_scheme1_kblock": None, "oztt_format_name": ctypes.c_char_p, "oztt_policy_vectors": None, "oztt_test_udiv_small": ctypes.c_uint32, "oztt_test_ext80_dot": ctypes.c_double, "oztt_ii_padded_dims": None, "oztt_eval_inputs": None,
             "oztt_eval_output_hash": ctypes.c_uint64}

# Symbols declared in include/oztt_cuda.h (the tests check that the library exports each of them).
C_ABI_SYMBOLS = [name for name in _SIGNATURES if not name.startswith("oztt_test_")]


def _load() -> ctypes.CDLL:
    if not library_path.exists():
        raise ImportError(f"{library_path} is not built; run `python -m oztt_b200.build` "
                          "(or __graft_entry__.build()) first")
    lib_ = ctypes.CDLL(str(library_path))
    for name, args in _SIGNATURES.items():
        fn = getattr(lib_, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    return lib_


_LIB = None


def _lib() -> ctypes.CDLL:
    """The loaded library (loaded on first use, so that building does not need it)."""
    global _LIB
    if _LIB is None:
        _LIB = _load()
    return _LIB


def __getattr__(name: str):
    if name == "lib":
        return _lib()
    raise AttributeError(name)


def _raise(code: int, msg: bytes | str) -> None:
    text = msg.decode(errors="replace") if isinstance(msg, bytes) else msg
    if code == EINVAL:
        raise ValueError(text)
    if code == ENOMEM:
        raise MemoryError(text)
    raise RuntimeError(text)


def _errbuf() -> ctypes.Array:
    return ctypes.create_string_buffer(1024)


def is_available(fmt) -> bool:
    """False for formats this build does not provide (ozTTgemm::is_available through oztt_is_available)."""
    return bool(_lib().oztt_is_available(int(fmt)))


def format_name(fmt) -> str:
    try:
        return Format(int(fmt)).name
    except ValueError:
        return "unknown"


def _as_f64(x, name: str) -> np.ndarray:
    arr = np.ascontiguousarray(x, dtype=np.float64).reshape(-1)
    return arr


class Context:
    """Owns one CUDA device (ozTTgemm::Context); calls of all contexts are serialised by the library."""

    def __init__(self, options: DeviceOptions | None = None):
        self.options = options or DeviceOptions()
        if self.options.device_id < 0:
            raise ValueError("device_id must be nonnegative")

    def gemm(self, a, b, c, m: int, n: int, k: int, options: Options | None = None) -> Info:
        """C = A*B for row-major FP64 A[m,k], B[k,n]; C (a writable float64 buffer of m*n) is
        overwritten. Raises ValueError / RuntimeError / MemoryError like the reference."""
        opt = options or Options()
        av, bv = _as_f64(a, "a"), _as_f64(b, "b")
        if not (isinstance(c, np.ndarray) and c.dtype == np.float64 and c.flags.c_contiguous and c.flags.writeable):
            raise ValueError("c must be a writable C-contiguous float64 array")
        cv = c.reshape(-1)
        co = _COptions(int(opt.scheme), int(opt.format), int(opt.slices), int(opt.max_moduli), int(opt.reconstruction))
        ci = _CInfo()
        err = _errbuf()
        rc = _lib().oztt_gemm(self.options.device_id, av.ctypes.data, av.size, bv.ctypes.data, bv.size, cv.ctypes.data,
                           cv.size, m, n, k, ctypes.byref(co), ctypes.byref(ci), err, len(err))
        if rc != OK:
            _raise(rc, err.value)
        return Info(Scheme(ci.scheme), Format(ci.format), ci.slices, ci.moduli, ci.integer_bits,
                    ci.reconstruction_passes, ci.padded_m, ci.padded_n, ci.padded_k)

    def multiply(self, a, b, m: int, n: int, k: int, options: Options | None = None) -> np.ndarray:
        if m <= 0 or n <= 0:
            # the library raises the reference's message for zero dimensions
            c = np.zeros(0, dtype=np.float64)
        else:
            c = np.empty(m * n, dtype=np.float64)
        self.gemm(a, b, c, m, n, k, options)
        return c


def ii_int8_plan(a, b, m: int, n: int, k: int, max_moduli: int = 0, reconstruction: int = 0,
                 fixed_bits: int = 0) -> IIPlan:
    """Scheme II INT8 plan for row-major host matrices (oztt_ii_int8_plan)."""
    av, bv = _as_f64(a, "a"), _as_f64(b, "b")
    if av.size != m * k or bv.size != k * n:
        raise ValueError("matrix span sizes do not match m, n, k")
    plan = IIPlan()
    err = _errbuf()
    rc = _lib().oztt_ii_int8_plan(av.ctypes.data, bv.ctypes.data, m, n, k, max_moduli, reconstruction, fixed_bits,
                               ctypes.byref(plan), err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return plan


def ii_int8_plan_device(a_ptr: int, b_ptr: int, m: int, n: int, k: int, max_moduli: int = 0, reconstruction: int = 0,
                        fixed_bits: int = 0, stream: int = 0, device_id: int = 0) -> IIPlan:
    """Scheme II INT8 plan for device-resident operands, the statistics measured on the device
    (oztt_ii_int8_plan_device)."""
    plan = IIPlan()
    err = _errbuf()
    rc = _lib().oztt_ii_int8_plan_device(device_id, a_ptr, b_ptr, m, n, k, max_moduli, reconstruction, fixed_bits,
                                         ctypes.byref(plan), stream, err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return plan


def digit_plan(a, b, m: int, n: int, k: int, max_moduli: int = 0, reconstruction: int = 0,
               fixed_bits: int = 0, fmt=Format.FP8) -> DigitPlan:
    """Scheme II plan of a digit format (FP8, BF16, FP16, TF32) for row-major host matrices
    (oztt_ii_digit_plan); a and b may be None with a fixed width and a fixed number of passes."""
    av = _as_f64(a, "a") if a is not None else None
    bv = _as_f64(b, "b") if b is not None else None
    plan = DigitPlan()
    err = _errbuf()
    rc = _lib().oztt_ii_digit_plan(int(fmt), av.ctypes.data if av is not None else None,
                                   bv.ctypes.data if bv is not None else None, m, n, k, max_moduli, reconstruction,
                                   fixed_bits, ctypes.byref(plan), err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return plan


def policy_vectors(N: int) -> np.ndarray:
    """The 8 x N Gaussian vectors of the precision policy's norm estimate (oztt_policy_vectors)."""
    out = np.empty((8, N), dtype=np.float64)
    _lib().oztt_policy_vectors(N, out.ctypes.data)
    return out


def ii_int8_last_phases() -> dict:
    """Host wall-clock phases (ms) of the last INT8 Scheme II call through Context.gemm in this process
    (oztt_ii_int8_last_phases): upload, statistics read-back, value checks, plan, pipeline with the
    read-back of C, total, the number of pieces of C read back (row bands or tiles); on the path that
    computes while its operands upload also when the first plan was made, whether the complete statistics
    replanned, whether the bounds left the decision open so that the exact sums were computed, whether C
    was read back as its pieces finished (before the plan was confirmed), the device timeline (ms from the
    first copy: A's first part done against every block of B, the last reconstruction, the end of C's
    read-back, the last band's bounded statistics) and when the host's value checks were ready."""
    out = np.zeros(16, dtype=np.float64)
    _lib().oztt_ii_int8_last_phases(out.ctypes.data, 16)
    keys = ("upload_ms", "stats_ms", "check_ms", "plan_ms", "pipeline_ms", "total_ms")
    d = {key: float(v) for key, v in zip(keys, out[:6])}
    d["bands"] = int(out[6])
    d["first_plan_ms"] = float(out[7])
    d["replanned"] = int(out[8])
    d["exact_stats"] = int(out[9])
    d["early_readback"] = int(out[10])
    d["gpu_prefix_ms"] = float(out[11])
    d["gpu_compute_ms"] = float(out[12])
    d["gpu_readback_ms"] = float(out[13])
    d["gpu_bounds_ms"] = float(out[14])
    d["host_checked_ms"] = float(out[15])
    return d


def policy_stats_combine(row_max, col_max, row_sumsq, col_sumsq, sketch_s, rgA: float,
                         rgB: float) -> tuple[float, float, float, float, float]:
    """(TA, TB, nA, nB, nC) from the whole problem's per-row and per-column measurements, summed in the
    reference's order (oztt_policy_stats_combine); sketch_s is 8 x m."""
    rm, cm = np.ascontiguousarray(row_max, np.float64), np.ascontiguousarray(col_max, np.float64)
    r2, c2 = np.ascontiguousarray(row_sumsq, np.float64), np.ascontiguousarray(col_sumsq, np.float64)
    sk = np.ascontiguousarray(sketch_s, np.float64)
    m, n = rm.size, cm.size
    if r2.size != m or c2.size != n or sk.size != 8 * m:
        raise ValueError("policy_stats_combine: sizes do not match")
    out = np.zeros(5)
    err = _errbuf()
    rc = _lib().oztt_policy_stats_combine(rm.ctypes.data, m, cm.ctypes.data, n, r2.ctypes.data, c2.ctypes.data,
                                          sk.ctypes.data, rgA, rgB, out.ctypes.data, err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return tuple(float(x) for x in out)


def ii_int8_plan_from_stats(m: int, n: int, k: int, TA: float, TB: float, nA: float, nB: float, nC: float,
                            max_moduli: int = 0, reconstruction: int = 0, fixed_bits: int = 0) -> IIPlan:
    """Scheme II INT8 plan from the precision policy's five input statistics
    (oztt_ii_int8_plan_from_stats)."""
    plan = IIPlan()
    err = _errbuf()
    rc = _lib().oztt_ii_int8_plan_from_stats(m, n, k, max_moduli, reconstruction, fixed_bits, TA, TB, nA, nB, nC,
                                             ctypes.byref(plan), err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return plan


def ii_int8_run(a, b, m: int, n: int, k: int, plan: IIPlan, device_id: int = 0) -> np.ndarray:
    """Run the Scheme II INT8 pipeline on host matrices with a given plan (oztt_ii_int8_run)."""
    av, bv = _as_f64(a, "a"), _as_f64(b, "b")
    c = np.empty(m * n, dtype=np.float64)
    err = _errbuf()
    rc = _lib().oztt_ii_int8_run(device_id, av.ctypes.data, bv.ctypes.data, c.ctypes.data, m, n, k, ctypes.byref(plan),
                              err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return c


def ii_int8_run_device(a_ptr: int, b_ptr: int, c_ptr: int, m: int, n: int, k: int, plan: IIPlan,
                       stream: int = 0, device_id: int = 0) -> None:
    """The pipeline on device pointers (oztt_ii_int8_run_device); synchronises `stream`."""
    err = _errbuf()
    rc = _lib().oztt_ii_int8_run_device(device_id, a_ptr, b_ptr, c_ptr, m, n, k, ctypes.byref(plan), stream, err,
                                     len(err))
    if rc != OK:
        _raise(rc, err.value)


def ii_int8_run_device_timed(a_ptr: int, b_ptr: int, c_ptr: int, m: int, n: int, k: int, plan: IIPlan,
                             stream: int = 0, device_id: int = 0) -> list[float]:
    """As ii_int8_run_device; returns the device milliseconds of the six stages (scale rows, scale
    columns, split rows, split columns, residue GEMM, reconstruction)."""
    ms = (ctypes.c_double * 6)()
    err = _errbuf()
    rc = _lib().oztt_ii_int8_run_device_timed(device_id, a_ptr, b_ptr, c_ptr, m, n, k, ctypes.byref(plan), stream, ms,
                                           err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return list(ms)


def digit_plan_device(a_ptr: int, b_ptr: int, m: int, n: int, k: int, max_moduli: int = 0, reconstruction: int = 0,
                      fixed_bits: int = 0, stream: int = 0, device_id: int = 0, fmt=Format.FP8) -> DigitPlan:
    """Scheme II plan of a digit format for device-resident operands, the statistics measured on the device
    (oztt_ii_digit_plan_device)."""
    plan = DigitPlan()
    err = _errbuf()
    rc = _lib().oztt_ii_digit_plan_device(device_id, int(fmt), a_ptr, b_ptr, m, n, k, max_moduli, reconstruction,
                                          fixed_bits, ctypes.byref(plan), stream, err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return plan


def digit_run(a, b, m: int, n: int, k: int, plan: DigitPlan, device_id: int = 0) -> np.ndarray:
    """The Scheme II digit-format pipeline on host matrices with a given plan (oztt_ii_digit_run)."""
    av, bv = _as_f64(a, "a"), _as_f64(b, "b")
    if av.size != m * k or bv.size != k * n:
        raise ValueError("matrix span sizes do not match m, n, k")
    c = np.empty(m * n, dtype=np.float64)
    err = _errbuf()
    rc = _lib().oztt_ii_digit_run(device_id, av.ctypes.data, bv.ctypes.data, c.ctypes.data, m, n, k, ctypes.byref(plan),
                                err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return c


def digit_run_device(a_ptr: int, b_ptr: int, c_ptr: int, m: int, n: int, k: int, plan: DigitPlan, stream: int = 0,
                   device_id: int = 0, timed: bool = False) -> list[float] | None:
    """The digit-format pipeline on device pointers (oztt_ii_digit_run_device); synchronises `stream`. With timed=True
    returns the device milliseconds of scale rows, scale columns, split rows, split columns, digit GEMM and
    reconstruction."""
    ms = (ctypes.c_double * 6)()
    err = _errbuf()
    rc = _lib().oztt_ii_digit_run_device(device_id, a_ptr, b_ptr, c_ptr, m, n, k, ctypes.byref(plan), stream,
                                       ms if timed else None, err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return list(ms) if timed else None


def i_int8_plan(a, b, m: int, n: int, k: int, slices: int = 0, fmt=None) -> IPlan:
    """Scheme I plan (oztt_i_int8_plan, or oztt_i_format_plan for another format fmt): slices > 0 fixes p,
    0 selects it from the input."""
    av, bv = _as_f64(a, "a"), _as_f64(b, "b")
    if av.size != m * k or bv.size != k * n:
        raise ValueError("matrix span sizes do not match m, n, k")
    plan = IPlan()
    err = _errbuf()
    if fmt is None or int(fmt) == Format.INT8:
        rc = _lib().oztt_i_int8_plan(av.ctypes.data, bv.ctypes.data, m, n, k, slices, ctypes.byref(plan), err,
                                     len(err))
    else:
        rc = _lib().oztt_i_format_plan(int(fmt), av.ctypes.data, bv.ctypes.data, m, n, k, slices, ctypes.byref(plan),
                                       err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return plan


def i_plan_device(a_dev: int, b_dev: int, m: int, n: int, k: int, slices: int = 0, fmt=Format.INT8,
                  stream: int = 0) -> IPlan:
    """Scheme I plan for device pointers a_dev (m x k), b_dev (k x n), the slice count selected from
    statistics measured on the device (oztt_i_format_plan_device)."""
    plan = IPlan()
    err = _errbuf()
    rc = _lib().oztt_i_format_plan_device(int(fmt), a_dev, b_dev, m, n, k, slices, ctypes.byref(plan), stream, err,
                                          len(err))
    if rc != OK:
        _raise(rc, err.value)
    return plan


def i_model1_errors(a, b, m: int, n: int, k: int, fmt=Format.INT8, a_dev: int = 0, b_dev: int = 0,
                    stream: int = 0, count: int = 40) -> np.ndarray:
    """Scheme I slice selection's model (1) errors (entries 2..) and its ||C||_F^2 estimate (entry 0),
    measured on the host (a_dev 0) or on the device (oztt_i_model1_errors)."""
    av = _as_f64(a, "a") if a is not None else None
    bv = _as_f64(b, "b") if b is not None else None
    out = np.zeros(count)
    err = _errbuf()
    rc = _lib().oztt_i_model1_errors(int(fmt), av.ctypes.data if av is not None else None,
                                     bv.ctypes.data if bv is not None else None, a_dev or None, b_dev or None, m, n, k,
                                     out.ctypes.data, count, stream, err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return out


def i_int8_run(a, b, m: int, n: int, k: int, plan: IPlan, device_id: int = 0) -> np.ndarray:
    """The Scheme I INT8 pipeline on host matrices with a given plan (oztt_i_int8_run)."""
    av, bv = _as_f64(a, "a"), _as_f64(b, "b")
    c = np.empty(m * n, dtype=np.float64)
    err = _errbuf()
    rc = _lib().oztt_i_int8_run(device_id, av.ctypes.data, bv.ctypes.data, c.ctypes.data, m, n, k, ctypes.byref(plan),
                                err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return c


def i_int8_run_device(a_ptr: int, b_ptr: int, c_ptr: int, m: int, n: int, k: int, plan: IPlan, stream: int = 0,
                      device_id: int = 0, timed: bool = False) -> list[float] | None:
    """The Scheme I pipeline on device pointers (oztt_i_int8_run_device); synchronises `stream`. With
    timed=True returns the device milliseconds of scale rows, scale columns, slicing, diagonal GEMMs and
    reconstruction."""
    ms = (ctypes.c_double * 5)()
    err = _errbuf()
    rc = _lib().oztt_i_int8_run_device(device_id, a_ptr, b_ptr, c_ptr, m, n, k, ctypes.byref(plan), stream,
                                       ms if timed else None, err, len(err))
    if rc != OK:
        _raise(rc, err.value)
    return list(ms) if timed else None


def eval_inputs(m: int, n: int, k: int, phi: float, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """The reference evaluator's seeded inputs (evaluation/numerics.hpp:19-38) with a seed parameter."""
    a = np.empty(m * k, dtype=np.float64)
    b = np.empty(k * n, dtype=np.float64)
    _lib().oztt_eval_inputs(a.ctypes.data, b.ctypes.data, m, n, k, phi, seed)
    return a, b


def eval_output_hash(c: np.ndarray) -> str:
    c = np.ascontiguousarray(c, dtype=np.float64).reshape(-1)
    return "%016x" % _lib().oztt_eval_output_hash(c.ctypes.data, c.size)


def padded_dims(m: int, n: int, k: int) -> tuple[int, int, int]:
    mp, np_, kp = _U64(), _U64(), _U64()
    _lib().oztt_ii_padded_dims(m, n, k, ctypes.byref(mp), ctypes.byref(np_), ctypes.byref(kp))
    return mp.value, np_.value, kp.value


class ResidentMatrix:
    """A matrix kept in HBM as the left ("A", m x k) or right ("B", k x n) operand of Scheme II INT8 products,
    with its precision-policy measurements and the residue planes of its last two plans cached
    (oztt_resident_*). x: row-major float64, a numpy array (host) or a CUDA tensor (device, device_id's)."""

    def __init__(self, x, rows: int, cols: int, role: str = "A", device_id: int = 0):
        self._h = None
        if role not in ("A", "B"):
            raise ValueError("role must be 'A' or 'B'")
        self.role, self.rows, self.cols, self.device_id = role, rows, cols, device_id
        on_device = hasattr(x, "data_ptr") and getattr(x, "is_cuda", False)
        if on_device:
            if x.numel() != rows * cols:
                raise ValueError("matrix span sizes do not match m, n, k")
            ptr = x.data_ptr()
        else:
            xv = _as_f64(x, "x")
            if xv.size != rows * cols:
                raise ValueError("matrix span sizes do not match m, n, k")
            ptr = xv.ctypes.data
        h = _P()
        err = _errbuf()
        rc = _lib().oztt_resident_create(device_id, 0 if role == "A" else 1, ptr, rows, cols, 1 if on_device else 0,
                                         ctypes.byref(h), err, len(err))
        if rc != OK:
            _raise(rc, err.value)
        self._h = h

    def close(self) -> None:
        if self._h is not None and _LIB is not None:
            _LIB.oztt_resident_destroy(self._h)
        self._h = None

    def __del__(self):
        self.close()

    def __matmul__(self, other: "ResidentMatrix") -> np.ndarray:
        return resident_gemm(self, other)[0]


def resident_gemm(a: ResidentMatrix, b: ResidentMatrix, c=None, options: Options | None = None):
    """C = A B of two resident operands (Scheme II INT8; oztt_resident_gemm): returns (C, Info). c: None (a new
    host array), a writable float64 host array of m*n, or a CUDA tensor of m*n doubles on the operands' device."""
    opt = options or Options(format=Format.INT8)
    m, n = a.rows, b.cols
    on_device = c is not None and hasattr(c, "data_ptr") and getattr(c, "is_cuda", False)
    if c is None:
        c = np.empty(m * n, dtype=np.float64)
    if on_device:
        if c.numel() != m * n:
            raise ValueError("matrix span sizes do not match m, n, k")
        ptr = c.data_ptr()
    else:
        if not (isinstance(c, np.ndarray) and c.dtype == np.float64 and c.flags.c_contiguous and c.size == m * n):
            raise ValueError("c must be a writable C-contiguous float64 array of m*n")
        ptr = c.ctypes.data
    co = _COptions(int(opt.scheme), int(opt.format), int(opt.slices), int(opt.max_moduli), int(opt.reconstruction))
    ci = _CInfo()
    err = _errbuf()
    rc = _lib().oztt_resident_gemm(a._h, b._h, ptr, 1 if on_device else 0, ctypes.byref(co), ctypes.byref(ci), err,
                                   len(err))
    if rc != OK:
        _raise(rc, err.value)
    return c, Info(Scheme(ci.scheme), Format(ci.format), ci.slices, ci.moduli, ci.integer_bits,
                   ci.reconstruction_passes, ci.padded_m, ci.padded_n, ci.padded_k)


# Kernel-variant options (OZTT_OPT_* of include/oztt_cuda.h): identical results, default 0.
OPT_GEMM_CTA_PAIRS, OPT_RECON_INT = 1, 2


def set_option(option: int, value: int) -> None:
    """Select a kernel variant process-wide (oztt_set_option)."""
    err = _errbuf()
    rc = _lib().oztt_set_option(option, int(value), err, len(err))
    if rc != OK:
        _raise(rc, err.value)


def get_option(option: int) -> int:
    v = _I32()
    rc = _lib().oztt_get_option(option, ctypes.byref(v))
    if rc != OK:
        _raise(rc, "unknown option")
    return v.value


def call(name: str, *args) -> None:
    """Call a stage entry point of the C ABI; the trailing (err, errlen) are appended here."""
    err = _errbuf()
    rc = getattr(_lib(), name)(*args, err, len(err))
    if rc != OK:
        _raise(rc, err.value)
