"""Scheme II INT8 over several GPUs of one node: 2-D output tiles of C, one process per GPU.

Rank (p, q) of a P x Q grid holds A's row panel p (m x k) and B's column panel q (k x n) in its own HBM
and computes the tile C_pq = A_p B_q with the whole single-GPU pipeline; scaling is per row of A and per
column of B, so scale, split, GEMM and reconstruction need nothing from other ranks. The one global step
is the precision decision of the reference's planner (choose_precision_policy,
src/backend/ozaki2/auto_precision.hpp:24-108), whose statistics run over the whole A and B:

  * the power-of-two normalisers come from the global maxima (all-reduce MAX);
  * TA, nA sum over all rows of A (ranks of grid column 0 contribute), TB, nB over all columns of B
    (ranks of grid row 0);
  * the norm estimate needs y_l = B g_l = sum_q B_q g_l[q-th slice] (all-reduce SUM of the K x 8
    partial sketches of grid row 0) and then ||A y_l||^2 = sum_p ||A_p y_l||^2 (grid column 0).

Every rank then makes the same plan from the same five numbers (oztt_ii_int8_plan_from_stats). On one
rank this is exactly the device measurement of the Context path, so its plan equals the reference's; on
several ranks the partial sums are added in a different order than the reference's single sequential
pass, which can move a statistic by a few ulps (a decision changes only if it sits that close to a
threshold).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Protocol

import numpy as np

VECTORS = 8


def _round_up(v: int, q: int) -> int:
    return (v + q - 1) // q * q


def inverse_pow2_scale(mx: float) -> float:
    """1 / 2^e for the exponent e of the largest magnitude, clamped to [-1000, 1000] (oz_pow2_scale,
    src/backend/common/norm_estimate.hpp:20-28)."""
    if not (mx > 0) or not math.isfinite(mx):
        return 1.0
    _, e = math.frexp(mx)
    e = min(max(e, -1000), 1000)
    return 1.0 / math.ldexp(1.0, e)


def tau_square_sum(maxima: np.ndarray, rg: float) -> float:
    """sum of (2^ceil(log2(mx*rg)))^2 over the nonzero maxima, in index order (the TA / TB terms)."""
    total = 0.0
    for mx in maxima:
        v = float(mx) * rg
        if v > 0:
            t = 2.0 ** math.ceil(math.log2(v))
            total += t * t
    return total


class LocalStats(Protocol):
    """The per-panel measurements (on the device by default)."""

    def absmax(self, x, rows: int, cols: int, mode: int) -> np.ndarray: ...

    def sumsq(self, x, rows: int, cols: int, mode: int, rg: float) -> np.ndarray: ...

    def sketch(self, x, rows: int, cols: int, rg: float, v: np.ndarray) -> np.ndarray: ...


class DeviceStats:
    """LocalStats on CUDA tensors through the library's statistics stages (oztt_stats_*)."""

    def __init__(self, lib_call, stream: int):
        import torch

        self.torch = torch
        self.call = lib_call
        self.stream = stream

    def absmax(self, x, rows, cols, mode):
        out = self.torch.empty(rows if mode == 0 else cols, dtype=self.torch.float64, device=x.device)
        self.call("oztt_stats_absmax", x.data_ptr(), rows, cols, mode, out.data_ptr(), self.stream)
        return out.cpu().numpy()

    def sumsq(self, x, rows, cols, mode, rg):
        out = self.torch.empty(rows if mode == 0 else cols, dtype=self.torch.float64, device=x.device)
        self.call("oztt_stats_sumsq", x.data_ptr(), rows, cols, mode, rg, out.data_ptr(), self.stream)
        return out.cpu().numpy()

    def sketch(self, x, rows, cols, rg, v):
        vd = self.torch.from_numpy(np.ascontiguousarray(v)).to(x.device)
        out = self.torch.empty((VECTORS, rows), dtype=self.torch.float64, device=x.device)
        self.call("oztt_stats_sketch", x.data_ptr(), rows, cols, rg, vd.data_ptr(), cols, out.data_ptr(), rows,
                  self.stream)
        return out.cpu().numpy()


@dataclass
class Grid:
    P: int
    Q: int
    p: int
    q: int


def policy_stats_tiled(a, b, m: int, n: int, k: int, grid: Grid, stats: LocalStats, allreduce_max, allreduce_sum,
                       vectors) -> tuple[float, float, float, float, float]:
    """The five statistics (TA, TB, nA, nB, nC) of the global problem from this rank's panels.

    allreduce_max / allreduce_sum take and return a float64 numpy array (the same result on every
    rank); vectors(N) returns the 8 x N Gaussian vectors of the reference (oztt_policy_vectors)."""
    rmax = stats.absmax(a, m, k, 0)
    cmax = stats.absmax(b, k, n, 1)
    g = allreduce_max(np.array([rmax.max(initial=0.0), cmax.max(initial=0.0)]))
    rgA, rgB = inverse_pow2_scale(float(g[0])), inverse_pow2_scale(float(g[1]))
    part = np.zeros(4)
    if grid.q == 0:  # rows of A: one grid column counts them
        part[0] = tau_square_sum(rmax, rgA)
        s2 = stats.sumsq(a, m, k, 0, rgA)
        acc = 0.0
        for v in s2:
            acc += float(v)
        part[2] = acc
    if grid.p == 0:  # columns of B: one grid row counts them
        part[1] = tau_square_sum(cmax, rgB)
        s2 = stats.sumsq(b, k, n, 1, rgB)
        acc = 0.0
        for v in s2:
            acc += float(v)
        part[3] = acc
    TA, TB, nA, nB = (float(x) for x in allreduce_sum(part))
    # the norm estimate over the global, padded N
    N = _round_up(grid.Q * n, 64)
    gv = vectors(N)[:, grid.q * n:(grid.q + 1) * n]
    y = stats.sketch(b, k, n, rgB, gv) if grid.p == 0 else np.zeros((VECTORS, k))
    y = allreduce_sum(np.ascontiguousarray(y).reshape(-1)).reshape(VECTORS, k)
    qpart = np.zeros(VECTORS)
    if grid.q == 0:
        s = stats.sketch(a, m, k, rgA, y)
        for l in range(VECTORS):
            acc = 0.0
            for v in s[l]:
                acc += float(v) * float(v)
            qpart[l] = acc
    qs = allreduce_sum(qpart)
    cs2, cmx = 0.0, 0.0
    for l in range(VECTORS):
        cs2 += float(qs[l])
        cmx = max(cmx, float(qs[l]))
    nC = (cs2 - cmx) / (VECTORS - 1) / (1.0 + 2.0 * math.sqrt(2.0 / VECTORS))
    return TA, TB, nA, nB, nC


def plan_ii_int8_tiled(a, b, m: int, n: int, k: int, grid: Grid, group=None, max_moduli: int = 0,
                       reconstruction: int = 0, stream: int = 0):
    """The Scheme II INT8 plan of the global (P m) x k by k x (Q n) problem, made on every rank from its
    CUDA panels a (m x k) and b (k x n) with NCCL all-reduces over `group`."""
    import torch
    import torch.distributed as dist

    from . import call, ii_int8_plan_from_stats, policy_vectors

    dev = a.device

    def allreduce(arr, op):
        t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float64)).to(dev)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(t, op=op, group=group)
        return t.cpu().numpy()

    stats = DeviceStats(call, stream)
    TA, TB, nA, nB, nC = policy_stats_tiled(
        a, b, m, n, k, grid, stats, lambda x: allreduce(x, dist.ReduceOp.MAX),
        lambda x: allreduce(x, dist.ReduceOp.SUM), policy_vectors)
    return ii_int8_plan_from_stats(grid.P * m, grid.Q * n, k, TA, TB, nA, nB, nC, max_moduli, reconstruction)
