"""Scheme II INT8 over several GPUs of one node: C in 2-D output tiles, one process per GPU.

Rank r = p*Q + q of a P x Q grid computes the tile C_pq = A_p B_q, where A_p is A's row panel p and B_q is
B's column panel q. Scaling is per row of A and per column of B, so the scaling, split, residue GEMM and
CRT reconstruction of a tile need nothing from other ranks: every tile is computed by the single-GPU
pipeline, and the whole C is bit for bit the single-GPU result under the same plan. The reference runs on
one device (src/context.cpp:155); this layer is the B200 build's own.

Three steps need the other ranks, all over torch.distributed (NCCL over NVLink for CUDA tensors, gloo for
the CPU tests):

  * placement (source = rank 0): rank 0 sends each grid row's A panel once, to the rank of grid column 0
    of that row, and each grid column's B panel (packed k x n_q) to the rank of grid row 0 of that column
    (one batched group of point-to-point transfers, so rank 0's outgoing NVLink carries every byte it does
    not keep exactly once); those ranks then broadcast the panel along their grid row / column.
  * the precision decision (choose_precision_policy, src/backend/ozaki2/auto_precision.hpp:24-108): its
    five statistics run over the whole A and B. Each rank measures its panels on the device; the per-row
    and per-column values are all-gathered and summed on the host in the reference's order
    (oztt_policy_stats_combine); the sketch y_l = B g_l runs along grid row 0 as one chain of extended-
    precision sums, each rank continuing the sums of the panel before it (oztt_stats_sketch_chain), so
    every statistic is bit-identical to the single-process measurement and every rank makes the
    reference's plan.
  * assembly (on request): the tiles are gathered to rank 0 (point-to-point) or to every rank
    (all-gather) and copied into a row-major C.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Callable, Optional, Protocol

import numpy as np

VECTORS = 8
EXT_BYTES = 16  # one extended-precision sum of the sketch chain


def _round_up(v: int, q: int) -> int:
    return (v + q - 1) // q * q


def grid_shape(world: int) -> tuple[int, int]:
    """P x Q with P >= Q and P*Q = world, as square as possible (2 -> 2x1, 4 -> 2x2, 8 -> 4x2)."""
    q = int(math.isqrt(world))
    while world % q:
        q -= 1
    return world // q, q


def split_ranges(total: int, parts: int) -> list[tuple[int, int]]:
    """`parts` consecutive, nearly equal ranges covering [0, total)."""
    return [(i * total // parts, (i + 1) * total // parts) for i in range(parts)]


def inverse_pow2_scale(mx: float) -> float:
    """1 / 2^e for the exponent e of the largest magnitude, clamped to [-1000, 1000] (oz_pow2_scale,
    src/backend/common/norm_estimate.hpp:20-28)."""
    if not (mx > 0) or not math.isfinite(mx):
        return 1.0
    _, e = math.frexp(mx)
    e = min(max(e, -1000), 1000)
    return 1.0 / math.ldexp(1.0, e)


@dataclass(frozen=True)
class Grid:
    P: int
    Q: int
    p: int
    q: int

    @property
    def rank(self) -> int:
        return self.p * self.Q + self.q

    @property
    def size(self) -> int:
        return self.P * self.Q

    @staticmethod
    def of(rank: int, world: int) -> "Grid":
        P, Q = grid_shape(world)
        return Grid(P, Q, rank // Q, rank % Q)

    def row_range(self, m: int, p: Optional[int] = None) -> tuple[int, int]:
        return split_ranges(m, self.P)[self.p if p is None else p]

    def col_range(self, n: int, q: Optional[int] = None) -> tuple[int, int]:
        return split_ranges(n, self.Q)[self.q if q is None else q]


class GridComm:
    """The grid's collectives over torch.distributed's default group: the row groups (the ranks that share
    A's row panel) and the column groups (those that share B's column panel). Every rank must construct it,
    at the same point of its program: each group is created by all ranks, in the same order."""

    def __init__(self, grid: Grid, device=None):
        import torch
        import torch.distributed as dist

        self.torch = torch
        self.grid = grid
        P, Q = grid.P, grid.Q
        self.single = grid.size == 1 and not (dist.is_available() and dist.is_initialized())
        self.dist = None if self.single else dist
        if device is not None:
            self.device = torch.device(device)
        elif self.single:
            self.device = torch.device("cuda", torch.cuda.current_device())
        else:
            self.device = torch.device("cuda", torch.cuda.current_device()) \
                if dist.get_backend() == "nccl" else torch.device("cpu")
        self.rows = self.cols = None
        if self.single:
            return
        self.rows = [dist.new_group([p * Q + q for q in range(Q)]) for p in range(P)] if Q > 1 else None
        self.cols = [dist.new_group([p * Q + q for p in range(P)]) for q in range(Q)] if P > 1 else None
        # one collective on the default group before any point-to-point transfer (NCCL wants every rank in
        # the first operation of a communicator)
        t = torch.zeros(1, device=self.device)
        dist.all_reduce(t)

    def broadcast(self, t, src: int, group=None) -> None:
        if not self.single:
            self.dist.broadcast(t, src=src, group=group)

    # -- small helpers -----------------------------------------------------------------------------
    def p2p(self, sends: list, recvs: list) -> None:
        """One batched group of point-to-point transfers: sends / recvs are (tensor, peer) pairs."""
        if self.single:
            return
        ops = [self.dist.P2POp(self.dist.isend, t, peer) for t, peer in sends]
        ops += [self.dist.P2POp(self.dist.irecv, t, peer) for t, peer in recvs]
        if ops:
            for req in self.dist.batch_isend_irecv(ops):
                req.wait()

    def all_gather(self, t):
        """Every rank's equally sized tensor t, in rank order."""
        if self.single:
            return [t]
        out = [self.torch.empty_like(t) for _ in range(self.grid.size)]
        self.dist.all_gather(out, t)
        return out


def place_panels(comm: GridComm, a0, b0, m: int, n: int, k: int):
    """Rank 0's row-major A (m x k) and B (k x n), flat tensors on rank 0's device (None elsewhere) ->
    this rank's A_p (rows of panel p, row-major, flat) and B_q (columns of panel q packed as k x n_q,
    row-major, flat), in its own memory."""
    torch, g = comm.torch, comm.grid
    if g.size == 1:
        return a0, b0
    r0, r1 = g.row_range(m)
    c0, c1 = g.col_range(n)
    a_p = torch.empty((r1 - r0) * k, dtype=torch.float64, device=comm.device)
    b_q = torch.empty(k * (c1 - c0), dtype=torch.float64, device=comm.device)
    sends, recvs, keep = [], [], []
    if g.rank == 0:
        A, B = a0.view(m, k), b0.view(k, n)
        for p in range(1, g.P):
            lo, hi = g.row_range(m, p)
            sends.append((A[lo:hi].reshape(-1), p * g.Q))
        for q in range(1, g.Q):
            lo, hi = g.col_range(n, q)
            packed = B[:, lo:hi].contiguous().view(-1)
            keep.append(packed)
            sends.append((packed, q))
        a_p.copy_(A[r0:r1].reshape(-1))
        b_q.view(k, c1 - c0).copy_(B[:, c0:c1])
    else:
        if g.q == 0:
            recvs.append((a_p, 0))
        if g.p == 0:
            recvs.append((b_q, 0))
    comm.p2p(sends, recvs)
    del keep
    if comm.rows is not None:
        comm.broadcast(a_p, src=g.p * g.Q, group=comm.rows[g.p])
    if comm.cols is not None:
        comm.broadcast(b_q, src=g.q, group=comm.cols[g.q])
    return a_p, b_q


class PanelStats(Protocol):
    """This rank's measurements for the precision decision (on the device by default)."""

    def absmax(self, x, rows: int, cols: int, mode: int): ...

    def sumsq(self, x, rows: int, cols: int, mode: int, rg: float): ...

    def sketch(self, x, rows: int, cols: int, rg: float, v): ...

    def sketch_chain(self, x, rows: int, cols: int, rg: float, v, state): ...

    def sketch_round(self, state, rows: int): ...

    def new_state(self, rows: int): ...


class DeviceStats:
    """PanelStats on CUDA tensors through the library's statistics stages (oztt_stats_*); results stay on
    the device."""

    def __init__(self, stream: int = 0):
        import torch

        from . import call

        self.torch = torch
        self.call = call
        self.stream = stream

    def _empty(self, count, like):
        return self.torch.empty(count, dtype=self.torch.float64, device=like.device)

    def absmax(self, x, rows, cols, mode):
        out = self._empty(rows if mode == 0 else cols, x)
        if out.numel():
            self.call("oztt_stats_absmax", x.data_ptr(), rows, cols, mode, out.data_ptr(), self.stream)
        return out

    def sumsq(self, x, rows, cols, mode, rg):
        out = self._empty(rows if mode == 0 else cols, x)
        if out.numel():
            self.call("oztt_stats_sumsq", x.data_ptr(), rows, cols, mode, rg, out.data_ptr(), self.stream)
        return out

    def sketch(self, x, rows, cols, rg, v):
        out = self._empty(VECTORS * rows, x)
        if rows:
            v = v.contiguous()
            self.call("oztt_stats_sketch", x.data_ptr(), rows, cols, rg, v.data_ptr(), v.shape[1], out.data_ptr(),
                      rows, self.stream)
        return out.view(VECTORS, rows)

    def new_state(self, rows):
        return self.torch.zeros(VECTORS * rows * EXT_BYTES, dtype=self.torch.uint8, device="cuda")

    def sketch_chain(self, x, rows, cols, rg, v, state):
        carry = 1 if state is not None else 0
        if state is None:
            state = self.new_state(rows)
        if rows:
            v = v.contiguous()
            self.call("oztt_stats_sketch_chain", x.data_ptr(), rows, cols, cols, rg, v.data_ptr(), v.shape[1],
                      state.data_ptr(), carry, self.stream)
        return state

    def sketch_round(self, state, rows):
        out = self.torch.empty(VECTORS * rows, dtype=self.torch.float64, device=state.device)
        if rows:
            self.call("oztt_stats_sketch_round", state.data_ptr(), VECTORS * rows, out.data_ptr(), self.stream)
        return out.view(VECTORS, rows)


def _padded(torch, t, count):
    out = torch.zeros(count, dtype=t.dtype, device=t.device)
    out[: t.numel()] = t.reshape(-1)
    return out


def policy_stats_tiled(comm: GridComm, a_p, b_q, m: int, n: int, k: int, stats: PanelStats,
                       vectors: Callable[[int], np.ndarray]) -> tuple[float, float, float, float, float]:
    """The five statistics (TA, TB, nA, nB, nC) of the whole m x k by k x n problem from this rank's panels,
    bit-identical to the single-process measurement (the reference's order of every sum); the same on
    every rank. vectors(N) gives the 8 x N Gaussian vectors of the norm estimate (oztt_policy_vectors)."""
    from . import policy_stats_combine

    torch, g = comm.torch, comm.grid
    rows, cols = split_ranges(m, g.P), split_ranges(n, g.Q)
    r0, r1 = rows[g.p]
    c0, c1 = cols[g.q]
    mt, nt = r1 - r0, c1 - c0
    mw = max(hi - lo for lo, hi in rows)
    nw = max(hi - lo for lo, hi in cols)

    def assemble(parts, offset, width, ranges, owners):
        # the pieces of ranks `owners` (one per range), each at `offset` of its buffer, in range order
        return np.concatenate([parts[r][offset: offset + (hi - lo)] for r, (lo, hi) in zip(owners, ranges)]) \
            if ranges else np.zeros(0)

    row_owner = [p * g.Q for p in range(g.P)]  # grid column 0 measures A's rows
    col_owner = list(range(g.Q))               # grid row 0 measures B's columns
    # 1. maxima of A's rows and B's columns, gathered in order
    rmax, cmax = stats.absmax(a_p, mt, k, 0), stats.absmax(b_q, k, nt, 1)
    buf = torch.cat([_padded(torch, rmax, mw), _padded(torch, cmax, nw)])
    parts = [t.cpu().numpy() for t in comm.all_gather(buf)]
    row_max = assemble(parts, 0, mw, rows, row_owner)
    col_max = assemble(parts, mw, nw, cols, col_owner)
    rgA = inverse_pow2_scale(float(row_max.max(initial=0.0)))
    rgB = inverse_pow2_scale(float(col_max.max(initial=0.0)))
    # 2. sums of squares; the sketch y_l = B g_l along grid row 0, one chain of extended sums
    s2r, s2c = stats.sumsq(a_p, mt, k, 0, rgA), stats.sumsq(b_q, k, nt, 1, rgB)
    N = _round_up(n, 64)
    gv = torch.from_numpy(np.ascontiguousarray(vectors(N)[:, c0:c1])).to(a_p.device)
    last = g.Q - 1  # rank (0, Q-1) ends the chain
    y = torch.empty(VECTORS * k, dtype=torch.float64, device=a_p.device)
    if g.p == 0:
        state = None
        if g.q > 0:
            state = stats.new_state(k)
            comm.p2p([], [(state, g.q - 1)])
        state = stats.sketch_chain(b_q, k, nt, rgB, gv, state)
        if g.q < last:
            comm.p2p([(state, g.q + 1)], [])
        else:
            y.copy_(stats.sketch_round(state, k).reshape(-1))
    comm.broadcast(y, src=last)
    # 3. s_l = A_p y_l on grid column 0
    s = stats.sketch(a_p, mt, k, rgA, y.view(VECTORS, k)) if g.q == 0 else \
        torch.zeros((VECTORS, mt), dtype=torch.float64, device=a_p.device)
    buf = torch.cat([_padded(torch, s2r, mw), _padded(torch, s2c, nw),
                     _padded(torch, s.reshape(-1), VECTORS * mw)])
    parts = [t.cpu().numpy() for t in comm.all_gather(buf)]
    row_s2 = assemble(parts, 0, mw, rows, row_owner)
    col_s2 = assemble(parts, mw, nw, cols, col_owner)
    sk = np.zeros((VECTORS, m))
    # the per-panel sketch blocks hold s_l[i] at l * m_p + i (the m_p rows of that panel)
    for (lo, hi), r in zip(rows, row_owner):
        block = parts[r][mw + nw: mw + nw + VECTORS * (hi - lo)].reshape(VECTORS, hi - lo)
        sk[:, lo:hi] = block
    return policy_stats_combine(row_max, col_max, row_s2, col_s2, sk, rgA, rgB)


def plan_ii_int8_tiled(comm: GridComm, a_p, b_q, m: int, n: int, k: int, max_moduli: int = 0,
                       reconstruction: int = 0, fixed_bits: int = 0, stats: Optional[PanelStats] = None):
    """The Scheme II INT8 plan of the whole problem, the same on every rank (the reference's decisions)."""
    from . import ii_int8_plan_from_stats, policy_vectors

    st = policy_stats_tiled(comm, a_p, b_q, m, n, k, stats or DeviceStats(), policy_vectors)
    return ii_int8_plan_from_stats(m, n, k, *st, max_moduli=max_moduli, reconstruction=reconstruction,
                                   fixed_bits=fixed_bits)


def gather_tiles(comm: GridComm, tile, m: int, n: int, to: str = "rank0"):
    """The whole row-major C (m x n, flat) from every rank's tile (row-major m_p x n_q, flat): on rank 0
    (to="rank0"; other ranks get None) or on every rank (to="all")."""
    torch, g = comm.torch, comm.grid
    rows, cols = split_ranges(m, g.P), split_ranges(n, g.Q)
    if to == "all":
        width = max((hi - lo) for lo, hi in rows) * max((hi - lo) for lo, hi in cols)
        parts = comm.all_gather(_padded(torch, tile, width))
    elif to == "rank0":
        parts = None
        if g.rank == 0:
            parts = []
            recvs = []
            for r in range(g.size):
                (lo, hi), (cl, ch) = rows[r // g.Q], cols[r % g.Q]
                if r == 0:
                    parts.append(tile)
                else:
                    t = torch.empty((hi - lo) * (ch - cl), dtype=tile.dtype, device=tile.device)
                    parts.append(t)
                    recvs.append((t, r))
            comm.p2p([], recvs)
        else:
            comm.p2p([(tile.contiguous(), 0)], [])
            return None
    else:
        raise ValueError("gather must be 'rank0' or 'all'")
    C = torch.empty(m * n, dtype=tile.dtype, device=tile.device)
    Cv = C.view(m, n)
    for r in range(g.size):
        (lo, hi), (cl, ch) = rows[r // g.Q], cols[r % g.Q]
        Cv[lo:hi, cl:ch].copy_(parts[r][: (hi - lo) * (ch - cl)].view(hi - lo, ch - cl))
    return C


@dataclass
class TiledResult:
    c: object                 # the gathered C (rank 0 or all ranks), or this rank's tile (gather="none")
    plan: object              # the plan every rank used
    phases_ms: dict           # wall-clock phases of this rank: upload, placement, plan, compute, gather, total


def gemm_tiled(comm: GridComm, a, b, m: int, n: int, k: int, source: str = "rank0", gather: str = "rank0",
               max_moduli: int = 0, reconstruction: int = 0, fixed_bits: int = 0, stream: int = 0,
               stats: Optional[PanelStats] = None, local_gemm=None, out=None) -> TiledResult:
    """C = A B in FP64 by Scheme II INT8 over the P x Q grid of `comm`, one tile per rank.

    source="rank0": a (m x k) and b (k x n) are rank 0's whole matrices, row-major, on its device or in
        host memory (uploaded first); the other ranks pass None. The panels are placed over NVLink
        (place_panels).
    source="panels": every rank passes its own panels: a = A_p (rows of panel p, m_p x k) and b = B_q
        (columns of panel q packed as k x n_q), on the device or in host memory.
    gather="rank0" returns the whole C (m x n, on the device) on rank 0 and None elsewhere; "all" on every
        rank; "none" leaves each rank its tile (m_p x n_q, on the device); "host" copies each rank's tile
        into host memory: into `out` (a host tensor of m_p * n_q doubles, pinned for a fast copy) when given,
        else a new numpy array.
    The plan is the reference's for the whole problem (plan_ii_int8_tiled). For the CPU tests of the
    collectives, `stats` (PanelStats on host tensors) and local_gemm(a_p, b_q, m_p, n_q, k, plan) -> tile
    replace the device measurements and the device pipeline."""
    torch, g = comm.torch, comm.grid
    t_start = time.perf_counter()
    ph = {}

    def mark(name, t0):
        if comm.device.type == "cuda":
            torch.cuda.synchronize()
        ph[name] = (time.perf_counter() - t0) * 1e3
        return time.perf_counter()

    def to_device(x, count):
        if x is None:
            return None
        t = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(x).reshape(-1))
        t = t.reshape(-1)
        if t.numel() != count:
            raise ValueError("matrix span sizes do not match m, n, k")
        return t.to(comm.device, non_blocking=True) if t.device != comm.device else t

    (r0, r1), (c0, c1) = g.row_range(m), g.col_range(n)
    mt, nt = r1 - r0, c1 - c0
    t0 = time.perf_counter()
    if source == "rank0":
        a0 = to_device(a, m * k) if g.rank == 0 else None
        b0 = to_device(b, k * n) if g.rank == 0 else None
        t0 = mark("upload_ms", t0)
        a_p, b_q = place_panels(comm, a0, b0, m, n, k)
        t0 = mark("placement_ms", t0)
    elif source == "panels":
        a_p, b_q = to_device(a, mt * k), to_device(b, k * nt)
        t0 = mark("upload_ms", t0)
        ph["placement_ms"] = 0.0
    else:
        raise ValueError("source must be 'rank0' or 'panels'")
    plan = plan_ii_int8_tiled(comm, a_p, b_q, m, n, k, max_moduli, reconstruction, fixed_bits, stats=stats)
    t0 = mark("plan_ms", t0)
    if local_gemm is not None:
        tile = local_gemm(a_p, b_q, mt, nt, k, plan)
    else:
        from . import ii_int8_run_device

        tile = torch.empty(mt * nt, dtype=torch.float64, device=comm.device)
        if mt and nt:
            ii_int8_run_device(a_p.data_ptr(), b_q.data_ptr(), tile.data_ptr(), mt, nt, k, plan, stream,
                               comm.device.index or 0)
    t0 = mark("compute_ms", t0)
    if gather in ("rank0", "all"):
        out = gather_tiles(comm, tile, m, n, to=gather)
    elif gather == "host":
        if out is not None:
            out.view(-1).copy_(tile.view(-1))
        else:
            out = tile.cpu().numpy()
    elif gather == "none":
        out = tile
    else:
        raise ValueError("gather must be 'rank0', 'all', 'host' or 'none'")
    t0 = mark("gather_ms", t0)
    ph["total_ms"] = (time.perf_counter() - t_start) * 1e3
    return TiledResult(out, plan, ph)
