"""The multi-GPU layer (oztt_b200/distributed.py) on CPU: gloo ranks, host implementations of the panel
measurements, a host stand-in for the device pipeline of a tile.

  * the plan made on every rank of a P x Q grid equals, byte for byte, the host planner's plan of the whole
    problem, and so do the five statistics (the tiled measurements are summed in the reference's order and
    the sketch is one chain of extended-precision sums along the grid row);
  * placement: rank 0's A and B reach every rank as its A row panel and packed B column panel;
  * assembly: the tiles gathered to rank 0, or to every rank, form the whole C.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oztt_b200.distributed import VECTORS, Grid, GridComm, gemm_tiled, grid_shape, place_panels, split_ranges


class HostStats:
    """The panel measurements in host arithmetic: float64 sums in index order (one rounding per multiply and
    add), the sketch in x87 extended precision (numpy longdouble), the chain state as its bytes."""

    @staticmethod
    def _np(x, rows, cols):
        return np.asarray(x.cpu() if isinstance(x, torch.Tensor) else x, dtype=np.float64).reshape(rows, cols)

    def absmax(self, x, rows, cols, mode):
        x = self._np(x, rows, cols)
        return torch.from_numpy(np.abs(x).max(axis=1 - mode) if x.size else np.zeros(rows if mode == 0 else cols))

    def sumsq(self, x, rows, cols, mode, rg):
        x = self._np(x, rows, cols)
        if mode == 1:
            x = x.T
        w = x * rg
        sq = w * w
        return torch.from_numpy(np.ascontiguousarray(np.cumsum(sq, axis=1)[:, -1]) if sq.shape[1] else
                                np.zeros(sq.shape[0]))

    @staticmethod
    def _sums(x, rg, v, start):
        # start (8 x rows, longdouble) + sum_j ext(x[r][j]*rg) * ext(v[l][j]), j ascending
        xs = (x * rg).astype(np.longdouble)
        out = np.empty((VECTORS, x.shape[0]), dtype=np.longdouble)
        for l in range(VECTORS):
            prods = xs * np.asarray(v[l], dtype=np.float64).astype(np.longdouble)[None, :]
            seq = np.concatenate([start[l][:, None], prods], axis=1)
            out[l] = np.cumsum(seq, axis=1)[:, -1]
        return out

    def sketch(self, x, rows, cols, rg, v):
        x = self._np(x, rows, cols)
        v = np.asarray(v.cpu() if isinstance(v, torch.Tensor) else v).reshape(VECTORS, -1)
        acc = self._sums(x, rg, v, np.zeros((VECTORS, rows), dtype=np.longdouble))
        return torch.from_numpy(acc.astype(np.float64))

    def new_state(self, rows):
        return torch.from_numpy(np.zeros(VECTORS * rows, dtype=np.longdouble).view(np.uint8).copy())

    def sketch_chain(self, x, rows, cols, rg, v, state):
        start = np.zeros((VECTORS, rows), dtype=np.longdouble) if state is None else \
            state.numpy().view(np.longdouble).reshape(VECTORS, rows).copy()
        x = self._np(x, rows, cols)
        v = np.asarray(v.cpu() if isinstance(v, torch.Tensor) else v).reshape(VECTORS, -1)
        acc = self._sums(x, rg, v, start)
        return torch.from_numpy(np.ascontiguousarray(acc).reshape(-1).view(np.uint8).copy())

    def sketch_round(self, state, rows):
        return torch.from_numpy(state.numpy().view(np.longdouble).astype(np.float64).reshape(VECTORS, rows))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exact_tile(a_p, b_q, mt, nt, k, plan):
    """The host stand-in for a tile's pipeline: the exact product of integer-valued panels."""
    return torch.from_numpy(np.asarray(a_p).reshape(mt, k) @ np.asarray(b_q).reshape(k, nt)).reshape(-1)


def _worker(rank, world, port, A, B, m, n, k, out, mode):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        comm = GridComm(Grid.of(rank, world), device="cpu")
        g = comm.grid
        a0 = torch.from_numpy(A.reshape(-1).copy()) if rank == 0 else None
        b0 = torch.from_numpy(B.reshape(-1).copy()) if rank == 0 else None
        if mode == "plan":
            res = gemm_tiled(comm, a0, b0, m, n, k, source="rank0", gather="none", stats=HostStats(),
                             local_gemm=lambda *args: torch.zeros(1, dtype=torch.float64))
            out[rank] = bytes(res.plan)
        elif mode == "place":
            a_p, b_q = place_panels(comm, a0, b0, m, n, k)
            (r0, r1), (c0, c1) = g.row_range(m), g.col_range(n)
            ok = np.array_equal(a_p.numpy(), A[r0:r1].reshape(-1)) and \
                np.array_equal(b_q.numpy(), np.ascontiguousarray(B[:, c0:c1]).reshape(-1))
            res = gemm_tiled(comm, a0, b0, m, n, k, source="rank0", gather="rank0", stats=HostStats(),
                             local_gemm=_exact_tile)
            c_rank0 = res.c.numpy() if rank == 0 else None
            # each rank passes its own panels; the tiles assembled on every rank
            res2 = gemm_tiled(comm, A[r0:r1].copy(), np.ascontiguousarray(B[:, c0:c1]), m, n, k, source="panels",
                              gather="all", stats=HostStats(), local_gemm=_exact_tile)
            out[rank] = (ok, c_rank0, res2.c.numpy(), bytes(res.plan) == bytes(res2.plan))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(world, A, B, m, n, k, mode):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        out = man.dict()
        mp.start_processes(_worker, args=(world, _free_port(), A, B, m, n, k, out, mode), nprocs=world, join=True,
                           start_method="spawn")
        return dict(out)


def test_grid_shapes_and_ranges():
    assert [grid_shape(w) for w in (1, 2, 4, 8)] == [(1, 1), (2, 1), (2, 2), (4, 2)]
    assert split_ranges(10, 3) == [(0, 3), (3, 6), (6, 10)]
    assert split_ranges(32768, 4) == [(0, 8192), (8192, 16384), (16384, 24576), (24576, 32768)]


@pytest.mark.parametrize("world,m,n,k,phi", [(2, 48, 40, 70, 1.0), (2, 37, 29, 33, 4.0), (4, 50, 44, 65, 0.5)])
def test_tiled_plan_equals_whole_problem_plan(oztt, oracle, world, m, n, k, phi):
    a, b = oracle.gen_inputs(m, n, k, phi, world + m)
    A, B = a.reshape(m, k), b.reshape(k, n)
    A[3] *= 2.0 ** 30  # a row scale far from the others
    B[:, 5] *= 2.0 ** -40
    plans = _run(world, A, B, m, n, k, "plan")
    host = oztt.ii_int8_plan(A.reshape(-1), B.reshape(-1), m, n, k)
    assert all(p == bytes(host) for p in plans.values()), "a rank's plan differs from the whole problem's"


@pytest.mark.parametrize("world,m,n,k", [(2, 30, 22, 17), (4, 33, 26, 12)])
def test_placement_and_assembly(world, m, n, k):
    rng = np.random.default_rng(world * 100 + m)
    A = rng.integers(-50, 50, (m, k)).astype(np.float64)
    B = rng.integers(-50, 50, (k, n)).astype(np.float64)
    res = _run(world, A, B, m, n, k, "place")
    want = (A @ B).reshape(-1)
    for r in range(world):
        ok, c0, c_all, same_plan = res[r]
        assert ok, f"rank {r}: panels differ from the slices of A and B"
        assert np.array_equal(c_all, want), f"rank {r}: all-gathered C differs"
        assert same_plan
    assert np.array_equal(res[0][1], want)
