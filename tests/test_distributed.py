"""The multi-GPU planning logic (oztt_b200/distributed.py) on CPU: gloo ranks with a host implementation
of the per-panel measurements. Every rank must make the same plan, and it must be the plan of the whole
problem made in one piece (the decisions of the reference's planner)."""

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from oztt_b200.distributed import Grid, VECTORS, policy_stats_tiled


class HostStats:
    """The measurements in plain host arithmetic (float64 sums in index order, long double sketches)."""

    def absmax(self, x, rows, cols, mode):
        x = np.asarray(x).reshape(rows, cols)
        return np.abs(x).max(axis=1 - mode)

    def sumsq(self, x, rows, cols, mode, rg):
        x = np.asarray(x).reshape(rows, cols)
        if mode == 1:
            x = x.T
        out = np.zeros(x.shape[0])
        for i, row in enumerate(x):
            acc = 0.0
            for v in row:
                w = float(v) * rg
                acc += w * w
            out[i] = acc
        return out

    def sketch(self, x, rows, cols, rg, v):
        x = np.asarray(x).reshape(rows, cols)
        out = np.zeros((VECTORS, rows))
        for l in range(VECTORS):
            for r in range(rows):
                acc = np.longdouble(0)
                for j in range(cols):
                    acc = acc + np.longdouble(float(x[r, j]) * rg) * np.longdouble(v[l, j])
                out[l, r] = float(acc)
        return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, P, Q, port, A, B, m, n, k, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch

    import oztt_b200 as oz

    p, q = rank // Q, rank % Q
    a = A[p * m:(p + 1) * m]
    b = np.ascontiguousarray(B[:, q * n:(q + 1) * n])

    def red(arr, op):
        t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float64))
        dist.all_reduce(t, op=op)
        return t.numpy()

    st = policy_stats_tiled(a, b, m, n, k, Grid(P, Q, p, q), HostStats(), lambda x: red(x, dist.ReduceOp.MAX),
                            lambda x: red(x, dist.ReduceOp.SUM), oz.policy_vectors)
    plan = oz.ii_int8_plan_from_stats(P * m, Q * n, k, *st)
    out[rank] = (st, bytes(plan))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("P,Q", [(2, 1), (1, 2), (2, 2)])
def test_tiled_plan_matches_whole_problem(oztt, P, Q):
    m, n, k = 24, 20, 40
    rng = np.random.default_rng(P * 10 + Q)
    A = rng.standard_normal((P * m, k)) * np.exp2(rng.integers(-8, 8, (P * m, 1)))
    B = rng.standard_normal((k, Q * n))
    world = P * Q
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        out = man.dict()
        mp.start_processes(_worker, args=(world, P, Q, _free_port(), A, B, m, n, k, out), nprocs=world, join=True,
                           start_method="spawn")
        results = dict(out)
    plans = {r: results[r][1] for r in range(world)}
    assert len(set(plans.values())) == 1  # every rank made the same plan
    whole = policy_stats_tiled(A, B, P * m, Q * n, k, Grid(1, 1, 0, 0), HostStats(), lambda x: x, lambda x: x,
                               oztt.policy_vectors)
    host = oztt.ii_int8_plan(A.reshape(-1), B.reshape(-1), P * m, Q * n, k)
    # one piece: the host planner's statistics exactly
    for got, f in zip(whole, ("TA", "TB", "nA", "nB", "nC")):
        assert np.float64(got).view(np.uint64) == np.float64(getattr(host, f)).view(np.uint64), f
    # tiled: the same decisions, statistics equal up to the order of the partial sums
    tiled = results[0][0]
    assert np.allclose(tiled, whole, rtol=1e-12, atol=0)
    plan = type(host).from_buffer_copy(plans[0])
    assert (plan.S, plan.b, plan.two_pass, plan.moduli_list) == (host.S, host.b, host.two_pass, host.moduli_list)
