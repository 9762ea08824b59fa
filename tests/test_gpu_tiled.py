"""The tiled multi-GPU Scheme II INT8 path (oztt_b200.distributed.gemm_tiled) on 2 or more B200s, one
process per GPU over NCCL. Skipped on a machine with one GPU (the collectives are covered on CPU by
tests/test_distributed.py).

  * every rank's plan is the host planner's plan of the whole problem, byte for byte;
  * the C assembled from the tiles equals, bit for bit, the single-GPU pipeline's C under that plan (each
    tile is the single-GPU computation of its rows and columns);
  * rank-0 placement and per-rank panels give the same result, gathered to rank 0 or to every rank.
"""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, k, phi, out):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import oztt_b200 as oz
        from oztt_b200.distributed import Grid, GridComm, gemm_tiled

        comm = GridComm(Grid.of(rank, world))
        g = comm.grid
        a, b = oz.eval_inputs(m, n, k, phi, 5)
        A, B = a.reshape(m, k), b.reshape(k, n)
        res = gemm_tiled(comm, a if rank == 0 else None, b if rank == 0 else None, m, n, k, source="rank0",
                         gather="rank0")
        (r0, r1), (c0, c1) = g.row_range(m), g.col_range(n)
        res2 = gemm_tiled(comm, A[r0:r1].copy(), np.ascontiguousarray(B[:, c0:c1]), m, n, k, source="panels",
                          gather="all")
        out[rank] = (bytes(res.plan), bytes(res2.plan), res.c.cpu().numpy() if rank == 0 else None,
                     res2.c.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tiled_equals_single_gpu(oztt, cuda, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    m, n, k, phi = 1000, 1300, 777, 1.0
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        out = man.dict()
        mp.start_processes(_worker, args=(world, _free_port(), m, n, k, phi, out), nprocs=world, join=True,
                           start_method="spawn")
        res = dict(out)
    a, b = oztt.eval_inputs(m, n, k, phi, 5)
    plan = oztt.ii_int8_plan(a, b, m, n, k)
    want = oztt.ii_int8_run(a, b, m, n, k, plan)
    for r in range(world):
        p1, p2, c0, c_all = res[r]
        assert p1 == bytes(plan) and p2 == bytes(plan), f"rank {r}: plan differs from the whole problem's"
        assert np.array_equal(c_all.view(np.uint64), want.view(np.uint64)), f"rank {r}: all-gathered C differs"
    assert np.array_equal(res[0][2].view(np.uint64), want.view(np.uint64))
