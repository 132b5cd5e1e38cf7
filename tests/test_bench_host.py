"""Host-side multi-rank logic of bench.py on CPU ranks (gloo, world size 2)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        got = bench.max_over_ranks([10.0 + rank, 5.0 - rank], world)
        out[rank] = got
    finally:
        dist.destroy_process_group()


def test_timing_is_the_max_over_ranks():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    assert out[0] == [11.0, 5.0] and out[1] == [11.0, 5.0]


def test_ops_per_step_matches_configs1():
    import bench

    # 4 x (5120 x 5120) + (5120 -> 13824) + (13824 -> 5120) at M = 32760.
    assert abs(bench.ops_per_step(32760) - 1.61448e13) / 1.61448e13 < 1e-4
