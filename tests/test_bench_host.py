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


def _gather_worker(rank, world, port, m_total, out):
    """One CPU rank of the sharded configs[1]/configs[4] layout: take this rank's rows,
    run the ConvRot W8A8 linear on them with the CPU oracle, all-gather the bf16 outputs
    (padded shards) and return the reassembled sequence."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        x, w, w_s, b = _linear_problem(m_total)
        start, rows = bench.shard_rows(m_total, world, rank)
        local = _oracle_linear(x[start:start + rows], w, w_s, b)
        per = -(-m_total // world)
        full = torch.empty((per * world, local.shape[1]), dtype=torch.bfloat16)
        bench.gather_rows(local, per, full, async_op=True).wait()
        out[rank] = (rows, full[:m_total].view(torch.int16).clone())
    finally:
        dist.destroy_process_group()


def _linear_problem(m, k=256, n=16):
    import bench

    g = bench.torch_generator(5)
    x = bench.synth_activation(m, k, g)
    w, w_s, b = bench.synth_weight(n, k, 6)
    return x, w, w_s, b


def _oracle_linear(x, w, w_s, b):
    import numpy as np

    import convrot_oracle as oracle

    if x.shape[0] == 0:
        return torch.empty((0, w.shape[0]), dtype=torch.bfloat16)
    codes, scales = oracle.convrot_quantize(x.view(torch.int16).numpy().view(np.uint16), 8)
    y = oracle.int8_linear(codes, w.numpy(), scales, w_s.numpy(), b.numpy())
    return torch.from_numpy(y.view(np.int16)).view(torch.bfloat16)


def test_shard_rows_cover_the_sequence_in_order():
    import bench

    for m_total in (1, 7, 4095, 32760, 32761):
        for world in (1, 2, 3, 4, 8):
            spans = [bench.shard_rows(m_total, world, r) for r in range(world)]
            per = -(-m_total // world)
            assert all(rows <= per for _, rows in spans)
            assert sum(rows for _, rows in spans) == m_total
            pos = 0
            for start, rows in spans:
                if rows:
                    assert start == pos
                pos += rows
    # configs[1] at 8 GPUs: 4095 rows on every rank.
    assert [bench.shard_rows(32760, 8, r)[1] for r in range(8)] == [4095] * 8


def test_sharded_linear_gathers_to_the_single_rank_result():
    """Two gloo ranks: the row-sharded linear plus the padded all-gather reassemble the
    one-rank output bit for bit -- with a short last shard (7 rows: 4 + 3) and with an
    empty one (1 row: 1 + 0)."""
    for m_total in (7, 1):
        x, w, w_s, b = _linear_problem(m_total)
        whole = _oracle_linear(x, w, w_s, b).view(torch.int16)
        mgr = mp.get_context("spawn").Manager()
        out = mgr.dict()
        mp.start_processes(_gather_worker, args=(2, _free_port(), m_total, out), nprocs=2, start_method="spawn",
                           join=True)
        per = -(-m_total // 2)
        assert out[0][0] == per and out[1][0] == m_total - per
        assert torch.equal(out[0][1], whole) and torch.equal(out[1][1], whole)


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
