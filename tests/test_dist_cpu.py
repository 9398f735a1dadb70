"""Multi-rank path on CPU: two gloo ranks shard a workload by LPT and gather
their outputs back to rank 0 in global sequence order (the one collective of
the sequence-sharded serving step)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cautreo_b200 as ct
from cautreo_b200.shard import gather_rows


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, lens, row, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rank_of = ct.lpt_shard(lens, world)
        mine = np.nonzero(rank_of == rank)[0]
        # a row per owned sequence whose values name the sequence (bf16 bits)
        local = torch.tensor(np.repeat((mine * 7 + 3).astype(np.int16)[:, None], row, 1))
        full = gather_rows(local.view(torch.bfloat16), rank_of, rank, world)
        tokens = torch.tensor([float(lens[mine].sum())], dtype=torch.float64)
        dist.all_reduce(tokens)
        if rank == 0:
            q.put((full.view(torch.int16).numpy(), float(tokens[0])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_gather_in_global_order(world):
    rng = np.random.default_rng(4)
    lens = np.exp(rng.uniform(np.log(512), np.log(65536), 37)).astype(np.uint32)
    row = 24
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, lens, row, q)) for r in range(world)]
    for p in procs:
        p.start()
    got, tokens = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = np.repeat((np.arange(len(lens)) * 7 + 3).astype(np.int16)[:, None], row, 1)
    assert np.array_equal(got, want)
    assert tokens == float(lens.sum())          # every sequence owned by exactly one rank


def test_rank_with_no_sequences():
    """More ranks than sequences: empty ranks still join the gather."""
    lens = np.array([100, 5000], np.uint32)
    rank_of = ct.lpt_shard(lens, 3)
    assert sorted(np.bincount(rank_of, minlength=3).tolist()) == [0, 1, 1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 3, port, lens, 8, q)) for r in range(3)]
    for p in procs:
        p.start()
    got, tokens = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.array_equal(got[:, 0], np.array([3, 10], np.int16))
