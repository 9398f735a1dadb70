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


# ---- the C-ABI NCCL backend: what runs without a GPU -------------------------

def test_nccl_unique_id_and_reference_contexts():
    """ct_dist_nccl_unique_id makes a fresh 128-byte id (NCCL's bootstrap
    needs no GPU); contexts from ct_dist_init keep the reference's
    single-process behaviour and refuse the NCCL gathers."""
    import ctypes as C
    import cautreo_b200 as ct
    a, b = ct.nccl_unique_id(), ct.nccl_unique_id()
    assert len(a) == 128 and a != b
    L = ct.lib()
    cfg = ct.DistConfig(0, 2, 1, None)
    h = L.ct_dist_init(C.byref(cfg))
    try:
        assert L.ct_dist_n_devices(h) == 2 and L.ct_dist_device_id(h) == 1 and not L.ct_dist_is_leader(h)
        x = (C.c_float * 4)(1, 2, 3, 4)
        assert L.ct_dist_allreduce(h, x, 4) and list(x) == [1, 2, 3, 4]     # identity, as the reference
        assert L.ct_dist_gather_rows(h, None, 0, 16, None, 0, None, None) == ct.CT_ERR_ARG
        st = ct.DistStats()
        assert L.ct_dist_gather_stats(h, C.byref(st), None) == ct.CT_ERR_ARG
    finally:
        L.ct_dist_destroy(h)
    bad = ct.DistConfig(0, 2, 2, None)                                    # rank beyond the world
    assert not L.ct_dist_init_nccl(C.byref(bad), (C.c_uint8 * 128)(), 0)
