"""GPU: the C-ABI NCCL gather of a sequence-sharded step (ct_dist_init_nccl,
ct_dist_gather_rows, ct_dist_gather_stats), two processes with one GPU
each, the communicator id passed through a file as a launcher would.  Every
rank's rows must land at their global positions on rank 0, bit for bit.
Skipped where fewer than two GPUs are visible."""
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

RANK = r"""
import sys, os, time, json, ctypes as C
import numpy as np, torch
sys.path.insert(0, sys.argv[1])
import cautreo_b200 as ct
rank, world, idfile, outfile = int(sys.argv[2]), int(sys.argv[3]), sys.argv[4], sys.argv[5]
torch.cuda.set_device(rank)
if rank == 0:
    uid = ct.nccl_unique_id()
    open(idfile + ".tmp", "wb").write(uid); os.rename(idfile + ".tmp", idfile)
else:
    t0 = time.time()
    while not os.path.exists(idfile):
        assert time.time() - t0 < 60, "no communicator id"
        time.sleep(0.05)
    uid = open(idfile, "rb").read()
ctx = ct.NcclContext(rank, world, uid, rank)
n_global, row = 1000, 128 * 512                          # 1000 sequences of 128 x 512 bf16
lens = (np.arange(n_global) * 7919) % 65536 + 512
rank_of = ct.lpt_shard(lens, world)
mine = np.nonzero(rank_of == rank)[0].astype(np.uint32)
rows = torch.empty((len(mine), row), dtype=torch.int16, device="cuda")
for i, g in enumerate(mine):
    rows[i].fill_(int(g) * 3 + 1)                        # a row tells where it belongs
out = torch.zeros((n_global, row), dtype=torch.int16, device="cuda") if rank == 0 else None
for _ in range(2):                                       # a second call reuses the staging
    ctx.gather_rows(rows.data_ptr(), len(mine), row * 2, mine, n_global, out.data_ptr() if out is not None else None,
                    torch.cuda.current_stream().cuda_stream)
st = ct.DistStats(int(lens[mine].sum()), int(lens[mine].sum()) * 1152, 1000.0 + rank, 0, len(mine))
allst = ctx.gather_stats(st)
res = {}
if rank == 0:
    want = torch.arange(n_global, dtype=torch.int32, device="cuda") * 3 + 1
    res["rows_ok"] = bool((out == want.to(torch.int16)[:, None]).all().item())
    res["stats"] = [[s.kv_tokens, s.n_seqs, s.decode_us] for s in allst]
    res["want_stats"] = [[int(lens[rank_of == r].sum()), int((rank_of == r).sum()), 1000.0 + r] for r in range(world)]
ctx.close()
json.dump(res, open(outfile, "w"))
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_gather_rows_and_stats_two_processes():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        idfile = os.path.join(d, "nccl.id")
        outs = [os.path.join(d, f"r{r}.json") for r in range(world)]
        env = dict(os.environ, NCCL_NVLS_ENABLE="0")
        procs = [subprocess.Popen([sys.executable, "-c", RANK, str(ROOT), str(r), str(world), idfile, outs[r]],
                                  env=env, cwd=str(ROOT)) for r in range(world)]
        rcs = [p.wait(timeout=300) for p in procs]
        assert rcs == [0] * world
        res = json.load(open(outs[0]))
    assert res["rows_ok"]
    assert res["stats"] == res["want_stats"]


@pytest.mark.parametrize("row_bytes", [131072, 10244, 100])
def test_gather_rows_one_rank_places_rows(row_bytes):
    """A one-rank NCCL context (one GPU): ct_dist_gather_rows places the
    rank's own rows at their global positions through the scatter kernel;
    long rows spread over many warps, rows that are not a multiple of 16
    bytes go as 4-byte words."""
    import cautreo_b200 as ct
    from gpu_util import dev, empty, host, stream
    n = 300
    ctx = ct.NcclContext(0, 1, ct.nccl_unique_id(), 0)
    try:
        src = np.random.default_rng(row_bytes).integers(0, 2**32, n * row_bytes // 4, dtype=np.uint64).astype(np.uint32)
        ids = np.random.default_rng(row_bytes + 1).permutation(n).astype(np.uint32)
        out = empty((n * row_bytes // 4,), np.uint32)
        src_d = dev(src)
        ctx.gather_rows(src_d.data_ptr(), n, row_bytes, ids, n, out.data_ptr(), stream())
        got = host(out, np.uint32).reshape(n, row_bytes // 4)
        assert np.array_equal(got[ids], src.reshape(n, row_bytes // 4))
    finally:
        ctx.close()
