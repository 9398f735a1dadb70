"""Sequence sharding across ranks and the one collective of the sharded path.

Sequences are independent, so each rank owns a subset (LPT by length, computed
by ct_dist_shard_lpt in the C library), its own page pool, block tables and
work list, and decodes with no cross-GPU traffic.  The only exchange is the
gather of the per-rank outputs to rank 0 after decode, put back in global
sequence order.  The gather moves bytes, not numbers, so the bf16 outputs
travel as a same-width float16 view (a dtype every backend carries).
"""
import numpy as np


def gather_rows(local, rank_of, rank, world, group=None):
    """Gathers each rank's rows to rank 0 in global sequence order.

    local: this rank's [n_local, row] tensor (any 2-byte dtype), rows in the
    order of np.nonzero(rank_of == rank).  rank_of: the rank of every global
    sequence.  Returns the [n_all, row] tensor on rank 0, None elsewhere.
    Every rank must call it (it is one collective)."""
    import torch
    import torch.distributed as dist

    if local.element_size() != 2 or local.dim() != 2:
        raise ValueError("gather_rows expects a 2-D tensor of a 2-byte dtype")
    rank_of = np.asarray(rank_of)
    counts = np.bincount(rank_of, minlength=world)
    n_max = int(counts.max()) if len(counts) else 0
    row = local.shape[1]
    pad = torch.zeros((max(n_max, 1), row), dtype=torch.float16, device=local.device)
    if local.shape[0]:
        pad[:local.shape[0]] = local.contiguous().view(torch.float16)
    parts = [torch.empty_like(pad) for _ in range(world)] if rank == 0 else None
    dist.gather(pad, parts, dst=0, group=group)
    if rank != 0:
        return None
    full = torch.empty((len(rank_of), row), dtype=torch.float16, device=local.device)
    for r in range(world):
        ids = np.nonzero(rank_of == r)[0]
        if len(ids):
            full[torch.from_numpy(ids).to(local.device)] = parts[r][:len(ids)]
    return full.view(local.dtype)
