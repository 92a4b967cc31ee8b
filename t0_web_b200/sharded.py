"""Data-parallel forecasting over the GPUs of one box.

Series are independent (group attention mixes only the variates of one
series, time attention only one row: mask.rs:49-82), so the batch is split
across ranks at series granularity with the weights replicated on every GPU.
The only collective is one all-gather of the quantile outputs (NCCL over
NVLink on GPUs; gloo in the CPU tests).

Shards are contiguous ranges of series balanced by token count (sum of
v_i * p over the shard), so the gathered output is the concatenation of the
rank outputs in rank order -- no permutation is needed.
"""
from __future__ import annotations

import numpy as np


def balanced_split(n_variates, world: int) -> list[tuple[int, int]]:
    """Contiguous series ranges [lo, hi) per rank with near-equal total rows.

    Tokens per series are v_i * p with p common to the call, so balancing
    rows balances tokens.  Every rank gets a (possibly empty) range."""
    nv = np.asarray(n_variates, np.int64)
    cum = np.concatenate([[0], np.cumsum(nv)])
    total = int(cum[-1])
    bounds = [0]
    for r in range(1, world):
        target = total * r / world
        idx = int(np.searchsorted(cum, target, side="left"))
        # pick the boundary closest to the target row count
        if idx > 0 and abs(cum[idx - 1] - target) <= abs(cum[min(idx, len(cum) - 1)] - target):
            idx -= 1
        bounds.append(max(bounds[-1], min(idx, len(nv))))
    bounds.append(len(nv))
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def shard_rows(n_variates, world: int) -> list[tuple[int, int]]:
    """Row ranges [r0, r1) of each rank's series (rows = variates)."""
    nv = np.asarray(n_variates, np.int64)
    cum = np.concatenate([[0], np.cumsum(nv)])
    return [(int(cum[lo]), int(cum[hi])) for lo, hi in balanced_split(nv, world)]


def gather_outputs(out_local, rows_per_rank: list[int], group=None):
    """All-gather each rank's [rows_r, horizon, nq] output into the full
    [sum rows, horizon, nq] tensor (identical on every rank).  Shards of
    unequal size are padded to the largest one for the collective."""
    import torch
    import torch.distributed as dist

    world = len(rows_per_rank)
    maxr = max(rows_per_rank)
    tail = tuple(out_local.shape[1:])
    buf = out_local.new_zeros((maxr,) + tail)
    if out_local.shape[0]:
        buf[: out_local.shape[0]].copy_(out_local)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([parts[r][: rows_per_rank[r]] for r in range(world)], dim=0)
