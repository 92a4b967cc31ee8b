"""Series sharding and the output all-gather (t0_web_b200/sharded.py), on CPU.

The multi-rank cases run two `gloo` ranks as spawned processes on
127.0.0.1: the same code path bench.py takes over NCCL on GPUs.  The
failure case makes one rank raise before the collective; the surviving rank
must get an error from the process group's short timeout, not hang.
"""
import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest

from t0_web_b200 import sharded


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_balanced_split_is_contiguous_and_balanced(world, seed):
    nv = np.random.default_rng(seed).integers(1, 9, size=97)
    parts = sharded.balanced_split(nv, world)
    assert len(parts) == world
    assert parts[0][0] == 0 and parts[-1][1] == len(nv)
    for (a, b), (c, _) in zip(parts, parts[1:]):
        assert a <= b == c
    rows = [int(nv[a:b].sum()) for a, b in parts]
    assert sum(rows) == int(nv.sum())
    # every boundary is the closest series boundary to its ideal row count
    assert max(rows) - min(rows) <= 2 * int(nv.max())
    rr = sharded.shard_rows(nv, world)
    assert [r1 - r0 for r0, r1 in rr] == rows


def test_balanced_split_more_ranks_than_series():
    parts = sharded.balanced_split([3, 5], 4)
    assert len(parts) == 4
    assert sum(b - a for a, b in parts) == 2
    assert all(a <= b for a, b in parts)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, nv, horizon, fail_rank, q, pg_timeout_s):
    try:
        import torch
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=pg_timeout_s))
        rr = sharded.shard_rows(nv, world)
        r0, r1 = rr[rank]
        local = torch.arange(r0, r1, dtype=torch.float32)[:, None, None].expand(r1 - r0, horizon, 5).contiguous()
        if rank == fail_rank:
            raise RuntimeError("planted failure before the collective")
        full = sharded.gather_outputs(local, [b - a for a, b in rr])
        q.put((rank, "ok", full.numpy()))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which decides pass/fail
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc(limit=2)}"))


def _run(world, nv, horizon=3, fail_rank=-1, limit=150, pg_timeout_s=60):
    # healthy runs get a long process-group timeout (it also bounds the
    # rendezvous, and a spawned rank can take seconds to import torch on a
    # loaded machine); the dead-rank case a short one, so the survivor's
    # collective ends with an error well within `limit`
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, nv, horizon, fail_rank, q, pg_timeout_s))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, payload = q.get(timeout=limit)
            results[rank] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=20)
            if p.is_alive():
                p.kill()  # exact child process started above
                p.join()
    return results


def test_gather_outputs_two_ranks_uneven():
    nv = np.array([3, 1, 4, 1, 5, 2], np.int64)
    res = _run(2, nv)
    total = int(nv.sum())
    for rank in (0, 1):
        status, full = res[rank]
        assert status == "ok", full
        assert full.shape == (total, 3, 5)
        assert np.array_equal(full[:, 0, 0], np.arange(total, dtype=np.float32))


def test_gather_outputs_rank_with_no_series():
    res = _run(2, np.array([4], np.int64))
    for rank in (0, 1):
        status, full = res[rank]
        assert status == "ok", full
        assert full.shape == (4, 3, 5)


def test_dead_rank_fails_collective_with_timeout():
    res = _run(2, np.array([2, 2, 2], np.int64), fail_rank=1, pg_timeout_s=10)
    assert res[1][0] == "error" and "planted failure" in res[1][1]
    assert res[0][0] == "error", "surviving rank must get an error, not a result"
