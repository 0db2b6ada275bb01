"""The N > 1 host logic on CPU ranks (gloo, world size 2): the rank ->
(party, shard) assignment covers the job with weak scaling, timing takes the
max over ranks, and sharded evaluation with idx_base reproduces the shares of
one call over the whole batch (reference-format AES-CTR counters depend on
the element index)."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, ws: int, port: int, q):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    import bench
    from oracle.oracle import Oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        parties, n, shard = bench.assignment(ws, rank, 1000)
        # every rank does the same work as a single GPU (2 party-evaluations of n_elem)
        assert len(parties) * n == 2 * 1000
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        assert t.item() == float(ws)
        # sharded interval-LUT evaluation with idx_base == single call
        orc = Oracle()
        seed = orc.seed_from_id(9, 7)
        cuts = np.array([0, 2**62, 2**63, 3 * 2**62], dtype=np.uint64)
        pay = np.arange(1, 3 * 4 + 1, dtype=np.uint64)
        # one party's key on every rank: the property under test is idx_base
        key = orc.interval_key(0, 9, 64, 4, cuts, pay, seed)
        total = 4000
        xs = np.random.default_rng(3).integers(0, 2**63, total, dtype=np.uint64) * np.uint64(2)
        per = total // ws
        mine = orc.interval_eval(key, key.size, True, xs[rank * per:(rank + 1) * per], 4, idx_base=rank * per)
        full = orc.interval_eval(key, key.size, True, xs, 4, idx_base=0)
        got = [torch.zeros(per * 4, dtype=torch.int64) for _ in range(ws)]
        dist.all_gather(got, torch.from_numpy(mine.view(np.int64).ravel().copy()))
        gathered = np.concatenate([g.numpy() for g in got]).view(np.uint64).reshape(total, 4)
        assert (gathered == full).all()
        # and the counters really depend on the index: a shard evaluated at
        # idx_base 0 differs from its slice of the whole-batch call
        if rank == 1:
            wrong = orc.interval_eval(key, key.size, True, xs[per:], 4, idx_base=0)
            assert not (wrong == full[per:]).all()
        q.put((rank, parties, n, shard))
    finally:
        dist.destroy_process_group()


def test_two_cpu_ranks_assignment_timing_and_sharding():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert res[0][1] == [0] and res[1][1] == [1]      # party 0 on rank 0, party 1 on rank 1
    assert res[0][3] == res[1][3] == 0                # paired ranks share the shard


def test_assignment_rules():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.assignment(1, 0) == ([0, 1], bench.N_ELEM, 0)
    for ws in (2, 4, 8):
        seen = {}
        for r in range(ws):
            parties, n, shard = bench.assignment(ws, r)
            assert n == 2 * bench.N_ELEM and len(parties) == 1
            seen.setdefault(shard, set()).add(parties[0])
        assert all(v == {0, 1} for v in seen.values()) and len(seen) == ws // 2
    with pytest.raises(ValueError):
        bench.assignment(3, 0)


def _id_worker(rank: int, port: int, q):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    from suf_b200.engine import share_open_id

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        q.put((rank, share_open_id(rank)))
    finally:
        dist.destroy_process_group()


def test_open_id_shared_over_gloo():
    """Rank 0 makes the NCCL id of the paired-GPU open; both ranks hold the
    same 128 bytes afterwards (the hand-off the communicator needs)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_id_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = dict(q.get(timeout=5) for _ in range(2))
    assert len(got[0]) == 128 and got[0] == got[1]
