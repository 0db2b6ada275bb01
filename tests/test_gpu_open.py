"""GPU: the paired-GPU open (sufb200_open_exchange) on two GPUs, one process
per GPU like the runtime (party 0 on GPU 0, party 1 on GPU 1), against the
plain arithmetic of OpenCollector::flush's packed path
(src/runtime/open_collector.cpp:357-895): opened = s0 + s1 mod 2^ring,
optionally sign-extended, for flushes packed to eff_bits.  The two-GPU
tests are skipped with fewer than two GPUs; the loopback test runs the fused
kernel (sufb200_p2p_open_*) on one."""
from __future__ import annotations

import os
import socket
import sys
import time
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu

CASES = [  # (n, eff_bits, ring_bits, signed)
    (1, 37, 37, False),
    (1001, 37, 37, True),
    (1001, 56, 37, True),
    ((1 << 20) + 3, 56, 56, False),
    ((1 << 20) + 3, 64, 64, True),
    (4097, 64, 64, False),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expected(x: np.ndarray, ring: int, signed: bool) -> np.ndarray:
    m = np.uint64((1 << ring) - 1) if ring < 64 else np.uint64(~np.uint64(0))
    v = x & m
    if signed and ring < 64:
        sign = (v >> np.uint64(ring - 1)) & np.uint64(1)
        v = v | (np.uint64(0) - sign) & ~m
    return v


def _worker(rank: int, port: int, q):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    from suf_b200.engine import Context, OpenComm, share_open_id

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.cuda.set_device(rank)
    ctx = Context(rank)
    comm = OpenComm(ctx, share_open_id(rank), 2, rank, timeout_s=60.0)
    try:
        stream = torch.cuda.Stream()
        results = []
        for ci, (n, eff, ring, signed) in enumerate(CASES):
            rng = np.random.default_rng([7, ci])  # same values on both ranks
            x = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
            s0 = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(3)
            m = np.uint64((1 << ring) - 1) if ring < 64 else np.uint64(~np.uint64(0))
            s0 &= m
            s1 = (x - s0) & m
            mine = s0 if rank == 0 else s1
            d = torch.from_numpy(mine.view(np.int64)).cuda()
            for _ in range(2):  # twice in a row: reused pool scratch
                out = comm.exchange(1 - rank, d, eff, ring, signed=signed, stream=stream)
            stream.synchronize()
            got = out.cpu().numpy().view(np.uint64)
            results.append(bool((got == _expected(x, ring, signed)).all()))
        dist.barrier()
        q.put((rank, results))
    finally:
        comm.close()
        ctx.close()
        dist.destroy_process_group()


def _run(target, args_of, nproc=2, timeout=300):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=args_of(r, q)) for r in range(nproc)]
    for p in procs:
        p.start()
    deadline = time.time() + timeout
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return procs, q


def test_open_exchange_two_gpus():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    port = _free_port()
    procs, q = _run(_worker, lambda r, q: (r, port, q))
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res[0] == res[1] == [True] * len(CASES), res


def _lonely_worker(q):
    sys.path.insert(0, str(ROOT))
    import torch

    from suf_b200 import SufB200Error
    from suf_b200._lib import ERR_COMM
    from suf_b200.engine import Context, OpenComm, open_unique_id

    torch.cuda.set_device(0)
    ctx = Context(0)
    t0 = time.time()
    try:
        OpenComm(ctx, open_unique_id(), 2, 0, timeout_s=3.0)
        q.put(("joined", 0.0))
    except SufB200Error as e:
        q.put(("error" if e.code == ERR_COMM else f"code {e.code}", time.time() - t0))
    finally:
        ctx.close()


def test_open_comm_create_times_out_without_peer():
    """A rank whose peer never joins gets SUFB200_ERR_COMM after its deadline
    (the failure is on the host: nothing runs on the GPU meanwhile)."""
    import torch

    if torch.cuda.device_count() < 1:
        pytest.skip("needs a GPU")
    procs, q = _run(_lonely_worker, lambda r, q: (q,), nproc=1, timeout=120)
    assert procs[0].exitcode == 0
    what, dt = q.get(timeout=5)
    assert what == "error" and dt < 60, (what, dt)


# ---- the open in one kernel: peer stores over NVLink (sufb200_p2p_open_*) ----

def _p2p_worker(rank: int, port: int, q):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    from suf_b200.engine import Context, OpenComm, P2POpen, share_open_id, share_p2p_handles

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.cuda.set_device(rank)
    ctx = Context(rank)
    ep = P2POpen(ctx, max_words=(1 << 20) + 64)
    comm = OpenComm(ctx, share_open_id(rank), 2, rank, timeout_s=60.0)
    try:
        ep.connect(share_p2p_handles(ep)[1 - rank])
        stream = torch.cuda.Stream()
        results = []
        for ci, (n, eff, ring, signed) in enumerate(CASES):
            rng = np.random.default_rng([9, ci])  # same values on both ranks
            x = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
            s0 = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(3)
            m = np.uint64((1 << ring) - 1) if ring < 64 else np.uint64(~np.uint64(0))
            s0 &= m
            s1 = (x - s0) & m
            d = torch.from_numpy((s0 if rank == 0 else s1).view(np.int64)).cuda()
            outs = []
            for _ in range(3):  # three calls in a row: both landing halves, flags of rising value
                outs.append(ep.exchange(d, eff, ring, signed=signed, timeout_s=10.0, stream=stream))
            ref = comm.exchange(1 - rank, d, eff, ring, signed=signed, stream=stream)
            ctx.sync(stream)
            want = _expected(x, ring, signed)
            ok = all(bool((o.cpu().numpy().view(np.uint64) == want).all()) for o in outs)
            ok = ok and bool((ref.cpu().numpy() == outs[-1].cpu().numpy()).all())  # same words as the NCCL path
            results.append(ok)
        dist.barrier()
        q.put((rank, results))
    finally:
        ep.close()
        comm.close()
        ctx.close()
        dist.destroy_process_group()


def test_p2p_open_two_gpus():
    """The fused open equals the plain Z_2^ring arithmetic and the NCCL path,
    word for word, for packed and raw flushes, three calls in a row."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    port = _free_port()
    procs, q = _run(_p2p_worker, lambda r, q: (r, port, q))
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res[0] == res[1] == [True] * len(CASES), res


def _p2p_silent_peer_worker(rank: int, port: int, q):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    from suf_b200 import SufB200Error
    from suf_b200.engine import Context, P2POpen, share_p2p_handles

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.cuda.set_device(rank)
    ctx = Context(rank)
    ep = P2POpen(ctx, max_words=4096)
    try:
        ep.connect(share_p2p_handles(ep)[1 - rank])
        dist.barrier()
        what, dt = "idle", 0.0
        if rank == 0:  # rank 1 never calls: rank 0's wait must end by itself
            d = torch.arange(1000, dtype=torch.int64, device="cuda")
            t0 = time.time()
            ep.exchange(d, 37, 37, timeout_s=0.5)
            try:
                ctx.sync()
                what = "completed"
            except SufB200Error as e:
                what = "timeout" if "bounded wait" in str(e) else f"other: {e}"
            dt = time.time() - t0
            ctx.sync()  # the status was cleared: the context stays usable
        dist.barrier()
        q.put((rank, what, dt))
    finally:
        ep.close()
        ctx.close()
        dist.destroy_process_group()


def test_p2p_open_times_out_when_the_peer_never_calls():
    """A peer that never calls ends the waiting kernel after its bounded wait
    (the kernel returns; sufb200_ctx_sync reports the timeout)."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    port = _free_port()
    procs, q = _run(_p2p_silent_peer_worker, lambda r, q: (r, port, q), timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = {r: (w, dt) for r, w, dt in (q.get(timeout=5) for _ in range(2))}
    assert res[0][0] == "timeout" and res[0][1] < 30, res


def test_p2p_open_loopback_one_gpu():
    """The whole fused-open kernel on one device: an endpoint connected to
    itself packs, stores, raises and waits on its own per-CTA flags, unpacks
    and adds -- out = local + (local mod 2^eff_bits), reduced to the ring and
    sign-extended -- over both landing halves; connecting to the endpoint's
    own handle as a peer is refused (the paired kernels need two devices)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from suf_b200 import SufB200Error
    from suf_b200.engine import Context, P2POpen

    ctx = Context(0)
    ep = P2POpen(ctx, max_words=(1 << 20) + 64)
    try:
        with pytest.raises(SufB200Error):
            ep.connect(ep.handle)
        ep.connect_self()
        stream = torch.cuda.Stream()
        for ci, (n, eff, ring, signed) in enumerate(CASES):
            rng = np.random.default_rng([11, ci])
            s = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
            d = torch.from_numpy(s.view(np.int64)).cuda()
            emask = np.uint64((1 << eff) - 1) if eff < 64 else np.uint64(~np.uint64(0))
            want = _expected(s + (s & emask), ring, signed)
            outs = [ep.exchange(d, eff, ring, signed=signed, timeout_s=5.0, stream=stream) for _ in range(3)]
            ctx.sync(stream)
            for o in outs:
                assert (o.cpu().numpy().view(np.uint64) == want).all(), (n, eff, ring, signed)
        # captured exchanges replay with fresh call numbers (the device
        # counter): two calls per replay, three replays, both halves in turn
        n, eff, ring, signed = CASES[1]
        rng = np.random.default_rng([11, 99])
        s = rng.integers(0, 2**63, n, dtype=np.uint64)
        d = torch.from_numpy(s.view(np.int64)).cuda()
        want = _expected(s + (s & np.uint64((1 << eff) - 1)), ring, signed)
        o = [torch.zeros_like(d), torch.zeros_like(d)]
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="relaxed"):
            for k in range(2):
                ep.exchange(d, eff, ring, signed=signed, d_out=o[k], timeout_s=5.0, stream=stream)
        for _ in range(3):
            o[0].zero_()
            o[1].zero_()
            g.replay()
            torch.cuda.synchronize()
            ctx.sync()
            for k in range(2):
                assert (o[k].cpu().numpy().view(np.uint64) == want).all(), k
        del g
    finally:
        ep.close()
        ctx.close()
