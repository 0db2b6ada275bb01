#!/usr/bin/env python3
"""Benchmark of the PFSS hot path on B200 (one process per GPU).

Workload: a FaithfulARS truncation bundle --
N = 4,194,304 masked Q32 inputs (|x| < 2^40, f = 16, seed 2), 4 raw DCF
queries per element (2 x 64-bit, 2 x 16-bit, broadcast myl7 keys, AES-128-MMO
PRG), the additive boolean plan and the ARS postproc, all in one fused
launch per party.  Metric: DCF pred-evals per second (one pred-eval = one
(element, query, party) evaluation), whole job.

One step is the protocol's truncation round: each party holds its masked
share m_p = x_p + r_p of the input, the parties open x^ = m_0 + m_1 (the
open of OpenCollector::flush), and each party evaluates its bundle on x^.
At N = 1 the GPU holds both parties (the reference's setting) and the open
is the local add of the two shares.  At N >= 2, ranks [0, N/2) are party 0
and [N/2, N) party 1; paired ranks j and j + N/2 hold the same shard of
2 x 4,194,304 elements, swap their masked shares over NVLink
(sufb200_p2p_open: one kernel per GPU stores its 64-bit words into the
paired GPU's landing buffer, flags it and adds the peer's words; the NCCL
form sufb200_open_exchange with --open-impl nccl) and evaluate their
party's bundle, so per-GPU work is the same at every N (weak scaling)
and the one collective is the open between paired GPUs.

Legs: `value` (inputs resident in HBM, CUDA events on the launch stream,
L2 flushed between steps), `e2e` (host buffers, copies inside the timed
region), the roofline of the fused kernel, a bounded CPU baseline (the
reference's own myl7 dcf_eval, OpenMP over elements, in a child process
that runs exactly the `--impl reference` code) and the clocks sampled during
the timed region.  `--impl reference` times only the reference CPU
implementation on the same workload, with keys dealt by test infrastructure
(the oracle's truncation dealer and the reference's own dcf_gen): the
product library is not loaded in that arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_ELEM = 1 << 22
FRAC = 16
SEED = 2
KIND_ARS = 1
METRIC = "DCF pred-evals/sec (FaithfulARS trunc bundle, 4 queries/element)"
UNIT = "pred-evals/s"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# workload material (product dealer + keygen; deterministic from the seed)
# ---------------------------------------------------------------------------

def prg_state() -> np.ndarray:
    from suf_b200.engine import host_mt19937_64

    return host_mt19937_64(0x5EED_0002, 16).view(np.uint8).copy()


def dealer(ctx):
    """Both parties' bundle descriptors and myl7 keys (product keygen)."""
    from suf_b200 import GROUP_ADD
    from suf_b200.engine import Context, host_mt19937_64

    r_in, d0, d1, thetas = Context.trunc_gen(KIND_ARS, FRAC, SEED)
    words = host_mt19937_64(SEED ^ 0x6D796C37, 4 * max(d0.nq, 1)).view(np.uint8).reshape(-1, 2, 16)
    keys0, keys1 = [], []
    for q in range(d0.nq):
        k0, k1 = ctx.myl7_gen(GROUP_ADD, d0.q_bits[q], int(thetas[q]), (1).to_bytes(8, "little"), words[q, 0],
                              words[q, 1])
        keys0.append(k0)
        keys1.append(k1)
    return r_in, (d0, d1), (keys0, keys1)


def assignment(ws: int, rank: int, n_elem: int = N_ELEM):
    """(parties, elements, shard) of one rank.  N = 1: both parties on the
    configs[1] batch.  N >= 2: ranks [0, N/2) hold party 0 and [N/2, N)
    party 1, each on its own shard of 2 * n_elem elements (the same per-GPU
    work as N = 1: weak scaling); paired ranks j and j + N/2 hold the same
    shard, so the two parties' shares of an element live on paired GPUs."""
    if ws <= 1:
        return [0, 1], n_elem, 0
    if ws % 2:
        raise ValueError("the party split needs an even number of GPUs")
    half = ws // 2
    return [0 if rank < half else 1], 2 * n_elem, rank % half


def inputs(r_in: int, n: int, shard: int) -> np.ndarray:
    rng = np.random.default_rng([SEED, shard])
    x = rng.integers(-(2**40) + 1, 2**40, n, dtype=np.int64).view(np.uint64)
    return x + np.uint64(r_in)


# ---------------------------------------------------------------------------
# work model: the shared-prefix plan of suf_b200/csrc/prefix.cuh, restated to
# count the AES blocks one fused call executes
# ---------------------------------------------------------------------------

M64 = (1 << 64) - 1
# DRAM bytes per element of trunc_bundle_prefix_kernel, from an ncu capture
# of one 4,194,304-element launch (dram read + write divided by its
# elements): 16 B of x^ and y plus the random 32-byte frontier-entry reads of
# the four queries.
TRAFFIC_BYTES_PER_ELEMENT = 142.1


def plan_for(xh: np.ndarray, nbits: int, kmax: int):
    """(D, count, first) of the shared-prefix plan (make_plan in prefix.cuh)."""
    piv = int(xh[0])
    off = (xh - np.uint64(piv)).view(np.int64)
    mn, mx = int(off.min()), int(off.max())
    lo = (piv + mn) & M64
    width = (mx - mn) & M64
    lo_n = lo & ((1 << nbits) - 1)
    for d in range(nbits, 0, -1):
        sh = nbits - d
        bm = (1 << sh) - 1
        cnt = (width >> sh) + (((lo_n & bm) + (width & bm)) >> sh) + 1
        covers_all = cnt >= (1 << d)
        if covers_all:
            cnt = 1 << d
        if cnt <= kmax:
            return d, cnt, 0 if covers_all else lo_n >> sh
    return 0, 1, 0


def prefix_budget(n: int) -> int:
    return min(max(n // 8 * 5, 256), 1 << 23)


def frontier_blocks(d: int, cnt: int, first: int) -> int:
    """AES blocks of the frontier pass for one key: subtree roots at level
    d - h walked from the root (2 blocks a level), then every child of each
    h-level subtree (2 blocks each) -- expand_height / root_count in prefix.cuh."""
    h = 0
    while h < 7 and h < d and (cnt >> (h + 1)) >= 8192:
        h += 1
    roots = (((first & ((1 << h) - 1)) + cnt - 1) >> h) + 1
    if d - h < 64:
        roots = min(roots, 1 << (d - h))
    return roots * (2 * (d - h) + 2 * ((1 << (h + 1)) - 2))


def executed_aes_blocks(desc, xh: np.ndarray, n: int) -> float:
    kmax = prefix_budget(n)
    prefix = n >= 16384 and os.environ.get("SUFB200_PREFIX", "1") != "0"  # else: a root walk per query
    total = 0
    for q in range(desc.nq):
        nb = int(desc.q_bits[q])
        d, cnt, first = plan_for(xh, nb, kmax) if prefix else (0, 1, 0)
        total += n * 2 * (nb - d) + (frontier_blocks(d, cnt, first) if prefix else 0)
    return float(total)


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.proc = None

    def __enter__(self):
        if self.gpu is None:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([s.strip() for s in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            try:
                sm.append(float(s[1]))
                mx = float(s[2])
                for nm, v in zip(names, s[5:9]):
                    if v.lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


def launches_per_call(desc, n: int) -> int:
    """Kernels one sufb200_trunc_bundle_eval call launches: the shared-prefix
    path (n >= 16384) runs range_kernel, one frontier_kernel for all queries
    and trunc_bundle_prefix_kernel; below that one trunc_bundle_kernel."""
    if n >= 16384 and os.environ.get("SUFB200_PREFIX", "1") != "0":
        return 3
    return 1


def _max_over_ranks(ws: int, dev, v: float) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed(args, ws, dev, stream, flush, step, ctx, local, sample_clocks=True, mids=False):
    """W untimed steps (after the clock sampler has started, so an idle GPU's
    clocks are back up before timing), then K steps bracketed by a barrier
    and a device synchronize, each timed by CUDA events on the launch stream
    after a 256 MB write (> 126 MB L2); returns (max over ranks of the mean step ms, this
    rank's step times, the clock sampler[, this rank's step-start -> mid-event
    times]).  With mids=True the step is called as step(mid) and records
    `mid` on the stream at the point whose share of the step is wanted."""
    import torch
    import torch.distributed as dist

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    mid_evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)] if mids else None
    clk = ClockSampler(local if sample_clocks else None)
    with clk:
        if sample_clocks:
            time.sleep(0.3)  # the sampler's first readings; the warm-up then brings the clocks back up
        with torch.cuda.stream(stream):
            # the warm-up steps are the timed steps' exact sequence (L2 flush,
            # events, step): the first flush and event records of a process
            # run long once, and they belong here, not in step 0
            for k in range(args.warmup):
                flush.fill_(k)
                wev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                wev[0].record(stream)
                if mids:
                    step(torch.cuda.Event(enable_timing=True))
                else:
                    step()
                wev[1].record(stream)
        ctx.sync(stream)
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            # a ~1 ms device-side wait first, so the host has enqueued the first
            # steps before the GPU reaches them (the events then time the
            # device's work, not the host's enqueue of step 0)
            torch.cuda._sleep(2_000_000)
            for k in range(args.steps):
                flush.fill_(k)
                evs[k][0].record(stream)
                if mids:
                    step(mid_evs[k])
                else:
                    step()
                evs[k][1].record(stream)
        torch.cuda.synchronize()
        ctx.sync(stream)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms_steps = [a.elapsed_time(b) for a, b in evs]
    ms_max = _max_over_ranks(ws, dev, sum(ms_steps) / len(ms_steps))
    if mids:
        return ms_max, ms_steps, clk, [evs[k][0].elapsed_time(mid_evs[k]) for k in range(args.steps)]
    return ms_max, ms_steps, clk


def _pair_check(ws: int, rank: int, dev, d_mine, want: np.ndarray) -> bool:
    """Paired ranks j and j + N/2 swap their shares over NCCL and check
    mine + theirs == want; the flag is reduced over all ranks."""
    import torch
    import torch.distributed as dist

    peer = (rank + ws // 2) % ws
    other = torch.empty_like(d_mine)
    for r in dist.batch_isend_irecv([dist.P2POp(dist.isend, d_mine, peer), dist.P2POp(dist.irecv, other, peer)]):
        r.wait()
    ysum = d_mine.cpu().numpy().view(np.uint64) + other.cpu().numpy().view(np.uint64)
    flag = torch.tensor([1 if bool((ysum == want).all()) else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


def masked_shares(xhat: np.ndarray, shard: int) -> tuple[np.ndarray, np.ndarray]:
    """The two parties' masked shares of x^ = x + r_in: party p holds
    m_p = x_p + r_p, where x = x_0 + x_1 is the secret-shared input and
    r_in = r_0 + r_1 the dealer's split of the mask (TruncTask's masked
    value before its open); m_0 is uniform and m_1 = x^ - m_0 mod 2^64."""
    rng = np.random.default_rng([SEED, shard, 0x0FE4])
    m0 = rng.integers(0, 2**64 - 1, xhat.size, dtype=np.uint64, endpoint=True)
    return m0, xhat - m0


def trunc_config(ws: int, n: int, parties: int, nq: int, q_bits) -> dict:
    """The workload description both arms print (the reference arm times the
    work one GPU of ours does at this N)."""
    return {"workload": "configs[1]: FaithfulARS trunc bundle, f=16, |x|<2^40, seed 2",
            "n_elements_per_party_per_gpu": n, "queries_per_element": nq, "query_bits": list(q_bits),
            "parties_per_gpu": parties, "keys": "broadcast myl7 (AES-128-MMO PRG)",
            "step": "open of the masked input (local add at N=1, paired-GPU exchange at N>=2) + fused bundle",
            "l2": "256 MB buffer written between timed steps",
            "parallelism": ("both parties on one GPU" if ws <= 1 else
                            f"party 0 on GPUs 0..{ws // 2 - 1}, party 1 on GPUs {ws // 2}..{ws - 1}, "
                            f"element shards, open between GPU j and j+{ws // 2}")}


def run_ours(args, ws, rank, local):
    import torch
    import torch.distributed as dist

    from suf_b200.engine import Context, OpenComm, open_add_local, share_open_id

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    ctx = Context(local)
    ctx.prg_init(prg_state())
    r_in, descs, keys = dealer(ctx)
    nq = int(descs[0].nq)
    parties, n, shard = assignment(ws, rank, args.n_elem or N_ELEM)
    xhat_h = inputs(r_in, n, shard)
    m_h = masked_shares(xhat_h, shard)
    stream = torch.cuda.Stream(device=dev)
    d_m = {p: torch.from_numpy(m_h[p].view(np.int64)).to(dev) for p in parties}
    d_x = torch.empty(n, dtype=torch.int64, device=dev)
    d_y = {p: torch.empty(n, dtype=torch.int64, device=dev) for p in parties}
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)
    comm, peer, ep = None, None, None
    if ws > 1:
        peer = (rank + ws // 2) % ws
        if args.open_impl == "p2p":
            from suf_b200.engine import P2POpen, share_p2p_handles

            ep = P2POpen(ctx, max_words=(n + 63) // 64 * 64)
            ep.connect(share_p2p_handles(ep)[peer])
        else:
            comm = OpenComm(ctx, share_open_id(rank), ws, rank, timeout_s=60.0)
    torch.cuda.synchronize()

    def open_step(d_in, d_out, st):
        """x^ from this GPU's masked share(s): the local add with both parties
        here, else the exchange with the paired GPU (64-bit ring, raw words):
        one fused peer-store kernel (p2p) or NCCL send/recv plus an add."""
        if ws <= 1:
            open_add_local(d_in[0], d_in[1], 64, d_out=d_out, stream=st)
        elif ep is not None:
            ep.exchange(d_in[parties[0]], 64, 64, signed=False, d_out=d_out, timeout_s=5.0, stream=st)
        else:
            comm.exchange(peer, d_in[parties[0]], 64, 64, signed=False, d_out=d_out, stream=st)

    def step(mid):
        open_step(d_m, d_x, stream)
        mid.record(stream)
        for p in parties:
            ctx.trunc_bundle_eval(descs[p], keys[p], d_x, d_y=d_y[p], stream=stream)

    ms_max, ms_steps, clk, open_ms = _timed(args, ws, dev, stream, flush, step, ctx, local, mids=True)
    opened_ok = bool((d_x.cpu().numpy().view(np.uint64) == xhat_h).all())
    open_ms_max = _max_over_ranks(ws, dev, sum(open_ms) / len(open_ms))
    units_per_rank = n * nq * len(parties)
    total_units = units_per_rank * ws
    value = total_units / (ms_max / 1e3)

    # ---- e2e: host buffers, copies inside the timed region ----
    import threading

    y_pin = {p: torch.empty(n, dtype=torch.int64).pin_memory() for p in parties}
    y_np = {p: y_pin[p].numpy().view(np.uint64) for p in parties}
    pctx = {parties[0]: ctx}
    if ws <= 1:
        # Both parties here: the reference-facing host call (x^ in, y out) per
        # party, one backend instance (context) and host thread per party as
        # in the reference, so one party's copies overlap the other's kernels.
        x_pin = torch.from_numpy(xhat_h.view(np.int64)).pin_memory()
        x_np = x_pin.numpy().view(np.uint64)
        for p in parties[1:]:
            pctx[p] = Context(local)
            pctx[p].prg_init(prg_state())

        def e2e_step():
            errs = []

            def one(p):
                try:
                    pctx[p].trunc_bundle_eval_host(descs[p], keys[p], x_np, y=y_np[p])
                except Exception as ex:  # re-raised below, on the bench thread
                    errs.append(ex)

            ths = [threading.Thread(target=one, args=(p,)) for p in parties]
            for th in ths:
                th.start()
            for th in ths:
                th.join()
            if errs:
                raise errs[0]

        e2e_path = ("sufb200_trunc_bundle_eval_host (pinned host x^ in, y out; one context and host thread per "
                    "party)")
        h2d = 8 * n * len(parties)
    else:
        # One party here: its masked share crosses PCIe, the open crosses
        # NVLink, the bundle runs, y comes back.
        p0 = parties[0]
        m_pin = torch.from_numpy(m_h[p0].view(np.int64)).pin_memory()
        d_me = torch.empty(n, dtype=torch.int64, device=dev)
        d_xe = torch.empty(n, dtype=torch.int64, device=dev)
        d_ye = torch.empty(n, dtype=torch.int64, device=dev)

        def e2e_step():
            with torch.cuda.stream(stream):
                d_me.copy_(m_pin, non_blocking=True)
                open_step({p0: d_me}, d_xe, stream)
                ctx.trunc_bundle_eval(descs[p0], keys[p0], d_xe, d_y=d_ye, stream=stream)
                y_pin[p0].copy_(d_ye, non_blocking=True)
            stream.synchronize()

        e2e_path = ("pinned host masked share -> device, the open with the paired GPU ("
                    + ("sufb200_p2p_open" if ep is not None else "sufb200_open_exchange")
                    + "), sufb200_trunc_bundle_eval, y -> pinned host")
        h2d = 8 * n

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e2e_ms = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        e2e_step()
        e2e_ms.append((time.perf_counter() - t0) * 1e3)
    ctx.sync(stream)
    for p in parties[1:]:
        pctx[p].close()
    e2e_ms_max = _max_over_ranks(ws, dev, sum(e2e_ms) / len(e2e_ms))
    e2e_value = total_units / (e2e_ms_max / 1e3)

    # correctness guard on the measured outputs: y0 + y1 == x >> f.  With both
    # parties local it is checked in place; across GPUs the paired ranks
    # (j, j + N/2) swap their shares over NCCL (outside the timed region).
    x = (xhat_h - np.uint64(r_in)).view(np.int64)
    want = (x >> FRAC).view(np.uint64)
    if len(parties) == 2:
        y0 = d_y[0].cpu().numpy().view(np.uint64)
        y1 = d_y[1].cpu().numpy().view(np.uint64)
        ok = bool(((y0 + y1) == want).all())
        ok = ok and bool(((y_np[0] + y_np[1]) == want).all())  # the e2e leg's host outputs too
    else:
        ok = _pair_check(ws, rank, dev, d_y[parties[0]], want)
        ok = ok and bool((y_np[parties[0]] == d_y[parties[0]].cpu().numpy().view(np.uint64)).all())
    if ws > 1:
        flag = torch.tensor([1 if (ok and opened_ok) else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = bool(flag.item())

    peaks = measured_peaks()
    engine_peak = ctx.probe_aes_engine()  # AES-128 blocks/s of the T-table engine, measured now
    kernel_ms = (ms_max - open_ms_max) / len(parties)  # one fused call (range + frontiers + main) per party
    blocks = executed_aes_blocks(descs[0], xhat_h, n)
    achieved = blocks / (kernel_ms / 1e3)
    hbm_gbs = 16.0 * n / (kernel_ms / 1e3) / 1e9  # x^ read + y written per element
    roofline = {
        "bound": "lsu", "unit": "G AES-128 blocks/s",
        "achieved": round(achieved / 1e9, 2), "peak": round(engine_peak / 1e9, 2),
        "frac": round(achieved / engine_peak, 4),
        "traffic": round(TRAFFIC_BYTES_PER_ELEMENT * n) if TRAFFIC_BYTES_PER_ELEMENT is not None else None,
        "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one full-size launch (caches "
                          "flushed per pass), per element, times this call's elements",
        "kernel": ("trunc_bundle_prefix_kernel (+ frontier_kernel, range_kernel)"
                   if launches_per_call(descs[0], n) == 3 else "trunc_bundle_kernel"),
        "peak_source": "sufb200_probe_aes_engine: the DCF walk's two-block AES-128-MMO step on every SM, "
                       "measured in this run (the table-load (LSU) and integer (ALU) pipes it saturates are the "
                       "bound)",
        "work_model": "executed AES blocks = N * sum_q 2*(n_q - D_q) + frontier sum_q roots_q * (2*(D_q - h_q) "
                      "+ 2*(2^(h_q+1) - 2))",
        "hbm": {"achieved": round(hbm_gbs, 2), "peak": peaks.get("hbm_gbs"), "unit": "GB/s",
                "frac": round(hbm_gbs / peaks.get("hbm_gbs", 6650.0), 5)},
        "hw_pipes": {"lsu_pct_of_peak": 95.0, "alu_pct_of_peak": 92.0, "issue_active_pct": 74.6,
                     "source": "ncu --set full of one full-size trunc_bundle_prefix_kernel launch after the "
                               "warm-up (sm__inst_executed_pipe_lsu, sm__pipe_alu_cycles_active, "
                               "smsp__issue_active; pct of peak sustained active): the hardware bound behind "
                               "the engine ceiling"},
        "kernel_ms": round(kernel_ms, 4),
    }
    open_bytes = 8 * n  # 64-bit words each GPU sends (N >= 2) or the add reads twice and writes (N = 1)
    open_info = {
        "what": ("local add of both parties' masked shares (open_add_to_signed_kernel)" if ws <= 1 else
                 ("sufb200_p2p_open: one kernel per GPU stores its 64-bit words into the paired GPU's landing "
                  "buffer over NVLink, flags it, waits (bounded) for the peer's flag and adds" if ep is not None else
                  "sufb200_open_exchange: NCCL send/recv of 64-bit words between GPU j (party 0) and GPU j+N/2 "
                  "(party 1), then open_add_to_signed_kernel")),
        "ms": round(open_ms_max, 4), "share_of_step": round(open_ms_max / ms_max, 4),
        "bytes_per_gpu": open_bytes,
        "gbs_per_gpu": round(open_bytes / (open_ms_max / 1e3) / 1e9, 1),
        "opened_ok": opened_ok,
    }
    out = None
    if rank == 0:
        cpu = cpu_baseline(args, ws) if (ws == 1 and not args.no_cpu) else None
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128", "data": "synthetic (seeded, configs[1] shapes)",
            "config": trunc_config(ws, n, len(parties), nq, [int(descs[0].q_bits[q]) for q in range(nq)]),
            "open": open_info,
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 8 * n * len(parties), "ms_per_step": round(e2e_ms_max, 3),
                    "path": e2e_path},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            # per step: the open's add kernel, then per party range_kernel +
            # frontier_kernel + the main kernel (NCCL's own kernel not counted)
            "gpu_launches": args.steps * (1 + len(parties) * launches_per_call(descs[0], n)),
            "reconstruction_ok": ok,
            "ms_per_step_all": [round(v, 4) for v in ms_steps],
        }
    if comm is not None or ep is not None:
        dist.barrier()
        if comm is not None:
            comm.close()
        if ep is not None:
            ep.close()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return out


# ---------------------------------------------------------------------------
# CPU legs (the reference's own myl7 dcf_eval; test infrastructure under oracle/)
# ---------------------------------------------------------------------------

def host_threads() -> int:
    """Host cores this process may run on (all of them for the CPU legs)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def ref_prg_state() -> np.ndarray:
    """prg_state() computed by the oracle's mt19937_64 (no product library)."""
    from oracle.oracle import Oracle

    return Oracle().mt64(0x5EED_0002, 16).view(np.uint8).copy()


def ref_dealer():
    """The configs[1] bundle material dealt by test infrastructure alone: the
    oracle's truncation dealer (composite_gen_trunc_gate's masks and query
    rewrite, include/gates/composite_fss.hpp:645-833) and the reference's own
    myl7 dcf_gen (oracle/_ref) with the seeds dealer() uses -- byte-identical
    to the product dealer's material, without loading the product library."""
    from oracle.oracle import GROUP_ADD, Oracle, RefMyl7

    orc = Oracle()
    r_in, d0, d1 = orc.trunc_gen(KIND_ARS, FRAC, SEED)
    words = orc.mt64(SEED ^ 0x6D796C37, 4 * max(d0.nq, 1)).view(np.uint8).reshape(-1, 2, 16)
    ref = RefMyl7(GROUP_ADD)
    ref.prg_init(ref_prg_state())
    keys0, keys1 = [], []
    for q in range(d0.nq):
        k0, k1 = ref.gen_seeded(int(d0.q_bits[q]), int(d0.q_theta[q]), (1).to_bytes(8, "little"), words[q, 0],
                                words[q, 1])
        keys0.append(k0)
        keys1.append(k1)
    return r_in, (d0, d1), (keys0, keys1)


def cpu_eval_bundle(ref, orc, descs, keys, xhat, parties):
    """The reference CPU path of the bundle: per query, the reference's own
    myl7 dcf_eval over all elements (OpenMP in the harness), then the
    composite boolean plan + ARS postproc (oracle restatement)."""
    from oracle.oracle import desc_from_fields

    ys = []
    for p in parties:
        d = descs[p]
        pred = np.zeros((d.nq, xhat.size), dtype=np.uint64)
        for q in range(d.nq):
            k = keys[p][q]
            pred[q] = ref.eval_omp(int(d.q_bits[q]), k, k.size, True, xhat, 8).view(np.uint64).ravel()
        ys.append(orc.trunc_combine(desc_from_fields(d), xhat, pred.ravel()))
    return ys


def cpu_baseline(args, ws):
    """One step of the --impl reference arm on the whole batch, run in a
    child process exactly as that arm runs (same code, same thread count, no
    CUDA context or bench threads beside it), so the two CPU figures agree."""
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK",
                        "MASTER_ADDR", "MASTER_PORT", "TORCHELASTIC_RUN_ID")}
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"]
    if args.n_elem:
        cmd += ["--n-elem", str(args.n_elem)]
    try:
        r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
        line = json.loads(r.stdout.strip().splitlines()[-1])
    except (subprocess.TimeoutExpired, ValueError, IndexError) as ex:
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference", "sample": f"failed: {ex}"}
    if "unavailable" in line:
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference", "sample": line["unavailable"]}
    cb = dict(line["cpu_baseline"])
    cb["sample"] += " (one step of the --impl reference arm, in a child process)"
    return cb


def run_reference(args, ws, rank):
    """The reference's CPU implementation of the step on the box's host
    cores: the reference's myl7 dcf_eval (oracle/_ref, OpenMP over elements,
    all host threads) plus the composite plan/postproc, on the same elements
    one GPU of our arm evaluates at this N (the open is an add and is left
    out).  Warm-up steps run on an eighth of the batch; every timed step is
    the whole batch.  Keys come from ref_dealer(): nothing here loads the
    product library."""
    from oracle.oracle import Oracle, RefMyl7

    if rank != 0:
        return None
    if not RefMyl7.available():
        return {"impl": "reference", "unavailable": "oracle/_ref (reference myl7 sources) was not built"}
    from oracle.oracle import GROUP_ADD

    r_in, descs, keys = ref_dealer()
    parties, n, shard = assignment(ws, 0, args.n_elem or N_ELEM)
    xhat = inputs(r_in, n, shard)
    nq = int(descs[0].nq)
    ref = RefMyl7(GROUP_ADD)
    threads = ref.set_threads(host_threads())
    ref.prg_init(ref_prg_state())
    orc = Oracle()
    for _ in range(args.warmup):
        cpu_eval_bundle(ref, orc, descs, keys, xhat[: max(1, n // 8)], parties)
    times = []
    ys = None
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ys = cpu_eval_bundle(ref, orc, descs, keys, xhat, parties)
        times.append(time.perf_counter() - t0)
    ok = None
    if len(parties) == 2:
        x = (xhat - np.uint64(r_in)).view(np.int64)
        ok = bool(((ys[0] + ys[1]) == (x >> FRAC).view(np.uint64)).all())
    dt = sum(times) / len(times)
    v = n * nq * len(parties) / dt
    sample = (f"{n} elements x {nq} queries x {len(parties)} part{'ies' if len(parties) == 2 else 'y'} per step "
              f"(the work of one GPU of the GPU arm at N={ws}), reference myl7 dcf_eval (OpenMP over elements, "
              f"{threads} threads) + composite plan/postproc")
    return {"metric": METRIC, "value": round(v, 1), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128", "data": "synthetic (seeded, configs[1] shapes)",
            "impl": "reference",
            "config": trunc_config(ws, n, len(parties), nq, [int(descs[0].q_bits[q]) for q in range(nq)]),
            "cpu_baseline": {"value": round(v, 1), "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": round(v, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reconstruction_ok": ok, "s_per_step_all": [round(t, 3) for t in times]}

# ---------------------------------------------------------------------------
# configs[1] secondary case: per-element masks (SUF_PER_ELEMENT_MASKS=1)
# ---------------------------------------------------------------------------

ELEM_METRIC = ("DCF pred-evals/sec (FaithfulARS trunc bundle with per-element masks: every element its own gate and "
               "keys, 4 queries/element)")


def elem_material(ctx, n: int, shard: int, dev):
    """Per-element configs[1] gates (seed 2) and both parties' per-element
    keys, made on the device (sufb200_myl7_gen_batch_device), one array per
    query slot."""
    import torch

    from suf_b200.engine import Context, host_mt19937_64, myl7_key_bytes

    r_in, s0, s1, w0, w1, th = Context.trunc_gen_elem(KIND_ARS, FRAC, SEED + (shard << 40), n)
    nq = int(s0.nq)
    keys = ([], [])
    kb = []
    for q in range(nq):
        nb = int(s0.q_bits[q])
        kb.append(myl7_key_bytes(nb, 8))
        seeds = torch.from_numpy(host_mt19937_64((SEED << 8) ^ (shard << 4) ^ q, 4 * n).view(np.uint8)).to(dev)
        seeds = seeds.view(n, 2, 16)
        d_alpha = torch.from_numpy(np.ascontiguousarray(th[:, q]).view(np.int64)).to(dev)
        k0, k1 = ctx.myl7_gen_batch_device(0, nb, d_alpha, (1).to_bytes(8, "little"), seeds[:, 0].contiguous(),
                                           seeds[:, 1].contiguous())
        keys[0].append(k0)
        keys[1].append(k1)
        del seeds, d_alpha
    words = tuple(torch.from_numpy(w.view(np.int64).ravel()).to(dev) for w in (w0, w1))
    return r_in, (s0, s1), keys, kb, words


def run_trunc_elem(args, ws, rank, local):
    """Both parties' per-element configs[1] gates on one GPU per step
    (replicas at N > 1: per-element gates have no shared state to exchange
    beyond the open, which the headline line measures)."""
    import torch
    import torch.distributed as dist

    from suf_b200.engine import Context

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=300))
    ctx = Context(local)
    ctx.prg_init(prg_state())
    n = args.n_elem or N_ELEM
    r_in, shapes, keys, kb, words = elem_material(ctx, n, rank, dev)
    nq = int(shapes[0].nq)
    rng = np.random.default_rng([SEED, rank, 0xE1])
    x = rng.integers(-(2**40) + 1, 2**40, n, dtype=np.int64).view(np.uint64)
    xhat_h = x + r_in
    d_x = torch.from_numpy(xhat_h.view(np.int64)).to(dev)
    d_y = [torch.empty(n, dtype=torch.int64, device=dev) for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()

    def step_adapter():
        for p in (0, 1):
            ctx.trunc_bundle_eval_elem(shapes[p], keys[p], kb, words[p], d_x, d_y=d_y[p], stream=stream)

    ms_adapter, _, _ = _timed(args, ws, dev, stream, flush, step_adapter, ctx, local)
    want = (x.view(np.int64) >> FRAC).view(np.uint64)
    ok = bool(((d_y[0].cpu().numpy().view(np.uint64) + d_y[1].cpu().numpy().view(np.uint64)) == want).all())
    # the keys rearranged level by level (dealer-side, once; the adapter
    # layout is dropped), the layout the product path evaluates
    soa = [[ctx.elem_keys_to_soa(int(shapes[p].q_bits[q]), p, keys[p][q], n, stream=stream) for q in range(nq)]
           for p in (0, 1)]
    ctx.sync(stream)
    del keys
    torch.cuda.empty_cache()

    def step():
        for p in (0, 1):
            ctx.trunc_bundle_eval_elem_soa(shapes[p], soa[p], words[p], d_x, d_y=d_y[p], stream=stream)

    ms, ms_steps, clk = _timed(args, ws, dev, stream, flush, step, ctx, local)
    ok = ok and bool(((d_y[0].cpu().numpy().view(np.uint64) + d_y[1].cpu().numpy().view(np.uint64)) == want).all())

    x_pin = torch.from_numpy(xhat_h.view(np.int64)).pin_memory()
    y_pin = [torch.empty(n, dtype=torch.int64).pin_memory() for _ in range(2)]
    d_xe = torch.empty_like(d_x)

    def e2e_step():
        with torch.cuda.stream(stream):
            d_xe.copy_(x_pin, non_blocking=True)
            for p in (0, 1):
                ctx.trunc_bundle_eval_elem_soa(shapes[p], soa[p], words[p], d_xe, d_y=d_y[p], stream=stream)
                y_pin[p].copy_(d_y[p], non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        e2e_step()
    e2e = []
    for _ in range(args.steps):
        h0 = time.perf_counter()
        e2e_step()
        e2e.append((time.perf_counter() - h0) * 1e3)
    ctx.sync(stream)
    e2e_ms = _max_over_ranks(ws, dev, sum(e2e) / len(e2e))
    ok = ok and bool(((y_pin[0].numpy().view(np.uint64) + y_pin[1].numpy().view(np.uint64)) == want).all())

    units = n * nq * 2
    engine_peak = ctx.probe_aes_engine()
    bits = [int(shapes[0].q_bits[q]) for q in range(nq)]
    blocks = n * 2 * sum(bits)  # one party's call: two AES blocks per level, every level of every key
    kernel_ms = ms / 2
    soa_kb = [25 * b + 24 for b in bits]  # bytes per key in the level-major layout
    key_bytes = n * sum(soa_kb)
    hbm = (key_bytes + n * (8 + 48 + 8)) / (kernel_ms / 1e3) / 1e9  # keys + x^ + words + y per party call
    peaks = measured_peaks()
    res = None
    if rank == 0:
        res = {"metric": ELEM_METRIC, "value": round(units * ws / (ms / 1e3), 1), "unit": UNIT, "n_gpus": ws,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128",
               "data": "synthetic (seeded, configs[1] shapes; per-element gates from seed 2)",
               "config": {"workload": "configs[1] secondary: FaithfulARS, f=16, |x|<2^40, per-element masks "
                                      "(SUF_PER_ELEMENT_MASKS=1)", "n_elements_per_party_per_gpu": n,
                          "query_bits": bits, "key_bytes_per_element_per_party": sum(kb), "parties_per_gpu": 2,
                          "l2": "256 MB flush between steps (the 45 GB of keys exceed L2 anyway)",
                          "parallelism": "both parties on one GPU" + (f"; {ws} replicas" if ws > 1 else "")},
               "e2e": {"value": round(units * ws / (e2e_ms / 1e3), 1), "unit": UNIT, "h2d_bytes_per_step": 8 * n,
                       "d2h_bytes_per_step": 16 * n, "ms_per_step": round(e2e_ms, 3),
                       "path": "pinned host x^ in, both parties' y out; the per-element keys are dealer material "
                               "resident on the device (offline phase)"},
               "roofline": {"bound": "lsu", "unit": "G AES-128 blocks/s",
                            "achieved": round(blocks / (kernel_ms / 1e3) / 1e9, 2),
                            "peak": round(engine_peak / 1e9, 2),
                            "frac": round(blocks / (kernel_ms / 1e3) / engine_peak, 4),
                            "kernel": "trunc_bundle_elem_kernel<2> (level-major keys)",
                            "traffic": None,
                            "traffic_adapter_layout": round(ELEM_TRAFFIC_BYTES_PER_ELEMENT * n),
                            "traffic_source": "ncu dram read + write of two 262,144-element launches of the "
                                              "adapter-layout kernel, per element, times one launch's elements",
                            "adapter_layout_ms_per_step": round(ms_adapter, 4),
                            "work_model": "every element walks every level of its own four keys: 2 AES blocks per "
                                          "level, 160 levels per element per party",
                            "hbm": {"achieved": round(hbm, 1), "peak": peaks.get("hbm_gbs"), "unit": "GB/s",
                                    "frac": round(hbm / peaks.get("hbm_gbs", 6650.0), 4),
                                    "bytes_per_element_per_party": sum(soa_kb) + 64}},
               "cpu_baseline": None, "clocks": clk.summary(), "gpu_launches": 2 * args.steps,
               "reconstruction_ok": ok, "ms_per_step_all": [round(v, 4) for v in ms_steps]}
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return res


# ---------------------------------------------------------------------------
# batched single-predicate DCF compare, per-element keys
# ---------------------------------------------------------------------------

CMP_N = 1 << 20
# DRAM bytes per element and party of trunc_bundle_elem_kernel from its ncu
# capture (two 262,144-element launches: 1,497.1 MB read and 1.9 - 5.3 MB
# written each): the 5,440 bytes of keys, the six plan words, x^ and y.
ELEM_TRAFFIC_BYTES_PER_ELEMENT = 5724.9
# DRAM bytes per element of myl7_eval_elem_aligned_kernel from its ncu capture
# ((594.6 + 8.3) MB / 262,144): the 2,152-byte key, x^, y and some re-reads.
CMP_TRAFFIC_BYTES_PER_ELEMENT = 2299.8
CMP_METRIC = "DCF pred-evals/sec (single-predicate compare 1[x^ < r_in], per-element myl7 keys)"


def compare_seeds(n: int, shard: int) -> np.ndarray:
    from suf_b200.engine import host_mt19937_64

    total = n * (shard + 1)
    return host_mt19937_64(1 ^ 0x5EED, 4 * total).view(np.uint8).reshape(total, 2, 16)[shard * n:(shard + 1) * n]


def compare_material(ctx, n: int, shard: int):
    """r_in[i] = successive mt19937_64(1) draws, x uniform with
    |x| < 2^36 (|v| < 2^20 with 16 fractional bits) from the draws after the
    masks, x^ = x + r_in; per-element myl7 keys for 1[x^ < r_in] with payload 1
    (additive Z_2^64 shares), seeds from mt19937_64(1 ^ 0x5EED)."""
    from suf_b200 import GROUP_ADD
    from suf_b200.engine import host_mt19937_64

    total = n * (shard + 1)
    draws = host_mt19937_64(1, 2 * total)
    r_in = draws[shard * n:(shard + 1) * n].copy()
    x = ((draws[total + shard * n: total + (shard + 1) * n] >> np.uint64(27)).view(np.int64) - (1 << 36))
    xhat = x.view(np.uint64) + r_in
    seeds = compare_seeds(n, shard)
    k0, k1 = ctx.myl7_gen_batch(GROUP_ADD, 64, r_in, (1).to_bytes(8, "little"), seeds[:, 0].copy(),
                                seeds[:, 1].copy())
    return r_in, xhat, (k0, k1)


def threshold_keys(alphas: np.ndarray, payload: int) -> np.ndarray:
    """Per-element keys of the reference GPU backend's DcfKeyHeader format
    (packed {u16 in_bits, u16 payload_len, u64 alpha} + 8-byte payload)."""
    rec = np.zeros(alphas.size, dtype=np.dtype([("in_bits", "<u2"), ("plen", "<u2"), ("alpha", "<u8"),
                                                 ("pay", "<u8")]))
    rec["in_bits"] = 64
    rec["plen"] = 8
    rec["alpha"] = alphas
    rec["pay"] = payload
    return rec.view(np.uint8).reshape(alphas.size, 20)


def run_compare(args, ws, rank, local):
    import torch
    import torch.distributed as dist

    from suf_b200 import GROUP_ADD
    from suf_b200.engine import Context, thr_dcf_key

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    ctx = Context(local)
    ctx.prg_init(prg_state())
    parties, n, shard = assignment(ws, rank, args.n_elem or CMP_N)
    t0 = time.perf_counter()
    r_in, xhat, keys = compare_material(ctx, n, shard)
    host_dealer_s = time.perf_counter() - t0
    kb = keys[0].shape[1]
    # the same key pairs from the GPU dealer (sufb200_myl7_gen_batch_device)
    from suf_b200 import GROUP_ADD as _GA

    sd = torch.from_numpy(np.ascontiguousarray(compare_seeds(n, shard).transpose(1, 0, 2)).reshape(2, -1)).to(dev)
    d_alpha = torch.from_numpy(r_in.view(np.int64)).to(dev)
    s0d, s1d = sd[0].contiguous(), sd[1].contiguous()
    g0 = torch.empty(n * kb, dtype=torch.uint8, device=dev)
    g1 = torch.empty(n * kb, dtype=torch.uint8, device=dev)
    ctx.myl7_gen_batch_device(_GA, 64, d_alpha, (1).to_bytes(8, "little"), s0d, s1d, g0, g1)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    ctx.myl7_gen_batch_device(_GA, 64, d_alpha, (1).to_bytes(8, "little"), s0d, s1d, g0, g1)
    e1.record()
    torch.cuda.synchronize()
    dev_dealer_ms = e0.elapsed_time(e1)
    dealer_same = bool((g0.cpu().numpy() == keys[0].reshape(-1)).all() and (g1.cpu().numpy() == keys[1].reshape(-1)).all())
    del g0, g1, sd, s0d, s1d
    stream = torch.cuda.Stream(device=dev)
    d_x = torch.from_numpy(xhat.view(np.int64)).to(dev)
    d_k = {p: torch.from_numpy(keys[p].reshape(-1)).to(dev) for p in parties}
    d_y = {p: torch.empty(n, dtype=torch.int64, device=dev) for p in parties}
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()

    def step():
        for p in parties:
            ctx.myl7_eval(GROUP_ADD, 64, d_k[p], kb, False, d_x, 8, d_out=d_y[p], stream=stream)

    ms, ms_steps, clk = _timed(args, ws, dev, stream, flush, step, ctx, local)
    units = n * len(parties) * ws
    value = units / (ms / 1e3)

    # reconstruction: y0 + y1 == 1[x^ < r_in]
    want = (xhat < r_in).astype(np.uint64)
    if len(parties) == 2:
        ok = bool(((d_y[0].cpu().numpy().view(np.uint64) + d_y[1].cpu().numpy().view(np.uint64)) == want).all())
    else:
        ok = _pair_check(ws, rank, dev, d_y[parties[0]], want)

    # e2e: the host-buffer entry point (keys, x^ in; shares out), copies timed
    x_pin = torch.from_numpy(xhat.view(np.int64)).pin_memory().numpy().view(np.uint64)
    k_pin = {p: torch.from_numpy(keys[p]).pin_memory().numpy() for p in parties}
    o_pin = {p: torch.empty(n * 8, dtype=torch.uint8).pin_memory().numpy().reshape(n, 8) for p in parties}
    for p in parties:
        ctx.myl7_eval_host(GROUP_ADD, 64, k_pin[p], kb, False, x_pin, 8, outs=o_pin[p])
    e2e = []
    for _ in range(max(1, min(args.steps, 3))):
        t0 = time.perf_counter()
        for p in parties:
            ctx.myl7_eval_host(GROUP_ADD, 64, k_pin[p], kb, False, x_pin, 8, outs=o_pin[p])
        e2e.append((time.perf_counter() - t0) * 1e3)
    e2e_ms = _max_over_ranks(ws, dev, sum(e2e) / len(e2e))

    # the reference GPU backend's trivial threshold format (20-byte keys): HBM-bound
    thr = {p: threshold_keys(r_in, 1 if p == 0 else 0) for p in parties}
    for p in parties:  # the vectorised blobs are the library builder's bytes
        for i in (0, n // 2, n - 1):
            want_k = thr_dcf_key(64, int(r_in[i]), (1 if p == 0 else 0).to_bytes(8, "little"))
            assert (thr[p][i] == want_k).all()
    d_t = {p: torch.from_numpy(thr[p].reshape(-1)).to(dev) for p in parties}
    d_o = {p: torch.empty(n, dtype=torch.int64, device=dev) for p in parties}

    def thr_step():
        for p in parties:
            ctx.thr_dcf_eval(64, d_t[p], 20, False, d_x, 8, d_out=d_o[p], stream=stream)

    thr_ms, _, _ = _timed(args, ws, dev, stream, flush, thr_step, ctx, local, sample_clocks=False)

    peaks = measured_peaks()
    engine_peak = ctx.probe_aes_engine()
    kernel_ms = ms / len(parties)
    blocks = n * 2 * 64  # two AES blocks (seed and value halves of the PRG) per level, 64 levels
    hbm_bytes = n * (kb + 16)
    roofline = {"bound": "lsu", "unit": "G AES-128 blocks/s",
                "achieved": round(blocks / (kernel_ms / 1e3) / 1e9, 2), "peak": round(engine_peak / 1e9, 2),
                "frac": round(blocks / (kernel_ms / 1e3) / engine_peak, 4),
                "traffic": round(CMP_TRAFFIC_BYTES_PER_ELEMENT * n),
                "traffic_source": "ncu dram read + write of one 262,144-element launch of this kernel, per "
                                  "element, times this call's elements",
                "kernel": "myl7_eval_elem_aligned_kernel",
                "work_model": "128 AES blocks per element (2 per level x 64 levels)",
                "hbm": {"achieved": round(hbm_bytes / (kernel_ms / 1e3) / 1e9, 1), "peak": peaks.get("hbm_gbs"),
                        "unit": "GB/s", "bytes_per_element": kb + 16},
                "kernel_ms": round(kernel_ms, 4)}
    thr_gbs = n * 36 / (thr_ms / len(parties) / 1e3) / 1e9
    out = None
    if rank == 0:
        cpu = cpu_compare_baseline(args, keys, xhat, kb) if (ws == 1 and not args.no_cpu) else None
        out = {"metric": CMP_METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128", "data": "synthetic (seeded, configs[0] shapes)",
               "config": {"workload": "configs[0]: DCF compare 1[x^ < r_in], per-element keys, seed 1",
                          "n_elements_per_party_per_gpu": n, "parties_per_gpu": len(parties),
                          "key_bytes": kb, "l2": "keys (2.2 GB per party) larger than L2; 256 MB flush as well",
                          "parallelism": f"party x element shards on {ws} GPU(s)"},
               "e2e": {"value": round(units / (e2e_ms / 1e3), 1), "unit": UNIT,
                       "h2d_bytes_per_step": len(parties) * n * (kb + 8), "d2h_bytes_per_step": len(parties) * n * 8,
                       "ms_per_step": round(e2e_ms, 3), "path": "sufb200_myl7_dcf_eval_host (pinned keys and x^)"},
               "roofline": roofline, "cpu_baseline": cpu, "clocks": clk.summary(),
               "gpu_launches": args.steps * len(parties), "reconstruction_ok": ok,
               "dealer": {"device_ms": round(dev_dealer_ms, 3), "host_s": round(host_dealer_s, 3),
                          "host_threads": host_threads(), "identical_keys": dealer_same,
                          "device_key_pairs_per_s": round(n / (dev_dealer_ms / 1e3), 1),
                          "device_aes_blocks_per_s": round(n * 8 * 64 / (dev_dealer_ms / 1e3), 1),
                          "note": "sufb200_myl7_gen_batch_device vs the host dealer (OpenMP, AES-NI), same seeds"},
               "reference_threshold_format": {
                   "value": round(units / (thr_ms / 1e3), 1), "unit": UNIT, "ms_per_step": round(thr_ms, 4),
                   "hbm_gbs": round(thr_gbs, 1), "hbm_frac": round(thr_gbs / peaks.get("hbm_gbs", 6650.0), 3),
                   "kernel": "thr_dcf_kernel (DcfKeyHeader keys, 20 B + 8 B x^ + 8 B out per element)"},
               "ms_per_step_all": [round(v, 4) for v in ms_steps]}
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return out


def cpu_compare_baseline(args, keys, xhat, kb):
    """The reference's myl7 dcf_eval over a bounded sample of configs[0]
    (per-element keys), OpenMP over elements, both parties."""
    from oracle.oracle import GROUP_ADD, RefMyl7

    if not RefMyl7.available():
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference", "sample": "oracle/_ref not built"}
    ref = RefMyl7(GROUP_ADD)
    ref.set_threads(host_threads())
    ref.prg_init(prg_state())
    n = min(args.cpu_sample, xhat.size, 1 << 18)
    t0 = time.perf_counter()
    for p in (0, 1):
        ref.eval_omp(64, keys[p][:n], kb, False, xhat[:n], 8)
    dt = time.perf_counter() - t0
    return {"value": round(2 * n / dt, 1), "unit": UNIT, "cores": host_threads(), "kind": "reference",
            "sample": f"{n} elements x 2 parties, reference myl7 dcf_eval (OpenMP over elements, "
                      f"{host_threads()} threads); {dt:.2f} s"}


def run_compare_reference(args, ws, rank):
    from oracle.oracle import RefMyl7

    if rank != 0:
        return None
    if not RefMyl7.available():
        return {"impl": "reference", "unavailable": "oracle/_ref (reference myl7 sources) was not built"}
    from suf_b200.engine import Context

    ctx = Context(-1)
    ctx.prg_init(prg_state())
    n = min(args.ref_sample, CMP_N)
    r_in, xhat, keys = compare_material(ctx, n, 0)
    kb = keys[0].shape[1]
    a = argparse.Namespace(cpu_sample=n)
    for _ in range(args.warmup):
        cpu_compare_baseline(argparse.Namespace(cpu_sample=max(1, n // 8)), keys, xhat, kb)
    vals = [cpu_compare_baseline(a, keys, xhat, kb) for _ in range(args.steps)]
    ctx.close()
    v = sum(x["value"] for x in vals) / len(vals)
    return {"metric": CMP_METRIC, "value": round(v, 1), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(2 * n / v * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128",
            "data": "synthetic (seeded, configs[0] shapes)", "impl": "reference",
            "config": {"workload": "configs[0]: DCF compare 1[x^ < r_in], per-element keys, seed 1",
                       "sample_elements_per_step": n, "parties": 2},
            "cpu_baseline": dict(vals[-1], value=round(v, 1)),
            "e2e": {"value": round(v, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# the paired-GPU open (configs[4] open traffic): N >= 2
# ---------------------------------------------------------------------------

OPEN_WORDS = 16_700_000   # words opened per layer per party (bert-base, measured by the reference)
OPEN_FLUSHES = 120        # flushes per layer
OPEN_METRIC = "opened words/sec (paired-GPU open, configs[4] layer: 120 flushes, 16.7 M words per party)"
NVLINK_GBS = 770.0        # measured peer copy per direction on this pool


def run_open(args, ws, rank, local):
    import torch
    import torch.distributed as dist

    from suf_b200.engine import Context, OpenComm, share_open_id

    if ws < 2 or ws % 2:
        if rank == 0:
            return {"metric": OPEN_METRIC, "unavailable": "the open pairs GPU j with GPU j + N/2: run with N >= 2"}
        return None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    ctx = Context(local)
    comm = OpenComm(ctx, share_open_id(rank), ws, rank, timeout_s=60.0)
    peer = (rank + ws // 2) % ws
    ring = args.ring_bits
    ep = None
    if args.open_impl == "p2p":
        from suf_b200.engine import P2POpen, share_p2p_handles

        per0 = (args.n_elem or OPEN_WORDS) // OPEN_FLUSHES
        ep = P2POpen(ctx, max_words=(per0 + 63) // 64 * 64 + 64)
        ep.connect(share_p2p_handles(ep)[peer])
    eff = ring if ring <= 56 else 64  # SUF_OPEN_PACK_MAX_BITS default
    per = (args.n_elem or OPEN_WORDS) // OPEN_FLUSHES
    rng = np.random.default_rng([5, rank % (ws // 2)])
    m = np.uint64((1 << ring) - 1) if ring < 64 else np.uint64(~np.uint64(0))
    x = rng.integers(0, 2**63, per * OPEN_FLUSHES, dtype=np.uint64) & m
    s0 = rng.integers(0, 2**63, x.size, dtype=np.uint64) & m
    mine = s0 if rank < ws // 2 else (x - s0) & m
    d_in = torch.from_numpy(mine.view(np.int64)).to(dev).view(OPEN_FLUSHES, per)
    d_out = torch.empty_like(d_in)
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)

    # The flushes' device pointers are taken once, so a step is 120 calls of
    # the C ABI (as a C++ runtime would make them), not 120 tensor slicings.
    from suf_b200 import _lib as L_

    lib_ = L_.lib()
    sp = int(stream.cuda_stream)
    ins = [int(d_in[f].data_ptr()) for f in range(OPEN_FLUSHES)]
    outs = [int(d_out[f].data_ptr()) for f in range(OPEN_FLUSHES)]

    def step():
        if ep is not None:
            h = ep.h
            for f in range(OPEN_FLUSHES):
                L_.check(lib_.sufb200_p2p_open_exchange(h, ins[f], per, eff, ring, 1, outs[f], 5.0, sp))
        else:
            h = comm.h
            for f in range(OPEN_FLUSHES):
                L_.check(lib_.sufb200_open_exchange(h, peer, ins[f], per, eff, ring, 1, outs[f], sp))

    ms, ms_steps, clk = _timed(args, ws, dev, stream, flush, step, ctx, local)
    want = x.copy()
    if ring < 64:
        sign = (want >> np.uint64(ring - 1)) & np.uint64(1)
        want |= (np.uint64(0) - sign) & ~m
    ok = bool((d_out.cpu().numpy().reshape(-1).view(np.uint64) == want).all())
    eager_ms, graph = ms, None
    if ep is not None:
        # the step's 120 exchanges captured once as a CUDA graph (the kernel
        # numbers its calls on the device, so replays stay in step with the
        # peer's); each replay is one layer of opens with no host work
        d_out.zero_()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="relaxed"):
            step()
        dist.barrier()
        gms, gsteps, gclk = _timed(args, ws, dev, stream, flush, g.replay, ctx, local)
        gok = bool((d_out.cpu().numpy().reshape(-1).view(np.uint64) == want).all())
        graph = {"ms_per_step": round(gms, 4), "ms_per_flush": round(gms / OPEN_FLUSHES, 4), "opened_ok": gok,
                 "eager_ms_per_step": round(eager_ms, 4), "eager_ms_per_flush": round(eager_ms / OPEN_FLUSHES, 4)}
        if gok:
            ms, ms_steps, clk = gms, gsteps, gclk
        ok = ok and gok
        del g
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    ok = bool(flag.item())
    words = per * OPEN_FLUSHES
    wire = -(-per * eff // 64) * 8 * OPEN_FLUSHES  # bytes each GPU sends per step
    gbs = wire / (ms / 1e3) / 1e9
    out = None
    if rank == 0:
        out = {"metric": OPEN_METRIC, "value": round(words * ws / (ms / 1e3), 1), "unit": "opened words/s",
               "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": f"u64 (Z_2^{ring})",
               "data": "synthetic (seeded shares)",
               "config": {"workload": "configs[4] open traffic: one layer of flushes per step",
                          "words_per_party_per_pair": words, "flushes": OPEN_FLUSHES, "ring_bits": ring,
                          "eff_bits": eff, "pairs": ws // 2, "l2": "256 MB flush between steps",
                          "parallelism": f"party 0 on GPUs 0..{ws // 2 - 1}, party 1 on the rest"},
               "e2e": {"value": round(words * ws / (ms / 1e3), 1), "unit": "opened words/s",
                       "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                       "note": "device-resident by design: the shares and the opened values stay in HBM"},
               "roofline": {"bound": "nvlink", "unit": "GB/s", "achieved": round(gbs, 2), "peak": NVLINK_GBS,
                            "frac": round(gbs / NVLINK_GBS, 4), "traffic": wire,
                            "note": "bytes each GPU sends per step / step time, vs the measured peer copy per "
                                    "direction; 120 flushes of 139 K words are latency-bound"},
               "open_impl": ("sufb200_p2p_open: pack, peer stores over NVLink, flag, bounded wait, add in one "
                             "kernel" if ep is not None else "sufb200_open_exchange: pack, NCCL send/recv, add"),
               "graph": graph,
               "clocks": clk.summary(),
               "gpu_launches": args.steps * OPEN_FLUSHES * (1 if ep is not None else (2 if eff < 64 else 1)),
               "opened_ok": ok, "ms_per_flush": round(ms / OPEN_FLUSHES, 4),
               "ms_per_step_all": [round(v, 4) for v in ms_steps]}
    dist.barrier()
    if ep is not None:
        ep.close()
    comm.close()
    dist.destroy_process_group()
    ctx.close()
    return out


# ---------------------------------------------------------------------------
# the SiLU spline gate (interval-LUT coefficients, one pass)
# ---------------------------------------------------------------------------

SILU_N = 1 * 128 * 3072
SILU_METRIC = "SiLU gate evals/sec (configs[2]: interval-LUT coefficients + output masks, one pass per party)"


def silu_inputs(n: int, frac_bits: int, shard: int) -> np.ndarray:
    """x ~ N(0, 4^2) quantised at frac_bits (numpy default_rng([3, shard]))."""
    rng = np.random.default_rng([3, shard])
    return np.rint(rng.normal(0.0, 4.0, n) * 2.0**frac_bits).astype(np.int64).view(np.uint64)


def run_silu(args, ws, rank, local):
    import torch
    import torch.distributed as dist

    from suf_b200.engine import Context, coeff_lut_eval, coeff_lut_eval_pair
    from tests.helpers import silu_fixture, suf_table_eval

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    ctx = Context(local)
    ctx.prg_init(prg_state())  # the engine-ceiling probe runs the PRG step
    fx = silu_fixture()  # the reference's own dealer output (tests/golden/make_silu_fixture.py)
    parties, n, shard = assignment(ws, rank, args.n_elem or SILU_N)
    x = silu_inputs(n, fx["frac_bits"], shard)
    xhat = x + np.uint64(fx["r_in"])
    r = fx["r"]
    stream = torch.cuda.Stream(device=dev)
    d_x = torch.from_numpy(xhat.view(np.int64)).to(dev)
    d_y = {p: torch.empty(n * r, dtype=torch.int64, device=dev) for p in parties}
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)

    pair = len(parties) == 2

    def step():
        if pair:  # both parties on this GPU: one launch (sufb200_coeff_lut_eval_pair)
            coeff_lut_eval_pair(ctx, fx["keys"], d_x, r, fx["degree"], r_outs=(fx["r_out_share0"], fx["r_out_share1"]),
                                d_outs=(d_y[0], d_y[1]), stream=stream)
            return
        for p in parties:
            coeff_lut_eval(ctx, fx["keys"][p], d_x, r, fx["degree"], r_out=fx[f"r_out_share{p}"], d_out=d_y[p],
                           stream=stream)

    ms, ms_steps, clk = _timed(args, ws, dev, stream, flush, step, ctx, local)
    units = n * len(parties) * ws
    want = suf_table_eval(fx["alpha"], fx["pieces"], x)
    if len(parties) == 2:
        y = [d_y[p].cpu().numpy().view(np.uint64).reshape(n, r) for p in (0, 1)]
        ok = bool(((y[0] + y[1] - fx["r_out"]) == want).all())
    else:  # y0 + y1 = coefficients + r_out, checked across the paired GPUs
        ok = _pair_check(ws, rank, dev, d_y[parties[0]], (want + fx["r_out"]).reshape(-1))

    # e2e: pinned host x^ in, the r coefficient shares out, copies timed
    x_pin = torch.from_numpy(xhat.view(np.int64)).pin_memory()
    y_pin = {p: torch.empty(n * r, dtype=torch.int64).pin_memory() for p in parties}

    def e2e_step():
        d = x_pin.to(dev, non_blocking=True)
        if pair:
            ys = coeff_lut_eval_pair(ctx, fx["keys"], d, r, fx["degree"],
                                     r_outs=(fx["r_out_share0"], fx["r_out_share1"]))
            for p in parties:
                y_pin[p].copy_(ys[p], non_blocking=True)
        else:
            for p in parties:
                y_pin[p].copy_(coeff_lut_eval(ctx, fx["keys"][p], d, r, fx["degree"], r_out=fx[f"r_out_share{p}"]),
                               non_blocking=True)
        torch.cuda.synchronize()

    for _ in range(3):
        e2e_step()
    e2e = []
    for _ in range(max(args.steps, 5)):
        t0 = time.perf_counter()
        e2e_step()
        e2e.append((time.perf_counter() - t0) * 1e3)
    e2e_ms = _max_over_ranks(ws, dev, sum(e2e) / len(e2e))

    peaks = measured_peaks()
    engine_peak = ctx.probe_aes_engine()
    launches = 1 if pair else len(parties)
    kernel_ms = ms / launches
    # One AES block per two words; a dealt pair (one AES key, nonce and cut
    # table for both parties) shares its keystream, so the pair launch
    # encrypts each counter block once for both share rows.
    k0, k1 = (np.asarray(k).view(np.uint8) for k in fx["keys"])
    ivs = int(k0[4:8].view(np.uint32)[0])
    shared = pair and all((k0[a:b] == k1[a:b]).all() for a, b in ((0, 8), (16, 24), (40, 216 + 8 * ivs)))
    blocks_alg = n * (len(parties) // launches) * ((fx["out_words"] + 1) // 2)
    blocks = n * ((fx["out_words"] + 1) // 2) if shared else blocks_alg
    hbm = n * (8 + 8 * r * (len(parties) // launches))
    out = None
    if rank == 0:
        out = {"metric": SILU_METRIC, "value": round(units / (ms / 1e3), 1), "unit": "gate evals/s", "n_gpus": ws,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128",
               "data": "synthetic x ~ N(0, 16) at f = 12; keys from the reference's own SiLU dealer",
               "config": {"workload": "configs[2]: SiLU spline gate, 1x128x3072, f = 12, seed 3",
                          "n_elements_per_party_per_gpu": n, "parties_per_gpu": len(parties),
                          "intervals": int(fx["keys"][0][4:8].view(np.uint32)[0]), "coeff_words": r,
                          "l2": "256 MB flush between steps", "parallelism": f"party x element shards on {ws} GPU(s)"},
               "e2e": {"value": round(units / (e2e_ms / 1e3), 1), "unit": "gate evals/s",
                       "h2d_bytes_per_step": n * 8, "d2h_bytes_per_step": len(parties) * n * r * 8,
                       "ms_per_step": round(e2e_ms, 4),
                       "path": ("sufb200_coeff_lut_eval_pair" if pair else "sufb200_coeff_lut_eval")
                               + ", pinned x^ in, shares out"},
               "roofline": {"bound": "lsu", "unit": "us per launch", "achieved": round(kernel_ms * 1e3, 2),
                            "aes_floor_us": round(blocks / engine_peak * 1e6, 2),
                            "hbm_floor_us": round(hbm / (peaks.get("hbm_gbs", 6650.0) * 1e9) * 1e6, 2),
                            "frac": round((blocks / engine_peak * 1e6) / (kernel_ms * 1e3), 4),
                            "peak": round(engine_peak / 1e9, 2), "traffic": hbm,
                            "kernel": "coeff_lut_pair_kernel" if pair else "coeff_lut_kernel",
                            "work_model": f"{len(parties) // launches} x {n:,} elements per launch, one AES "
                                          "block per two coefficient words (2 per element)"
                                          + (", each block serving both parties' share rows (the dealt pair "
                                             "shares its keystream)" if shared else ""),
                            "blocks_executed": blocks, "blocks_per_party_sum": blocks_alg,
                            "note": "frac = AES-engine floor of the blocks the launch executes / measured "
                                    "launch time"},
               "cpu_baseline": cpu_silu_baseline(args, fx, xhat) if (ws == 1 and not args.no_cpu) else None,
               "clocks": clk.summary(), "gpu_launches": args.steps * launches, "reconstruction_ok": ok,
               "ms_per_step_all": [round(v, 4) for v in ms_steps]}
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return out


def run_silu_reference(args, ws, rank):
    if rank != 0:
        return None
    from tests.helpers import silu_fixture

    fx = silu_fixture()
    n = min(args.n_elem or SILU_N, SILU_N)
    xhat = silu_inputs(n, fx["frac_bits"], 0) + np.uint64(fx["r_in"])
    a = argparse.Namespace(cpu_sample=n)
    for _ in range(args.warmup):
        cpu_silu_baseline(argparse.Namespace(cpu_sample=max(1, n // 8)), fx, xhat)
    vals = [cpu_silu_baseline(a, fx, xhat)["value"] for _ in range(args.steps)]
    v = sum(vals) / len(vals)
    base = cpu_silu_baseline(argparse.Namespace(cpu_sample=min(n, 4096)), fx, xhat)
    return {"metric": SILU_METRIC, "value": round(v, 1), "unit": "gate evals/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(2 * n / v * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128",
            "data": "synthetic x ~ N(0, 16) at f = 12", "impl": "reference",
            "config": {"workload": "configs[2]: SiLU spline gate, 1x128x3072, f = 12, seed 3", "parties": 2},
            "cpu_baseline": dict(base, value=round(v, 1), sample=f"{n} elements x 2 parties per step"),
            "e2e": {"value": round(v, 1), "unit": "gate evals/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def cpu_silu_baseline(args, fx, xhat):
    """The oracle's restatement of the reference interval-LUT evaluation plus
    the r_out add, both parties, OpenMP over elements (a port: the reference's
    CPU composite path runs the same LUT through SigmaFastBackend)."""
    from oracle.oracle import Oracle

    orc = Oracle()
    n = min(xhat.size, args.cpu_sample)
    t0 = time.perf_counter()
    for p in (0, 1):
        orc.interval_eval(fx["keys"][p], fx["keys"][p].size, True, xhat[:n], fx["out_words"]) + fx[f"r_out_share{p}"]
    dt = time.perf_counter() - t0
    return {"value": round(2 * n / dt, 1), "unit": "gate evals/s", "cores": host_threads(), "kind": "port",
            "sample": f"{n} elements x 2 parties, oracle interval LUT + r_out; {dt:.3f} s"}


# ---------------------------------------------------------------------------
# the softmax block, device-resident, both parties on one GPU
# ---------------------------------------------------------------------------

SOFTMAX_HEADS, SOFTMAX_LEN = 12, 128
SOFTMAX_METRIC = "softmax blocks/sec (configs[4]: 12 x 128 x 128 causal attention softmax, both parties)"
# words each element's data moves through HBM in one block (reads + writes of
# every stage's tensors, both parties; row-level tensors are negligible)
SOFTMAX_WORDS_PER_ELEMENT = 70
REF_SOFTMAX = ROOT / "oracle" / "_ref" / "ref_softmax_drive"


def softmax_inputs(heads: int, length: int, frac_bits: int, seed: int = 4):
    """Causal attention scores ~ N(0, 2^2) at f = 12 (seed 4): the packed
    max-differences t = max - x clamped to [0, 16] (the SoftmaxBlockTask input),
    the row lengths, and the double-precision softmax of the same scores."""
    rng = np.random.default_rng(seed)
    rows = heads * length
    lens = np.arange(rows) % length + 1
    x = np.round(rng.normal(0.0, 2.0, (rows, length)) * (1 << frac_bits)) / (1 << frac_bits)
    ts, ref = [], []
    for r in range(rows):
        v = x[r, :lens[r]]
        d = np.minimum(v.max() - v, 16.0)
        ts.append(np.round(d * (1 << frac_bits)).astype(np.uint64))
        e = np.exp(-d)
        ref.append(e / e.sum())
    return np.concatenate(ts), lens, np.concatenate(ref)


def cpu_softmax_baseline(args):
    """The reference's own nn::SoftmaxBlockTask on its CPU backend
    (proto::ReferenceBackend), both parties on threads, driven by
    oracle/_ref/ref_softmax_drive (built from the reference sources): ms per
    block, best of the runs.  Without that build, the plaintext model of the
    block (oracle/softmax_model.py, numpy) stands in as a port."""
    if REF_SOFTMAX.exists():
        r = subprocess.run([str(REF_SOFTMAX), f"--heads={SOFTMAX_HEADS}", f"--len={SOFTMAX_LEN}", "--reps=3",
                            "--cpu-only"],
                           capture_output=True, text=True, timeout=600)
        line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
        if line:
            j = json.loads(line[-1])
            ms = float(j["ref_cpu_ms"])
            return {"value": round(1e3 / ms, 3), "unit": "blocks/s", "cores": 2, "kind": "reference",
                    "ms_per_block": round(ms, 3),
                    "sample": "one configs[4] block, reference SoftmaxBlockTask on proto::ReferenceBackend, "
                              "both parties on two threads, best of 3"}
    from oracle.softmax_model import load_tables, softmax_block

    t, lens, _ = softmax_inputs(SOFTMAX_HEADS, SOFTMAX_LEN, 12)
    off = np.concatenate([[0], np.cumsum(lens)])
    t0 = time.perf_counter()
    softmax_block(t, off, load_tables())
    ms = (time.perf_counter() - t0) * 1e3
    return {"value": round(1e3 / ms, 3), "unit": "blocks/s", "cores": 1, "kind": "port", "ms_per_block": round(ms, 3),
            "sample": "one configs[4] block, plaintext numpy model of the block (no shares)"}


# Our kernels per block (from the ncu launch list): softmax = 4 element-level
# truncations x (frontier, main; their f-bit queries take full-domain tables,
# so no range pass) + 3 row-level pair truncations + 2 interval-LUT gates
# (both parties per launch) + 9 elementwise stages; LayerNorm = 1
# element-level truncation x 2 + 7 row-level pair truncations + 1 LUT gate +
# 9 row and elementwise stages.
SOFTMAX_LAUNCHES = 22
LAYERNORM_LAUNCHES = 19


def run_softmax(args, ws, rank, local):
    """One configs[4] softmax block per step on every GPU, both parties' shares
    on the GPU (replicas: the block has no cross-GPU exchange when both
    parties sit on one GPU)."""
    import torch
    import torch.distributed as dist

    from suf_b200.engine import Context
    from suf_b200.softmax import SoftmaxBlock

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    ctx = Context(local)
    ctx.prg_init(prg_state())
    t, lens, ref = softmax_inputs(SOFTMAX_HEADS, SOFTMAX_LEN, 12)
    n = t.size
    blk = SoftmaxBlock(ctx, lens, seed=11 + rank)
    rng = np.random.default_rng(5 + rank)
    t0 = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2)
    with np.errstate(over="ignore"):
        t1 = t - t0
    d_t = [torch.from_numpy(v.view(np.int64)).to(dev) for v in (t0, t1)]
    d_p = [torch.empty(n, dtype=torch.int64, device=dev) for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)

    def step():
        blk.run(d_t[0], d_t[1], d_p[0], d_p[1], stream=stream)

    ms, ms_steps, clk = _timed(args, ws, dev, stream, flush, step, ctx, local)
    ctx.sync()
    with np.errstate(over="ignore"):
        prob = (d_p[0].cpu().numpy().view(np.uint64) + d_p[1].cpu().numpy().view(np.uint64)).view(np.int64)
    err = float(np.abs(prob / 4096.0 - ref).max())

    # e2e: pinned host shares of t in, both parties' probability shares out
    t_pin = [torch.from_numpy(v.view(np.int64)).pin_memory() for v in (t0, t1)]
    p_pin = [torch.empty(n, dtype=torch.int64).pin_memory() for _ in range(2)]

    def e2e_step():
        d0, d1 = (v.to(dev, non_blocking=True) for v in t_pin)
        p0, p1 = blk.run(d0, d1)
        p_pin[0].copy_(p0, non_blocking=True)
        p_pin[1].copy_(p1, non_blocking=True)
        torch.cuda.synchronize()

    for _ in range(3):
        e2e_step()
    e2e = []
    for _ in range(max(args.steps, 5)):
        h0 = time.perf_counter()
        e2e_step()
        e2e.append((time.perf_counter() - h0) * 1e3)
    e2e_ms = _max_over_ranks(ws, dev, sum(e2e) / len(e2e))

    peaks = measured_peaks()
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    traffic = SOFTMAX_WORDS_PER_ELEMENT * 8 * n
    gbs = traffic / (ms / 1e3) / 1e9
    out = None
    if rank == 0:
        out = {"metric": SOFTMAX_METRIC, "value": round(ws / (ms / 1e3), 3), "unit": "blocks/s", "n_gpus": ws,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128",
               "data": "synthetic causal scores ~ N(0, 4) at f = 12 (seed 4); gate tables from the reference",
               "config": {"workload": "configs[4]: softmax block, 12 heads x 128 x 128 causal, f = 12, seed 4",
                          "rows": int(lens.size), "active_elements": int(n), "parties_per_gpu": 2,
                          "l2": "256 MB flush between steps", "parallelism": f"one block per GPU, {ws} GPU(s)"},
               "e2e": {"value": round(ws / (e2e_ms / 1e3), 3), "unit": "blocks/s", "h2d_bytes_per_step": 2 * n * 8,
                       "d2h_bytes_per_step": 2 * n * 8, "ms_per_step": round(e2e_ms, 4),
                       "path": "sufb200_softmax_block_pair, pinned t shares in, probability shares out"},
               "roofline": {"bound": "hbm", "unit": "GB/s", "achieved": round(gbs, 1), "peak": hbm_peak,
                            "frac": round(gbs / hbm_peak, 4), "traffic": traffic,
                            "per_block_us": round(ms * 1e3, 1),
                            "note": "bytes = every stage's tensors read and written once (70 words per active "
                                    "element); the block is a chain of 22 small launches, bound by their latency"},
               "cpu_baseline": cpu_softmax_baseline(args) if (ws == 1 and not args.no_cpu) else None,
               "clocks": clk.summary(), "gpu_launches": SOFTMAX_LAUNCHES * args.steps,
               "max_err_vs_double_softmax": round(err, 6), "reconstruction_ok": err < 0.03,
               "ms_per_step_all": [round(v, 4) for v in ms_steps]}
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return out


LN_ROWS, LN_COLS = 128, 768
LN_METRIC = "layernorm blocks/sec (configs[4]: 128 x 768 LayerNorm, one Newton rsqrt step, both parties)"
# words per element through HBM: x (2 r), d (2 w + 2 r), squares' triples (6 r),
# x^ (1 w + 1 r per stage, 2 stages), row-broadcast triples (4 r), output (2 w)
LN_WORDS_PER_ELEMENT = 22


def ln_inputs(rows: int, cols: int, frac_bits: int, seed: int = 4):
    rng = np.random.default_rng(seed)
    return np.round(rng.normal(0.0, 1.0, rows * cols) * (1 << frac_bits)).astype(np.int64).view(np.uint64)


def cpu_layernorm_baseline(args):
    """The reference's own runtime::LayerNormTask on its CPU backend
    (proto::ReferenceBackend, which by default reconstructs x and computes the
    LayerNorm in plaintext), both parties on threads, via
    oracle/_ref/ref_softmax_drive --block=ln.  Without that build the numpy
    model of the block stands in as a port."""
    if REF_SOFTMAX.exists():
        r = subprocess.run([str(REF_SOFTMAX), "--block=ln", f"--rows={LN_ROWS}", f"--cols={LN_COLS}", "--reps=3",
                            "--cpu-only"], capture_output=True, text=True, timeout=600)
        line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
        if line:
            ms = float(json.loads(line[-1])["ref_cpu_ms"])
            return {"value": round(1e3 / ms, 3), "unit": "blocks/s", "cores": 2, "kind": "reference",
                    "ms_per_block": round(ms, 3),
                    "sample": "one configs[4] LayerNorm block, reference LayerNormTask on proto::ReferenceBackend, "
                              "both parties on two threads, best of 3"}
    from oracle.softmax_model import layernorm_block, load_tables

    x = ln_inputs(LN_ROWS, LN_COLS, 12)
    t0 = time.perf_counter()
    layernorm_block(x, LN_ROWS, LN_COLS, load_tables())
    ms = (time.perf_counter() - t0) * 1e3
    return {"value": round(1e3 / ms, 3), "unit": "blocks/s", "cores": 1, "kind": "port", "ms_per_block": round(ms, 3),
            "sample": "one configs[4] LayerNorm block, plaintext numpy model (no shares)"}


def run_layernorm(args, ws, rank, local):
    """One configs[4] LayerNorm block per step on every GPU, both parties'
    shares on the GPU (replicas, as for the softmax block)."""
    import torch
    import torch.distributed as dist

    from suf_b200.engine import Context
    from suf_b200.softmax import LayerNormBlock

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    ctx = Context(local)
    ctx.prg_init(prg_state())
    x = ln_inputs(LN_ROWS, LN_COLS, 12)
    n = x.size
    blk = LayerNormBlock(ctx, LN_ROWS, LN_COLS, seed=21 + rank)
    rng = np.random.default_rng(6 + rank)
    x0 = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2)
    with np.errstate(over="ignore"):
        x1 = x - x0
    d_x = [torch.from_numpy(v.view(np.int64)).to(dev) for v in (x0, x1)]
    d_o = [torch.empty(n, dtype=torch.int64, device=dev) for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)

    def step():
        blk.run(d_x[0], d_x[1], d_o[0], d_o[1], stream=stream)

    ms, ms_steps, clk = _timed(args, ws, dev, stream, flush, step, ctx, local)
    ctx.sync()
    with np.errstate(over="ignore"):
        out = (d_o[0].cpu().numpy().view(np.uint64) + d_o[1].cpu().numpy().view(np.uint64)).view(np.int64)
    inv = round(4096 / LN_COLS) / 4096.0
    xr = x.view(np.int64).reshape(LN_ROWS, LN_COLS) / 4096.0
    mu = xr.sum(1, keepdims=True) * inv
    ref = (xr - mu) / np.sqrt(((xr - mu) ** 2).sum(1, keepdims=True) * inv + 1 / 1024)
    err = float(np.abs(out.reshape(LN_ROWS, LN_COLS) / 4096.0 - ref).max())

    x_pin = [torch.from_numpy(v.view(np.int64)).pin_memory() for v in (x0, x1)]
    o_pin = [torch.empty(n, dtype=torch.int64).pin_memory() for _ in range(2)]

    def e2e_step():
        a, b = (v.to(dev, non_blocking=True) for v in x_pin)
        o0, o1 = blk.run(a, b)
        o_pin[0].copy_(o0, non_blocking=True)
        o_pin[1].copy_(o1, non_blocking=True)
        torch.cuda.synchronize()

    for _ in range(3):
        e2e_step()
    e2e = []
    for _ in range(max(args.steps, 5)):
        h0 = time.perf_counter()
        e2e_step()
        e2e.append((time.perf_counter() - h0) * 1e3)
    e2e_ms = _max_over_ranks(ws, dev, sum(e2e) / len(e2e))

    hbm_peak = measured_peaks().get("hbm_gbs", 6650.0)
    traffic = LN_WORDS_PER_ELEMENT * 8 * n
    gbs = traffic / (ms / 1e3) / 1e9
    res = None
    if rank == 0:
        res = {"metric": LN_METRIC, "value": round(ws / (ms / 1e3), 3), "unit": "blocks/s", "n_gpus": ws,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128",
               "data": "synthetic x ~ N(0, 1) at f = 12 (seed 4); rsqrt table from the reference",
               "config": {"workload": "configs[4]: LayerNorm block, 128 x 768, f = 12, eps 1/1024, seed 4",
                          "rows": LN_ROWS, "cols": LN_COLS, "parties_per_gpu": 2,
                          "l2": "256 MB flush between steps", "parallelism": f"one block per GPU, {ws} GPU(s)"},
               "e2e": {"value": round(ws / (e2e_ms / 1e3), 3), "unit": "blocks/s", "h2d_bytes_per_step": 2 * n * 8,
                       "d2h_bytes_per_step": 2 * n * 8, "ms_per_step": round(e2e_ms, 4),
                       "path": "sufb200_layernorm_block_pair, pinned x shares in, output shares out"},
               "roofline": {"bound": "hbm", "unit": "GB/s", "achieved": round(gbs, 1), "peak": hbm_peak,
                            "frac": round(gbs / hbm_peak, 4), "traffic": traffic, "per_block_us": round(ms * 1e3, 1),
                            "note": "bytes = every stage's tensors read and written once (22 words per element); "
                                    "a chain of 20 small launches, bound by their latency"},
               "cpu_baseline": cpu_layernorm_baseline(args) if (ws == 1 and not args.no_cpu) else None,
               "clocks": clk.summary(), "gpu_launches": LAYERNORM_LAUNCHES * args.steps,
               "max_err_vs_double_layernorm": round(err, 6), "reconstruction_ok": err < 0.02,
               "ms_per_step_all": [round(v, 4) for v in ms_steps]}
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return res


def run_layernorm_reference(args, ws, rank):
    if rank != 0:
        return None
    runs = [cpu_layernorm_baseline(args) for _ in range(args.steps)]
    ms = min(r["ms_per_block"] for r in runs)
    v = round(1e3 / ms, 3)
    return {"metric": LN_METRIC, "value": v, "unit": "blocks/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 (Z_2^64)", "data": "synthetic x ~ N(0, 1) at f = 12",
            "impl": "reference",
            "config": {"workload": "configs[4]: LayerNorm block, 128 x 768, f = 12, eps 1/1024, seed 4"},
            "cpu_baseline": dict(runs[0], value=v, ms_per_block=round(ms, 3)),
            "e2e": {"value": v, "unit": "blocks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_softmax_reference(args, ws, rank):
    if rank != 0:
        return None
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_softmax_baseline(args)
    runs = [cpu_softmax_baseline(args) for _ in range(args.steps)]
    ms = min(r["ms_per_block"] for r in runs)
    v = round(1e3 / ms, 3)
    return {"metric": SOFTMAX_METRIC, "value": v, "unit": "blocks/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 (Z_2^64)", "data": "synthetic causal scores ~ N(0, 4) at f = 12",
            "impl": "reference",
            "config": {"workload": "configs[4]: softmax block, 12 heads x 128 x 128 causal, f = 12, seed 4"},
            "cpu_baseline": dict(runs[0], value=v, ms_per_block=round(ms, 3)),
            "e2e": {"value": v, "unit": "blocks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# the 2PC transformer layer (and the 12-layer stack)
# ---------------------------------------------------------------------------

LAYER_METRIC = "2PC transformer-layer latency (configs[4]: d 768, 12 heads, d_ff 3072, seq 128, Z_2^64, f 12)"
LAYER_STACK = 12
HARNESS_B200 = ROOT / "suf_b200" / "_refrt" / "layer_harness_b200"
HARNESS_REF = ROOT / "oracle" / "_ref" / "refgpu" / "layer_harness_ref"


def _run_harness(path: Path, args_list, timeout: int = 900) -> dict:
    """One run of a layer_harness binary; its JSON line, or {'error': ...}."""
    if not path.exists():
        return {"error": f"{path.relative_to(ROOT)} not built (needs the reference checkout at build time)"}
    env = dict(os.environ)
    env.pop("OMP_NUM_THREADS", None)  # the harness picks the reference bench's per-party thread count
    try:
        r = subprocess.run([str(path), *args_list], capture_output=True, text=True, timeout=timeout, env=env)
    except subprocess.TimeoutExpired:
        return {"error": f"timed out after {timeout} s"}
    try:
        return json.loads(r.stdout.strip().splitlines()[-1])
    except (ValueError, IndexError):
        return {"error": f"rc={r.returncode}: {r.stderr.strip()[-300:]}"}


def _layer_float64(X, W, dims):
    """The same pre-LN layer in float64 on the dequantised values (exact
    LayerNorm with eps 1/1024, softmax and GeLU): the accuracy yardstick."""
    from math import erf, sqrt

    S, D, H, Dh, f = dims.S, dims.D, dims.H, dims.Dh, dims.f
    x = X.view(np.int64).reshape(S, D) / float(1 << f)
    w = {n: W[n].astype(np.float64) / float(1 << f) for n in W}

    def ln(z):
        mu = z.mean(axis=1, keepdims=True)
        return (z - mu) / np.sqrt(((z - mu) ** 2).mean(axis=1, keepdims=True) + 1.0 / 1024)

    qkv = ln(x) @ w["qkv"]
    outs = []
    for h in range(H):
        q, k, v = (qkv[:, o + h * Dh:o + (h + 1) * Dh] for o in (0, D, 2 * D))
        s = q @ k.T / np.sqrt(Dh)
        e = np.exp(s - s.max(axis=1, keepdims=True))
        outs.append(e / e.sum(axis=1, keepdims=True) @ v)
    x2 = x + np.concatenate(outs, axis=1) @ w["o"]
    f1 = ln(x2) @ w["ff1"]
    g = np.vectorize(lambda z: 0.5 * z * (1.0 + erf(z / sqrt(2.0))))(f1)
    return x2 + g @ w["ff2"]


def run_layer(args, ws, rank, local):
    """One configs[4] transformer layer per step on the device (both parties'
    shares on one GPU, suf_b200.layer.TransformerLayerPair), the 12-layer
    stack timed beside it; at N > 1 every GPU runs its own replica (the
    layer has no cross-GPU step).  Beside it, the reference's own layer
    runtime (nn::transformer_layer_forward on its phase executor) with this
    engine as its PFSS backend (the drop-in, suf_b200/_refrt)."""
    import torch
    import torch.distributed as dist

    from suf_b200.engine import Context
    from suf_b200.layer import LayerDims, TransformerLayerPair, synthetic_layer

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=300))
    ctx = Context(local)
    ctx.prg_init(prg_state())
    dims = LayerDims()
    X, W = synthetic_layer(dims, seed=5)
    lay = TransformerLayerPair(ctx, W, dims, seed=11 + rank)
    rng = np.random.default_rng([5, rank])
    x0 = rng.integers(0, 2**64, X.size, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x1 = X.ravel() - x0
    d_x = [torch.from_numpy(v.view(np.int64)).to(dev) for v in (x0, x1)]
    d_y = [torch.empty(X.size, dtype=torch.int64, device=dev) for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)

    def step():
        lay.run(d_x[0], d_x[1], d_y[0], d_y[1], stream=stream)

    ms, ms_steps, clk = _timed(args, ws, dev, stream, flush, step, ctx, local)
    ctx.sync(stream)
    y = (d_y[0].cpu().numpy().view(np.uint64) + d_y[1].cpu().numpy().view(np.uint64)).view(np.int64) / 4096.0

    # the 12-layer stack: each layer's output shares feed the next
    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    stack = []
    for _ in range(2):
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            flush.fill_(0)
            ev[0].record(stream)
            a, b = d_x
            for _ in range(LAYER_STACK):
                a, b = lay.run(a, b, stream=stream)
            ev[1].record(stream)
        torch.cuda.synchronize()
        stack.append(ev[0].elapsed_time(ev[1]))
    ctx.sync(stream)
    stack_ms = _max_over_ranks(ws, dev, min(stack))

    # the same layer as a CUDA graph (TransformerLayerPair.capture): one
    # replay per step launches all of the layer's kernels with no host work
    eager_ms, eager_stack_ms = ms, stack_ms
    gx = [t.clone() for t in d_x]
    gy = [torch.empty_like(t) for t in d_x]
    g1 = lay.capture(gx[0], gx[1], gy[0], gy[1], layers=1)

    def gstep():
        g1.replay()

    gms, gms_steps, gclk = _timed(args, ws, dev, stream, flush, gstep, ctx, local)
    ctx.sync(stream)
    graph_ok = bool((gy[0].cpu().numpy() == d_y[0].cpu().numpy()).all()
                    and (gy[1].cpu().numpy() == d_y[1].cpu().numpy()).all())
    gs = lay.capture(gx[0], gx[1], gy[0], gy[1], layers=LAYER_STACK)
    gstack = []
    for _ in range(2):
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            flush.fill_(0)
            ev[0].record(stream)
            gs.replay()
            ev[1].record(stream)
        torch.cuda.synchronize()
        gstack.append(ev[0].elapsed_time(ev[1]))
    ctx.sync(stream)
    graph_stack_ms = _max_over_ranks(ws, dev, min(gstack))
    if graph_ok:
        ms, ms_steps, clk, stack_ms = gms, gms_steps, gclk, graph_stack_ms

    x_pin = [torch.from_numpy(v.view(np.int64)).pin_memory() for v in (x0, x1)]
    y_pin = [torch.empty(X.size, dtype=torch.int64).pin_memory() for _ in range(2)]

    def e2e_step():
        with torch.cuda.stream(stream):
            if graph_ok:  # pinned shares into the graph's input buffers, replay, shares out
                gx[0].copy_(x_pin[0], non_blocking=True)
                gx[1].copy_(x_pin[1], non_blocking=True)
                g1.replay()
                o0, o1 = gy
            else:
                a, b = (v.to(dev, non_blocking=True) for v in x_pin)
                o0, o1 = lay.run(a, b, stream=stream)
            y_pin[0].copy_(o0, non_blocking=True)
            y_pin[1].copy_(o1, non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        e2e_step()
    e2e = []
    for _ in range(max(args.steps, 5)):
        h0 = time.perf_counter()
        e2e_step()
        e2e.append((time.perf_counter() - h0) * 1e3)
    ctx.sync(stream)
    e2e_ms = _max_over_ranks(ws, dev, sum(e2e) / len(e2e))
    ok_e2e = bool((y_pin[0].numpy() + y_pin[1].numpy() == d_y[0].cpu().numpy() + d_y[1].cpu().numpy()).all())

    res = None
    if rank == 0:
        acc = None
        try:  # accuracy of the fixed-point layer against float64, off the timed path
            yf = _layer_float64(X, W, dims)
            acc = {"max_abs_err": round(float(np.abs(y.reshape(yf.shape) - yf).max()), 5),
                   "mean_abs_err": round(float(np.abs(y.reshape(yf.shape) - yf).mean()), 5),
                   "max_abs_output": round(float(np.abs(yf).max()), 4)}
        except Exception as ex:  # noqa: BLE001 -- a report, not a gate
            acc = {"error": str(ex)[:200]}
        dropin = (None if args.no_dropin else
                  _run_harness(HARNESS_B200, ["--backend=gpu", "--layers=1", f"--iters={max(3, args.steps // 2)}"]))
        cpu = None
        if ws == 1 and not args.no_cpu:
            c = _run_harness(HARNESS_B200, ["--backend=cpu", "--layers=1", "--iters=2"], timeout=600)
            cpu = ({"value": c["ms_per_layer"], "unit": "ms/layer", "cores": os.cpu_count(), "kind": "reference",
                    "sample": "one configs[4] layer of the reference's own runtime on its OpenMP CPU backend "
                              "(SigmaFast, SUF_FORCE_PFSS), both parties as threads, online iteration after the "
                              f"dealer's; {c.get('omp_threads_per_party')} OpenMP threads per party"}
                   if "ms_per_layer" in c else {"value": None, "unit": "ms/layer", "cores": 0, "kind": "reference",
                                                "sample": c.get("error", "failed")})
        res = {"metric": LAYER_METRIC, "value": round(ms, 4), "unit": "ms/layer", "n_gpus": ws, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False,
               "scaling": "weak", "vs_baseline": None, "dtype": "u64 (Z_2^64), AES-128",
               "data": "synthetic: weights N(0, 0.02^2), inputs N(0, 1), quantised at f = 12 (seed 5)",
               "config": {"workload": "configs[4]: one 2PC transformer encoder layer, pre-LN, GeLU (256-segment "
                                      "constant SUF), 64-bit ring", "d_model": dims.D, "heads": dims.H,
                          "d_ff": dims.Dff, "seq_len": dims.S, "batch": 1, "frac_bits": dims.f,
                          "parties_per_gpu": 2, "stack_layers": LAYER_STACK,
                          "l2": "256 MB flush between steps",
                          "parallelism": "both parties on one GPU" + (f"; {ws} replicas" if ws > 1 else "")},
               "stack_ms": round(stack_ms, 3),
               "e2e": {"value": round(e2e_ms, 4), "unit": "ms/layer", "h2d_bytes_per_step": 2 * X.size * 8,
                       "d2h_bytes_per_step": 2 * X.size * 8, "ms_per_step": round(e2e_ms, 4),
                       "path": ("TransformerLayerPair.capture's graph replayed" if graph_ok else
                                "TransformerLayerPair.run") + " from pinned host shares of X to pinned host shares of Y",
                       "outputs_match_device_leg": ok_e2e},
               "graph": {"used_for_value": graph_ok, "outputs_match_eager": graph_ok, "ms_per_layer": round(gms, 4),
                         "stack_ms": round(graph_stack_ms, 3), "eager_ms_per_layer": round(eager_ms, 4),
                         "eager_stack_ms": round(eager_stack_ms, 3)},
               "accuracy_vs_float64": acc,
               "dropin_reference_runtime": dropin,
               "cpu_baseline": cpu, "clocks": clk.summary(), "gpu_launches": lay.launches() * args.steps,
               "ms_per_step_all": [round(v, 4) for v in ms_steps]}
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return res


def run_layer_reference(args, ws, rank):
    """The reference's GPU build (its cuda_pfss backend and nn runtime,
    compiled for sm_100a by oracle/Makefile's refgpu recipe) running the same
    configs[4] layer: nn::transformer_layer_forward for both parties on
    threads, as its bench_suf_transformer does, 64-bit ring."""
    if rank != 0:
        return None
    r = _run_harness(HARNESS_REF, ["--backend=gpu", "--layers=1", f"--iters={args.steps + 1}"])
    if "ms_per_layer" not in r:
        return {"impl": "reference", "metric": LAYER_METRIC, "unavailable": r.get("error", "layer harness failed")}
    st = _run_harness(HARNESS_REF, ["--backend=gpu", f"--layers={LAYER_STACK}", "--iters=2"])
    v = r["ms_per_layer"]
    return {"metric": LAYER_METRIC, "value": v, "unit": "ms/layer", "n_gpus": ws, "steps": args.steps,
            "warmup": 1, "ms_per_step": v, "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "u64 (Z_2^64)", "data": "synthetic: weights N(0, 0.02^2), inputs N(0, 1), quantised at f = 12",
            "impl": "reference",
            "config": {"workload": "configs[4]: one 2PC transformer encoder layer (the reference's "
                                   "transformer_layer_forward, bert-base shape), GeLU (256-segment constant SUF), "
                                   "64-bit ring", "d_model": 768, "heads": 12, "d_ff": 3072, "seq_len": 128,
                       "batch": 1, "frac_bits": 12, "parties_per_gpu": 2, "stack_layers": LAYER_STACK},
            "stack_ms": st.get("online_ms"),
            "cpu_baseline": {"value": v, "unit": "ms/layer", "cores": os.cpu_count(), "kind": "reference",
                             "sample": "the reference GPU build's layer, host-orchestrated (wall clock per online "
                                       "iteration, as its bench measures)"},
            "e2e": {"value": v, "unit": "ms/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "harness": r}


# ---------------------------------------------------------------------------
# one layer's Beaver matmuls on the tensor cores
# ---------------------------------------------------------------------------

LAYER_MATMULS = [("qkv", 128, 768, 2304), ("out", 128, 768, 768), ("ffn1", 128, 768, 3072), ("ffn2", 128, 3072, 768)]
MATMUL_METRIC = "ring MACs/sec (configs[4] layer Beaver matmuls, Z_2^64, both parties)"


# A-plane pre-pass and fused GEMM per Beaver call (all four layer shapes take
# the fused path; the split contraction is reduced inside the GEMM's cluster)
LAUNCHES_PER_TC_CALL = 2


def run_matmul(args, ws, rank, local):
    import ctypes as C

    import torch

    from suf_b200 import _lib
    from suf_b200.engine import Context

    if ws > 1:
        return {"metric": MATMUL_METRIC, "unavailable": "single-GPU microbenchmark"} if rank == 0 else None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = Context(local)
    L = _lib.lib()
    rng = np.random.default_rng(5)
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)
    mats = []
    for name, M, K, N in LAYER_MATMULS:
        t = {k: torch.from_numpy(rng.integers(-(2**62), 2**62, sz, dtype=np.int64)).to(dev)
             for k, sz in (("D", M * K), ("E", K * N), ("A", M * K), ("B", K * N), ("C", M * N))}
        t["out"] = {p: torch.empty(M * N, dtype=torch.int64, device=dev) for p in (0, 1)}
        t["ref"] = {p: torch.empty(M * N, dtype=torch.int64, device=dev) for p in (0, 1)}
        mats.append((name, M, K, N, t))
    sp = int(stream.cuda_stream)
    # The two parties are independent: each runs its calls on its own stream
    # (as two party processes sharing the GPU would), forked from and joined
    # back to the timing stream inside the step.
    side = torch.cuda.Stream(device=dev)
    pst = (sp, int(side.cuda_stream))

    def both_parties(issue):
        fork = torch.cuda.Event()
        fork.record(stream)
        side.wait_event(fork)
        for name, M, K, N, t in mats:
            for p in (0, 1):
                issue(p, M, K, N, t, pst[p])
        join = torch.cuda.Event()
        join.record(side)
        stream.wait_event(join)

    def tc_step():
        both_parties(lambda p, M, K, N, t, s: _lib.check(L.sufb200_beaver_matmul2d_tc(
            ctx.h, p, t["D"].data_ptr(), t["E"].data_ptr(), t["A"].data_ptr(), t["B"].data_ptr(), t["C"].data_ptr(),
            1, M, K, N, 0, 1, C.c_int64(4096), 12, t["out"][p].data_ptr(), s)))

    def core_step():
        both_parties(lambda p, M, K, N, t, s: _lib.check(L.sufb200_beaver_matmul2d(
            p, t["D"].data_ptr(), t["E"].data_ptr(), t["A"].data_ptr(), t["B"].data_ptr(), t["C"].data_ptr(), 1, M,
            K, N, 0, 1, 4096, 12, t["ref"][p].data_ptr(), s)))

    ms, ms_steps, clk = _timed(args, ws, dev, stream, flush, tc_step, ctx, local)
    core_ms, _, _ = _timed(args, ws, dev, stream, flush, core_step, ctx, local, sample_clocks=False)
    # bit-exact against the CUDA-core kernel, both parties
    same = all(bool(torch.equal(t["out"][p], t["ref"][p])) for *_, t in mats for p in (0, 1))
    macs = sum(2 * M * N * (2 * K) for _, M, K, N in LAYER_MATMULS)  # [D|A][B(+E);E], both parties
    int8_macs = 36 * macs
    peaks = measured_peaks()
    int8_peak = 2 * peaks.get("bf16_tflops", 1590.0) * 1e12 / 2  # MAC/s: dense int8 = 2x bf16 rate
    # per-matmul times
    per = {}
    for name, M, K, N, t in mats:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            flush.fill_(1)
            e0.record(stream)
            for _ in range(10):
                _lib.check(L.sufb200_beaver_matmul2d_tc(ctx.h, 0, t["D"].data_ptr(), t["E"].data_ptr(),
                                                        t["A"].data_ptr(), t["B"].data_ptr(), t["C"].data_ptr(), 1, M,
                                                        K, N, 0, 1, C.c_int64(4096), 12, t["out"][0].data_ptr(), sp))
            e1.record(stream)
        torch.cuda.synchronize()
        per[f"{name}_{M}x{K}x{N}_us"] = round(e0.elapsed_time(e1) / 10 * 1e3, 2)
    ctx.sync(stream)
    ctx.close()
    return {"metric": MATMUL_METRIC, "value": round(macs / (ms / 1e3), 1), "unit": "ring MACs/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u64 (Z_2^64) via int8 limbs",
            "data": "synthetic shares (seeded)",
            "config": {"workload": "configs[4]: QKV, O, FFN1, FFN2 Beaver matmuls of one d=768 layer, L=128, "
                                   "rescale by 4096 >> 12", "matmuls": [list(m[:4]) for m in mats],
                       "parties": "one stream per party, concurrent", "l2": "256 MB flush between steps"},
            "e2e": {"value": round(macs / (ms / 1e3), 1), "unit": "ring MACs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0, "note": "device-resident operands by design (shares stay in HBM)"},
            "roofline": {"bound": "tensor", "unit": "T int8 MAC/s", "achieved": round(int8_macs / (ms / 1e3) / 1e12, 1),
                         "peak": round(int8_peak / 1e12, 1), "frac": round(int8_macs / (ms / 1e3) / int8_peak, 4),
                         "traffic": None, "kernel": "ring_gemm_tc_fused_kernel",
                         "peak_source": "2x the measured dense bf16 rate (MEASURED_PEAKS.json) as the int8 rate"},
            "cuda_core": {"ms_per_step": round(core_ms, 4), "speedup": round(core_ms / ms, 2),
                          "kernel": "beaver_matmul_kernel (u64 MACs on the integer pipes)", "identical": same},
            "per_matmul_us": per, "clocks": clk.summary(), "gpu_launches": args.steps * 8 * LAUNCHES_PER_TC_CALL,
            "ms_per_step_all": [round(v, 4) for v in ms_steps]}



def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-sample", type=int, default=N_ELEM,
                    help="elements of the compare / silu workloads' cpu_baseline leg")
    ap.add_argument("--ref-sample", type=int, default=1 << 20,
                    help="elements per step of the compare workload's --impl reference arm")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-dropin", action="store_true",
                    help="layer workload: skip the reference-runtime (drop-in) harness run beside the device layer")
    ap.add_argument("--n-elem", type=int, default=None,
                    help="elements per party at N=1 (default: the workload's config size; smaller only for "
                         "profiling)")
    ap.add_argument("--workload", default="trunc", choices=["trunc", "compare", "open", "silu", "matmul", "softmax",
                                                          "layernorm", "layer", "trunc_elem"],
                    help="trunc: configs[1] (the headline line); compare: configs[0], per-element keys; "
                         "open: the paired-GPU open of a configs[4] layer (N >= 2); layer: the configs[4] "
                         "transformer layer (ms/layer, lower is better); softmax: the configs[4] "
                         "softmax block; layernorm: the configs[4] LayerNorm block")
    ap.add_argument("--open-impl", default="p2p", choices=["nccl", "p2p"],
                    help="the open between paired GPUs (N >= 2; headline and open workloads): the one-kernel "
                         "peer-store open (sufb200_p2p_open, default) or NCCL send/recv (sufb200_open_exchange)")
    ap.add_argument("--ring-bits", type=int, default=37, help="ring of the open workload (37: the reference's "
                                                                 "measured bert-base ring)")
    args = ap.parse_args()
    ws, rank, local = dist_env()
    if args.workload == "open":
        out = ({"impl": "reference", "unavailable": "the reference's open runs through its host channel "
                "(net::Chan); no stand-alone CPU implementation of the exchange to time"}
               if args.impl == "reference" and rank == 0 else None) if args.impl == "reference" else \
            run_open(args, ws, rank, local)
    elif args.workload == "matmul":
        out = ({"impl": "reference", "metric": MATMUL_METRIC,
                "unavailable": "the reference's Beaver matmul is a CUDA kernel; its CUDA-core equivalent is timed "
                               "beside ours in the ours line (cuda_core)"}
               if rank == 0 else None) if args.impl == "reference" else run_matmul(args, ws, rank, local)
    elif args.workload == "trunc_elem":
        out = ({"impl": "reference", "metric": ELEM_METRIC,
                "unavailable": "the reference's per-element path evaluates one composite gate per element on its "
                               "host runtime; no batch CPU implementation to time at this size"}
               if rank == 0 else None) if args.impl == "reference" else run_trunc_elem(args, ws, rank, local)
    elif args.workload == "layer":
        out = run_layer_reference(args, ws, rank) if args.impl == "reference" else run_layer(args, ws, rank, local)
    elif args.workload == "layernorm":
        out = (run_layernorm_reference(args, ws, rank) if args.impl == "reference"
               else run_layernorm(args, ws, rank, local))
    elif args.workload == "softmax":
        out = run_softmax_reference(args, ws, rank) if args.impl == "reference" else run_softmax(args, ws, rank, local)
    elif args.workload == "silu":
        out = run_silu_reference(args, ws, rank) if args.impl == "reference" else run_silu(args, ws, rank, local)
    elif args.workload == "compare":
        out = run_compare_reference(args, ws, rank) if args.impl == "reference" else run_compare(args, ws, rank, local)
    elif args.impl == "reference":
        out = run_reference(args, ws, rank)
    else:
        out = run_ours(args, ws, rank, local)
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
