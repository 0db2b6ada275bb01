"""GPU parity: myl7 DCF tree walk (per-element and broadcast keys) against the
oracle, the reference-generated golden keys and, at full size, the
reconstruction property.  Bit-exact: all arithmetic is in Z_2^64."""
from __future__ import annotations

import zlib
from pathlib import Path

import numpy as np
import pytest

from oracle.oracle import GROUP_ADD, GROUP_XOR
from tests.conftest import from_dev, rand_u64, to_dev
from tests.helpers import seeds_for

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _gen_many(oracle, group, in_bits, n, out_bytes, seed):
    """n per-element key pairs (oracle dealer) with alphas from mt19937_64(seed)."""
    alphas = oracle.mt64(seed, n) & np.uint64((1 << in_bits) - 1 if in_bits < 64 else 2**64 - 1)
    s0, s1 = seeds_for(seed + 1, n, oracle)
    payload = np.random.default_rng(seed).integers(0, 256, out_bytes, dtype=np.uint8).tobytes()
    kb = oracle.myl7_key_bytes(in_bits, out_bytes)
    k0 = np.empty((n, kb), np.uint8)
    k1 = np.empty((n, kb), np.uint8)
    for i in range(n):
        k0[i], k1[i] = oracle.myl7_gen(group, in_bits, int(alphas[i]), payload, s0[i], s1[i])
    return alphas, payload, k0, k1


@pytest.mark.parametrize("group", [GROUP_ADD, GROUP_XOR])
@pytest.mark.parametrize("in_bits", [1, 7, 8, 16, 37, 63, 64])
def test_per_element_keys_bit_exact(ctx, torch_cuda, oracle, prg_state, group, in_bits):
    oracle.prg_init(prg_state)
    n, ob = 301, 8
    alphas, _, k0, k1 = _gen_many(oracle, group, in_bits, n, ob, 1000 + in_bits)
    rng = np.random.default_rng(in_bits)
    xs = rand_u64(rng, n)
    with np.errstate(over="ignore"):
        xs[:3] = [alphas[0], alphas[1] - np.uint64(1), alphas[2] + np.uint64(1)]
    dx = to_dev(torch_cuda, xs)
    for k in (k0, k1):
        dk = to_dev(torch_cuda, k.ravel())
        out = ctx.myl7_eval(group, in_bits, dk, k.shape[1], False, dx, ob)
        ctx.sync()
        exp = np.stack([oracle.myl7_eval(group, k[i], k.shape[1], True, xs[i:i + 1], ob)[0] for i in range(n)])
        assert (from_dev(out, np.uint8).reshape(n, ob) == exp).all()


@pytest.mark.parametrize("group", [GROUP_ADD, GROUP_XOR])
@pytest.mark.parametrize("in_bits,out_bytes", [(64, 8), (16, 8), (13, 1), (64, 3), (40, 8)])
def test_broadcast_key_bit_exact(ctx, torch_cuda, oracle, prg_state, group, in_bits, out_bytes):
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(7 * in_bits + out_bytes)
    alpha = int(rng.integers(0, 2**63)) & ((1 << in_bits) - 1)
    payload = rng.integers(0, 256, out_bytes, dtype=np.uint8).tobytes()
    s0, s1 = seeds_for(77 + in_bits, 1, oracle)
    k0, k1 = oracle.myl7_gen(group, in_bits, alpha, payload, s0[0], s1[0])
    n = 5000
    xs = rand_u64(rng, n)
    xs[:4] = [alpha, max(alpha - 1, 0), 0, 2**64 - 1]
    dx = to_dev(torch_cuda, xs)
    for k in (k0, k1):
        out = ctx.myl7_eval(group, in_bits, to_dev(torch_cuda, k), k.size, True, dx, out_bytes)
        ctx.sync()
        exp = oracle.myl7_eval(group, k, k.size, True, xs, out_bytes)
        assert (from_dev(out, np.uint8).reshape(n, out_bytes) == exp).all()


@pytest.mark.parametrize("group,fname", [(GROUP_ADD, "myl7_add.npz"), (GROUP_XOR, "myl7_xor.npz")])
def test_reference_golden_keys(torch_cuda, group, fname):
    """Keys made by the reference's dcf_gen, outputs of the reference's eval."""
    from suf_b200.engine import Context

    g = np.load(GOLDEN / fname)
    with Context(0) as c:
        c.prg_init(g["prg_state"])
        for ci in g["cases"]:
            in_bits, _, plen = (int(v) for v in g[f"c{ci}_meta"])
            xs = g[f"c{ci}_xs"]
            for p in (0, 1):
                k = g[f"c{ci}_key{p}"]
                out = c.myl7_eval(group, in_bits, to_dev(torch_cuda, k), k.size, True, to_dev(torch_cuda, xs), plen)
                c.sync()
                assert (from_dev(out, np.uint8).reshape(xs.size, plen) == g[f"c{ci}_out{p}"]).all()


def test_keys_from_reference_adapter(ctx, torch_cuda, prg_state):
    """Keys produced by the reference adapter's own gen_dcf (random seeds)."""
    from oracle.oracle import RefMyl7

    if not RefMyl7.available():
        pytest.skip("oracle/_ref not built")
    ref = RefMyl7(GROUP_ADD)
    ref.prg_init(prg_state)
    rng = np.random.default_rng(21)
    xs = rand_u64(rng, 2048)
    for alpha in (0, 1, 2**63, 2**64 - 1, 0x0123456789ABCDEF):
        k0, k1 = ref.adapter_gen(64, alpha, (1).to_bytes(8, "little"))
        for k in (k0, k1):
            out = ctx.myl7_eval(GROUP_ADD, 64, to_dev(torch_cuda, k), k.size, True, to_dev(torch_cuda, xs), 8)
            ctx.sync()
            assert (from_dev(out) == ref.eval_omp(64, k, k.size, True, xs, 8).view(np.uint64).ravel()).all()


def test_host_buffer_entry_point(ctx, oracle, prg_state):
    oracle.prg_init(prg_state)
    n = 257
    alphas, payload, k0, k1 = _gen_many(oracle, GROUP_ADD, 64, n, 8, 4242)
    xs = rand_u64(np.random.default_rng(5), n)
    o0 = ctx.myl7_eval_host(GROUP_ADD, 64, k0, k0.shape[1], False, xs, 8).view(np.uint64).ravel()
    o1 = ctx.myl7_eval_host(GROUP_ADD, 64, k1, k1.shape[1], False, xs, 8).view(np.uint64).ravel()
    pay = np.frombuffer(payload, np.uint64)[0]
    assert ((o0 + o1) == np.where(xs < alphas, pay, np.uint64(0))).all()


def test_empty_and_rejected_inputs(ctx, torch_cuda, oracle, prg_state):
    from suf_b200 import SufB200Error

    oracle.prg_init(prg_state)
    k0, _ = oracle.myl7_gen(GROUP_ADD, 64, 5, (1).to_bytes(8, "little"), np.zeros(16, np.uint8),
                            np.ones(16, np.uint8))
    dk = to_dev(torch_cuda, k0)
    empty = torch_cuda.empty(0, dtype=torch_cuda.int64, device="cuda")
    ctx.myl7_eval(GROUP_ADD, 64, dk, k0.size, True, empty, 8)  # N = 0 is a no-op
    dx = to_dev(torch_cuda, np.arange(8, dtype=np.uint64))
    with pytest.raises(SufB200Error):  # key_bytes inconsistent with in_bits
        ctx.myl7_eval(GROUP_ADD, 64, dk, k0.size - 1, True, dx, 8)
    with pytest.raises(SufB200Error):  # out_bytes beyond one chunk's low 8 bytes
        ctx.myl7_eval(GROUP_ADD, 64, dk, k0.size, True, dx, 9)
    with pytest.raises(SufB200Error):  # header says 64 bits, call says 63: host path rejects
        ctx.myl7_eval_host(GROUP_ADD, 63, k0[: k0.size - 33], k0.size - 33, True, np.arange(4, dtype=np.uint64), 8)
    # device path: wrong party byte is flagged through the status word
    bad = k0.copy()
    bad[2] = 7
    ctx.myl7_eval(GROUP_ADD, 64, to_dev(torch_cuda, bad), bad.size, True, dx, 8)
    with pytest.raises(SufB200Error) as ei:
        ctx.sync()
    assert ei.value.code == -3
    ctx.sync()  # the status word is cleared after being reported


def test_full_size_reconstruction_property(ctx, torch_cuda, oracle, prg_state):
    """N = 2^20 broadcast: p0 + p1 == 1[x^ < alpha] for every element (config-1 size)."""
    oracle.prg_init(prg_state)
    n = 1 << 20
    rng = np.random.default_rng(1)
    alpha = int(rng.integers(0, 2**63)) * 2
    s0, s1 = seeds_for(5, 1, oracle)
    k0, k1 = oracle.myl7_gen(GROUP_ADD, 64, alpha, (1).to_bytes(8, "little"), s0[0], s1[0])
    xs = rand_u64(rng, n)
    dx = to_dev(torch_cuda, xs)
    o0 = from_dev(ctx.myl7_eval(GROUP_ADD, 64, to_dev(torch_cuda, k0), k0.size, True, dx, 8))
    o1 = from_dev(ctx.myl7_eval(GROUP_ADD, 64, to_dev(torch_cuda, k1), k1.size, True, dx, 8))
    ctx.sync()
    assert ((o0 + o1) == (xs < np.uint64(alpha)).astype(np.uint64)).all()
    # spot-check shares against the oracle
    idx = rng.integers(0, n, 512)
    assert (o0[idx] == oracle.myl7_eval(GROUP_ADD, k0, k0.size, True, xs[idx], 8).view(np.uint64).ravel()).all()


def _window_inputs(rng, n, mode, in_bits):
    """Inputs shaped to stress the shared-prefix plan (prefix.cuh)."""
    mask = np.uint64((1 << in_bits) - 1 if in_bits < 64 else 2**64 - 1)
    if mode == "uniform":
        xs = rand_u64(rng, n)
    elif mode == "clustered":  # x^ = x + r with |x| < 2^40, the bench's shape
        r = np.uint64(int(rng.integers(0, 2**63)) * 2 + 1)
        xs = rng.integers(-(2**40) + 1, 2**40, n, dtype=np.int64).view(np.uint64) + r
    elif mode == "wrap":  # straddles 2^64 (and 2^in_bits after masking)
        xs = rng.integers(-(2**20), 2**20, n, dtype=np.int64).view(np.uint64)
    else:  # constant
        xs = np.full(n, np.uint64(int(rng.integers(0, 2**63))))
    return xs & mask if in_bits < 64 else xs


@pytest.mark.parametrize("group", [GROUP_ADD, GROUP_XOR])
@pytest.mark.parametrize("in_bits", [64, 37, 16])
@pytest.mark.parametrize("mode", ["uniform", "clustered", "wrap", "constant"])
def test_broadcast_shared_prefix_path_bit_exact(ctx, torch_cuda, oracle, prg_state, group, in_bits, mode):
    """N above the shared-prefix threshold: every share equals the oracle's."""
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(zlib.crc32(f"{group}-{in_bits}-{mode}".encode()))
    n = 40_000
    xs = _window_inputs(rng, n, mode, in_bits)
    alpha = int(xs[n // 2]) & ((1 << in_bits) - 1)  # threshold inside the window
    s0, s1 = seeds_for(900 + in_bits, 1, oracle)
    k0, k1 = oracle.myl7_gen(group, in_bits, alpha, (0x0102030405060708).to_bytes(8, "little"), s0[0], s1[0])
    dx = to_dev(torch_cuda, xs)
    for k in (k0, k1):
        out = ctx.myl7_eval(group, in_bits, to_dev(torch_cuda, k), k.size, True, dx, 8)
        ctx.sync()
        assert (from_dev(out, np.uint8).reshape(n, 8) == oracle.myl7_eval(group, k, k.size, True, xs, 8)).all()
