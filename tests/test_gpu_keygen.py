"""GPU parity: myl7 DCF keys generated on the GPU (sufb200_myl7_gen_batch_device)
are byte-identical to the host dealer's (sufb200_myl7_gen_batch) and to the
reference's own dcf_gen keys (tests/golden/myl7_*.npz) for the same party
seeds, and evaluate to the right shares at the configs[0] size."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle.oracle import GROUP_ADD, GROUP_XOR
from tests.conftest import from_dev, to_dev

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"


@pytest.mark.parametrize("group", [GROUP_ADD, GROUP_XOR])
@pytest.mark.parametrize("in_bits,plen", [(64, 8), (8, 1), (16, 16), (24, 3), (56, 9)])
def test_device_keys_match_host_dealer(ctx, torch_cuda, group, in_bits, plen):
    rng = np.random.default_rng(in_bits * 31 + plen + 7 * group)
    n = 3001
    alphas = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
    alphas[:4] = [0, 2**64 - 1, 1, 2**63]
    seeds0 = rng.integers(0, 256, (n, 16), dtype=np.uint8)
    seeds1 = rng.integers(0, 256, (n, 16), dtype=np.uint8)
    payload = rng.integers(0, 256, plen, dtype=np.uint8).tobytes()
    h0, h1 = ctx.myl7_gen_batch(group, in_bits, alphas, payload, seeds0, seeds1)
    d0, d1 = ctx.myl7_gen_batch_device(group, in_bits, to_dev(torch_cuda, alphas), payload,
                                       torch_cuda.from_numpy(seeds0.reshape(-1)).cuda(),
                                       torch_cuda.from_numpy(seeds1.reshape(-1)).cuda())
    ctx.sync()
    assert (from_dev(d0, np.uint8).reshape(h0.shape) == h0).all()
    assert (from_dev(d1, np.uint8).reshape(h1.shape) == h1).all()


@pytest.mark.parametrize("group,fname", [(GROUP_ADD, "myl7_add.npz"), (GROUP_XOR, "myl7_xor.npz")])
def test_device_keys_match_reference_dcf_gen(torch_cuda, group, fname):
    """The reference's dcf_gen keys (oracle/_ref, fixed seeds) for the golden
    cases whose input width is a multiple of 8."""
    from suf_b200.engine import Context

    g = np.load(GOLDEN / fname)
    checked = 0
    with Context(0) as c:
        c.prg_init(g["prg_state"])
        for ci in g["cases"]:
            in_bits, alpha, plen = (int(v) for v in g[f"c{ci}_meta"])
            if in_bits % 8:
                continue
            payload = g[f"c{ci}_payload"][:plen].tobytes()
            d0, d1 = c.myl7_gen_batch_device(
                group, in_bits, to_dev(torch_cuda, np.array([alpha], dtype=np.uint64)), payload,
                torch_cuda.from_numpy(g[f"c{ci}_seed0"].copy()).cuda(),
                torch_cuda.from_numpy(g[f"c{ci}_seed1"].copy()).cuda())
            c.sync()
            assert (from_dev(d0, np.uint8) == g[f"c{ci}_key0"]).all()
            assert (from_dev(d1, np.uint8) == g[f"c{ci}_key1"]).all()
            checked += 1
    assert checked >= 2


def test_device_keys_configs0_roundtrip(ctx, torch_cuda):
    """2^20 per-element key pairs for 1[x^ < alpha] made on the GPU and
    evaluated on the GPU: y0 + y1 is the comparison bit for every element."""
    n = 1 << 20
    rng = np.random.default_rng(1)
    alphas = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2)
    xs = alphas + rng.integers(-(2**20), 2**20, n, dtype=np.int64).view(np.uint64)
    s = torch_cuda.from_numpy(rng.integers(0, 256, (2, n, 16), dtype=np.uint8).reshape(2, -1)).cuda()
    d0, d1 = ctx.myl7_gen_batch_device(GROUP_ADD, 64, to_dev(torch_cuda, alphas), (1).to_bytes(8, "little"),
                                       s[0].contiguous(), s[1].contiguous())
    dx = to_dev(torch_cuda, xs)
    kb = d0.numel() // n
    y0 = from_dev(ctx.myl7_eval(GROUP_ADD, 64, d0, kb, False, dx, 8), np.uint64)
    y1 = from_dev(ctx.myl7_eval(GROUP_ADD, 64, d1, kb, False, dx, 8), np.uint64)
    ctx.sync()
    assert ((y0 + y1) == (xs < alphas).astype(np.uint64)).all()


def test_device_keygen_rejects(ctx, torch_cuda):
    from suf_b200 import SufB200Error

    a = to_dev(torch_cuda, np.arange(4, dtype=np.uint64))
    s = torch_cuda.zeros(64, dtype=torch_cuda.uint8, device="cuda")
    with pytest.raises(SufB200Error):
        ctx.myl7_gen_batch_device(GROUP_ADD, 63, a, b"\x01", s, s)  # not a multiple of 8
    with pytest.raises(SufB200Error):
        ctx.myl7_gen_batch_device(GROUP_ADD, 64, a, bytes(17), s, s)  # two payload chunks
    with pytest.raises(SufB200Error):
        ctx.myl7_gen_batch_device(GROUP_ADD, 64, a, b"\x01", s[1:], s)  # misaligned seeds
