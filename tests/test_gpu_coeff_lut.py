"""GPU parity: the composite coefficient gate in one pass
(sufb200_coeff_lut_eval) -- interval-LUT coefficient words, the polynomial
over the public x^, the output-mask shares -- against the oracle's interval
LUT plus the plain Z_2^64 polynomial, per share, and against the reference's
own SiLU dealer and eval_suf_ref (tests/golden/silu_gate_f12_seed3.json)."""
from __future__ import annotations

import numpy as np
import pytest

from suf_b200.engine import coeff_lut_eval
from tests.conftest import from_dev, to_dev
from tests.helpers import silu_fixture

pytestmark = pytest.mark.gpu


def _poly(words: np.ndarray, xh: np.ndarray, r: int, degree: int, r_out: np.ndarray, ring: int) -> np.ndarray:
    """out[i, j] = sum_k words[i, j*(d+1)+k] * x^_i^k + r_out[j] mod 2^ring."""
    out = np.zeros((xh.size, r), dtype=np.uint64)
    with np.errstate(over="ignore"):
        for j in range(r):
            acc = np.zeros(xh.size, dtype=np.uint64)
            pw = np.ones(xh.size, dtype=np.uint64)
            for k in range(degree + 1):
                acc += words[:, j * (degree + 1) + k] * pw
                pw *= xh
            out[:, j] = acc + r_out[j]
    if ring < 64:
        out &= np.uint64((1 << ring) - 1)
    return out


def test_silu_gate_from_reference_dealer(ctx, torch_cuda, oracle):
    """configs[2]'s gate: both parties' keys and r_out shares from the
    reference's composite_gen_backend_with_masks; each share equals the
    interval-LUT fast path (LUT share + r_out share), and y0 + y1 - r_out is
    the reference's eval_suf_ref on every sample."""
    d = silu_fixture()
    xhat = d["x"] + np.uint64(d["r_in"])
    dx = to_dev(torch_cuda, xhat)
    ys = []
    for p in (0, 1):
        ro = d[f"r_out_share{p}"]
        y = from_dev(coeff_lut_eval(ctx, d["keys"][p], dx, 4, 0, r_out=ro)).reshape(-1, 4)
        ctx.sync()
        lut = oracle.interval_eval(d["keys"][p], d["keys"][p].size, True, xhat, 4)
        assert (y == lut + ro).all()
        ys.append(y)
    assert ((ys[0] + ys[1] - d["r_out"]) == d["expect"]).all()


@pytest.mark.parametrize("r,degree,ring", [(1, 3, 64), (2, 1, 64), (4, 0, 37), (3, 2, 50), (8, 0, 64)])
def test_coeff_lut_random_keys(ctx, torch_cuda, oracle, r, degree, ring):
    rng = np.random.default_rng(100 * r + degree)
    ow = r * (degree + 1)
    ivs = 19
    cuts = np.sort(rng.integers(0, 2**63, ivs - 1, dtype=np.uint64) * np.uint64(2))
    cuts = np.concatenate([[np.uint64(0)], cuts, [np.uint64(0)]]).astype(np.uint64)  # last: wrap sentinel
    pay = rng.integers(0, 2**63, ivs * ow, dtype=np.uint64) * np.uint64(2) + np.uint64(1)
    seed = oracle.seed_from_id(31 + r, 7)
    n = 20_000
    xh = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
    xh[:3] = [0, 2**64 - 1, int(cuts[5])]
    dx = to_dev(torch_cuda, xh)
    r_out = rng.integers(0, 2**63, (2, r), dtype=np.uint64)
    keys = [oracle.interval_key(p, 31 + r, 64, ow, cuts, pay, seed) for p in (0, 1)]
    ys = []
    for p in (0, 1):
        key = keys[p]
        y = from_dev(coeff_lut_eval(ctx, key, dx, r, degree, r_out=r_out[p], ring_bits=ring, idx_base=5)).reshape(n, r)
        ctx.sync()
        words = oracle.interval_eval(key, key.size, True, xh, ow, idx_base=5)
        assert (y == _poly(words, xh, r, degree, r_out[p], ring)).all()
        ys.append(y)
    # reconstruction: the payload row's polynomial at x^, plus the masks
    full = sum(oracle.interval_eval(k, k.size, True, xh, ow) for k in keys)
    want = _poly(full, xh, r, degree, r_out[0] + r_out[1], ring)
    mask = np.uint64((1 << ring) - 1) if ring < 64 else np.uint64(2**64 - 1)
    assert (((ys[0] + ys[1]) & mask) == want).all()


def test_coeff_lut_rejects_shape_mismatch(ctx, torch_cuda, oracle):
    from suf_b200 import SufB200Error

    d = silu_fixture()
    dx = to_dev(torch_cuda, np.arange(8, dtype=np.uint64))
    with pytest.raises(SufB200Error):
        coeff_lut_eval(ctx, d["keys"][0], dx, 2, 0)  # the key has 4 words per interval, not 2
    with pytest.raises(SufB200Error):
        coeff_lut_eval(ctx, d["keys"][0][:300], dx, 4, 0)  # shorter than its table


@pytest.mark.parametrize("r,degree,n,dealt", [(4, 0, 393_216, True), (1, 1, 20_001, True), (3, 2, 1, True),
                                              (8, 0, 77_777, True), (1, 0, 5_003, True), (3, 0, 40_003, True),
                                              (1, 2, 9_999, True), (4, 0, 70_001, False), (1, 1, 33, False)])
def test_coeff_lut_pair_equals_per_party(ctx, torch_cuda, oracle, r, degree, n, dealt):
    """sufb200_coeff_lut_eval_pair: both parties in one launch give each
    party's sufb200_coeff_lut_eval output word for word (item counts that
    split a warp chunk between the parties, a single element, several waves).
    A dealt pair (one seed and nonce) takes the launch's shared-keystream
    path; keys of two different seeds take the per-party path."""
    from suf_b200.engine import coeff_lut_eval_pair

    rng = np.random.default_rng(7 * r + n)
    ow = r * (degree + 1)
    ivs = 20
    cuts = np.sort(rng.integers(0, 2**63, ivs - 1, dtype=np.uint64) * np.uint64(2))
    cuts = np.concatenate([[np.uint64(0)], cuts, [np.uint64(0)]]).astype(np.uint64)
    pay = rng.integers(0, 2**63, ivs * ow, dtype=np.uint64) * np.uint64(2)
    seed = oracle.seed_from_id(55 + r, 7)
    seeds = (seed, seed if dealt else oracle.seed_from_id(56 + r, 7))
    keys = [oracle.interval_key(p, 55 + r, 64, ow, cuts, pay, seeds[p]) for p in (0, 1)]
    xh = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
    dx = to_dev(torch_cuda, xh)
    r_out = rng.integers(0, 2**63, (2, r), dtype=np.uint64)
    y0, y1 = coeff_lut_eval_pair(ctx, keys, dx, r, degree, r_outs=(r_out[0], r_out[1]), idx_base=3)
    ctx.sync()
    for p, y in ((0, y0), (1, y1)):
        want = coeff_lut_eval(ctx, keys[p], dx, r, degree, r_out=r_out[p], idx_base=3)
        ctx.sync()
        assert (from_dev(y)[:n * r] == from_dev(want)[:n * r]).all(), p
