"""GPU parity: the reference GPU backend's own key formats (threshold DCF,
packed compare, interval LUT) against the oracle's restatement of the
reference kernels' counter layout, and the reference tests' fixed vectors."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from tests.conftest import from_dev, rand_u64, to_dev

pytestmark = pytest.mark.gpu
VEC = json.loads((Path(__file__).parent / "golden" / "ref_vectors.json").read_text())


def test_threshold_dcf(ctx, torch_cuda, oracle):
    from suf_b200 import engine as E

    d = VEC["dcf_threshold"]
    k0 = E.thr_dcf_key(d["in_bits"], d["alpha"], bytes(d["payload"]))
    xs = np.array(d["xs"], dtype=np.uint64)
    out = ctx.thr_dcf_eval(d["in_bits"], to_dev(torch_cuda, k0), k0.size, True, to_dev(torch_cuda, xs), 1)
    ctx.sync()
    assert list(from_dev(out, np.uint8)[: len(xs)]) == d["party0_expect"]
    rng = np.random.default_rng(4)
    n = 4096
    for in_bits, ob in ((64, 8), (37, 8), (6, 1), (64, 3)):
        alphas = rand_u64(rng, n)
        keys = np.stack([oracle.thr_dcf_key(in_bits, int(a), rng.integers(0, 256, ob, np.uint8).tobytes())
                         for a in alphas])
        xs = rand_u64(rng, n)
        out = ctx.thr_dcf_eval(in_bits, to_dev(torch_cuda, keys.ravel()), keys.shape[1], False,
                               to_dev(torch_cuda, xs), ob)
        ctx.sync()
        exp = oracle.thr_dcf_eval(in_bits, keys, keys.shape[1], False, xs, ob)
        assert (from_dev(out, np.uint8)[: n * ob].reshape(n, ob) == exp).all()


@pytest.mark.parametrize("broadcast", [True, False])
def test_packed_compare(ctx, torch_cuda, oracle, broadcast):
    p = VEC["packed"]
    seed = oracle.seed_from_id(1, 0)
    keys = [oracle.packed_key(party, 1, p["in_bits"], p["thresholds"], seed) for party in (0, 1)]
    xs = np.array(p["xs"], dtype=np.uint64)
    outs = []
    for k in keys:
        kk = k if broadcast else np.tile(k, len(xs))
        o = ctx.packed_lt_eval(to_dev(torch_cuda, kk), k.size, broadcast, to_dev(torch_cuda, xs), p["in_bits"], 1)
        ctx.sync()
        outs.append(from_dev(o))
        assert (outs[-1] == oracle.packed_eval(kk, k.size, broadcast, xs, 1).ravel()).all()
    assert list(outs[0] ^ outs[1]) == p["expect"]
    # larger: sorted and unsorted thresholds, multi-word masks, non-zero idx_base
    rng = np.random.default_rng(8)
    for num_thr, sort, in_bits in ((130, True, 64), (70, False, 64), (5, True, 20), (200, False, 33)):
        thr = rand_u64(rng, num_thr)
        if sort:
            thr = np.sort(thr & np.uint64((1 << in_bits) - 1 if in_bits < 64 else 2**64 - 1))
        seed = oracle.seed_from_id(num_thr, 0)
        words = (num_thr + 63) // 64
        n = 3000
        xs = rand_u64(rng, n)
        for party in (0, 1):
            k = oracle.packed_key(party, 99, in_bits, thr, seed)
            o = ctx.packed_lt_eval(to_dev(torch_cuda, k), k.size, True, to_dev(torch_cuda, xs), in_bits, words,
                                   idx_base=12345)
            ctx.sync()
            exp = oracle.packed_eval(k, k.size, True, xs, words, idx_base=12345)
            assert (from_dev(o).reshape(n, words) == exp).all()


@pytest.mark.parametrize("broadcast", [True, False])
def test_interval_lut(ctx, torch_cuda, oracle, broadcast):
    for name in ("interval", "interval_small"):
        iv = VEC[name]
        seed = oracle.seed_from_id(2, 7)
        xs = np.array(iv["xs"], dtype=np.uint64)
        outs = []
        for party in (0, 1):
            k = oracle.interval_key(party, 2, iv["in_bits"], iv["out_words"], iv["cutpoints"], iv["payload"], seed)
            kk = k if broadcast else np.tile(k, len(xs))
            o = ctx.interval_lut_eval(to_dev(torch_cuda, kk), k.size, broadcast, to_dev(torch_cuda, xs),
                                      iv["out_words"])
            ctx.sync()
            outs.append(from_dev(o))
            assert (outs[-1] == oracle.interval_eval(kk, k.size, broadcast, xs, iv["out_words"]).ravel()).all()
        rec = (outs[0] + outs[1]).reshape(len(xs), iv["out_words"])
        assert (rec == np.array(iv["expect"], dtype=np.uint64).reshape(rec.shape)).all()
    # SiLU-shaped table: 19 cutpoints in the masked domain, 4 coefficient words
    rng = np.random.default_rng(3)
    cuts = np.sort(rand_u64(rng, 18))
    cuts = np.concatenate([np.zeros(1, np.uint64), cuts])
    pay = rand_u64(rng, (cuts.size - 1) * 4)
    seed = oracle.seed_from_id(3, 7)
    n = 5000
    xs = rand_u64(rng, n)
    for party in (0, 1):
        k = oracle.interval_key(party, 3, 64, 4, cuts, pay, seed)
        o = ctx.interval_lut_eval(to_dev(torch_cuda, k), k.size, True, to_dev(torch_cuda, xs), 4, idx_base=77)
        ctx.sync()
        assert (from_dev(o).reshape(n, 4) == oracle.interval_eval(k, k.size, True, xs, 4, idx_base=77)).all()
