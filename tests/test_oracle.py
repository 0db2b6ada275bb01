"""The oracle against known answers, golden fixtures and the reference code."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle.oracle import GROUP_ADD, GROUP_XOR, KIND_ARS, KIND_GAPARS, KIND_TR, RefMyl7
from tests.helpers import oracle_trunc_eval, seeds_for, trunc_material

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_mt19937_64_known_answer(oracle):
    # C++ [rand.predef]: the 10000th output of a default-constructed mt19937_64.
    assert int(oracle.mt64(5489, 10000)[-1]) == 9981545732273789042


def test_aes_fips197_and_test_cuda_prg_vectors(oracle):
    g = json.loads((GOLDEN / "aes_ctr.json").read_text())
    c1 = g["fips197_c1"]
    ct = oracle.aes_ecb(bytes.fromhex(c1["key"]), np.frombuffer(bytes.fromhex(c1["pt"]), np.uint8))
    assert ct.tobytes().hex() == c1["ct"]
    key = bytes.fromhex(g["test_cuda_prg_key"])
    assert key == bytes(int(v) & 0xFF for v in oracle.mt64(12345, 16))
    for b in g["test_cuda_prg_blocks"]:
        pt = np.frombuffer(b["ctr"].to_bytes(8, "little") + bytes(8), np.uint8)
        assert oracle.aes_ecb(key, pt).tobytes().hex() == b["ct"]


def test_aes_against_openssl_random(oracle):
    from cryptography.hazmat.primitives.ciphers import Cipher, algorithms, modes

    rng = np.random.default_rng(7)
    for _ in range(8):
        key = rng.integers(0, 256, 16, dtype=np.uint8).tobytes()
        pts = rng.integers(0, 256, (32, 16), dtype=np.uint8)
        enc = Cipher(algorithms.AES(key), modes.ECB()).encryptor()
        assert oracle.aes_ecb(key, pts).tobytes() == enc.update(pts.tobytes())


@pytest.mark.parametrize("group,fname", [(GROUP_ADD, "myl7_add.npz"), (GROUP_XOR, "myl7_xor.npz")])
def test_myl7_oracle_matches_reference_golden(oracle, group, fname):
    g = np.load(GOLDEN / fname)
    oracle.prg_init(g["prg_state"])
    for ci in g["cases"]:
        in_bits, alpha, plen = (int(v) for v in g[f"c{ci}_meta"])
        payload = g[f"c{ci}_payload"].tobytes()
        k0, k1 = oracle.myl7_gen(group, in_bits, alpha, payload, g[f"c{ci}_seed0"], g[f"c{ci}_seed1"])
        assert (k0 == g[f"c{ci}_key0"]).all() and (k1 == g[f"c{ci}_key1"]).all()
        xs = g[f"c{ci}_xs"]
        for p, k in ((0, k0), (1, k1)):
            out = oracle.myl7_eval(group, k, k.size, True, xs, plen)
            assert (out == g[f"c{ci}_out{p}"]).all()


@pytest.mark.skipif(not RefMyl7.available(), reason="oracle/_ref not built (needs the reference checkout)")
@pytest.mark.parametrize("group", [GROUP_ADD, GROUP_XOR])
def test_myl7_oracle_matches_live_reference(oracle, prg_state, group):
    ref = RefMyl7(group)
    ref.prg_init(prg_state)
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(11 + group)
    for in_bits in (3, 8, 33, 64):
        alpha = int(rng.integers(0, 2**63)) & ((1 << in_bits) - 1)
        payload = rng.integers(0, 256, 8, dtype=np.uint8).tobytes()
        s0, s1 = rng.integers(0, 256, (2, 16), dtype=np.uint8)
        k0, k1 = oracle.myl7_gen(group, in_bits, alpha, payload, s0, s1)
        r0, r1 = ref.gen_seeded(in_bits, alpha, payload, s0, s1)
        assert (k0 == r0).all() and (k1 == r1).all()
        xs = rng.integers(0, 2**63, 64, dtype=np.uint64)
        for k in (k0, k1):
            assert (oracle.myl7_eval(group, k, k.size, True, xs, 8) == ref.adapter_eval(in_bits, k, k.size, True,
                                                                                         xs, 8)).all()
    # keys made by the reference adapter itself (std::random_device seeds)
    a0, a1 = ref.adapter_gen(64, 0x0123456789ABCDEF, (1).to_bytes(8, "little"))
    xs = rng.integers(0, 2**63, 64, dtype=np.uint64)
    for k in (a0, a1):
        assert (oracle.myl7_eval(group, k, k.size, True, xs, 8) == ref.adapter_eval(64, k, k.size, True, xs,
                                                                                     8)).all()


def test_myl7_reconstruction_property(oracle, prg_state):
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(3)
    s0, s1 = seeds_for(99, 1, oracle)
    for in_bits in (1, 2, 7, 64):
        alpha = int(rng.integers(0, 2**63)) & ((1 << in_bits) - 1)
        pay = 0x1122334455667788
        k0, k1 = oracle.myl7_gen(GROUP_ADD, in_bits, alpha, pay.to_bytes(8, "little"), s0[0], s1[0])
        xs = rng.integers(0, 2**63, 200, dtype=np.uint64)
        if in_bits <= 8:
            xs = np.arange(1 << in_bits, dtype=np.uint64)  # the whole domain
        o0 = oracle.myl7_eval(GROUP_ADD, k0, k0.size, True, xs, 8).view(np.uint64).ravel()
        o1 = oracle.myl7_eval(GROUP_ADD, k1, k1.size, True, xs, 8).view(np.uint64).ravel()
        lt = (xs & np.uint64((1 << in_bits) - 1)) < np.uint64(alpha)
        assert ((o0 + o1) == np.where(lt, np.uint64(pay), np.uint64(0))).all()


def test_reference_format_vectors(oracle):
    v = json.loads((GOLDEN / "ref_vectors.json").read_text())
    d = v["dcf_threshold"]
    k0 = oracle.thr_dcf_key(d["in_bits"], d["alpha"], bytes(d["payload"]))
    k1 = oracle.thr_dcf_key(d["in_bits"], d["alpha"], bytes(len(d["payload"])))
    xs = np.array(d["xs"], dtype=np.uint64)
    assert list(oracle.thr_dcf_eval(d["in_bits"], k0, k0.size, True, xs, 1).ravel()) == d["party0_expect"]
    assert not oracle.thr_dcf_eval(d["in_bits"], k1, k1.size, True, xs, 1).any()
    p = v["packed"]
    seed = oracle.seed_from_id(1, 0)
    keys = [oracle.packed_key(party, 1, p["in_bits"], p["thresholds"], seed) for party in (0, 1)]
    xs = np.array(p["xs"], dtype=np.uint64)
    o = [oracle.packed_eval(k, k.size, True, xs, 1) for k in keys]
    assert list((o[0] ^ o[1]).ravel()) == p["expect"]
    for name in ("interval", "interval_small"):
        iv = v[name]
        seed = oracle.seed_from_id(2, 7)
        keys = [oracle.interval_key(party, 2, iv["in_bits"], iv["out_words"], iv["cutpoints"], iv["payload"], seed)
                for party in (0, 1)]
        xs = np.array(iv["xs"], dtype=np.uint64)
        o = [oracle.interval_eval(k, k.size, True, xs, iv["out_words"]) for k in keys]
        rec = (o[0] + o[1]).reshape(len(xs), iv["out_words"])
        exp = np.array(iv["expect"], dtype=np.uint64).reshape(len(xs), iv["out_words"])
        assert (rec == exp).all()


@pytest.mark.parametrize("kind", [KIND_TR, KIND_ARS, KIND_GAPARS])
def test_trunc_oracle_reference_vectors(oracle, prg_state, kind):
    oracle.prg_init(prg_state)
    v = json.loads((Path(__file__).parent / "golden" / "ref_vectors.json").read_text())["trunc"]
    plain = np.array(v["plain"], dtype=np.int64)
    f = v["frac_bits"]
    for seed in v["seeds"]:
        r_in, (d0, d1), (k0, k1) = trunc_material(oracle, kind, f, seed)
        xhat = plain.view(np.uint64) + np.uint64(r_in)
        y = oracle_trunc_eval(oracle, d0, k0, xhat) + oracle_trunc_eval(oracle, d1, k1, xhat)
        if kind == KIND_TR:
            exp = plain.view(np.uint64) >> np.uint64(f)
        else:
            exp = (plain >> f).view(np.uint64)
        assert (y == exp).all(), (kind, seed, y, exp)


@pytest.mark.parametrize("kind", [KIND_TR, KIND_ARS, KIND_GAPARS])
def test_trunc_oracle_random_and_edges(oracle, prg_state, kind):
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(100 + kind)
    f = 16
    x = rng.integers(-(2**40) + 1, 2**40, 300, dtype=np.int64)
    x[:6] = [0, 1, -1, 2**40 - 1, -(2**40) + 1, 1 << f]
    for seed in (2, 3):
        r_in, (d0, d1), (k0, k1) = trunc_material(oracle, kind, f, seed)
        xhat = x.view(np.uint64) + np.uint64(r_in)
        y = oracle_trunc_eval(oracle, d0, k0, xhat) + oracle_trunc_eval(oracle, d1, k1, xhat)
        exp = (x.view(np.uint64) >> np.uint64(f)) if kind == KIND_TR else (x >> f).view(np.uint64)
        assert (y == exp).all()


# ---- configs[2] SiLU gate fixture (the reference's own dealer) ----

def test_silu_fixture_table_and_lut_semantics(oracle):
    """The fixture's SUF table restated (select_interval + degree-0 piece)
    reproduces the reference's eval_suf_ref on every sample; the compiled
    interval LUT, evaluated by the oracle at x^ = x + r_in, reconstructs the
    same coefficient words; the r_out shares add up to r_out."""
    from tests.helpers import silu_fixture, suf_table_eval

    d = silu_fixture()
    assert (d["degree"], d["r"], d["out_words"]) == (0, 4, 4)
    assert (suf_table_eval(d["alpha"], d["pieces"], d["x"]) == d["expect"]).all()
    assert ((d["r_out_share0"] + d["r_out_share1"]) == d["r_out"]).all()
    xhat = d["x"] + np.uint64(d["r_in"])
    s = [oracle.interval_eval(k, k.size, True, xhat, 4) for k in d["keys"]]
    assert ((s[0] + s[1]) == d["expect"]).all()
