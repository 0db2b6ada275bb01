"""Test helpers: seeded dealer material built with the ORACLE (the checker).

Inputs follow the bench workloads' shapes and seeds (synthetic stand-ins for
the reference's configs): x is fixed-point with `frac` fractional bits and
|x| < 2^bound, masked as x^ = x + r_in mod 2^64.
"""
from __future__ import annotations

import numpy as np

from oracle.oracle import GROUP_ADD, Oracle, TruncDesc as OrcDesc

ONE_LE = (1).to_bytes(8, "little")


def signed_fixed(rng: np.random.Generator, n: int, bound_bits: int) -> np.ndarray:
    """Uniform integers in (-2^bound, 2^bound) as uint64 two's complement."""
    v = rng.integers(-(2**bound_bits) + 1, 2**bound_bits, n, dtype=np.int64)
    return v.view(np.uint64)


def seeds_for(seed: int, count: int, oracle: Oracle) -> tuple[np.ndarray, np.ndarray]:
    """Deterministic party seeds: mt19937_64(seed) stream, 16 bytes each."""
    words = oracle.mt64(seed, 4 * count)
    s = words.view(np.uint8).reshape(count, 2, 16)
    return np.ascontiguousarray(s[:, 0, :]), np.ascontiguousarray(s[:, 1, :])


def trunc_material(oracle: Oracle, kind: int, f: int, seed: int):
    """Dealer material for one bundle: oracle descriptors and myl7 keys."""
    r_in, d0, d1 = oracle.trunc_gen(kind, f, seed)
    s0, s1 = seeds_for(seed ^ 0x6D796C37, max(d0.nq, 1), oracle)
    keys0, keys1 = [], []
    for q in range(d0.nq):
        k0, k1 = oracle.myl7_gen(GROUP_ADD, d0.q_bits[q], int(d0.q_theta[q]), ONE_LE, s0[q], s1[q])
        keys0.append(k0)
        keys1.append(k1)
    return r_in, (d0, d1), (keys0, keys1)


def oracle_trunc_eval(oracle: Oracle, desc: OrcDesc, keys: list[np.ndarray], xhat: np.ndarray, want_bools=False):
    """Per-query DCF shares with the oracle, then the oracle's plan + postproc."""
    n = xhat.size
    pred = np.zeros((max(desc.nq, 1), n), dtype=np.uint64)
    for q in range(desc.nq):
        out = oracle.myl7_eval(GROUP_ADD, keys[q], keys[q].size, True, xhat, 8)
        pred[q] = out.view(np.uint64).ravel()
    return oracle.trunc_combine(desc, xhat, pred.ravel(), want_bools=want_bools)


def to_product_desc(d: OrcDesc):
    """Oracle descriptor -> suf_b200.TruncDesc (same fields, no thresholds)."""
    from suf_b200 import TruncDesc

    p = TruncDesc()
    for name in ("kind", "frac_bits", "party", "nq", "carry_a", "carry_b", "sign_a", "sign_b", "wrap_q",
                 "carry_w", "sign_w", "haty", "r_hi", "m"):
        setattr(p, name, getattr(d, name))
    for i in range(4):
        p.q_bits[i] = d.q_bits[i]
    return p


# ---- the SiLU gate fixture (tests/golden/make_silu_fixture.py) ----

def silu_fixture() -> dict:
    import json
    from pathlib import Path

    d = json.loads((Path(__file__).parent / "golden" / "silu_gate_f12_seed3.json").read_text())
    u = lambda v: np.array([int(t) for t in v], dtype=np.uint64)  # noqa: E731
    d["r_in"] = int(d["r_in"])
    for k in ("r_out", "r_out_share0", "r_out_share1", "alpha"):
        d[k] = u(d[k])
    d["pieces"] = np.array([[int(t) for t in p] for p in d["pieces"]], dtype=np.uint64)
    d["keys"] = [np.frombuffer(bytes.fromhex(d["key0"]), dtype=np.uint8).copy(),
                 np.frombuffer(bytes.fromhex(d["key1"]), dtype=np.uint8).copy()]
    d["x"] = u([s["x"] for s in d["samples"]])
    d["expect"] = np.array([[int(t) for t in s["expect"]] for s in d["samples"]], dtype=np.uint64)
    return d


def suf_table_eval(alpha: np.ndarray, pieces: np.ndarray, x: np.ndarray) -> np.ndarray:
    """suf::eval_suf_ref (include/suf/ref_eval.hpp:47-77) for degree-0 pieces:
    the piece whose [alpha_i, alpha_i+1) holds x, else the last piece."""
    idx = np.searchsorted(alpha, x, side="right").astype(np.int64) - 1
    idx[(idx < 0) | (idx > alpha.size - 2)] = alpha.size - 2
    return pieces[idx]
