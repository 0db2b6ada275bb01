"""The plaintext model of the configs[4] softmax block (oracle/softmax_model.py)
against the reference's own SoftmaxBlockTask reconstruction: the committed
64 x 64 causal fixture always, and the full 12 x 128 x 128 causal block when
oracle/_ref/ref_softmax_drive is built (it runs the reference CPU backend)."""
from __future__ import annotations

import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle.softmax_model import load_tables, softmax_block

GOLDEN = Path(__file__).parent / "golden"
DRIVE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "ref_softmax_drive"


def causal_pack(dense: np.ndarray, rows: int, length: int):
    lens = np.arange(rows) % length + 1
    d = dense.reshape(rows, length)
    packed = np.concatenate([d[r, :lens[r]] for r in range(rows)])
    return packed, np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)


def test_tables_are_the_reference_suf_programs():
    tb = load_tables()
    assert tb["frac_bits"] == 12
    alpha, coeffs = tb["nexp"]
    assert len(alpha) == len(coeffs) + 1 == 18 and alpha[16] == 16 << 12 and alpha[-1] == np.uint64(2**64 - 1)
    assert int(coeffs[0, 0]) == 1 << 12  # exp(0) = 1
    alpha, coeffs = tb["recip"]
    assert len(alpha) == len(coeffs) + 1 and (coeffs[:, 2:] == 0).all()  # affine init


def test_model_matches_reference_fixture():
    g = np.load(GOLDEN / "softmax_ref_h1_l64.npz")
    t, off = causal_pack(g["t"], 64, 64)
    y, _ = causal_pack(g["y"], 64, 64)
    assert (softmax_block(t, off, load_tables()) == y).all()


@pytest.mark.skipif(not DRIVE.exists(), reason="oracle/_ref/ref_softmax_drive not built (needs the reference checkout)")
def test_model_matches_reference_configs4(tmp_path):
    out = tmp_path / "d.bin"
    subprocess.run([str(DRIVE), "--reps=1", f"--dump={out}"], capture_output=True, text=True, timeout=600)
    raw = np.fromfile(out, dtype=np.uint64)
    n = raw.size // 2
    t, off = causal_pack(raw[:n], 1536, 128)
    y, _ = causal_pack(raw[n:], 1536, 128)
    assert len(t) == 99072
    assert (softmax_block(t, off, load_tables()) == y).all()


def test_layernorm_model_matches_reference_protocol_where_it_is_exact():
    """runtime::LayerNormTask run as the protocol (SUF_FORCE_PFSS=1) on the
    reference CPU backend, 32 x 64 (tests/golden/layernorm_ref_r32_c64.npz).
    Its RsqrtTask forms the initial guess from each party's coefficient share
    (a per-share floor) and halves x y^2 by shifting each share, so on
    additive shares some rows come out wrapped (2^50-scale values) and some
    off by a few units.  The model is the same fixed-point function with
    exact steps: it equals the reference on most rows that did not wrap and
    is within 4 units on all of them."""
    from oracle.softmax_model import layernorm_block

    g = np.load(GOLDEN / "layernorm_ref_r32_c64.npz")
    y = g["y"].reshape(32, 64).view(np.int64)
    m = layernorm_block(g["x"], 32, 64, load_tables()).reshape(32, 64).view(np.int64)
    sane = (np.abs(y) < (1 << 24)).all(axis=1)
    assert sane.sum() >= 12
    assert (np.abs(m[sane] - y[sane]) <= 4).all()
    assert (m[sane] == y[sane]).all(axis=1).sum() >= 0.7 * sane.sum()
