"""The plaintext model of the device transformer layer (oracle/layer_model.py):
its ReLU tournament is the row maximum, its gate tables are the reference's,
and the whole layer stays within a fixed-point error of the float64 layer
on the configs[4] synthetic inputs (the GPU test pins the device layer to this
model bit for bit)."""
from __future__ import annotations

import numpy as np

from oracle.layer_model import Dims, layer, layer_float, load_layer_tables, piecewise, rowmax


def test_rowmax_tournament_is_the_row_max():
    rng = np.random.default_rng(1)
    s = rng.integers(-(2**40), 2**40, (64, 128)).astype(np.int64).view(np.uint64)
    m = rowmax(s, load_layer_tables()["relu"])
    assert (m.view(np.int64) == s.view(np.int64).max(axis=1)).all()


def test_gate_tables():
    t = load_layer_tables()
    x = np.array([0, 5, 2**63 - 1, 2**63, 2**64 - 1], dtype=np.uint64)
    assert (piecewise(t["relu"], x) == np.array([0, 5, 2**63 - 1, 0, 0], dtype=np.uint64)).all()
    # the constant GeLU at f = 12: about x for large x, about 0 for negative x
    g = piecewise(t["gelu_const"], np.array([3 * 4096, (-3 * 4096) & (2**64 - 1)], dtype=np.uint64)).view(np.int64)
    assert abs(g[0] - 3 * 4096) < 128 and abs(g[1]) < 128  # the 256-segment table is coarse in the tails


def test_layer_model_close_to_float():
    from suf_b200.layer import LayerDims, synthetic_layer

    d = Dims(S=32, D=128, H=2, Dff=256)
    X, W = synthetic_layer(LayerDims(S=32, D=128, H=2, Dff=256), seed=5)
    y = layer(X, W, d).view(np.int64) / 4096.0
    yf = layer_float(X, W, d)
    assert np.abs(y - yf).max() < 0.15
    assert np.abs(y - yf).mean() < 0.03
