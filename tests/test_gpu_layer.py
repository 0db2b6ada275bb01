"""The device-resident 2PC transformer layer (suf_b200/layer.py) against its
plaintext model (oracle/layer_model.py), bit for bit: every step is exact in
Z_2^64, so the reconstruction y0 + y1 must equal the model's output word for
word (tolerance zero).  A small shape, the configs[4] shape, and two calls in
a row (the second on new inputs, same dealer material).  The model's own
accuracy against a float64 layer is checked in tests/test_layer_model.py."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.layer_model import Dims, layer
from tests.conftest import from_dev, to_dev

pytestmark = pytest.mark.gpu


def _shares(rng, X):
    s0 = rng.integers(0, 2**64, X.size, dtype=np.uint64)
    return s0, X.ravel() - s0


@pytest.mark.parametrize("dims", [Dims(S=32, D=128, H=2, Dff=256), Dims()], ids=["small", "configs4"])
def test_layer_matches_model(ctx, torch_cuda, dims):
    from suf_b200.layer import LayerDims, TransformerLayerPair, synthetic_layer

    ld = LayerDims(S=dims.S, D=dims.D, H=dims.H, Dff=dims.Dff, f=dims.f)
    X, W = synthetic_layer(ld, seed=5)
    lay = TransformerLayerPair(ctx, W, ld, seed=11)
    rng = np.random.default_rng(3)
    for call in range(2):
        if call == 1:
            X = np.rint(rng.normal(0.0, 1.0, X.shape) * 4096).astype(np.int64).view(np.uint64)
        x0, x1 = _shares(rng, X)
        y0, y1 = lay.run(to_dev(torch_cuda, x0), to_dev(torch_cuda, x1))
        ctx.sync()
        got = from_dev(y0) + from_dev(y1)
        want = layer(X, W, dims).ravel()
        bad = np.flatnonzero(got != want)
        assert bad.size == 0, f"call {call}: {bad.size} of {want.size} outputs differ (first at {bad[:5]})"
