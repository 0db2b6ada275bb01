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


def test_layer_graph_replay_matches_eager(ctx, torch_cuda):
    """TransformerLayerPair.capture: a CUDA graph of three chained layers
    replays to the same output shares as the eager calls, word for word, and
    picks up new inputs written into its input buffers between replays."""
    from suf_b200.layer import LayerDims, TransformerLayerPair, synthetic_layer

    torch = torch_cuda
    ld = LayerDims(S=32, D=128, H=2, Dff=256)
    X, W = synthetic_layer(ld, seed=5)
    lay = TransformerLayerPair(ctx, W, ld, seed=11)
    rng = np.random.default_rng(4)
    x0, x1 = _shares(rng, X)
    dx = [to_dev(torch, x0), to_dev(torch, x1)]
    dy = [torch.empty_like(dx[0]), torch.empty_like(dx[1])]
    g = lay.capture(dx[0], dx[1], dy[0], dy[1], layers=3)
    for rep in range(2):
        if rep == 1:  # new inputs, same buffers
            X = np.rint(rng.normal(0.0, 1.0, X.shape) * 4096).astype(np.int64).view(np.uint64)
            x0, x1 = _shares(rng, X)
            dx[0].copy_(to_dev(torch, x0))
            dx[1].copy_(to_dev(torch, x1))
        g.replay()
        torch.cuda.synchronize()
        ctx.sync()
        a, b = to_dev(torch, x0), to_dev(torch, x1)
        for _ in range(3):
            a, b = lay.run(a, b)
        ctx.sync()
        assert (from_dev(dy[0]) == from_dev(a)).all() and (from_dev(dy[1]) == from_dev(b)).all(), rep
