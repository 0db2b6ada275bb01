"""configs[4] softmax block on the device (sufb200_softmax_block_pair,
suf_b200/softmax.py): the dealer's masked interval tables on the CPU, and on
the GPU the reconstruction of both parties' outputs against the plaintext
model pinned to the reference's SoftmaxBlockTask (oracle/softmax_model.py,
tests/test_softmax_model.py) -- bit for bit -- and against the reference's
own 64 x 64 reconstruction fixture."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle.softmax_model import softmax_block as model_block
from suf_b200.softmax import load_tables, masked_lut_table

GOLDEN = Path(__file__).parent / "golden"


def _lut_search(cuts: np.ndarray, x: np.ndarray) -> np.ndarray:
    """The interval-LUT kernel's rule: the last cut <= x among cuts[0..iv-1],
    clamped to interval 0."""
    iv = len(cuts) - 1
    return np.clip(np.searchsorted(cuts[:iv], x, side="right").astype(np.int64) - 1, 0, iv - 1)


@pytest.mark.parametrize("gate", ["nexp", "recip"])
def test_masked_table_returns_the_piece_of_x(gate):
    alpha, coeffs = load_tables()[gate]
    rng = np.random.default_rng(3)
    for r_in in [0, 1, 2**64 - 1, 2**63, *[int(v) for v in rng.integers(0, 2**64, 20, dtype=np.uint64)]]:
        cuts, rows = masked_lut_table(alpha, coeffs, r_in)
        assert cuts[0] == 0 and (np.diff(cuts[:-1].astype(object)) > 0).all()
        xs = np.concatenate([alpha[:-1], alpha[:-1] - np.uint64(1), rng.integers(0, 2**64, 2000, dtype=np.uint64),
                             np.array([0, 2**64 - 1], dtype=np.uint64)])
        with np.errstate(over="ignore"):
            xh = xs + np.uint64(r_in)
        got = rows[_lut_search(cuts, xh)]
        piece = np.clip(np.searchsorted(alpha[:-1], xs, side="right").astype(np.int64) - 1, 0, len(coeffs) - 1)
        assert (got == coeffs[piece]).all()


def _shares(rng, v: np.ndarray):
    s0 = rng.integers(0, 2**64, v.size, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return s0, v - s0


@pytest.mark.gpu
@pytest.mark.parametrize("heads,length", [(1, 64), (12, 128), (2, 200)])
def test_softmax_block_matches_model(ctx, torch_cuda, heads, length):
    from suf_b200.softmax import SoftmaxBlock
    from tests.conftest import from_dev, to_dev

    rng = np.random.default_rng(heads * 1000 + length)
    lens = np.arange(heads * length) % length + 1
    off = np.concatenate([[0], np.cumsum(lens)])
    t = rng.integers(0, 16 << 12, off[-1], dtype=np.uint64)
    t[rng.random(t.size) < 0.05] = 0
    t[rng.random(t.size) < 0.02] = 16 << 12
    blk = SoftmaxBlock(ctx, lens, seed=heads + length)
    t0, t1 = _shares(rng, t)
    p0, p1 = blk.run(to_dev(torch_cuda, t0), to_dev(torch_cuda, t1))
    ctx.sync()
    with np.errstate(over="ignore"):
        got = from_dev(p0, np.uint64) + from_dev(p1, np.uint64)
    want = model_block(t, off, load_tables())
    assert (got == want).all(), int((got != want).sum())


@pytest.mark.gpu
def test_softmax_block_matches_reference_fixture(ctx, torch_cuda):
    """The reference's own SoftmaxBlockTask reconstruction (64 x 64 causal,
    seed 4, its CPU backend) from the committed fixture."""
    from suf_b200.softmax import SoftmaxBlock
    from tests.conftest import from_dev, to_dev

    g = np.load(GOLDEN / "softmax_ref_h1_l64.npz")
    lens = np.arange(64) % 64 + 1
    t = np.concatenate([g["t"].reshape(64, 64)[r, :lens[r]] for r in range(64)])
    y = np.concatenate([g["y"].reshape(64, 64)[r, :lens[r]] for r in range(64)])
    blk = SoftmaxBlock(ctx, lens, seed=9)
    p0, p1 = blk.run(to_dev(torch_cuda, t), to_dev(torch_cuda, np.zeros_like(t)))
    ctx.sync()
    with np.errstate(over="ignore"):
        assert ((from_dev(p0, np.uint64) + from_dev(p1, np.uint64)) == y).all()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(128, 768), (7, 100), (64, 64)])
def test_layernorm_block_matches_model(ctx, torch_cuda, rows, cols):
    from oracle.softmax_model import layernorm_block
    from suf_b200.softmax import LayerNormBlock
    from tests.conftest import from_dev, to_dev

    rng = np.random.default_rng(rows * 7 + cols)
    x = np.round(rng.normal(0.0, 1.0, rows * cols) * 4096).astype(np.int64).view(np.uint64)
    blk = LayerNormBlock(ctx, rows, cols, seed=rows + cols)
    x0, x1 = _shares(rng, x)
    o0, o1 = blk.run(to_dev(torch_cuda, x0), to_dev(torch_cuda, x1))
    ctx.sync()
    with np.errstate(over="ignore"):
        got = from_dev(o0, np.uint64) + from_dev(o1, np.uint64)
    want = layernorm_block(x, rows, cols, load_tables())
    assert (got == want).all(), int((got != want).sum())
    # double-precision LayerNorm with the block's public 1/L = round(2^f / cols) / 2^f
    # (the reference's inv_len_qf), against which only rounding remains
    inv = round(4096 / cols) / 4096.0
    xr = x.view(np.int64).reshape(rows, cols) / 4096.0
    mu = xr.sum(1, keepdims=True) * inv
    ref = (xr - mu) / np.sqrt(((xr - mu) ** 2).sum(1, keepdims=True) * inv + 1 / 1024)
    assert np.abs(got.view(np.int64).reshape(rows, cols) / 4096.0 - ref).max() < 0.02


@pytest.mark.gpu
def test_layernorm_block_against_reference_protocol_rows(ctx, torch_cuda):
    """The device LayerNorm block directly against the reference's own
    runtime::LayerNormTask reconstruction (run as the protocol on its CPU
    backend, tests/golden/layernorm_ref_r32_c64.npz), on the rows where that
    protocol did not wrap (its RsqrtTask works on shares with share-local
    floors; wrapped rows come out at 2^50 scale): within 4 units on every such
    row and identical on most of them."""
    from pathlib import Path

    from suf_b200.softmax import LayerNormBlock
    from tests.conftest import from_dev, to_dev

    g = np.load(Path(__file__).parent / "golden" / "layernorm_ref_r32_c64.npz")
    x = g["x"].astype(np.uint64)
    ref = g["y"].reshape(32, 64).view(np.int64)
    blk = LayerNormBlock(ctx, 32, 64, seed=5)
    rng = np.random.default_rng(11)
    x0, x1 = _shares(rng, x)
    o0, o1 = blk.run(to_dev(torch_cuda, x0), to_dev(torch_cuda, x1))
    ctx.sync()
    with np.errstate(over="ignore"):
        got = (from_dev(o0, np.uint64) + from_dev(o1, np.uint64)).view(np.int64).reshape(32, 64)
    sane = (np.abs(ref) < (1 << 24)).all(axis=1)
    assert sane.sum() >= 12
    assert (np.abs(got[sane] - ref[sane]) <= 4).all()
    assert (got[sane] == ref[sane]).all(axis=1).sum() >= 0.7 * sane.sum()


@pytest.mark.gpu
@pytest.mark.parametrize("which,shape", [("softmax", (12, 128)), ("softmax", (2, 200)), ("layernorm", (128, 768)),
                                         ("layernorm", (7, 100))])
def test_block_tables_give_the_walks_shares(ctx, torch_cuda, which, shape):
    """prepare_tables(): the blocks' truncation bundles evaluated against
    their full-domain tables (sufb200_trunc_bundle_eval_pair_tables_dev)
    give each party the share words of the key walks, bundle by bundle."""
    from suf_b200.softmax import LayerNormBlock, SoftmaxBlock
    from tests.conftest import from_dev, to_dev

    rng = np.random.default_rng(sum(shape) + len(which))
    if which == "softmax":
        heads, length = shape
        lens = np.arange(heads * length) % length + 1
        blk = SoftmaxBlock(ctx, lens, seed=heads + length)
        v = rng.integers(0, 16 << 12, int(lens.sum()), dtype=np.uint64)
    else:
        blk = LayerNormBlock(ctx, *shape, seed=sum(shape))
        v = np.round(rng.normal(0.0, 1.0, shape[0] * shape[1]) * 4096).astype(np.int64).view(np.uint64)
    s0, s1 = (to_dev(torch_cuda, a) for a in _shares(rng, v))
    walk = [from_dev(o, np.uint64) for o in blk.run(s0, s1)]
    blk.prepare_tables()
    assert any(T.any() for T in blk._tables.values()), "no bundle qualified for tables"
    tab = [from_dev(o, np.uint64) for o in blk.run(s0, s1)]
    ctx.sync()
    for p in (0, 1):
        assert (tab[p] == walk[p]).all(), p


@pytest.mark.gpu
def test_block_tables_ready_event_orders_a_side_stream_fill(ctx, torch_cuda):
    """Tables filled on another stream with a `ready` event: the block call
    on the current stream, issued right after with no wait of its own,
    waits on the event before each such bundle and gives the walks' shares."""
    from suf_b200.softmax import LayerNormBlock
    from tests.conftest import from_dev, to_dev

    rng = np.random.default_rng(77)
    rows, cols = 128, 768
    blk = LayerNormBlock(ctx, rows, cols, seed=71)
    v = np.round(rng.normal(0.0, 1.0, rows * cols) * 4096).astype(np.int64).view(np.uint64)
    s0, s1 = (to_dev(torch_cuda, a) for a in _shares(rng, v))
    walk = [from_dev(o, np.uint64) for o in blk.run(s0, s1)]
    side = torch_cuda.cuda.Stream()
    for _ in range(2):  # a second fill rewrites the same tables
        ev = torch_cuda.cuda.Event()
        side.wait_stream(torch_cuda.cuda.current_stream())
        blk.prepare_tables(side, bundles=(2, 3, 4, 6, 7), ready=ev)
        tab = [from_dev(o, np.uint64) for o in blk.run(s0, s1)]
        for p in (0, 1):
            assert (tab[p] == walk[p]).all(), p
    ctx.sync()
