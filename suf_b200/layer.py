"""A 2PC transformer encoder layer (d_model 768, 12
heads, d_ff 3072, sequence 128, f = 12, 64-bit ring) resident on one GPU for
both parties: the dealer that makes its correlated randomness and the layer
call.  No host round trip happens inside the layer.

Structure (pre-LN, the order of nn::transformer_layer_forward,
src/nn/transformer_layer.cpp: LayerNorm, attention, residual, LayerNorm, MLP,
residual):
  H1 = LN(X)                      LayerNormBlock (runtime::LayerNormTask with RsqrtTask)
  QKV = T_f(H1 Wqkv)              public-weight matmul on the tensor cores
                                  (matmul_publicW_gpu) + GapARS truncation
  S_h = T_{f+3}(Q_h K_h^T)        Beaver matmul per head (nn::matmul_beaver),
                                  1/sqrt(64) folded into the truncation
  t = rowmax(S) - S               ReLU tournament of nn::RowMaxDiffTask
  P = softmax(t)                  SoftmaxBlock (nn::SoftmaxBlockTask), non-causal rows
  O_h = T_f(P_h V_h);  X2 = X + T_f(O Wo)
  H2 = LN(X2);  F1 = T_f(H2 W1)
  G = GeLU_const(F1)              the reference bench's GPU GeLU: 256-segment
                                  degree-0 SUF (SUF_GELU_CONST, src/nn/mlp_block.cpp:531-580)
  Y = X2 + T_f(G W2)
Every truncation is a GapARS bundle; the ReLU and GeLU gates are coefficient
gates over the opened x^ (composite_eval_batch_backend's interval-LUT path
with the polynomial shifted to the x^ domain).  The gate tables are the
reference's own (suf_b200/tables/{softmax,layer}_suf_f12.json).  Every step
is exact in Z_2^64, so the reconstruction does not depend on the dealer's
draws.
"""
from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _lib
from ._lib import TruncDesc, check
from .engine import Context, TruncTables, _stream_ptr, _t_ptr, interval_lut_key, seed_from_id
from .softmax import TRUNC_GAPARS, LayerNormBlock, SoftmaxBlock, load_tables, masked_lut_table

LAYER_TABLES = Path(__file__).resolve().parent / "tables" / "layer_suf_f12.json"
M64 = (1 << 64) - 1
GROUP_ADD = 0


@dataclass
class LayerDims:
    S: int = 128
    D: int = 768
    H: int = 12
    Dff: int = 3072
    f: int = 12

    @property
    def Dh(self) -> int:
        return self.D // self.H


def synthetic_layer(dims: LayerDims, seed: int = 5):
    """configs[4]'s synthetic layer: weights Gaussian sigma 0.02, inputs
    Gaussian sigma 1, quantised at f (numpy default_rng(seed)).  Returns
    (X [S, D] u64, {'qkv', 'o', 'ff1', 'ff2'} int64)."""
    rng = np.random.default_rng(seed)
    sc = float(1 << dims.f)
    W = {n: np.rint(rng.normal(0.0, 0.02, shp) * sc).astype(np.int64)
         for n, shp in (("qkv", (dims.D, 3 * dims.D)), ("o", (dims.D, dims.D)), ("ff1", (dims.D, dims.Dff)),
                        ("ff2", (dims.Dff, dims.D)))}
    X = np.rint(rng.normal(0.0, 1.0, (dims.S, dims.D)) * sc).astype(np.int64).view(np.uint64)
    return X, W


def load_layer_tables(path: Path = LAYER_TABLES) -> dict:
    d = json.loads(Path(path).read_text())
    out = {}
    for g in ("relu", "gelu_const"):
        deg = int(d[g]["degree"])
        alpha = np.array([int(v) for v in d[g]["alpha"]], dtype=np.uint64)
        coeffs = np.zeros((len(d[g]["pieces"]), deg + 1), dtype=np.uint64)
        for i, piece in enumerate(d[g]["pieces"]):
            for k, c in enumerate(piece[0]):
                coeffs[i, k] = np.uint64(int(c))
        out[g] = (alpha, coeffs, deg)
    return out


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def _rand64(rng) -> int:
    return int(rng.integers(0, 2**64, dtype=np.uint64))


class _Trunc:
    """One GapARS truncation bundle for both parties: descriptors, myl7 keys
    (on the device) and the split of its input mask r_in = r[0] + r[1]."""

    def __init__(self, ctx: Context, rng, frac_bits: int, dev=None):
        import torch

        r_in, d0, d1, thetas = Context.trunc_gen(TRUNC_GAPARS, frac_bits, int(rng.integers(1, 2**63)))
        r0 = _rand64(rng)
        self.r = (r0, (r_in - r0) & M64)
        self.desc = (d0, d1)
        self.keys = ([], [])  # device copies: the bundle's keys stay resident
        for q in range(int(d0.nq)):
            s0 = rng.integers(0, 256, 16, dtype=np.uint8)
            s1 = rng.integers(0, 256, 16, dtype=np.uint8)
            k0, k1 = ctx.myl7_gen(GROUP_ADD, int(d0.q_bits[q]), int(thetas[q]), (1).to_bytes(8, "little"), s0, s1)
            self.keys[0].append(torch.from_numpy(k0).to(dev))
            self.keys[1].append(torch.from_numpy(k1).to(dev))
        nq = int(d0.nq)
        self.kptr = [(C.c_void_p * 4)(*[k.data_ptr() for k in ks], *([None] * (4 - nq))) for ks in self.keys]
        self.ksz = [(C.c_size_t * 4)(*[k.numel() for k in ks], *([0] * (4 - nq))) for ks in self.keys]
        # (TruncTables, party 0's index, party 1's) when the layer keeps this
        # bundle's full-domain tables; `ready` is the event after their fill
        self.tables = None
        self.ready = None

    def bundles(self):
        return [(self.desc[p], self.kptr[p], self.ksz[p]) for p in (0, 1)]

    def eval_pair(self, ctx: Context, d_xhat, d_y0, d_y1, stream):
        if self.tables is not None and self.ready is not None:
            import torch

            T, i0, i1 = self.tables
            (stream if stream is not None else torch.cuda.current_stream()).wait_event(self.ready)
            check(_lib.lib().sufb200_trunc_bundle_eval_pair_tables_dev(
                ctx.h, C.byref(self.desc[0]), C.cast(self.kptr[0], C.c_void_p), C.cast(self.ksz[0], C.c_void_p),
                T.ptr(i0), C.byref(self.desc[1]), C.cast(self.kptr[1], C.c_void_p),
                C.cast(self.ksz[1], C.c_void_p), T.ptr(i1), _t_ptr(d_xhat), d_xhat.numel(),
                _t_ptr(d_y0), _t_ptr(d_y1), _stream_ptr(stream)))
            self.ready = None
            return
        check(_lib.lib().sufb200_trunc_bundle_eval_pair_dev(
            ctx.h, C.byref(self.desc[0]), C.cast(self.kptr[0], C.c_void_p), C.cast(self.ksz[0], C.c_void_p),
            C.byref(self.desc[1]), C.cast(self.kptr[1], C.c_void_p), C.cast(self.ksz[1], C.c_void_p), _t_ptr(d_xhat),
            d_xhat.numel(), _t_ptr(d_y0), _t_ptr(d_y1), _stream_ptr(stream)))


class _CoeffGate:
    """A coefficient gate (one output word, polynomial of degree <= 1 per
    piece) for both parties: the table moved to the x^ domain (cut list
    shifted by r_in, the wrapped piece split at 0, each piece's polynomial
    a0 + a1 x rewritten as (a0 - a1 r_in) + a1 x^), one interval-LUT key per
    party, the split of r_in and zero-sum output-mask shares."""

    def __init__(self, rng, table):
        alpha, coeffs, deg = table
        if deg > 1:
            raise ValueError("coefficient gates of degree <= 1 only")
        self.degree = deg
        r_in = _rand64(rng)
        rows = coeffs.copy()
        if deg == 1:
            with np.errstate(over="ignore"):
                rows[:, 0] = coeffs[:, 0] - coeffs[:, 1] * np.uint64(r_in)
        cuts, payload = masked_lut_table(alpha, rows, r_in)
        nonce = int(rng.integers(1, 2**62))
        sd = seed_from_id(nonce, 7)
        self.keys = [interval_lut_key(p, nonce, 64, deg + 1, cuts, payload.reshape(-1), sd) for p in (0, 1)]
        r0 = _rand64(rng)
        self.r = (r0, (r_in - r0) & M64)
        s = _rand64(rng)
        self.r_out = (np.array([s], dtype=np.uint64), np.array([(-s) & M64], dtype=np.uint64))

    def eval(self, ctx: Context, p: int, d_xhat, d_out, stream):
        key = self.keys[p]
        ro = self.r_out[p]
        check(ctx._L.sufb200_coeff_lut_eval(ctx.h, key.ctypes.data, key.size, _t_ptr(d_xhat), d_xhat.numel(), 1,
                                            self.degree, ro.ctypes.data, 64, C.c_uint64(0), _t_ptr(d_out),
                                            _stream_ptr(stream)))

    def eval_pair(self, ctx: Context, d_xhat, d_out0, d_out1, stream):
        """Both parties in one launch (sufb200_coeff_lut_eval_pair)."""
        k0, k1 = self.keys
        check(ctx._L.sufb200_coeff_lut_eval_pair(ctx.h, k0.ctypes.data, k0.size, k1.ctypes.data, k1.size,
                                                 _t_ptr(d_xhat), d_xhat.numel(), 1, self.degree,
                                                 self.r_out[0].ctypes.data, self.r_out[1].ctypes.data, 64,
                                                 C.c_uint64(0), _t_ptr(d_out0), _t_ptr(d_out1), _stream_ptr(stream)))


class _Triples:
    """Beaver matmul triples, one per head: A [H][M][K], B [H][K][N] (or
    [H][N][K] when transposed), C = A B, additively shared."""

    def __init__(self, rng, dev, H: int, M: int, K: int, N: int, transposed: bool):
        import torch

        A = rng.integers(0, 2**64, (H, M, K), dtype=np.uint64, endpoint=False)
        B = rng.integers(0, 2**64, (H, N, K) if transposed else (H, K, N), dtype=np.uint64)
        with np.errstate(over="ignore"):
            Cm = np.matmul(A, B.transpose(0, 2, 1) if transposed else B)
        self.parts = []
        for v in (A, B, Cm):
            s0 = rng.integers(0, 2**64, v.shape, dtype=np.uint64)
            with np.errstate(over="ignore"):
                s1 = v - s0
            self.parts.append(tuple(torch.from_numpy(np.ascontiguousarray(s).view(np.int64).ravel()).to(dev)
                                    for s in (s0, s1)))

    def ptrs(self, which: int):
        return (C.c_void_p * 2)(*[t.data_ptr() for t in self.parts[which]])


class TransformerLayerPair:
    """Dealer material for one layer (both parties, resident on the
    context's device) and the layer call.  W: {'qkv' [D, 3D], 'o' [D, D],
    'ff1' [D, Dff], 'ff2' [Dff, D]} public int64 weights (Q f)."""

    def __init__(self, ctx: Context, W: dict, dims: LayerDims | None = None, seed: int = 1):
        import torch

        self.ctx = ctx
        d = self.dims = dims or LayerDims()
        S, D, H, Dh, Dff, f = d.S, d.D, d.H, d.Dh, d.Dff, d.f
        if S & (S - 1):
            raise ValueError("the row-max tournament needs a power-of-two sequence length")
        dev = self.dev = torch.device("cuda", ctx.device)
        sm_tab = load_tables()
        if int(sm_tab["frac_bits"]) != f:
            raise ValueError("the gate tables are for f = %d" % sm_tab["frac_bits"])
        tabs = load_layer_tables()
        rng = np.random.default_rng(seed)
        self.W = {n: torch.from_numpy(np.ascontiguousarray(W[n], dtype=np.int64).ravel()).to(dev)
                  for n in ("qkv", "o", "ff1", "ff2")}
        self.ln1 = LayerNormBlock(ctx, S, D, seed=int(rng.integers(1, 2**62)), tables=sm_tab)
        self.ln2 = LayerNormBlock(ctx, S, D, seed=int(rng.integers(1, 2**62)), tables=sm_tab)
        self.softmax = SoftmaxBlock(ctx, [S] * (H * S), seed=int(rng.integers(1, 2**62)), tables=sm_tab)
        self.tr = {name: _Trunc(ctx, rng, fk, dev)
                   for name, fk in (("qkv", f), ("scores", f + 3), ("pv", f), ("o", f), ("ff1", f), ("ff2", f))}
        # the truncations' full-domain tables, in the three groups the layer
        # fills them in (one launch per group)
        self._tab_groups = []
        for names in (("qkv", "scores"), ("pv", "o"), ("ff1", "ff2")):
            T = TruncTables([b for nm in names for b in self.tr[nm].bundles()], dev)
            for j, nm in enumerate(names):
                if T.ptr(2 * j) and T.ptr(2 * j + 1):
                    self.tr[nm].tables = (T, 2 * j, 2 * j + 1)
            self._tab_groups.append((names, T))
        self.trip_s = _Triples(rng, dev, H, S, Dh, S, transposed=True)
        self.trip_pv = _Triples(rng, dev, H, S, S, Dh, transposed=False)
        self.rounds = S.bit_length() - 1
        self.relu = [_CoeffGate(rng, tabs["relu"]) for _ in range(self.rounds)]
        self.gelu = _CoeffGate(rng, tabs["gelu_const"])

        def buf(n):
            return torch.empty(n, dtype=torch.int64, device=dev)

        self._side = self._fork = self._join = None  # party 1's stream (created on first use)
        self._tab_stream = self._tab_fork = self._tab_ev = None  # the truncation tables' stream
        wide = max(S * 3 * D, S * Dff)  # the widest public-weight product
        self.b = {
            "h": (buf(S * D), buf(S * D)), "acc": (buf(wide), buf(wide)), "xhat": buf(max(wide, H * S * S)),
            "qkv": (buf(S * 3 * D), buf(S * 3 * D)), "s": (buf(H * S * S), buf(H * S * S)),
            "c": (buf(H * S * S // 2), buf(H * S * S // 2)), "c2": (buf(H * S * S // 4), buf(H * S * S // 4)),
            "relu": (buf(H * S * S // 2), buf(H * S * S // 2)), "t": (buf(H * S * S), buf(H * S * S)),
            "p": (buf(H * S * S), buf(H * S * S)), "o": (buf(S * D), buf(S * D)), "a": (buf(S * D), buf(S * D)),
            "x2": (buf(S * D), buf(S * D)), "f1": (buf(S * Dff), buf(S * Dff)), "g": (buf(S * Dff), buf(S * Dff)),
        }

    # -- steps ---------------------------------------------------------------
    def _both_parties(self, stream, fn):
        """fn(p, stream_p) for both parties, party 1 on a side stream forked
        from and joined back to `stream`: the parties' independent launches
        (their matmuls, their gate evaluations) overlap on the GPU, as two
        party processes sharing it would."""
        import torch

        main = stream if stream is not None else torch.cuda.current_stream(self.dev)
        if self._side is None:
            self._side = torch.cuda.Stream(device=self.dev)
            self._fork = torch.cuda.Event()
            self._join = torch.cuda.Event()
        self._fork.record(main)
        self._side.wait_event(self._fork)
        fn(0, main)
        fn(1, self._side)
        self._join.record(self._side)
        main.wait_event(self._join)

    def _matmul_trunc(self, x, wname, K, N, tr: _Trunc, out, stream):
        """out_p = T(x_p W): each party's public-weight product, the open of
        the masked products and the truncation bundle of both parties."""
        L = _lib.lib()
        S = self.dims.S
        acc = self.b["acc"]
        self._both_parties(stream, lambda p, st: check(L.sufb200_ring_matmul(
            self.ctx.h, _t_ptr(x[p]), _t_ptr(self.W[wname]), None, _t_ptr(acc[p]), 1, S, K, N, 0, _stream_ptr(st))))
        n = S * N
        if acc[0].numel() < n or self.b["xhat"].numel() < n or out[0].numel() < n or x[0].numel() < S * K:
            raise ValueError("layer: a staging buffer is smaller than the product")
        xh = self.b["xhat"][:n]
        check(L.sufb200_open_masked_pair(_t_ptr(acc[0]), _t_ptr(acc[1]), C.c_uint64(tr.r[0]), C.c_uint64(tr.r[1]),
                                         _t_ptr(xh), n, _stream_ptr(stream)))
        tr.eval_pair(self.ctx, xh, out[0][:n], out[1][:n], stream)

    def _beaver_trunc(self, x, off_x, sx, ldx, y, off_y, sy, ldy, trans, trip: _Triples, M, K, N, so, ldo,
                      tr: _Trunc, out, stream):
        H = self.dims.H
        n = H * M * N
        if self.b["xhat"].numel() < n or out[0].numel() < n:
            raise ValueError("layer: a staging buffer is smaller than the product")
        xh = self.b["xhat"][:n]
        xs = (C.c_void_p * 2)(*[x[p].data_ptr() + 8 * off_x for p in (0, 1)])
        ys = (C.c_void_p * 2)(*[y[p].data_ptr() + 8 * off_y for p in (0, 1)])
        rr = (C.c_uint64 * 2)(*tr.r)
        check(_lib.lib().sufb200_beaver_open_pair(
            C.cast(xs, C.c_void_p), sx, ldx, C.cast(ys, C.c_void_p), sy, ldy, int(trans),
            C.cast(trip.ptrs(0), C.c_void_p), C.cast(trip.ptrs(1), C.c_void_p), C.cast(trip.ptrs(2), C.c_void_p),
            C.cast(rr, C.c_void_p), H, M, K, N, _t_ptr(xh), so, ldo, _stream_ptr(stream)))
        tr.eval_pair(self.ctx, xh, out[0][:n], out[1][:n], stream)

    def _rowmax_diff(self, s, t, stream):
        """t_p = rowmax(s) - s_p over rows of S columns (H * S rows)."""
        L = _lib.lib()
        d = self.dims
        rows, w = d.H * d.S, d.S
        cur = s
        bufs = [self.b["c"], self.b["c2"]]
        for i, g in enumerate(self.relu):
            half = rows * (w // 2)
            xh = self.b["xhat"][:half]
            check(L.sufb200_relu_open_pair(_t_ptr(cur[0]), _t_ptr(cur[1]), rows, w, C.c_uint64(g.r[0]),
                                           C.c_uint64(g.r[1]), _t_ptr(xh), _stream_ptr(stream)))
            rl = self.b["relu"]
            g.eval_pair(self.ctx, xh, rl[0][:half], rl[1][:half], stream)
            nxt = bufs[i % 2]
            check(L.sufb200_relu_update_pair(_t_ptr(cur[0]), _t_ptr(cur[1]), _t_ptr(rl[0]), _t_ptr(rl[1]), rows, w,
                                             _t_ptr(nxt[0]), _t_ptr(nxt[1]), _stream_ptr(stream)))
            cur = nxt
            w //= 2
        check(L.sufb200_maxdiff_pair(_t_ptr(cur[0]), _t_ptr(cur[1]), _t_ptr(s[0]), _t_ptr(s[1]), rows, d.S,
                                     _t_ptr(t[0]), _t_ptr(t[1]), _stream_ptr(stream)))

    def run(self, d_x0, d_x1, d_y0=None, d_y1=None, stream=None, trace: dict | None = None):
        """Both parties' shares of X ([S, D] Q f, int64 tensors on the device)
        -> shares of the layer output.  Asynchronous on `stream`.  With a
        `trace` dict, copies of both parties' shares after each stage are
        stored in it (for stage-by-stage checks)."""
        import torch

        def keep(name, pair, n):
            if trace is not None:
                with torch.cuda.stream(stream) if stream is not None else _nullctx():
                    trace[name] = (pair[0][:n].clone(), pair[1][:n].clone())

        d = self.dims
        S, D, H, Dh, Dff = d.S, d.D, d.H, d.Dh, d.Dff
        if d_x0.numel() != S * D or d_x1.numel() != S * D:
            raise ValueError(f"layer: expected {S * D} elements per share")
        if d_y0 is None:
            d_y0 = torch.empty_like(d_x0)
        if d_y1 is None:
            d_y1 = torch.empty_like(d_x1)
        L = _lib.lib()
        b = self.b
        x = (d_x0, d_x1)
        # the truncations' full-domain tables depend on their keys only: they
        # are filled on a side stream, in the order the layer needs them,
        # while LayerNorm and the first matmuls run (the first LayerNorm's
        # mean and variance bundles walk their keys: they start the layer)
        main = stream if stream is not None else torch.cuda.current_stream(self.dev)
        if self._tab_stream is None:
            self._tab_stream = torch.cuda.Stream(device=self.dev)
            self._tab_fork = torch.cuda.Event()
            self._tab_ev = [torch.cuda.Event() for _ in range(7)]
        ts, ev = self._tab_stream, self._tab_ev
        self._tab_fork.record(main)
        ts.wait_event(self._tab_fork)
        # the first LayerNorm's normalised-output bundle (its last step): the
        # block waits on the event right before it
        self.ln1.prepare_tables(ts, bundles=(7,), ready=ev[6])
        g = self._tab_groups
        for (grp, block), e in zip(((g[0], None), (None, self.softmax), (g[1], None), (None, self.ln2),
                                    (g[2], None)), ev):
            if grp is not None and grp[1].any():
                grp[1].fill(self.ctx, ts)
                for name in grp[0]:
                    if self.tr[name].tables is not None:
                        self.tr[name].ready = e
            if block is not None:
                block.prepare_tables(ts)
            e.record(ts)
        # attention
        h = self.ln1.run(x[0], x[1], b["h"][0], b["h"][1], stream=stream)
        keep("h1", h, S * D)
        self._matmul_trunc(h, "qkv", D, 3 * D, self.tr["qkv"], b["qkv"], stream)
        keep("qkv", b["qkv"], S * 3 * D)
        self._beaver_trunc(b["qkv"], 0, Dh, 3 * D, b["qkv"], D, Dh, 3 * D, True, self.trip_s, S, Dh, S, S * S, S,
                           self.tr["scores"], b["s"], stream)
        keep("scores", b["s"], H * S * S)
        self._rowmax_diff(b["s"], b["t"], stream)
        keep("t", b["t"], H * S * S)
        main.wait_event(ev[1])
        self.softmax.run(b["t"][0], b["t"][1], b["p"][0], b["p"][1], stream=stream)
        keep("probs", b["p"], H * S * S)
        self._beaver_trunc(b["p"], 0, S * S, S, b["qkv"], 2 * D, Dh, 3 * D, False, self.trip_pv, S, S, Dh, Dh, D,
                           self.tr["pv"], b["o"], stream)
        keep("o", b["o"], S * D)
        self._matmul_trunc(b["o"], "o", D, D, self.tr["o"], b["a"], stream)
        keep("attn", b["a"], S * D)
        check(L.sufb200_add_pair(_t_ptr(x[0]), _t_ptr(b["a"][0]), _t_ptr(x[1]), _t_ptr(b["a"][1]),
                                 _t_ptr(b["x2"][0]), _t_ptr(b["x2"][1]), S * D, _stream_ptr(stream)))
        # MLP
        main.wait_event(ev[3])
        h = self.ln2.run(b["x2"][0], b["x2"][1], b["h"][0], b["h"][1], stream=stream)
        keep("h2", h, S * D)
        self._matmul_trunc(h, "ff1", D, Dff, self.tr["ff1"], b["f1"], stream)
        keep("f1", b["f1"], S * Dff)
        n = S * Dff
        xh = b["xhat"][:n]
        g = self.gelu
        check(L.sufb200_open_masked_pair(_t_ptr(b["f1"][0]), _t_ptr(b["f1"][1]), C.c_uint64(g.r[0]),
                                         C.c_uint64(g.r[1]), _t_ptr(xh), n, _stream_ptr(stream)))
        g.eval_pair(self.ctx, xh, b["g"][0], b["g"][1], stream)
        keep("gelu", b["g"], S * Dff)
        self._matmul_trunc(b["g"], "ff2", Dff, D, self.tr["ff2"], b["a"], stream)
        keep("f2", b["a"], S * D)
        check(L.sufb200_add_pair(_t_ptr(b["x2"][0]), _t_ptr(b["a"][0]), _t_ptr(b["x2"][1]), _t_ptr(b["a"][1]),
                                 _t_ptr(d_y0), _t_ptr(d_y1), S * D, _stream_ptr(stream)))
        return d_y0, d_y1

    def capture(self, d_x0, d_x1, d_y0, d_y1, layers: int = 1):
        """A CUDA graph of `layers` runs of this layer, each layer's output
        shares feeding the next and the last one's written to d_y0 / d_y1;
        replay() reads d_x0 / d_x1 as they are at replay time and launches
        the whole sequence (about 150 kernels a layer) with no host work.
        Everything the calls use stays resident on the device (keys, triples,
        tables); the scratch the calls allocate becomes graph memory."""
        import torch

        d = self.dims
        tmp = [(torch.empty(d.S * d.D, dtype=torch.int64, device=self.dev),
                torch.empty(d.S * d.D, dtype=torch.int64, device=self.dev)) for _ in range(2 if layers > 1 else 0)]

        def chain(stream):
            a, b = d_x0, d_x1
            for i in range(layers):
                o = (d_y0, d_y1) if i == layers - 1 else tmp[i % 2]
                self.run(a, b, o[0], o[1], stream=stream)
                a, b = o

        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        chain(s)  # warm-up outside the capture: lazily made streams, events and pool memory
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.ctx.sync(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s, capture_error_mode="relaxed"):
            chain(s)
        g._sufb200_keep = tmp  # the graph's intermediate buffers live as long as it does
        return g

    # launches of our kernels per layer (counted from the calls above).  Every
    # truncation bundle with tables is one launch against them; the side
    # stream fills the tables with one frontier launch per 16 keys of a
    # group: three for the layer's own six bundles (three groups of 8 keys),
    # two for the softmax block (28 keys), one for the first LayerNorm's
    # normalised output (4 keys) and two for the second LayerNorm (24 keys);
    # their element-level bundles then skip their own frontier launch.
    def launches(self) -> int:
        d = self.dims
        # each LayerNorm's element-level bundle against tables, one frontier
        # launch fewer than bench.py's LAYERNORM_LAUNCHES; table fills: one
        # for the first (that bundle only), two for the second (every f-bit bundle)
        ln = (19 - 1 + 1) + (19 - 1 + 2)
        sm = 22 - 4 + 2  # the softmax block against tables (bench.py's SOFTMAX_LAUNCHES)
        mm = 4 * (2 * 2 + 1 + 1)  # qkv, o, ff1, ff2: two ring matmuls (pre-pass + GEMM each), open, truncation
        bv = 2 * (1 + 1)  # scores, pv: the Beaver open, the truncation
        relu = self.rounds * 3 + 1  # open, the pair gate launch, update per round; the final max-difference
        gelu = 1 + 1  # open, the pair gate launch
        return ln + sm + mm + bv + relu + gelu + 2 + 3
