"""Plaintext model of the device-resident 2PC transformer layer -- TEST
INFRASTRUCTURE (never imported by the product).

The layer suf_b200/layer.py runs on secret shares, restated on the
reconstructed values.  Every step is exact in Z_2^64, so the reconstruction
does not depend on the dealer's masks, keys or triples:

  H1  = LN(X)                                (configs[4] LayerNorm block)
  QKV = T_f(H1 Wqkv)                         (public-weight matmul + GapARS)
  S_h = T_{f+3}(Q_h K_h^T)                   (Beaver matmul per head, 1/sqrt(64) folded)
  m   = rowmax(S) by max(a, b) = b + ReLU(a - b)   (nn::RowMaxDiffTask)
  P   = softmax block on t = m - S           (nn::SoftmaxBlockTask)
  O_h = T_f(P_h V_h);  A = T_f(O Wo);  X2 = X + A
  H2  = LN(X2);  F1 = T_f(H2 W1);  G = GeLU_const(F1);  F2 = T_f(G W2)
  Y   = X2 + F2

T_k is the signed floor shift (the GapARS truncation), LN the LayerNorm block
model of oracle/softmax_model.py, the softmax block its softmax model, ReLU
and GeLU_const the reference's own SUF tables (relu: make_relu_value_suf_u64,
include/gates/relu_gate.hpp:39; gelu_const: build_gelu_suf_const_from_piecewise
of make_gelu_spline_spec(f, 256), include/suf/suf_gelu_builders.hpp:107),
dumped to suf_b200/tables/layer_suf_f12.json by oracle/softmax_tables.cpp.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from oracle.softmax_model import layernorm_block, load_tables, softmax_block, tshift

LAYER_TABLES = Path(__file__).resolve().parents[1] / "suf_b200" / "tables" / "layer_suf_f12.json"


@dataclass
class Dims:
    S: int = 128
    D: int = 768
    H: int = 12
    Dff: int = 3072
    f: int = 12

    @property
    def Dh(self) -> int:
        return self.D // self.H


def load_layer_tables(path: Path = LAYER_TABLES) -> dict:
    """{'relu': (alpha, coeffs [m][2]), 'gelu_const': (alpha, coeffs [m][1])}:
    piece i covers alpha[i] <= x < alpha[i+1] (the last piece runs to 2^64 - 1),
    its polynomial is sum_k coeffs[i][k] x^k."""
    d = json.loads(Path(path).read_text())
    out = {"frac_bits": int(d["frac_bits"])}
    for g in ("relu", "gelu_const"):
        deg = int(d[g]["degree"])
        alpha = np.array([int(v) for v in d[g]["alpha"]], dtype=np.uint64)
        coeffs = np.zeros((len(d[g]["pieces"]), deg + 1), dtype=np.uint64)
        for i, piece in enumerate(d[g]["pieces"]):
            for k, c in enumerate(piece[0]):
                coeffs[i, k] = np.uint64(int(c))
        out[g] = (alpha, coeffs)
    return out


def piecewise(table, x: np.ndarray) -> np.ndarray:
    """The SUF's polynomial of the piece containing x (suf::eval_suf_ref)."""
    alpha, coeffs = table
    idx = np.clip(np.searchsorted(alpha[:-1], x, side="right").astype(np.int64) - 1, 0, len(coeffs) - 1)
    c = coeffs[idx]
    y = np.zeros_like(x)
    with np.errstate(over="ignore"):
        for k in range(coeffs.shape[1] - 1, -1, -1):
            y = y * x + c[:, k]
    return y


def matmul(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """X (u64 shares or values) times a public int64 matrix, mod 2^64."""
    with np.errstate(over="ignore"):
        return np.matmul(x.astype(np.uint64), w.astype(np.int64).view(np.uint64))


def rowmax(s: np.ndarray, relu) -> np.ndarray:
    """The tournament of nn::RowMaxDiffTask: pairs (2j, 2j+1), max = b + ReLU(a - b)."""
    c = s
    with np.errstate(over="ignore"):
        while c.shape[1] > 1:
            a, b = c[:, 0::2], c[:, 1::2]
            c = b + piecewise(relu, (a - b).ravel()).reshape(a.shape)
    return c[:, 0]


def layer(X: np.ndarray, W: dict, dims: Dims, sm_tables: dict | None = None, tables: dict | None = None,
          trace: dict | None = None) -> np.ndarray:
    """X: [S, D] u64 (Q f).  W: {'qkv': [D, 3D], 'o': [D, D], 'ff1': [D, Dff],
    'ff2': [Dff, D]} int64 (Q f).  Returns Y [S, D] u64."""
    sm_tables = sm_tables or load_tables()
    tables = tables or load_layer_tables()
    S, D, H, Dh, Dff, f = dims.S, dims.D, dims.H, dims.Dh, dims.Dff, dims.f
    X = X.astype(np.uint64).reshape(S, D)
    with np.errstate(over="ignore"):
        h1 = layernorm_block(X.ravel(), S, D, sm_tables).reshape(S, D)
        qkv = tshift(matmul(h1, W["qkv"]), f)
        q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
        scores = np.stack([tshift(np.matmul(q[:, h * Dh:(h + 1) * Dh], k[:, h * Dh:(h + 1) * Dh].T), f + 3)
                           for h in range(H)])  # [H, S, S]
        s2 = scores.reshape(H * S, S)
        m = rowmax(s2, tables["relu"])
        t = m[:, None] - s2
        if trace is not None:
            trace["t"] = t
        offs = np.arange(0, H * S * S + 1, S, dtype=np.int64)
        p = softmax_block(t.ravel(), offs, sm_tables).reshape(H, S, S)
        o = np.concatenate([tshift(np.matmul(p[h], v[:, h * Dh:(h + 1) * Dh]), f) for h in range(H)], axis=1)
        a = tshift(matmul(o, W["o"]), f)
        x2 = X + a
        h2 = layernorm_block(x2.ravel(), S, D, sm_tables).reshape(S, D)
        f1 = tshift(matmul(h2, W["ff1"]), f)
        g = piecewise(tables["gelu_const"], f1.ravel()).reshape(S, Dff)
        f2 = tshift(matmul(g, W["ff2"]), f)
        y = x2 + f2
    if trace is not None:
        trace.update(h1=h1, qkv=qkv, scores=scores, rowmax=m, probs=p, o=o, attn=a, x2=x2, h2=h2, f1=f1, gelu=g, f2=f2)
    return y


def layer_float(X: np.ndarray, W: dict, dims: Dims) -> np.ndarray:
    """The same pre-LN layer in float64 on the dequantised values (exact
    LayerNorm with eps 1/1024, exact softmax and GeLU), for accuracy reports."""
    from math import erf, sqrt

    S, D, H, Dh, f = dims.S, dims.D, dims.H, dims.Dh, dims.f
    sc = float(1 << f)
    x = X.astype(np.uint64).view(np.int64).reshape(S, D) / sc
    w = {n: W[n].astype(np.float64) / sc for n in W}

    def ln(z):
        mu = z.mean(axis=1, keepdims=True)
        var = ((z - mu) ** 2).mean(axis=1, keepdims=True)
        return (z - mu) / np.sqrt(var + 1.0 / 1024)

    h1 = ln(x)
    qkv = h1 @ w["qkv"]
    q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
    outs = []
    for h in range(H):
        sl = slice(h * Dh, (h + 1) * Dh)
        s = q[:, sl] @ k[:, sl].T / np.sqrt(Dh)
        e = np.exp(s - s.max(axis=1, keepdims=True))
        outs.append((e / e.sum(axis=1, keepdims=True)) @ v[:, sl])
    x2 = x + np.concatenate(outs, axis=1) @ w["o"]
    f1 = ln(x2) @ w["ff1"]
    g = np.vectorize(lambda z: 0.5 * z * (1.0 + erf(z / sqrt(2.0))))(f1)
    return x2 + g @ w["ff2"]
