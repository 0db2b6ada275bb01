"""Plaintext model of the configs[4] softmax block -- TEST INFRASTRUCTURE.

The arithmetic nn::SoftmaxBlockTask performs on secret shares, restated on
the reconstructed values (every step is exact in Z_2^64, so the
reconstruction does not depend on the masks):
  nExp   (CubicPolyTask, include/runtime/phase_tasks.hpp:2960-3060):
           c0..c3 = LUT_nexp(t); p2 = T_f((c3 t + c2 2^f) t);
           e = T_2f((p2 + c1 2^f) t) + c0
  sums   (SoftmaxBlockTask SumLocal, include/nn/softmax_block_task.hpp):
           s_r = sum of e over row r's valid prefix
  recip  (RecipTask, phase_tasks.hpp:3355-3540, one Newton step):
           a0, a1 = LUT_recip(s); y = T_f(a1 s) + a0;
           y = T_f(y (2 2^f - T_f(y s)))
  probs  (MulRowBroadcastTask + TruncTask): prob = T_f(e y_row)
where T_k is the signed floor shift (the ARS / GapARS truncations) and
LUT_g(x) the coefficient words of the SUF piece containing x (alpha[i] <=
x < alpha[i+1]).  The tables are the reference's own SUF programs
(suf_b200/tables/softmax_suf_f12.json, from oracle/softmax_tables.cpp).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

TABLES = Path(__file__).resolve().parents[1] / "suf_b200" / "tables" / "softmax_suf_f12.json"


def load_tables(path: Path = TABLES) -> dict:
    d = json.loads(Path(path).read_text())
    out = {"frac_bits": int(d["frac_bits"])}
    for g in ("nexp", "recip", "rsqrt"):
        if g not in d:
            continue
        alpha = np.array([int(v) for v in d[g]["alpha"]], dtype=np.uint64)
        coeffs = np.zeros((len(d[g]["pieces"]), 4), dtype=np.uint64)
        for i, piece in enumerate(d[g]["pieces"]):
            for j, poly in enumerate(piece[:4]):
                coeffs[i, j] = np.uint64(int(poly[0]))
        out[g] = (alpha, coeffs)
    return out


def lut(table, x: np.ndarray) -> np.ndarray:
    alpha, coeffs = table
    idx = np.searchsorted(alpha[:-1], x, side="right").astype(np.int64) - 1
    return coeffs[np.clip(idx, 0, len(coeffs) - 1)]


def tshift(v: np.ndarray, k: int) -> np.ndarray:
    return (v.view(np.int64) >> np.int64(k)).view(np.uint64)


def softmax_block(t: np.ndarray, row_offsets: np.ndarray, tables: dict) -> np.ndarray:
    """t: packed active elements (u64, Q f); row_offsets: rows + 1 offsets.
    Returns the packed probabilities (u64, Q f)."""
    f = tables["frac_bits"]
    F = np.uint64(1 << f)
    t = t.astype(np.uint64)
    with np.errstate(over="ignore"):
        c = lut(tables["nexp"], t)
        p2 = tshift((c[:, 3] * t + c[:, 2] * F) * t, f)
        e = tshift((p2 + c[:, 1] * F) * t, 2 * f) + c[:, 0]
        rows = len(row_offsets) - 1
        lens = np.diff(row_offsets)
        s = np.add.reduceat(e, row_offsets[:-1]) if len(e) else np.zeros(rows, np.uint64)
        s = np.where(lens > 0, s, np.uint64(0)).astype(np.uint64)
        a = lut(tables["recip"], s)
        y = tshift(a[:, 1] * s, f) + a[:, 0]
        y = tshift(y * (np.uint64(2 << f) - tshift(y * s, f)), f)
        row_of = np.repeat(np.arange(rows), lens)
        return tshift(e * y[row_of], f)


def layernorm_block(x: np.ndarray, rows: int, cols: int, tables: dict, eps_qf: int | None = None) -> np.ndarray:
    """The configs[4] LayerNorm block (runtime::LayerNormTask with RsqrtTask,
    include/runtime/phase_tasks.hpp:1383-1700, 2186-2600; one Newton step, no
    affine), with signed truncations:
      mu = T_f(sum_row(x) invL)            d = x - mu
      v  = T_2f(sum_row(d^2) invL) + eps
      y  = c0 + T_f(c1 v)                  (c0, c1 = LUT_rsqrt(v))
      y  = T_f(y (3 2^(f-1) - floor(T_f(v T_f(y y)) / 2)))
      out = T_f(d y_row)
    invL = round(2^f / cols), eps = round(2^f / 1024)."""
    f = tables["frac_bits"]
    inv_len = np.uint64(round((1 << f) / cols))
    eps = np.uint64(round((1 << f) / 1024) if eps_qf is None else eps_qf)
    x = x.astype(np.uint64).reshape(rows, cols)
    with np.errstate(over="ignore"):
        mu = tshift(x.sum(axis=1, dtype=np.uint64) * inv_len, f)
        d = x - mu[:, None]
        v = tshift((d * d).sum(axis=1, dtype=np.uint64) * inv_len, 2 * f) + eps
        c = lut(tables["rsqrt"], v)
        y = c[:, 0] + tshift(c[:, 1] * v, f)
        xy2 = tshift(v * tshift(y * y, f), f)
        t = np.uint64(3 << (f - 1)) - (xy2 >> np.uint64(1))
        y = tshift(y * t, f)
        return tshift(d * y[:, None], f).reshape(-1)
