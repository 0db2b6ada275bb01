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
    for g in ("nexp", "recip"):
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
