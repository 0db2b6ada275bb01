"""configs[4] softmax block on the device for both parties of one GPU
(sufb200_softmax_block_pair): the dealer that makes its correlated
randomness, and the call.

The block is nn::SoftmaxBlockTask (include/nn/softmax_block_task.hpp) of the
reference: nExp cubic gate (CubicPolyTask), ragged row sums, reciprocal with
one Newton step (RecipTask), row-broadcast Beaver product and probability
truncation.  Its gate tables are the reference's own SUF programs
(suf_b200/tables/softmax_suf_f12.json, dumped from the reference by
tests/golden/make_softmax_tables.py):
  nexp : make_nexp_spec(NExpGateParams{f, 16}) via build_silu_suf_from_piecewise
  recip: make_recip_affine_init_spec(f, 1024) via build_silu_suf_from_piecewise
Every truncation is a GapARS bundle, as dealer_make_nexp_task_material and the
reciprocal's AutoTrunc choose for these ranges; CubicPolyTask's T_2f is done
as two f-bit bundles (the same floor).  The dealer's masks are its
own draws: the reconstruction of every step is exact in Z_2^64 and does not
depend on them.
"""
from __future__ import annotations

import ctypes as C
import json
from pathlib import Path

import numpy as np

from . import _lib
from ._lib import TruncDesc, check
from .engine import Context, interval_lut_key, seed_from_id

TABLES = Path(__file__).resolve().parent / "tables" / "softmax_suf_f12.json"
N_TRUNCS = 7
TRUNC_GAPARS = 2  # SUFB200_TRUNC_GAPARS
GROUP_ADD = 0
M64 = (1 << 64) - 1


class SoftmaxParty(C.Structure):
    """Mirror of sufb200_softmax_party."""

    _fields_ = [
        ("nexp_rin", C.c_uint64), ("recip_rin", C.c_uint64),
        ("d_nexp_lut", C.c_void_p), ("nexp_lut_bytes", C.c_size_t),
        ("d_recip_lut", C.c_void_p), ("recip_lut_bytes", C.c_size_t),
        ("d_nexp_triples", C.c_void_p), ("d_recip_triples", C.c_void_p),
        ("d_row_a", C.c_void_p), ("d_row_b", C.c_void_p), ("d_row_c", C.c_void_p),
        ("trunc", TruncDesc * N_TRUNCS),
        ("trunc_rin", C.c_uint64 * N_TRUNCS),
        ("trunc_keys", (C.c_void_p * 4) * N_TRUNCS),
        ("trunc_key_bytes", (C.c_size_t * 4) * N_TRUNCS),
        ("trunc_keys_device", C.c_int32),
        ("trunc_tables", C.c_void_p * N_TRUNCS),
        ("trunc_ready", C.c_void_p * N_TRUNCS),
    ]


def load_tables(path: Path = TABLES) -> dict:
    """{'frac_bits': f, 'nexp': (alpha [m+1] u64, coeffs [m][4] u64), 'recip': ...}"""
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


def masked_lut_table(alpha: np.ndarray, coeffs: np.ndarray, r_in: int):
    """The gate's pieces moved to the x^ = x + r_in domain: the cut list
    (ascending, first cut 0, last entry the end sentinel) and the payload
    rows, for an interval LUT that returns piece i's coefficients when
    alpha[i] <= x^ - r_in < alpha[i+1] (the wrapped piece split at 0)."""
    m = len(coeffs)
    starts = [(int(alpha[j]) + r_in) & M64 for j in range(m)]
    order = sorted(range(m), key=lambda j: starts[j])
    cuts = [starts[j] for j in order]
    rows = [coeffs[j] for j in order]
    if cuts[0] != 0:  # x^ = 0 is x = -r_in: the piece containing it
        x0 = (-r_in) & M64
        j0 = int(np.searchsorted(alpha[:-1], np.uint64(x0), side="right")) - 1
        cuts.insert(0, 0)
        rows.insert(0, coeffs[min(max(j0, 0), m - 1)])
    cuts.append(M64)
    return np.array(cuts, dtype=np.uint64), np.ascontiguousarray(np.stack(rows), dtype=np.uint64)


def _split(rng: np.random.Generator, v: np.ndarray):
    s0 = rng.integers(0, 2**64, v.shape, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return s0, v - s0


def _triples(rng: np.random.Generator, n: int):
    """(a, b, c) shares of n triples, interleaved per party: [n][3]."""
    a = rng.integers(0, 2**64, n, dtype=np.uint64)
    b = rng.integers(0, 2**64, n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        c = a * b
    out = []
    for sh in zip(_split(rng, a), _split(rng, b), _split(rng, c)):
        out.append(np.ascontiguousarray(np.stack(sh, axis=1)))
    return out


def _block_tables(parts, dev, ks):
    """Both parties' tables of a block's truncation bundles ks (TruncTables
    over party 0's bundles, then party 1's)."""
    from .engine import TruncTables

    return TruncTables([(parts[p].trunc[k], parts[p].trunc_keys[k], parts[p].trunc_key_bytes[k])
                        for p in (0, 1) for k in ks], dev)


def _prepare_tables(blk, stream, bundles, ready):
    import torch

    K = len(blk.parts[0].trunc)
    ks = tuple(range(K)) if bundles is None else tuple(bundles)
    T = blk._tables.get(ks)
    if T is None:
        T = blk._tables[ks] = _block_tables(blk.parts, blk._dev, ks)
    T.fill(blk.ctx, stream)
    if ready is not None:
        ready.record(stream if stream is not None else torch.cuda.current_stream())
    for j, k in enumerate(ks):
        for p in (0, 1):
            blk.parts[p].trunc_tables[k] = T.ptr(p * len(ks) + j)
            blk.parts[p].trunc_ready[k] = ready.cuda_event if ready is not None else None


class SoftmaxBlock:
    """Dealer material for one softmax block shape (rows, ragged row lengths)
    for both parties, resident on the context's device, and the block call.

    row_lengths: valid entries per row (the causal prefix lengths); the
    block's inputs and outputs are packed row after row."""

    def __init__(self, ctx: Context, row_lengths, seed: int = 1, tables: dict | None = None):
        import torch

        self.ctx = ctx
        self.tables = tables or load_tables()
        f = self.frac_bits = int(self.tables["frac_bits"])
        lens = np.asarray(row_lengths, dtype=np.int64)
        self.rows = int(lens.size)
        off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        self.n = int(off[-1])
        dev = self._dev = torch.device("cuda", ctx.device if hasattr(ctx, "device") else 0)
        self._keep = []  # host key arrays and device tensors the structs point at
        self._tables = {}  # prepare_tables(): bundle subset -> TruncTables

        def dcopy(a: np.ndarray):
            t = torch.from_numpy(np.ascontiguousarray(a).view(np.int64) if a.dtype == np.uint64 else a).to(dev)
            self._keep.append(t)
            return t

        self.d_row_off = dcopy(off)
        rng = np.random.default_rng(seed)
        parts = [SoftmaxParty(), SoftmaxParty()]

        # interval-LUT gates: one input mask each, keys on the x^ domain
        for gate, rin_field, lut_field, bytes_field in (("nexp", "nexp_rin", "d_nexp_lut", "nexp_lut_bytes"),
                                                        ("recip", "recip_rin", "d_recip_lut", "recip_lut_bytes")):
            r_in = int(rng.integers(0, 2**64, dtype=np.uint64))
            r0 = int(rng.integers(0, 2**64, dtype=np.uint64))
            cuts, payload = masked_lut_table(*self.tables[gate], r_in)
            nonce = int(rng.integers(1, 2**62))
            sd = seed_from_id(nonce, 7)
            for p in (0, 1):
                key = interval_lut_key(p, nonce, 64, 4, cuts, payload.reshape(-1), sd)
                dk = dcopy(key)
                setattr(parts[p], rin_field, r0 if p == 0 else (r_in - r0) & M64)
                setattr(parts[p], lut_field, dk.data_ptr())
                setattr(parts[p], bytes_field, key.size)

        # Beaver triples: three per element (nExp Horner), three per row
        # (reciprocal), and the row-broadcast triple of the probability product
        for field, count in (("d_nexp_triples", 3 * self.n), ("d_recip_triples", 3 * self.rows)):
            sh = _triples(rng, count)
            for p in (0, 1):
                setattr(parts[p], field, dcopy(sh[p]).data_ptr())
        A = rng.integers(0, 2**64, self.n, dtype=np.uint64)
        B = rng.integers(0, 2**64, self.rows, dtype=np.uint64)
        with np.errstate(over="ignore"):
            Cm = A * B[np.repeat(np.arange(self.rows), lens)]
        for field, v in (("d_row_a", A), ("d_row_b", B), ("d_row_c", Cm)):
            sh = _split(rng, v)
            for p in (0, 1):
                setattr(parts[p], field, dcopy(sh[p]).data_ptr())

        # the seven GapARS truncations: nExp T_f(p), the first T_f of T_2f(r);
        # reciprocal init, Newton x2; probabilities; the second T_f of T_2f(r)
        # (floor(floor(r / 2^f) / 2^f) = floor(r / 2^2f): two f-bit bundles,
        # each a full-domain table lookup, in place of one 2f-bit bundle)
        payload1 = (1).to_bytes(8, "little")
        for k, fk in enumerate((f, f, f, f, f, f, f)):
            r_in, d0, d1, thetas = Context.trunc_gen(TRUNC_GAPARS, fk, int(rng.integers(1, 2**63)))
            r0 = int(rng.integers(0, 2**64, dtype=np.uint64))
            for p, d in ((0, d0), (1, d1)):
                parts[p].trunc[k] = d
                parts[p].trunc_rin[k] = r0 if p == 0 else (r_in - r0) & M64
            for q in range(int(d0.nq)):
                s0 = rng.integers(0, 256, 16, dtype=np.uint8)
                s1 = rng.integers(0, 256, 16, dtype=np.uint8)
                k0, k1 = ctx.myl7_gen(GROUP_ADD, int(d0.q_bits[q]), int(thetas[q]), payload1, s0, s1)
                for p, key in ((0, k0), (1, k1)):  # resident on the device, like the rest of the material
                    parts[p].trunc_keys[k][q] = dcopy(key).data_ptr()
                    parts[p].trunc_key_bytes[k][q] = key.size
        for p in (0, 1):
            parts[p].trunc_keys_device = 1
        self.parts = parts

    def prepare_tables(self, stream=None, bundles=None, ready=None):
        """Fill the tables of the truncation bundles `bundles` (default all)
        whose queries are at most 16 bits wide, on `stream` (they depend on
        the keys only), and switch those bundles to table evaluation.  Block
        calls ordered after this on the device read them; with a
        torch.cuda.Event `ready` (recorded here after the fill) a block call
        on another stream waits for it right before each such bundle."""
        _prepare_tables(self, stream, bundles, ready)

    def run(self, d_t0, d_t1, d_prob0=None, d_prob1=None, stream=None):
        """Both parties' shares of the packed max-differences t (Q f, int64
        tensors of n words on the device) -> shares of the packed
        probabilities.  Asynchronous on `stream` (default: torch's current)."""
        import torch

        from .engine import _stream_ptr, _t_ptr

        if d_t0.numel() != self.n or d_t1.numel() != self.n:
            raise ValueError(f"softmax block: expected {self.n} packed elements")
        if d_prob0 is None:
            d_prob0 = torch.empty_like(d_t0)
        if d_prob1 is None:
            d_prob1 = torch.empty_like(d_t1)
        L = _lib.lib()
        check(L.sufb200_softmax_block_pair(self.ctx.h, C.byref(self.parts[0]), C.byref(self.parts[1]), self.rows,
                                           _t_ptr(self.d_row_off), _t_ptr(d_t0), _t_ptr(d_t1), self.n,
                                           self.frac_bits, _t_ptr(d_prob0), _t_ptr(d_prob1), _stream_ptr(stream)))
        return d_prob0, d_prob1


# ---------------------------------------------------------------------------
# configs[4] LayerNorm block (sufb200_layernorm_block_pair)
# ---------------------------------------------------------------------------

N_LN_TRUNCS = 8


class LayerNormParty(C.Structure):
    """Mirror of sufb200_layernorm_party."""

    _fields_ = [
        ("rsqrt_rin", C.c_uint64),
        ("d_rsqrt_lut", C.c_void_p), ("rsqrt_lut_bytes", C.c_size_t),
        ("d_sq_triples", C.c_void_p), ("d_row_triples", C.c_void_p),
        ("d_norm_a", C.c_void_p), ("d_norm_b", C.c_void_p), ("d_norm_c", C.c_void_p),
        ("trunc", TruncDesc * N_LN_TRUNCS),
        ("trunc_rin", C.c_uint64 * N_LN_TRUNCS),
        ("trunc_keys", (C.c_void_p * 4) * N_LN_TRUNCS),
        ("trunc_key_bytes", (C.c_size_t * 4) * N_LN_TRUNCS),
        ("trunc_keys_device", C.c_int32),
        ("trunc_tables", C.c_void_p * N_LN_TRUNCS),
        ("trunc_ready", C.c_void_p * N_LN_TRUNCS),
    ]


class LayerNormBlock:
    """Dealer material for one LayerNorm block (rows x cols, dense) for both
    parties on the context's device, and the block call.  All eight
    truncations are GapARS bundles (signed floors; the reference's bench uses
    logical shifts for the mean and the output, which are wrong for the
    negative values of Gaussian inputs, and FaithfulARS for the Newton steps,
    which floors identically in this range)."""

    def __init__(self, ctx: Context, rows: int, cols: int, seed: int = 1, tables: dict | None = None):
        import torch

        self.ctx = ctx
        self.tables = tables or load_tables()
        f = self.frac_bits = int(self.tables["frac_bits"])
        self.rows, self.cols = int(rows), int(cols)
        n = self.n = self.rows * self.cols
        self.inv_len = int(round((1 << f) / cols))
        self.eps = int(round((1 << f) / 1024))
        dev = self._dev = torch.device("cuda", ctx.device)
        self._keep = []
        self._tables = {}  # prepare_tables(): bundle subset -> TruncTables

        def dcopy(a: np.ndarray):
            t = torch.from_numpy(np.ascontiguousarray(a).view(np.int64) if a.dtype == np.uint64 else a).to(dev)
            self._keep.append(t)
            return t

        rng = np.random.default_rng(seed)
        parts = [LayerNormParty(), LayerNormParty()]
        r_in = int(rng.integers(0, 2**64, dtype=np.uint64))
        r0 = int(rng.integers(0, 2**64, dtype=np.uint64))
        cuts, payload = masked_lut_table(*self.tables["rsqrt"], r_in)
        nonce = int(rng.integers(1, 2**62))
        sd = seed_from_id(nonce, 7)
        for p in (0, 1):
            key = interval_lut_key(p, nonce, 64, 4, cuts, payload.reshape(-1), sd)
            parts[p].rsqrt_rin = r0 if p == 0 else (r_in - r0) & M64
            parts[p].d_rsqrt_lut = dcopy(key).data_ptr()
            parts[p].rsqrt_lut_bytes = key.size
        for field, count in (("d_sq_triples", n), ("d_row_triples", 4 * self.rows)):
            sh = _triples(rng, count)
            for p in (0, 1):
                setattr(parts[p], field, dcopy(sh[p]).data_ptr())
        A = rng.integers(0, 2**64, n, dtype=np.uint64)
        B = rng.integers(0, 2**64, self.rows, dtype=np.uint64)
        with np.errstate(over="ignore"):
            Cm = A * np.repeat(B, self.cols)
        for field, v in (("d_norm_a", A), ("d_norm_b", B), ("d_norm_c", Cm)):
            sh = _split(rng, v)
            for p in (0, 1):
                setattr(parts[p], field, dcopy(sh[p]).data_ptr())
        payload1 = (1).to_bytes(8, "little")
        # every value truncated here stays below 2^40 in magnitude, far inside
        # GapARS's exactness bound, where it floors exactly like FaithfulARS with
        # two f-bit queries instead of two 64-bit ones
        kinds = [(TRUNC_GAPARS, fk) for fk in (f, 2 * f, f, f, f, 1, f, f)]
        for k, (kind, fk) in enumerate(kinds):
            r_t, d0, d1, thetas = Context.trunc_gen(kind, fk, int(rng.integers(1, 2**63)))
            rr = int(rng.integers(0, 2**64, dtype=np.uint64))
            for p, d in ((0, d0), (1, d1)):
                parts[p].trunc[k] = d
                parts[p].trunc_rin[k] = rr if p == 0 else (r_t - rr) & M64
            for q in range(int(d0.nq)):
                s0 = rng.integers(0, 256, 16, dtype=np.uint8)
                s1 = rng.integers(0, 256, 16, dtype=np.uint8)
                k0, k1 = ctx.myl7_gen(GROUP_ADD, int(d0.q_bits[q]), int(thetas[q]), payload1, s0, s1)
                for p, key in ((0, k0), (1, k1)):  # resident on the device, like the rest of the material
                    parts[p].trunc_keys[k][q] = dcopy(key).data_ptr()
                    parts[p].trunc_key_bytes[k][q] = key.size
        for p in (0, 1):
            parts[p].trunc_keys_device = 1
        self.parts = parts

    def prepare_tables(self, stream=None, bundles=None, ready=None):
        """Fill the tables of the truncation bundles `bundles` (default all)
        whose queries are at most 16 bits wide, on `stream` (they depend on
        the keys only), and switch those bundles to table evaluation.  Block
        calls ordered after this on the device read them; with a
        torch.cuda.Event `ready` (recorded here after the fill) a block call
        on another stream waits for it right before each such bundle."""
        _prepare_tables(self, stream, bundles, ready)

    def run(self, d_x0, d_x1, d_out0=None, d_out1=None, stream=None):
        """Both parties' shares of x (rows * cols, Q f, int64 tensors on the
        device) -> shares of the normalised values.  Asynchronous."""
        import torch

        from .engine import _stream_ptr, _t_ptr

        if d_x0.numel() != self.n or d_x1.numel() != self.n:
            raise ValueError(f"layernorm block: expected {self.n} elements")
        if d_out0 is None:
            d_out0 = torch.empty_like(d_x0)
        if d_out1 is None:
            d_out1 = torch.empty_like(d_x1)
        check(_lib.lib().sufb200_layernorm_block_pair(
            self.ctx.h, C.byref(self.parts[0]), C.byref(self.parts[1]), self.rows, self.cols, _t_ptr(d_x0),
            _t_ptr(d_x1), self.frac_bits, C.c_uint64(self.inv_len), C.c_uint64(self.eps), _t_ptr(d_out0),
            _t_ptr(d_out1), _stream_ptr(stream)))
        return d_out0, d_out1
