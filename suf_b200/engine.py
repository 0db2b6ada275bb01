"""Python host side of the engine: a thin object layer over the C ABI.

Device buffers are torch tensors on the context's device (PyTorch supplies
device memory and streams; the arithmetic runs in libsufb200's kernels).
Host buffers are numpy arrays.  Every call checks the C status code and
raises `SufB200Error` on failure -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import _lib
from ._lib import GROUP_ADD, GROUP_XOR, SufB200Error, TruncDesc, check  # noqa: F401


def _np_ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _t_ptr(t) -> int:
    return int(t.data_ptr())


def _stream_ptr(stream) -> int | None:
    if stream is None:
        import torch

        return int(torch.cuda.current_stream().cuda_stream) or None
    if isinstance(stream, int):
        return stream or None
    return int(stream.cuda_stream) or None


class TruncTables:
    """Device tables of a list of truncation bundles (either party's), each
    bundle given as (desc, key pointers [4], key sizes [4]) with its keys on
    the device; bundles with a query wider than 16 bits (or none) get no
    tables.  fill(stream) evaluates every table in as few launches as the
    keys allow (sufb200_trunc_tables_many_dev); ptr(i) is bundle i's table
    buffer or None."""

    def __init__(self, bundles, dev):
        import torch

        L = _lib.lib()
        n = len(bundles)
        self._descs = (TruncDesc * n)(*[b[0] for b in bundles])
        self._keys = (C.c_void_p * (4 * n))(*[k for b in bundles for k in list(b[1])[:4]])
        self._ksz = (C.c_size_t * (4 * n))(*[k for b in bundles for k in list(b[2])[:4]])
        sizes = [int(L.sufb200_trunc_tables_bytes(C.byref(self._descs[i]))) for i in range(n)]
        self._bufs = [torch.empty(b, dtype=torch.uint8, device=dev) if b else None for b in sizes]
        self._ptrs = (C.c_void_p * n)(*[t.data_ptr() if t is not None else None for t in self._bufs])
        self._bytes = (C.c_size_t * n)(*sizes)
        self.count = n

    def ptr(self, i: int):
        return self._ptrs[i]

    def any(self) -> bool:
        return any(t is not None for t in self._bufs)

    def fill(self, ctx, stream=None):
        check(_lib.lib().sufb200_trunc_tables_many_dev(ctx.h, self.count, self._descs, self._keys, self._ksz,
                                                       self._ptrs, self._bytes, _stream_ptr(stream)))


def host_mt19937_64(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint64)
    check(_lib.lib().sufb200_host_mt19937_64(C.c_uint64(seed), _np_ptr(out) if n else None, n))
    return out


def myl7_key_bytes(in_bits: int, payload_len: int) -> int:
    return int(_lib.lib().sufb200_myl7_key_bytes(in_bits, payload_len))


class Context:
    """One engine context: a device, the AES tables and the PRG keys."""

    def __init__(self, device: int = 0):
        self._L = _lib.lib()
        h = C.c_void_p()
        check(self._L.sufb200_ctx_create(device, C.byref(h)))
        self.h = h
        self.device = device

    def close(self) -> None:
        if self.h:
            self._L.sufb200_ctx_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def sm_count(self) -> int:
        return int(self._L.sufb200_ctx_sm_count(self.h))

    def probe_aes_engine(self) -> float:
        """Measured AES-128 blocks/s of the shared-memory engine (roofline peak)."""
        v = C.c_double()
        check(self._L.sufb200_probe_aes_engine(self.h, C.byref(v)))
        return float(v.value)

    def sync(self, stream=None) -> None:
        check(self._L.sufb200_ctx_sync(self.h, _stream_ptr(stream)))

    # -- myl7 PRG-tree DCF --------------------------------------------------
    def prg_init(self, state) -> None:
        s = np.ascontiguousarray(np.frombuffer(bytes(state), dtype=np.uint8) if isinstance(state, (bytes, bytearray))
                                 else state, dtype=np.uint8)
        check(self._L.sufb200_prg_init(self.h, _np_ptr(s), s.size))

    def myl7_gen(self, group: int, in_bits: int, alpha: int, payload: bytes, seeds0, seeds1):
        kb = myl7_key_bytes(in_bits, len(payload))
        k0 = np.zeros(kb, dtype=np.uint8)
        k1 = np.zeros(kb, dtype=np.uint8)
        pl = np.frombuffer(bytes(payload), dtype=np.uint8).copy()
        s0 = np.ascontiguousarray(seeds0, dtype=np.uint8)
        s1 = np.ascontiguousarray(seeds1, dtype=np.uint8)
        check(self._L.sufb200_myl7_gen(self.h, group, in_bits, C.c_uint64(alpha & (2**64 - 1)), _np_ptr(pl),
                                       len(payload), _np_ptr(s0), _np_ptr(s1), _np_ptr(k0), _np_ptr(k1)))
        return k0, k1

    def myl7_gen_batch(self, group: int, in_bits: int, alphas: np.ndarray, payload: bytes, seeds0: np.ndarray,
                       seeds1: np.ndarray):
        alphas = np.ascontiguousarray(alphas, dtype=np.uint64)
        n = alphas.size
        kb = myl7_key_bytes(in_bits, len(payload))
        keys0 = np.empty((n, kb), dtype=np.uint8)
        keys1 = np.empty((n, kb), dtype=np.uint8)
        pl = np.frombuffer(bytes(payload), dtype=np.uint8).copy()
        s0 = np.ascontiguousarray(seeds0, dtype=np.uint8)
        s1 = np.ascontiguousarray(seeds1, dtype=np.uint8)
        check(self._L.sufb200_myl7_gen_batch(self.h, group, in_bits, _np_ptr(alphas), n, _np_ptr(pl), len(payload),
                                             _np_ptr(s0), _np_ptr(s1), _np_ptr(keys0), _np_ptr(keys1)))
        return keys0, keys1

    def myl7_gen_batch_device(self, group: int, in_bits: int, d_alphas, payload: bytes, d_seeds0, d_seeds1,
                              d_keys0=None, d_keys1=None, stream=None):
        """Key pairs generated on the GPU (device tensors in and out)."""
        import torch

        n = d_alphas.numel()
        kb = myl7_key_bytes(in_bits, len(payload))
        if d_keys0 is None:
            d_keys0 = torch.empty(n * kb, dtype=torch.uint8, device=d_alphas.device)
        if d_keys1 is None:
            d_keys1 = torch.empty(n * kb, dtype=torch.uint8, device=d_alphas.device)
        pl = np.frombuffer(bytes(payload), dtype=np.uint8).copy()
        check(self._L.sufb200_myl7_gen_batch_device(self.h, group, in_bits, _t_ptr(d_alphas), n, _np_ptr(pl),
                                                    len(payload), _t_ptr(d_seeds0), _t_ptr(d_seeds1),
                                                    _t_ptr(d_keys0), _t_ptr(d_keys1), _stream_ptr(stream)))
        return d_keys0, d_keys1

    def myl7_eval(self, group: int, in_bits: int, d_keys, key_bytes: int, broadcast: bool, d_xs, out_bytes: int,
                  d_out=None, stream=None):
        import torch

        n = d_xs.numel()
        if d_out is None:
            d_out = torch.empty(n * out_bytes, dtype=torch.uint8, device=d_xs.device)
        check(self._L.sufb200_myl7_dcf_eval(self.h, group, in_bits, _t_ptr(d_keys), key_bytes, int(broadcast),
                                            _t_ptr(d_xs), n, out_bytes, _t_ptr(d_out), _stream_ptr(stream)))
        return d_out

    def myl7_eval_host(self, group: int, in_bits: int, keys: np.ndarray, key_bytes: int, broadcast: bool,
                       xs: np.ndarray, out_bytes: int, outs: np.ndarray | None = None) -> np.ndarray:
        keys = np.ascontiguousarray(keys, dtype=np.uint8)
        xs = np.ascontiguousarray(xs, dtype=np.uint64)
        if outs is None:
            outs = np.zeros((xs.size, out_bytes), dtype=np.uint8)
        check(self._L.sufb200_myl7_dcf_eval_host(self.h, group, in_bits, _np_ptr(keys), key_bytes, int(broadcast),
                                                 _np_ptr(xs), xs.size, out_bytes, _np_ptr(outs)))
        return outs

    # -- truncation bundles ---------------------------------------------------
    @staticmethod
    def trunc_gen(kind: int, frac_bits: int, seed: int):
        d0, d1 = TruncDesc(), TruncDesc()
        thetas = np.zeros(4, dtype=np.uint64)
        r_in = C.c_uint64()
        check(_lib.lib().sufb200_trunc_gen(kind, frac_bits, C.c_uint64(seed), C.byref(d0), C.byref(d1),
                                           _np_ptr(thetas), C.byref(r_in)))
        return int(r_in.value), d0, d1, thetas

    def trunc_bundle_eval(self, desc: TruncDesc, keys: Sequence[np.ndarray], d_xhat, d_y=None, d_bools=None,
                          stream=None):
        import torch

        n = d_xhat.numel()
        if d_y is None:
            d_y = torch.empty(n, dtype=torch.int64, device=d_xhat.device)
        nq = int(desc.nq)
        karr = [np.ascontiguousarray(k, dtype=np.uint8) for k in keys[:nq]]
        ptrs = (C.c_void_p * 4)(*[_np_ptr(k) for k in karr], *([None] * (4 - nq)))
        sizes = (C.c_size_t * 4)(*[k.size for k in karr], *([0] * (4 - nq)))
        check(self._L.sufb200_trunc_bundle_eval(self.h, C.byref(desc), C.cast(ptrs, C.c_void_p),
                                                C.cast(sizes, C.c_void_p), _t_ptr(d_xhat), n, _t_ptr(d_y),
                                                _t_ptr(d_bools) if d_bools is not None else None,
                                                _stream_ptr(stream)))
        return d_y

    @staticmethod
    def trunc_gen_elem(kind: int, frac_bits: int, seed: int, n: int):
        """Per-element gates (sufb200_trunc_gen_elem): (r_in [n], shape0,
        shape1, words0 [n][6], words1 [n][6], thetas [n][4])."""
        s0, s1 = TruncDesc(), TruncDesc()
        w0 = np.zeros((n, 6), dtype=np.uint64)
        w1 = np.zeros((n, 6), dtype=np.uint64)
        th = np.zeros((n, 4), dtype=np.uint64)
        r = np.zeros(n, dtype=np.uint64)
        check(_lib.lib().sufb200_trunc_gen_elem(kind, frac_bits, C.c_uint64(seed), n, C.byref(s0), C.byref(s1),
                                                _np_ptr(w0), _np_ptr(w1), _np_ptr(th), _np_ptr(r)))
        return r, s0, s1, w0, w1, th

    def trunc_bundle_eval_elem(self, shape: TruncDesc, d_keys: Sequence, key_bytes: Sequence[int], d_words, d_xhat,
                               d_y=None, d_bools=None, stream=None):
        """One party's per-element gates: d_keys[q] is slot q's [n][key_bytes[q]]
        device key array, d_words the party's [n][6] device words."""
        import torch

        n = d_xhat.numel()
        if d_y is None:
            d_y = torch.empty(n, dtype=torch.int64, device=d_xhat.device)
        nq = int(shape.nq)
        ptrs = (C.c_void_p * 4)(*[_t_ptr(k) for k in d_keys[:nq]], *([None] * (4 - nq)))
        sizes = (C.c_size_t * 4)(*[int(b) for b in key_bytes[:nq]], *([0] * (4 - nq)))
        check(self._L.sufb200_trunc_bundle_eval_elem(self.h, C.byref(shape), C.cast(ptrs, C.c_void_p),
                                                     C.cast(sizes, C.c_void_p), _t_ptr(d_words), _t_ptr(d_xhat), n,
                                                     _t_ptr(d_y), _t_ptr(d_bools) if d_bools is not None else None,
                                                     _stream_ptr(stream)))
        return d_y

    # -- composite tapes (gates::write_composite_tape format) -------------------
    @staticmethod
    def trunc_write_tapes(kind: int, frac_bits: int, seed: int, keys0: Sequence[np.ndarray],
                          keys1: Sequence[np.ndarray], bit_order: int = 1) -> tuple[bytes, bytes]:
        """Both parties' composite tapes of the gate trunc_gen(kind, frac_bits,
        seed) deals, with its queries' myl7 keys (composite_write_tapes)."""
        L = _lib.lib()
        nk = len(keys0)
        k0 = [np.ascontiguousarray(k, dtype=np.uint8) for k in keys0]
        k1 = [np.ascontiguousarray(k, dtype=np.uint8) for k in keys1]
        p0 = (C.c_void_p * max(nk, 1))(*[_np_ptr(k) for k in k0])
        p1 = (C.c_void_p * max(nk, 1))(*[_np_ptr(k) for k in k1])
        sizes = (C.c_size_t * max(nk, 1))(*[k.size for k in k0])
        n = C.c_size_t()
        args = (kind, frac_bits, C.c_uint64(seed), bit_order, C.cast(p0, C.c_void_p), C.cast(p1, C.c_void_p),
                C.cast(sizes, C.c_void_p), nk)
        check(L.sufb200_trunc_write_tapes(*args, None, None, 0, C.byref(n)))
        t0 = np.zeros(n.value, dtype=np.uint8)
        t1 = np.zeros(n.value, dtype=np.uint8)
        check(L.sufb200_trunc_write_tapes(*args, _np_ptr(t0), _np_ptr(t1), n.value, C.byref(n)))
        return t0.tobytes(), t1.tobytes()

    @staticmethod
    def trunc_read_tape(tape: bytes, kind: int, r_in: int, party: int):
        """(desc, [key arrays], r_in share) of one party's composite tape of a
        truncation gate of `kind` with mask r_in (read_composite_tape)."""
        buf = np.frombuffer(bytes(tape), dtype=np.uint8).copy()
        d = TruncDesc()
        off = (C.c_size_t * 4)()
        kb = (C.c_size_t * 4)()
        share = C.c_uint64()
        check(_lib.lib().sufb200_trunc_read_tape(_np_ptr(buf), buf.size, kind, C.c_uint64(r_in), party, C.byref(d),
                                                 C.cast(off, C.c_void_p), C.cast(kb, C.c_void_p), C.byref(share)))
        keys = [buf[off[q]:off[q] + kb[q]].copy() for q in range(int(d.nq))]
        return d, keys, int(share.value)

    @staticmethod
    def trunc_gen_elem_rin_shares(kind: int, frac_bits: int, seed: int, n: int) -> np.ndarray:
        """Party 0's r_in shares of trunc_gen_elem's n gates (party 1's: r_in - these)."""
        out = np.zeros(n, dtype=np.uint64)
        check(_lib.lib().sufb200_trunc_gen_elem_rin_shares(kind, frac_bits, C.c_uint64(seed), n, _np_ptr(out)))
        return out

    def trunc_write_tapes_elem(self, shape: TruncDesc, d_keys: Sequence, key_bytes: Sequence[int], d_words, d_r_in,
                               d_r_in_share, bit_order: int = 1, stream=None):
        """One party's per-element tapes on the device: ([n][stride] uint8, [n] lengths)."""
        import torch

        n = d_r_in.numel()
        nq = int(shape.nq)
        sizes = (C.c_size_t * 4)(*[int(b) for b in key_bytes[:nq]], *([0] * (4 - nq)))
        stride = int(self._L.sufb200_trunc_tape_elem_stride(C.byref(shape), C.cast(sizes, C.c_void_p)))
        if stride == 0:
            raise SufB200Error(_lib.ERR_INVALID, "bad per-element shape")
        out = torch.empty((n, stride), dtype=torch.uint8, device=d_r_in.device)
        lens = torch.empty(n, dtype=torch.int64, device=d_r_in.device)
        ptrs = (C.c_void_p * 4)(*[_t_ptr(k) for k in d_keys[:nq]], *([None] * (4 - nq)))
        check(self._L.sufb200_trunc_write_tapes_elem(self.h, C.byref(shape), C.cast(ptrs, C.c_void_p),
                                                     C.cast(sizes, C.c_void_p), _t_ptr(d_words), _t_ptr(d_r_in),
                                                     _t_ptr(d_r_in_share), n, bit_order, _t_ptr(out), stride,
                                                     _t_ptr(lens), _stream_ptr(stream)))
        return out, lens

    def elem_keys_to_soa(self, in_bits: int, party: int, d_keys, n: int, stream=None):
        """One slot's n per-element keys (device [n][key_bytes]) in the
        level-major layout the per-element kernel reads coalesced."""
        import torch

        nbytes = int(self._L.sufb200_elem_keys_soa_bytes(in_bits, n))
        out = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=d_keys.device)
        check(self._L.sufb200_elem_keys_to_soa(self.h, in_bits, party, _t_ptr(d_keys), myl7_key_bytes(in_bits, 8), n,
                                               _t_ptr(out), _stream_ptr(stream)))
        return out

    def trunc_bundle_eval_elem_soa(self, shape: TruncDesc, d_soa: Sequence, d_words, d_xhat, d_y=None,
                                   d_bools=None, stream=None):
        """trunc_bundle_eval_elem over level-major key layouts (elem_keys_to_soa)."""
        import torch

        n = d_xhat.numel()
        if d_y is None:
            d_y = torch.empty(n, dtype=torch.int64, device=d_xhat.device)
        nq = int(shape.nq)
        ptrs = (C.c_void_p * 4)(*[_t_ptr(k) for k in d_soa[:nq]], *([None] * (4 - nq)))
        check(self._L.sufb200_trunc_bundle_eval_elem_soa(self.h, C.byref(shape), C.cast(ptrs, C.c_void_p),
                                                         _t_ptr(d_words), _t_ptr(d_xhat), n, _t_ptr(d_y),
                                                         _t_ptr(d_bools) if d_bools is not None else None,
                                                         _stream_ptr(stream)))
        return d_y

    def trunc_bundle_eval_host(self, desc: TruncDesc, keys: Sequence[np.ndarray], xhat: np.ndarray,
                               y: np.ndarray | None = None, bools: np.ndarray | None = None) -> np.ndarray:
        """Host buffers in and out (pinned memory makes the copies true DMA)."""
        xhat = np.ascontiguousarray(xhat, dtype=np.uint64)
        if y is None:
            y = np.empty(xhat.size, dtype=np.uint64)
        nq = int(desc.nq)
        karr = [np.ascontiguousarray(k, dtype=np.uint8) for k in keys[:nq]]
        ptrs = (C.c_void_p * 4)(*[_np_ptr(k) for k in karr], *([None] * (4 - nq)))
        sizes = (C.c_size_t * 4)(*[k.size for k in karr], *([0] * (4 - nq)))
        check(self._L.sufb200_trunc_bundle_eval_host(self.h, C.byref(desc), C.cast(ptrs, C.c_void_p),
                                                     C.cast(sizes, C.c_void_p), _np_ptr(xhat), xhat.size,
                                                     _np_ptr(y), _np_ptr(bools) if bools is not None else None))
        return y

    # -- reference GPU-backend formats ------------------------------------------
    def thr_dcf_eval(self, in_bits, d_keys, key_bytes, broadcast, d_xs, out_bytes, d_out=None, stream=None):
        import torch

        n = d_xs.numel()
        if d_out is None:
            d_out = torch.empty(max(n * out_bytes, 1), dtype=torch.uint8, device=d_xs.device)
        check(self._L.sufb200_thr_dcf_eval(self.h, in_bits, _t_ptr(d_keys), key_bytes, int(broadcast),
                                           _t_ptr(d_xs), n, out_bytes, _t_ptr(d_out), _stream_ptr(stream)))
        return d_out

    def packed_lt_eval(self, d_keys, key_bytes, broadcast, d_xs, in_bits, out_words, idx_base=0, d_out=None,
                       stream=None):
        import torch

        n = d_xs.numel()
        if d_out is None:
            d_out = torch.empty(n * out_words, dtype=torch.int64, device=d_xs.device)
        check(self._L.sufb200_packed_lt_eval(self.h, _t_ptr(d_keys), key_bytes, int(broadcast), _t_ptr(d_xs), n,
                                             in_bits, out_words, C.c_uint64(idx_base), _t_ptr(d_out),
                                             _stream_ptr(stream)))
        return d_out

    def interval_lut_eval(self, d_keys, key_bytes, broadcast, d_xs, out_words, idx_base=0, d_out=None, stream=None):
        import torch

        n = d_xs.numel()
        if d_out is None:
            d_out = torch.empty(n * out_words, dtype=torch.int64, device=d_xs.device)
        check(self._L.sufb200_interval_lut_eval(self.h, _t_ptr(d_keys), key_bytes, int(broadcast), _t_ptr(d_xs), n,
                                                out_words, C.c_uint64(idx_base), _t_ptr(d_out),
                                                _stream_ptr(stream)))
        return d_out


def coeff_lut_eval(ctx: "Context", key: np.ndarray, d_xhat, r: int, degree: int, r_out=None, ring_bits: int = 64,
                   idx_base: int = 0, d_out=None, stream=None):
    """sufb200_coeff_lut_eval: the composite coefficient gate (interval-LUT
    coefficients, polynomial over the public x^, output masks) in one pass."""
    import torch

    key = np.ascontiguousarray(key, dtype=np.uint8)
    n = d_xhat.numel()
    if d_out is None:
        d_out = torch.empty(max(n * r, 1), dtype=torch.int64, device=d_xhat.device)
    ro = None if r_out is None else np.ascontiguousarray(r_out, dtype=np.uint64)
    check(ctx._L.sufb200_coeff_lut_eval(ctx.h, _np_ptr(key), key.size, _t_ptr(d_xhat), n, r, degree,
                                        _np_ptr(ro) if ro is not None else None, ring_bits, C.c_uint64(idx_base),
                                        _t_ptr(d_out), _stream_ptr(stream)))
    return d_out


def coeff_lut_eval_pair(ctx: "Context", keys, d_xhat, r: int, degree: int, r_outs=(None, None), ring_bits: int = 64,
                        idx_base: int = 0, d_outs=(None, None), stream=None):
    """sufb200_coeff_lut_eval_pair: both parties' coefficient gates over one
    x^ in one launch; returns (party 0's, party 1's) outputs."""
    import torch

    ks = [np.ascontiguousarray(k, dtype=np.uint8) for k in keys]
    n = d_xhat.numel()
    outs = [d if d is not None else torch.empty(max(n * r, 1), dtype=torch.int64, device=d_xhat.device)
            for d in d_outs]
    ro = [None if v is None else np.ascontiguousarray(v, dtype=np.uint64) for v in r_outs]
    check(ctx._L.sufb200_coeff_lut_eval_pair(ctx.h, _np_ptr(ks[0]), ks[0].size, _np_ptr(ks[1]), ks[1].size,
                                             _t_ptr(d_xhat), n, r, degree,
                                             _np_ptr(ro[0]) if ro[0] is not None else None,
                                             _np_ptr(ro[1]) if ro[1] is not None else None, ring_bits,
                                             C.c_uint64(idx_base), _t_ptr(outs[0]), _t_ptr(outs[1]),
                                             _stream_ptr(stream)))
    return outs[0], outs[1]


# -- paired-GPU open ---------------------------------------------------------------

OPEN_ID_BYTES = 128


def open_unique_id() -> bytes:
    """A fresh NCCL id for sufb200_open_comm_create (made on one rank)."""
    buf = (C.c_uint8 * OPEN_ID_BYTES)()
    check(_lib.lib().sufb200_open_unique_id(C.cast(buf, C.c_void_p)))
    return bytes(buf)


def open_add_local(d_share0, d_share1, ring_bits: int = 64, d_out=None, stream=None):
    """The open when both parties' shares live on this GPU: d_out = share0 +
    share1 mod 2^ring_bits, sign-extended from ring_bits (the add step of
    OpenCollector::flush, src/runtime/open_collector.cpp:357-895, with no
    exchange)."""
    import torch

    if d_share0.numel() != d_share1.numel():
        raise ValueError("the two shares differ in length")
    if d_out is None:
        d_out = torch.empty_like(d_share0)
    check(_lib.lib().sufb200_open_add_to_signed(_t_ptr(d_share0), _t_ptr(d_share1), _t_ptr(d_out),
                                                d_share0.numel(), ring_bits, _stream_ptr(stream)))
    return d_out


def share_open_id(rank: int, group=None) -> bytes:
    """Rank 0 makes the id and every rank of the torch.distributed group gets
    it (any backend: the id is 128 host bytes)."""
    import torch.distributed as dist

    box = [open_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0, group=group)
    return box[0]


class OpenComm:
    """The communicator of the paired-GPU open (sufb200_open_*): party 0 on
    GPU j and party 1 on GPU j + N/2 swap eff_bits-packed shares over NVLink
    and add them, on the caller's stream."""

    def __init__(self, ctx: Context, uid: bytes, nranks: int, rank: int, timeout_s: float = 60.0):
        if len(uid) != OPEN_ID_BYTES:
            raise ValueError("the NCCL id is 128 bytes")
        self._L = ctx._L
        self.ctx = ctx
        self.rank = rank
        self.nranks = nranks
        h = C.c_void_p()
        idb = (C.c_uint8 * OPEN_ID_BYTES).from_buffer_copy(uid)
        check(self._L.sufb200_open_comm_create(ctx.h, C.cast(idb, C.c_void_p), nranks, rank, float(timeout_s),
                                               C.byref(h)))
        self.h = h

    def exchange(self, peer: int, d_local, eff_bits: int, ring_bits: int, signed: bool = False, d_out=None,
                 stream=None):
        import torch

        if d_out is None:
            d_out = torch.empty_like(d_local)
        check(self._L.sufb200_open_exchange(self.h, peer, _t_ptr(d_local), d_local.numel(), eff_bits, ring_bits,
                                            int(signed), _t_ptr(d_out), _stream_ptr(stream)))
        return d_out

    def abort(self) -> None:
        if self.h:
            check(self._L.sufb200_open_comm_abort(self.h))

    def close(self) -> None:
        if self.h:
            h, self.h = self.h, C.c_void_p()
            check(self._L.sufb200_open_comm_destroy(h))


class P2POpen:
    """The paired-GPU open in one kernel (sufb200_p2p_open_*): this rank's
    landing buffer, mapped by the peer, receives the peer's packed shares by
    direct peer stores over NVLink.  `handles` is every rank's export blob
    (share_p2p_handles gathers them); the endpoint connects to `peer`'s."""

    HANDLE_BYTES = 128

    def __init__(self, ctx: Context, max_words: int):
        self._L = ctx._L
        self.ctx = ctx
        h = C.c_void_p()
        buf = (C.c_uint8 * self.HANDLE_BYTES)()
        check(self._L.sufb200_p2p_open_create(ctx.h, int(max_words), C.byref(h), C.cast(buf, C.c_void_p)))
        self.h = h
        self.handle = bytes(buf)

    def connect(self, peer_handle: bytes) -> None:
        buf = (C.c_uint8 * self.HANDLE_BYTES).from_buffer_copy(peer_handle)
        check(self._L.sufb200_p2p_open_connect(self.h, C.cast(buf, C.c_void_p)))

    def connect_self(self) -> None:
        """Loopback: this endpoint becomes its own peer (one-device check of
        the exchange kernel; exchange gives local + (local mod 2^eff_bits))."""
        check(self._L.sufb200_p2p_open_connect_self(self.h))

    def exchange(self, d_local, eff_bits: int, ring_bits: int, signed: bool = False, d_out=None, timeout_s=2.0,
                 stream=None):
        import torch

        if d_out is None:
            d_out = torch.empty_like(d_local)
        check(self._L.sufb200_p2p_open_exchange(self.h, _t_ptr(d_local), d_local.numel(), eff_bits, ring_bits,
                                                int(signed), _t_ptr(d_out), float(timeout_s), _stream_ptr(stream)))
        return d_out

    def close(self) -> None:
        if self.h:
            h, self.h = self.h, C.c_void_p()
            check(self._L.sufb200_p2p_open_destroy(h))


def share_p2p_handles(ep: P2POpen, group=None) -> list:
    """Every rank's P2P export blob, gathered over torch.distributed (any backend)."""
    import torch.distributed as dist

    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, ep.handle, group=group)
    return out


# -- key builders for the reference formats (host) ---------------------------------

def thr_dcf_key(in_bits: int, alpha: int, payload: bytes) -> np.ndarray:
    L = _lib.lib()
    n = int(L.sufb200_thr_dcf_build(in_bits, C.c_uint64(alpha & (2**64 - 1)), None, len(payload), None))
    if n == 0:
        raise SufB200Error(_lib.ERR_INVALID, "bad threshold DCF arguments")
    out = np.zeros(n, dtype=np.uint8)
    pl = np.frombuffer(bytes(payload), dtype=np.uint8).copy() if payload else None
    L.sufb200_thr_dcf_build(in_bits, C.c_uint64(alpha & (2**64 - 1)), _np_ptr(pl) if pl is not None else None,
                            len(payload), _np_ptr(out))
    return out


def seed_from_id(nid: int, tweak: int) -> np.ndarray:
    s = np.zeros(16, dtype=np.uint8)
    check(_lib.lib().sufb200_seed_from_id(C.c_uint64(nid), C.c_uint64(tweak), _np_ptr(s)))
    return s


def packed_lt_key(party: int, nonce: int, in_bits: int, thresholds, seed) -> np.ndarray:
    L = _lib.lib()
    thr = np.ascontiguousarray(thresholds, dtype=np.uint64)
    sd = np.ascontiguousarray(seed, dtype=np.uint8)
    n = int(L.sufb200_packed_lt_build(party, C.c_uint64(nonce), in_bits, None, thr.size, None, None))
    if n == 0:
        raise SufB200Error(_lib.ERR_INVALID, "bad packed-compare arguments")
    out = np.zeros(n, dtype=np.uint8)
    L.sufb200_packed_lt_build(party, C.c_uint64(nonce), in_bits, _np_ptr(thr), thr.size, _np_ptr(sd), _np_ptr(out))
    return out


def interval_lut_key(party: int, nonce: int, in_bits: int, out_words: int, cuts, payload, seed) -> np.ndarray:
    L = _lib.lib()
    cuts = np.ascontiguousarray(cuts, dtype=np.uint64)
    pay = np.ascontiguousarray(payload, dtype=np.uint64)
    sd = np.ascontiguousarray(seed, dtype=np.uint8)
    iv = cuts.size - 1
    n = int(L.sufb200_interval_lut_build(party, C.c_uint64(nonce), in_bits, out_words, None, iv, None, None, None))
    if n == 0:
        raise SufB200Error(_lib.ERR_INVALID, "bad interval-LUT arguments")
    out = np.zeros(n, dtype=np.uint8)
    L.sufb200_interval_lut_build(party, C.c_uint64(nonce), in_bits, out_words, _np_ptr(cuts), iv, _np_ptr(pay),
                                 _np_ptr(sd), _np_ptr(out))
    return out
