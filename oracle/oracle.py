"""Test-infrastructure wrapper around the CPU oracles (never the product).

`Oracle` loads ``oracle/liboracle.so`` (the C restatement in ``suf_oracle.c``);
`RefMyl7` loads ``oracle/_ref/libmyl7ref_{add,xor}.so`` (the reference's own
myl7 DCF sources compiled by ``oracle/Makefile``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs
import this module; the product package ``suf_b200`` never does.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
GROUP_ADD = 0
GROUP_XOR = 1
KIND_TR, KIND_ARS, KIND_GAPARS = 0, 1, 2

_u8p = C.POINTER(C.c_uint8)
_u64p = C.POINTER(C.c_uint64)


def _p8(a: np.ndarray):
    return a.ctypes.data_as(_u8p)


def _p64(a: np.ndarray):
    return a.ctypes.data_as(_u64p)


class TruncDesc(C.Structure):
    """Mirror of ``orc_trunc_desc`` (one party's trunc/ARS bundle material)."""

    _fields_ = [
        ("kind", C.c_int32), ("frac_bits", C.c_int32), ("party", C.c_int32), ("nq", C.c_int32),
        ("q_bits", C.c_int32 * 4), ("q_theta", C.c_uint64 * 4),
        ("carry_a", C.c_int32), ("carry_b", C.c_int32),
        ("sign_a", C.c_int32), ("sign_b", C.c_int32),
        ("wrap_q", C.c_int32), ("pad", C.c_int32),
        ("carry_w", C.c_uint64), ("sign_w", C.c_uint64),
        ("haty", C.c_uint64), ("r_hi", C.c_uint64), ("m", C.c_uint64),
    ]


def desc_from_fields(src) -> TruncDesc:
    """Copy a bundle descriptor with the same field names (e.g. the product's
    sufb200_trunc_desc mirror) into the oracle's layout."""
    d = TruncDesc()
    for name in ("kind", "frac_bits", "party", "nq", "carry_a", "carry_b", "sign_a", "sign_b", "wrap_q",
                 "carry_w", "sign_w", "haty", "r_hi", "m"):
        setattr(d, name, getattr(src, name))
    for i in range(4):
        d.q_bits[i] = src.q_bits[i]
    return d


def reference_root() -> Path | None:
    """The reference checkout, if this machine has one: $SUF_REFERENCE, else
    the `reference_path` that BASELINE.json at the repository root records.
    None when neither names an existing directory (as on a GPU box, which
    only uses the prebuilt oracle/_ref files)."""
    cand = os.environ.get("SUF_REFERENCE")
    if not cand:
        import json

        try:
            cand = json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            cand = None
    return Path(cand) if cand and Path(cand).is_dir() else None


def build_oracle(quiet: bool = True) -> None:
    """Compile liboracle.so (and oracle/_ref when the reference is present)."""
    import subprocess

    targets = ["oracle"]
    ref = reference_root()
    extra = []
    if ref is not None and (ref / "third_party" / "myl7_fss").is_dir():
        extra = [f"REF={ref}"]
        targets.append("ref")
        if (HERE.parent / "suf_b200" / "libsufb200.so").exists():
            targets += ["drive", "softmax", "refgpu"]
    subprocess.run(["make", "-C", str(HERE), f"-j{os.cpu_count() or 1}"] + extra + targets, check=True,
                   stdout=subprocess.DEVNULL if quiet else None, stderr=subprocess.DEVNULL if quiet else None)


class Oracle:
    def __init__(self, path: str | os.PathLike | None = None):
        p = Path(path) if path else HERE / "liboracle.so"
        if not p.exists():
            build_oracle()
        L = C.CDLL(str(p))
        self.L = L
        L.orc_mt64_fill.argtypes = [C.c_uint64, _u64p, C.c_size_t]
        L.orc_aes128_ecb.argtypes = [_u8p, _u8p, _u8p, C.c_size_t]
        L.orc_aes128_expand.argtypes = [_u8p, _u8p]
        L.orc_prg_init.argtypes = [_u8p, C.c_size_t]
        L.orc_myl7_key_bytes.argtypes = [C.c_int, C.c_int]
        L.orc_myl7_key_bytes.restype = C.c_size_t
        L.orc_myl7_gen_key_pair.argtypes = [C.c_int, C.c_int, C.c_uint64, _u8p, C.c_int, _u8p, _u8p, _u8p, _u8p]
        L.orc_myl7_eval_many.argtypes = [C.c_int, _u8p, C.c_size_t, C.c_int, _u64p, C.c_size_t, _u8p, C.c_int]
        L.orc_seed_from_id.argtypes = [C.c_uint64, C.c_uint64, _u8p]
        L.orc_thr_dcf_build.argtypes = [C.c_int, C.c_uint64, _u8p, C.c_int, _u8p]
        L.orc_thr_dcf_build.restype = C.c_size_t
        L.orc_thr_dcf_eval_many.argtypes = [C.c_int, _u8p, C.c_size_t, C.c_int, _u64p, C.c_size_t, C.c_int, _u8p]
        L.orc_packed_key_build.argtypes = [C.c_int, C.c_uint64, C.c_int, _u64p, C.c_int, _u8p, _u8p]
        L.orc_packed_key_build.restype = C.c_size_t
        L.orc_packed_eval_many.argtypes = [_u8p, C.c_size_t, C.c_int, _u64p, C.c_size_t, C.c_uint64, C.c_int, _u64p]
        L.orc_interval_key_build.argtypes = [C.c_int, C.c_uint64, C.c_int, C.c_int, _u64p, C.c_int, _u64p, _u8p, _u8p]
        L.orc_interval_key_build.restype = C.c_size_t
        L.orc_interval_eval_many.argtypes = [_u8p, C.c_size_t, C.c_int, _u64p, C.c_size_t, C.c_uint64, C.c_int, _u64p]
        L.orc_trunc_gen.argtypes = [C.c_int, C.c_int, C.c_uint64, C.POINTER(TruncDesc), C.POINTER(TruncDesc)]
        L.orc_trunc_gen.restype = C.c_uint64
        L.orc_trunc_combine.argtypes = [C.POINTER(TruncDesc), _u64p, _u64p, C.c_size_t, _u64p, _u64p]
        L.orc_pack_eff_bits.argtypes = [_u64p, C.c_size_t, C.c_int, _u64p, C.c_size_t]
        L.orc_unpack_eff_bits.argtypes = [_u64p, C.c_size_t, C.c_int, _u64p]
        L.orc_beaver_mul.argtypes = [C.c_int] + [_u64p] * 6 + [C.c_size_t]
        L.orc_horner_cubic.argtypes = [_u64p] * 6 + [C.c_size_t]
        L.orc_row_sum.argtypes = [_u64p, C.c_int, C.c_int, C.POINTER(C.c_int), _u64p]
        L.orc_row_variance.argtypes = [_u64p, _u64p, C.c_int, C.c_int, C.POINTER(C.c_int), _u64p]

    # -- rng / AES -----------------------------------------------------------
    def mt64(self, seed: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint64)
        self.L.orc_mt64_fill(C.c_uint64(seed), _p64(out), n)
        return out

    def aes_ecb(self, key: bytes, blocks: np.ndarray) -> np.ndarray:
        k = np.frombuffer(bytes(key), dtype=np.uint8).copy()
        b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 16)
        out = np.empty_like(b)
        self.L.orc_aes128_ecb(_p8(k), _p8(b), _p8(out), b.shape[0])
        return out

    def aes_expand(self, key: bytes) -> np.ndarray:
        k = np.frombuffer(bytes(key), dtype=np.uint8).copy()
        rk = np.empty(176, dtype=np.uint8)
        self.L.orc_aes128_expand(_p8(k), _p8(rk))
        return rk

    # -- myl7 DCF ------------------------------------------------------------
    def prg_init(self, state: np.ndarray) -> None:
        s = np.ascontiguousarray(state, dtype=np.uint8)
        self.L.orc_prg_init(_p8(s), s.size)

    def myl7_key_bytes(self, in_bits: int, payload_len: int) -> int:
        return int(self.L.orc_myl7_key_bytes(in_bits, payload_len))

    def myl7_gen(self, group: int, in_bits: int, alpha: int, payload: bytes, seed0: np.ndarray, seed1: np.ndarray):
        kb = self.myl7_key_bytes(in_bits, len(payload))
        k0 = np.zeros(kb, dtype=np.uint8)
        k1 = np.zeros(kb, dtype=np.uint8)
        pl = np.frombuffer(bytes(payload), dtype=np.uint8).copy()
        s0 = np.ascontiguousarray(seed0, dtype=np.uint8)
        s1 = np.ascontiguousarray(seed1, dtype=np.uint8)
        rc = self.L.orc_myl7_gen_key_pair(group, in_bits, C.c_uint64(alpha & (2**64 - 1)), _p8(pl), len(payload),
                                          _p8(s0), _p8(s1), _p8(k0), _p8(k1))
        if rc:
            raise RuntimeError(f"orc_myl7_gen_key_pair rc={rc}")
        return k0, k1

    def myl7_eval(self, group: int, keys: np.ndarray, key_bytes: int, broadcast: bool, xs: np.ndarray,
                  out_len: int) -> np.ndarray:
        xs = np.ascontiguousarray(xs, dtype=np.uint64)
        keys = np.ascontiguousarray(keys, dtype=np.uint8)
        out = np.zeros((xs.size, out_len), dtype=np.uint8)
        rc = self.L.orc_myl7_eval_many(group, _p8(keys), key_bytes, int(broadcast), _p64(xs), xs.size, _p8(out),
                                       out_len)
        if rc:
            raise RuntimeError(f"orc_myl7_eval_many rc={rc}")
        return out

    # -- reference GPU key formats -------------------------------------------
    def seed_from_id(self, nid: int, tweak: int) -> np.ndarray:
        s = np.empty(16, dtype=np.uint8)
        self.L.orc_seed_from_id(C.c_uint64(nid), C.c_uint64(tweak), _p8(s))
        return s

    def thr_dcf_key(self, in_bits: int, alpha: int, payload: bytes) -> np.ndarray:
        out = np.zeros(12 + len(payload), dtype=np.uint8)
        pl = np.frombuffer(bytes(payload), dtype=np.uint8).copy() if payload else np.zeros(1, np.uint8)
        self.L.orc_thr_dcf_build(in_bits, C.c_uint64(alpha), _p8(pl), len(payload), _p8(out))
        return out

    def thr_dcf_eval(self, in_bits, keys, key_bytes, broadcast, xs, out_bytes):
        xs = np.ascontiguousarray(xs, dtype=np.uint64)
        out = np.zeros((xs.size, out_bytes), dtype=np.uint8)
        self.L.orc_thr_dcf_eval_many(in_bits, _p8(np.ascontiguousarray(keys, np.uint8)), key_bytes,
                                     int(broadcast), _p64(xs), xs.size, out_bytes, _p8(out))
        return out

    def packed_key(self, party, nonce, in_bits, thresholds, seed) -> np.ndarray:
        thr = np.ascontiguousarray(thresholds, dtype=np.uint64)
        out = np.zeros(208 + 8 * thr.size, dtype=np.uint8)
        self.L.orc_packed_key_build(party, C.c_uint64(nonce), in_bits, _p64(thr), thr.size,
                                    _p8(np.ascontiguousarray(seed, np.uint8)), _p8(out))
        return out

    def packed_eval(self, keys, key_bytes, broadcast, xs, out_words, idx_base=0):
        xs = np.ascontiguousarray(xs, dtype=np.uint64)
        out = np.zeros((xs.size, out_words), dtype=np.uint64)
        rc = self.L.orc_packed_eval_many(_p8(np.ascontiguousarray(keys, np.uint8)), key_bytes, int(broadcast),
                                         _p64(xs), xs.size, C.c_uint64(idx_base), out_words, _p64(out))
        if rc:
            raise RuntimeError(f"orc_packed_eval_many rc={rc}")
        return out

    def interval_key(self, party, nonce, in_bits, out_words, cuts, payload, seed) -> np.ndarray:
        cuts = np.ascontiguousarray(cuts, dtype=np.uint64)
        pay = np.ascontiguousarray(payload, dtype=np.uint64)
        iv = cuts.size - 1
        out = np.zeros(216 + 8 * cuts.size + 8 * pay.size, dtype=np.uint8)
        self.L.orc_interval_key_build(party, C.c_uint64(nonce), in_bits, out_words, _p64(cuts), iv, _p64(pay),
                                      _p8(np.ascontiguousarray(seed, np.uint8)), _p8(out))
        return out

    def interval_eval(self, keys, key_bytes, broadcast, xs, out_words, idx_base=0):
        xs = np.ascontiguousarray(xs, dtype=np.uint64)
        out = np.zeros((xs.size, out_words), dtype=np.uint64)
        rc = self.L.orc_interval_eval_many(_p8(np.ascontiguousarray(keys, np.uint8)), key_bytes, int(broadcast),
                                           _p64(xs), xs.size, C.c_uint64(idx_base), out_words, _p64(out))
        if rc:
            raise RuntimeError(f"orc_interval_eval_many rc={rc}")
        return out

    # -- truncation bundles ----------------------------------------------------
    def trunc_gen(self, kind: int, f: int, seed: int):
        d0, d1 = TruncDesc(), TruncDesc()
        r = self.L.orc_trunc_gen(kind, f, C.c_uint64(seed), C.byref(d0), C.byref(d1))
        return int(r), d0, d1

    def trunc_combine(self, desc: TruncDesc, xhat: np.ndarray, pred: np.ndarray, want_bools=False):
        xhat = np.ascontiguousarray(xhat, dtype=np.uint64)
        pred = np.ascontiguousarray(pred, dtype=np.uint64)
        n = xhat.size
        y = np.zeros(n, dtype=np.uint64)
        bools = np.zeros((n, 3), dtype=np.uint64) if want_bools else None
        self.L.orc_trunc_combine(C.byref(desc), _p64(xhat), _p64(pred), n, _p64(y),
                                 _p64(bools) if want_bools else None)
        return (y, bools) if want_bools else y

    # -- primitives ------------------------------------------------------------
    def pack_eff_bits(self, xs, eff_bits):
        xs = np.ascontiguousarray(xs, dtype=np.uint64)
        words = (xs.size * eff_bits + 63) // 64 if eff_bits < 64 else xs.size
        out = np.zeros(max(words, 1), dtype=np.uint64)
        self.L.orc_pack_eff_bits(_p64(xs), xs.size, eff_bits, _p64(out), words)
        return out[:words]

    def unpack_eff_bits(self, packed, n, eff_bits):
        packed = np.ascontiguousarray(np.concatenate([packed, np.zeros(1, np.uint64)]), dtype=np.uint64)
        out = np.zeros(n, dtype=np.uint64)
        self.L.orc_unpack_eff_bits(_p64(packed), n, eff_bits, _p64(out))
        return out

    def beaver_mul(self, party, a, b, c, d, e):
        arrs = [np.ascontiguousarray(v, dtype=np.uint64) for v in (a, b, c, d, e)]
        z = np.zeros_like(arrs[0])
        self.L.orc_beaver_mul(party, *[_p64(v) for v in arrs], _p64(z), z.size)
        return z

    def horner_cubic(self, x, c0, c1, c2, c3):
        arrs = [np.ascontiguousarray(v, dtype=np.uint64) for v in (x, c0, c1, c2, c3)]
        out = np.zeros_like(arrs[0])
        self.L.orc_horner_cubic(*[_p64(v) for v in arrs], _p64(out), out.size)
        return out

    def row_sum(self, mat, valid=None):
        mat = np.ascontiguousarray(mat, dtype=np.uint64)
        rows, cols = mat.shape
        out = np.zeros(rows, dtype=np.uint64)
        vp = None
        if valid is not None:
            valid = np.ascontiguousarray(valid, dtype=np.int32)
            vp = valid.ctypes.data_as(C.POINTER(C.c_int))
        self.L.orc_row_sum(_p64(mat), rows, cols, vp, _p64(out))
        return out

    def row_variance(self, mat, mean, valid=None):
        mat = np.ascontiguousarray(mat, dtype=np.uint64)
        mean = np.ascontiguousarray(mean, dtype=np.uint64)
        rows, cols = mat.shape
        out = np.zeros(rows, dtype=np.uint64)
        vp = None
        if valid is not None:
            valid = np.ascontiguousarray(valid, dtype=np.int32)
            vp = valid.ctypes.data_as(C.POINTER(C.c_int))
        self.L.orc_row_variance(_p64(mat), _p64(mean), rows, cols, vp, _p64(out))
        return out


class RefMyl7:
    """The reference's own myl7 DCF code (oracle/_ref), for pinning."""

    def __init__(self, group: int = GROUP_ADD):
        name = "libmyl7ref_add.so" if group == GROUP_ADD else "libmyl7ref_xor.so"
        p = HERE / "_ref" / name
        if not p.exists():
            raise FileNotFoundError(f"{p} not built (needs the reference checkout at build time)")
        L = C.CDLL(str(p))
        self.L = L
        L.ref_prg_init.argtypes = [_u8p, C.c_int]
        L.ref_gen_seeded.argtypes = [C.c_int, C.c_uint64, _u8p, C.c_int, _u8p, _u8p, _u8p, _u8p]
        L.ref_adapter_gen.argtypes = [C.c_int, C.c_uint64, _u8p, C.c_int, _u8p, _u8p, C.c_size_t]
        L.ref_adapter_eval_many.argtypes = [C.c_int, _u8p, C.c_size_t, C.c_int, _u64p, C.c_size_t, _u8p, C.c_int]
        L.ref_eval_many_omp.argtypes = [C.c_int, _u8p, C.c_size_t, C.c_int, _u64p, C.c_size_t, _u8p, C.c_int]
        L.ref_set_threads.argtypes = [C.c_int]
        L.ref_set_threads.restype = C.c_int

    @staticmethod
    def available(group: int = GROUP_ADD) -> bool:
        name = "libmyl7ref_add.so" if group == GROUP_ADD else "libmyl7ref_xor.so"
        return (HERE / "_ref" / name).exists()

    def prg_init(self, state: np.ndarray) -> None:
        s = np.ascontiguousarray(state, dtype=np.uint8)
        rc = self.L.ref_prg_init(_p8(s), s.size)
        if rc:
            raise RuntimeError(f"ref_prg_init rc={rc}")

    def gen_seeded(self, in_bits, alpha, payload: bytes, seed0, seed1):
        kb = 8 + ((len(payload) + 15) // 16) * (32 + 33 * in_bits)
        k0 = np.zeros(kb, dtype=np.uint8)
        k1 = np.zeros(kb, dtype=np.uint8)
        pl = np.frombuffer(bytes(payload), dtype=np.uint8).copy()
        rc = self.L.ref_gen_seeded(in_bits, C.c_uint64(alpha & (2**64 - 1)), _p8(pl), len(payload),
                                   _p8(np.ascontiguousarray(seed0, np.uint8)),
                                   _p8(np.ascontiguousarray(seed1, np.uint8)), _p8(k0), _p8(k1))
        if rc:
            raise RuntimeError(f"ref_gen_seeded rc={rc}")
        return k0, k1

    def adapter_gen(self, in_bits, alpha, payload: bytes):
        cap = 8 + ((len(payload) + 15) // 16) * (32 + 33 * in_bits)
        k0 = np.zeros(cap, dtype=np.uint8)
        k1 = np.zeros(cap, dtype=np.uint8)
        pl = np.frombuffer(bytes(payload), dtype=np.uint8).copy()
        n = self.L.ref_adapter_gen(in_bits, C.c_uint64(alpha & (2**64 - 1)), _p8(pl), len(payload), _p8(k0),
                                   _p8(k1), cap)
        if n < 0:
            raise RuntimeError(f"ref_adapter_gen rc={n}")
        return k0[:n], k1[:n]

    def adapter_eval(self, in_bits, keys, key_bytes, broadcast, xs, out_len):
        xs = np.ascontiguousarray(xs, dtype=np.uint64)
        out = np.zeros((xs.size, out_len), dtype=np.uint8)
        rc = self.L.ref_adapter_eval_many(in_bits, _p8(np.ascontiguousarray(keys, np.uint8)), key_bytes,
                                          int(broadcast), _p64(xs), xs.size, _p8(out), out_len)
        if rc:
            raise RuntimeError(f"ref_adapter_eval_many rc={rc}")
        return out

    def set_threads(self, n: int) -> int:
        """OpenMP threads of eval_omp (n <= 0 leaves it); returns the count in effect."""
        return int(self.L.ref_set_threads(int(n)))

    def eval_omp(self, in_bits, keys, key_bytes, broadcast, xs, out_len):
        xs = np.ascontiguousarray(xs, dtype=np.uint64)
        out = np.zeros((xs.size, out_len), dtype=np.uint8)
        rc = self.L.ref_eval_many_omp(in_bits, _p8(np.ascontiguousarray(keys, np.uint8)), key_bytes,
                                      int(broadcast), _p64(xs), xs.size, _p8(out), out_len)
        if rc:
            raise RuntimeError(f"ref_eval_many_omp rc={rc}")
        return out
