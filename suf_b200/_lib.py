"""ctypes binding of libsufb200.so (include/sufb200.h).

The library is loaded from this package directory; importing this module
raises if it is missing, so no Python path can silently stand in for the
CUDA kernels.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libsufb200.so"

OK = 0
ERR_INVALID = -1
ERR_CUDA = -2
ERR_KEY = -3
ERR_UNSUPPORTED = -4
ERR_NOT_READY = -5
ERR_COMM = -6

GROUP_ADD = 0
GROUP_XOR = 1

TRUNC_FAITHFUL_TR = 0
TRUNC_FAITHFUL_ARS = 1
TRUNC_GAPARS = 2

NOALLOC_KEY_BYTES = 16384  # SUFB200_NOALLOC_KEY_BYTES


class SufB200Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"sufb200 error {code}: {msg}")
        self.code = code


class TruncDesc(C.Structure):
    """Mirror of sufb200_trunc_desc."""

    _fields_ = [
        ("kind", C.c_int32), ("frac_bits", C.c_int32), ("party", C.c_int32), ("nq", C.c_int32),
        ("q_bits", C.c_int32 * 4),
        ("carry_a", C.c_int32), ("carry_b", C.c_int32), ("sign_a", C.c_int32), ("sign_b", C.c_int32),
        ("wrap_q", C.c_int32), ("reserved", C.c_int32),
        ("carry_w", C.c_uint64), ("sign_w", C.c_uint64), ("haty", C.c_uint64), ("r_hi", C.c_uint64),
        ("m", C.c_uint64),
    ]


_vp = C.c_void_p
_sz = C.c_size_t
_u64 = C.c_uint64
_i = C.c_int

# name -> (restype, argtypes)
_SIGS = {
    "sufb200_version": (_i, []),
    "sufb200_last_error": (C.c_char_p, []),
    "sufb200_ctx_create": (_i, [_i, C.POINTER(_vp)]),
    "sufb200_ctx_destroy": (_i, [_vp]),
    "sufb200_ctx_sync": (_i, [_vp, _vp]),
    "sufb200_ctx_sm_count": (_i, [_vp]),
    "sufb200_probe_aes_engine": (_i, [_vp, C.POINTER(C.c_double)]),
    "sufb200_prg_init": (_i, [_vp, _vp, _sz]),
    "sufb200_myl7_key_bytes": (_sz, [_i, _i]),
    "sufb200_myl7_gen": (_i, [_vp, _i, _i, _u64, _vp, _i, _vp, _vp, _vp, _vp]),
    "sufb200_myl7_gen_batch": (_i, [_vp, _i, _i, _vp, _sz, _vp, _i, _vp, _vp, _vp, _vp]),
    "sufb200_myl7_dcf_eval": (_i, [_vp, _i, _i, _vp, _sz, _i, _vp, _sz, _i, _vp, _vp]),
    "sufb200_myl7_dcf_eval_host": (_i, [_vp, _i, _i, _vp, _sz, _i, _vp, _sz, _i, _vp]),
    "sufb200_trunc_gen": (_i, [_i, _i, _u64, C.POINTER(TruncDesc), C.POINTER(TruncDesc), _vp, _vp]),
    "sufb200_trunc_bundle_eval": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, _vp, _sz, _vp, _vp, _vp]),
    "sufb200_trunc_bundle_eval_jobs": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, _vp, _vp, _vp, _i, _vp]),
    "sufb200_trunc_bundle_eval_pair": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, C.POINTER(TruncDesc), _vp, _vp, _vp,
                                            _sz, _vp, _vp, _vp]),
    "sufb200_trunc_bundle_eval_pair_dev": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, C.POINTER(TruncDesc), _vp, _vp,
                                                _vp, _sz, _vp, _vp, _vp]),
    "sufb200_trunc_tables_bytes": (_sz, [C.POINTER(TruncDesc)]),
    "sufb200_trunc_tables_dev": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, _vp, _sz, _vp]),
    "sufb200_trunc_tables_many_dev": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sufb200_trunc_bundle_eval_pair_tables_dev": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, _vp, C.POINTER(TruncDesc),
                                                       _vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp]),
    "sufb200_trunc_bundle_eval_host": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, _vp, _sz, _vp, _vp]),
    "sufb200_trunc_bundle_eval_noalloc": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, _vp, _sz, _vp, _vp, _vp]),
    "sufb200_trunc_gen_elem": (_i, [_i, _i, _u64, _sz, C.POINTER(TruncDesc), C.POINTER(TruncDesc), _vp, _vp, _vp,
                                    _vp]),
    "sufb200_trunc_bundle_eval_elem": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp]),
    "sufb200_elem_keys_soa_bytes": (_sz, [_i, _sz]),
    "sufb200_elem_keys_to_soa": (_i, [_vp, _i, _i, _vp, _sz, _sz, _vp, _vp]),
    "sufb200_trunc_bundle_eval_elem_soa": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, _vp, _sz, _vp, _vp, _vp]),
    "sufb200_trunc_write_tapes": (_i, [_i, _i, _u64, _i, _vp, _vp, _vp, _i, _vp, _vp, _sz, _vp]),
    "sufb200_trunc_read_tape": (_i, [_vp, _sz, _i, _u64, _i, C.POINTER(TruncDesc), _vp, _vp, _vp]),
    "sufb200_trunc_gen_elem_rin_shares": (_i, [_i, _i, _u64, _sz, _vp]),
    "sufb200_trunc_tape_elem_stride": (_sz, [C.POINTER(TruncDesc), _vp]),
    "sufb200_trunc_write_tapes_elem": (_i, [_vp, C.POINTER(TruncDesc), _vp, _vp, _vp, _vp, _vp, _sz, _i, _vp, _sz,
                                            _vp, _vp]),
    "sufb200_thr_dcf_build": (_sz, [_i, _u64, _vp, _i, _vp]),
    "sufb200_thr_dcf_eval": (_i, [_vp, _i, _vp, _sz, _i, _vp, _sz, _i, _vp, _vp]),
    "sufb200_packed_lt_build": (_sz, [_i, _u64, _i, _vp, _i, _vp, _vp]),
    "sufb200_packed_lt_eval": (_i, [_vp, _vp, _sz, _i, _vp, _sz, _i, _i, _u64, _vp, _vp]),
    "sufb200_interval_lut_build": (_sz, [_i, _u64, _i, _i, _vp, _i, _vp, _vp, _vp]),
    "sufb200_interval_lut_eval": (_i, [_vp, _vp, _sz, _i, _vp, _sz, _i, _u64, _vp, _vp]),
    "sufb200_seed_from_id": (_i, [_u64, _u64, _vp]),
    "sufb200_beaver_mul": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "sufb200_beaver_mul_aos": (_i, [_i, _vp, _vp, _vp, _vp, _sz, _vp]),
    "sufb200_horner_cubic": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "sufb200_trunc_postproc": (_i, [_i, _i, _i, _u64, _u64, _vp, _vp, _sz, _i, _vp, _sz, _i, _i, _i, _vp, _sz, _vp]),
    "sufb200_add_rout_aos": (_i, [_vp, _sz, _i, _vp, _sz, _vp]),
    "sufb200_row_sum": (_i, [_vp, _i, _i, _vp, _vp, _vp]),
    "sufb200_row_sum_ragged": (_i, [_vp, _vp, _i, _vp, _vp]),
    "sufb200_row_variance": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp]),
    "sufb200_row_broadcast_mul": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp]),
    "sufb200_pack_eff_bits": (_i, [_vp, _i, _vp, _sz, _vp]),
    "sufb200_unpack_eff_bits": (_i, [_vp, _i, _vp, _sz, _vp]),
    "sufb200_unpack_add_mod": (_i, [_vp, _vp, _i, _vp, _sz, _i, _vp]),
    "sufb200_unpack_add_to_signed": (_i, [_vp, _vp, _i, _vp, _sz, _i, _vp]),
    "sufb200_open_add_to_signed": (_i, [_vp, _vp, _vp, _sz, _i, _vp]),
    "sufb200_myl7_gen_batch_device": (_i, [_vp, _i, _i, _vp, _sz, _vp, _i, _vp, _vp, _vp, _vp, _vp]),
    "sufb200_ring_matmul": (_i, [_vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _i, _vp]),
    "sufb200_beaver_matmul2d_tc": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, C.c_int64, _i, _vp,
                                        _vp]),
    "sufb200_coeff_lut_eval": (_i, [_vp, _vp, _sz, _vp, _sz, _i, _i, _vp, _i, _u64, _vp, _vp]),
    "sufb200_coeff_lut_eval_pair": (_i, [_vp, _vp, _sz, _vp, _sz, _vp, _sz, _i, _i, _vp, _vp, _i, _u64, _vp, _vp,
                                         _vp]),
    "sufb200_open_unique_id": (_i, [_vp]),
    "sufb200_open_comm_create": (_i, [_vp, _vp, _i, _i, C.c_double, C.POINTER(_vp)]),
    "sufb200_open_comm_destroy": (_i, [_vp]),
    "sufb200_open_comm_abort": (_i, [_vp]),
    "sufb200_open_exchange": (_i, [_vp, _i, _vp, _sz, _i, _i, _i, _vp, _vp]),
    "sufb200_row_mean": (_i, [_vp, _i, _i, _vp, _vp, _vp]),
    "sufb200_trunc_shift": (_i, [_vp, _vp, _i, _sz, _vp]),
    "sufb200_beaver_matmul2d": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, C.c_int64, _i, _vp, _vp]),
    "sufb200_host_mt19937_64": (_i, [_u64, _vp, _sz]),
    "sufb200_softmax_block_pair": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _sz, _i, _vp, _vp, _vp]),
    "sufb200_layernorm_block_pair": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _i, _u64, _u64, _vp, _vp, _vp]),
    "sufb200_open_masked_pair": (_i, [_vp, _vp, _u64, _u64, _vp, _sz, _vp]),
    "sufb200_p2p_open_create": (_i, [_vp, _sz, C.POINTER(_vp), _vp]),
    "sufb200_p2p_open_connect": (_i, [_vp, _vp]),
    "sufb200_p2p_open_connect_self": (_i, [_vp]),
    "sufb200_p2p_open_exchange": (_i, [_vp, _vp, _sz, _i, _i, _i, _vp, C.c_double, _vp]),
    "sufb200_p2p_open_destroy": (_i, [_vp]),
    "sufb200_add_pair": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "sufb200_relu_open_pair": (_i, [_vp, _vp, _i, _i, _u64, _u64, _vp, _vp]),
    "sufb200_relu_update_pair": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp]),
    "sufb200_maxdiff_pair": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp]),
    "sufb200_beaver_open_pair": (_i, [_vp, _sz, _i, _vp, _sz, _i, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz,
                                      _i, _vp]),
}


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(
            f"{p} is missing: build it with `python -m suf_b200.build` (nvcc, sm_100a); there is no fallback")
    lib = C.CDLL(str(p))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB: C.CDLL | None = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB


def check(rc: int) -> int:
    if rc != OK:
        msg = lib().sufb200_last_error().decode(errors="replace")
        raise SufB200Error(rc, msg)
    return rc


def exported_symbols() -> list[str]:
    return list(_SIGS)
