"""The allocation-free bundle entry point against the allocating one.

sufb200_trunc_bundle_eval_noalloc serves callers that cannot allocate device
memory while they evaluate (a runtime that owns all device memory through its
own arena, or code that must not re-enter or grow the CUDA allocator): it
stages the bundle keys in a fixed 16 KiB array instead of a cudaMallocAsync
buffer.  This file calls it through the C ABI twice in a row, with different
bundles, and checks each result bit-for-bit (the outputs are Z_2^64 shares,
so the tolerance is zero) against sufb200_trunc_bundle_eval on the same
inputs.  It sits in a file of its own, collected last.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle.oracle import KIND_ARS, KIND_GAPARS
from tests.conftest import from_dev, to_dev
from tests.helpers import signed_fixed, to_product_desc, trunc_material

pytestmark = pytest.mark.gpu


def _eval_noalloc(ctx, desc, keys, d_xhat, d_y, d_bools):
    from suf_b200 import _lib

    nq = int(desc.nq)
    karr = [np.ascontiguousarray(k, dtype=np.uint8) for k in keys[:nq]]
    ptrs = (C.c_void_p * 4)(*[k.ctypes.data for k in karr], *([None] * (4 - nq)))
    sizes = (C.c_size_t * 4)(*[k.size for k in karr], *([0] * (4 - nq)))
    _lib.check(_lib.lib().sufb200_trunc_bundle_eval_noalloc(
        ctx.h, C.byref(desc), C.cast(ptrs, C.c_void_p), C.cast(sizes, C.c_void_p), int(d_xhat.data_ptr()),
        d_xhat.numel(), int(d_y.data_ptr()), int(d_bools.data_ptr()), None))


def test_noalloc_matches_allocating_entry_point_twice(ctx, torch_cuda, oracle, prg_state):
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(2024)
    n = 50_000
    # two different bundles back to back: the second call must not see the
    # first call's keys, which the shared staging array still holds
    for kind, f, seed, party in ((KIND_ARS, 16, 2, 0), (KIND_GAPARS, 12, 7, 1)):
        r_in, descs, keys = trunc_material(oracle, kind, f, seed)
        x = signed_fixed(rng, n, 40)
        dx = to_dev(torch_cuda, x + np.uint64(r_in))
        desc = to_product_desc(descs[party])
        b_ref = torch_cuda.zeros(3 * n, dtype=torch_cuda.int64, device="cuda")
        y_ref = ctx.trunc_bundle_eval(desc, keys[party], dx, d_bools=b_ref)
        y_na = torch_cuda.full((n,), -1, dtype=torch_cuda.int64, device="cuda")
        b_na = torch_cuda.full((3 * n,), -1, dtype=torch_cuda.int64, device="cuda")
        _eval_noalloc(ctx, desc, keys[party], dx, y_na, b_na)
        ctx.sync()
        assert (from_dev(y_na) == from_dev(y_ref)).all()
        assert (from_dev(b_na) == from_dev(b_ref)).all()


def test_noalloc_rejects_bad_keys_before_staging(ctx, torch_cuda, oracle, prg_state):
    """A key of the wrong size or with a header that does not match the
    bundle is refused (SUFB200_ERR_KEY) by the host-side checks, before the
    shared staging array is written; a valid call afterwards still matches
    the allocating entry point."""
    from suf_b200 import _lib

    oracle.prg_init(prg_state)
    rng = np.random.default_rng(77)
    n = 4096
    r_in, descs, keys = trunc_material(oracle, KIND_ARS, 16, 2)
    dx = to_dev(torch_cuda, signed_fixed(rng, n, 40) + np.uint64(r_in))
    desc = to_product_desc(descs[0])
    y = torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda")
    b = torch_cuda.empty(3 * n, dtype=torch_cuda.int64, device="cuda")
    short = [k.copy() for k in keys[0]]
    short[0] = short[0][:-1]
    wrong_party = [k.copy() for k in keys[0]]
    wrong_party[1][2] ^= 1
    for bad in (short, wrong_party):
        with pytest.raises(_lib.SufB200Error) as ei:
            _eval_noalloc(ctx, desc, bad, dx, y, b)
        assert ei.value.code == _lib.ERR_KEY
    y_ref = ctx.trunc_bundle_eval(desc, keys[0], dx)
    _eval_noalloc(ctx, desc, keys[0], dx, y, b)
    ctx.sync()
    assert (from_dev(y) == from_dev(y_ref)).all()
