"""GPU parity: fused truncation / ARS bundles (FaithfulTR, FaithfulARS,
GapARS) against the oracle's composite eval + postproc, per share and per
boolean port, plus exact reconstruction at the configs[1] size."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle.oracle import KIND_ARS, KIND_GAPARS, KIND_TR
from tests.conftest import from_dev, to_dev
from tests.helpers import oracle_trunc_eval, signed_fixed, to_product_desc, trunc_material

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", [KIND_TR, KIND_ARS, KIND_GAPARS])
@pytest.mark.parametrize("f", [4, 12, 16])
def test_bundle_bit_exact_per_share(ctx, torch_cuda, oracle, prg_state, kind, f):
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(31 * kind + f)
    n = 3000
    x = signed_fixed(rng, n, 40)
    for seed in (2, 12345):
        r_in, descs, keys = trunc_material(oracle, kind, f, seed)
        xhat = x + np.uint64(r_in)
        dx = to_dev(torch_cuda, xhat)
        ys = []
        for p in (0, 1):
            db = torch_cuda.zeros(3 * n, dtype=torch_cuda.int64, device="cuda")
            dy = ctx.trunc_bundle_eval(to_product_desc(descs[p]), keys[p], dx, d_bools=db)
            ctx.sync()
            exp_y, exp_b = oracle_trunc_eval(oracle, descs[p], keys[p], xhat, want_bools=True)
            got = from_dev(dy)
            assert (got == exp_y).all()
            assert (from_dev(db).reshape(n, 3) == exp_b).all()
            ys.append(got)
        exp = (x >> np.uint64(f)) if kind == KIND_TR else (x.view(np.int64) >> f).view(np.uint64)
        assert ((ys[0] + ys[1]) == exp).all()


def test_reference_trunc_vectors(ctx, torch_cuda, oracle, prg_state):
    """src/demo/test_cuda_trunc_gapars.cpp / test_pfss_gpu.cpp inputs {16,-8,3,-1}, f=4."""
    oracle.prg_init(prg_state)
    v = json.loads((Path(__file__).parent / "golden" / "ref_vectors.json").read_text())["trunc"]
    plain = np.array(v["plain"], dtype=np.int64)
    for kind in (KIND_TR, KIND_ARS, KIND_GAPARS):
        for seed in v["seeds"]:
            r_in, descs, keys = trunc_material(oracle, kind, v["frac_bits"], seed)
            dx = to_dev(torch_cuda, plain.view(np.uint64) + np.uint64(r_in))
            y = sum(from_dev(ctx.trunc_bundle_eval(to_product_desc(descs[p]), keys[p], dx)) for p in (0, 1))
            ctx.sync()
            if kind == KIND_TR:
                exp = plain.view(np.uint64) >> np.uint64(v["frac_bits"])
            else:
                exp = np.array(v["expect_ars"], dtype=np.int64).view(np.uint64)
            assert (y == exp).all()


def test_bundle_rejects_mismatched_keys(ctx, torch_cuda, oracle, prg_state):
    from suf_b200 import SufB200Error

    oracle.prg_init(prg_state)
    r_in, descs, keys = trunc_material(oracle, KIND_ARS, 16, 2)
    dx = to_dev(torch_cuda, np.arange(16, dtype=np.uint64))
    with pytest.raises(SufB200Error):  # party-1 keys with the party-0 descriptor
        ctx.trunc_bundle_eval(to_product_desc(descs[0]), keys[1], dx)


def test_config2_size_reconstruction(ctx, torch_cuda, oracle, prg_state):
    """N = 4,194,304, |x| < 2^40 with 32 fractional bits, f = 16, seed 2."""
    oracle.prg_init(prg_state)
    n = 1 << 22
    rng = np.random.default_rng(2)
    x = signed_fixed(rng, n, 40)
    r_in, descs, keys = trunc_material(oracle, KIND_ARS, 16, 2)
    xhat = x + np.uint64(r_in)
    dx = to_dev(torch_cuda, xhat)
    y0 = from_dev(ctx.trunc_bundle_eval(to_product_desc(descs[0]), keys[0], dx))
    y1 = from_dev(ctx.trunc_bundle_eval(to_product_desc(descs[1]), keys[1], dx))
    ctx.sync()
    assert ((y0 + y1) == (x.view(np.int64) >> 16).view(np.uint64)).all()
    idx = rng.integers(0, n, 256)
    assert (y0[idx] == oracle_trunc_eval(oracle, descs[0], keys[0], xhat[idx])).all()


@pytest.mark.parametrize("kind", [KIND_TR, KIND_ARS, KIND_GAPARS])
def test_bundle_shared_prefix_path_bit_exact(ctx, torch_cuda, oracle, prg_state, kind):
    """N above the shared-prefix threshold (frontier tables for the 64-bit
    queries, full-domain tables for the 16-bit ones), per share and bool."""
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(77 + kind)
    n = 40_000
    x = signed_fixed(rng, n, 40)
    x[:4] = np.array([0, 1, -1, 2**40 - 1], dtype=np.int64).view(np.uint64)
    r_in, descs, keys = trunc_material(oracle, kind, 16, 5)
    xhat = x + np.uint64(r_in)
    dx = to_dev(torch_cuda, xhat)
    ys = []
    for p in (0, 1):
        db = torch_cuda.zeros(3 * n, dtype=torch_cuda.int64, device="cuda")
        y = from_dev(ctx.trunc_bundle_eval(to_product_desc(descs[p]), keys[p], dx, d_bools=db))
        ctx.sync()
        exp_y, exp_b = oracle_trunc_eval(oracle, descs[p], keys[p], xhat, want_bools=True)
        assert (y == exp_y).all()
        assert (from_dev(db).reshape(n, 3) == exp_b).all()
        ys.append(y)
    exp = (x >> np.uint64(16)) if kind == KIND_TR else (x.view(np.int64) >> 16).view(np.uint64)
    assert ((ys[0] + ys[1]) == exp).all()


def test_host_entry_chunked_matches_device_entry(ctx, torch_cuda, oracle, prg_state):
    """sufb200_trunc_bundle_eval_host above 2^20 elements runs the main pass
    in eight chunks with the copies back overlapped: same y and bool shares
    as the device entry, for a size that does not divide into eight, twice
    in a row (reused host-io buffers)."""
    oracle.prg_init(prg_state)
    n = (1 << 20) + 13
    rng = np.random.default_rng(4)
    x = signed_fixed(rng, n, 40)
    r_in, descs, keys = trunc_material(oracle, KIND_GAPARS, 12, 3)
    xhat = x + np.uint64(r_in)
    dx = to_dev(torch_cuda, xhat)
    ys = []
    for p in (0, 1):
        d = to_product_desc(descs[p])
        db = torch_cuda.zeros(3 * n, dtype=torch_cuda.int64, device="cuda")
        dy = from_dev(ctx.trunc_bundle_eval(d, keys[p], dx, d_bools=db))
        ctx.sync()
        for _ in range(2):
            hb = np.zeros(3 * n, dtype=np.uint64)
            hy = ctx.trunc_bundle_eval_host(d, keys[p], xhat, bools=hb)
            assert (hy == dy).all()
            assert (hb == from_dev(db)).all()
        ys.append(hy)
    assert ((ys[0] + ys[1]) == (x.view(np.int64) >> 12).view(np.uint64)).all()
    idx = rng.integers(0, n, 128)
    assert (ys[1][idx] == oracle_trunc_eval(oracle, descs[1], keys[1], xhat[idx])).all()


@pytest.mark.parametrize("kind", [KIND_TR, KIND_ARS, KIND_GAPARS])
@pytest.mark.parametrize("n", [1, 7, 1536, 20_000, 99_072])
def test_pair_entry_matches_per_party_entry(ctx, torch_cuda, oracle, prg_state, kind, n):
    """sufb200_trunc_bundle_eval_pair (one query-parallel launch for both
    parties below the shared-prefix size, the per-party path above it) gives
    each party exactly the oracle's shares, and sufb200_trunc_bundle_eval_pair_dev
    (keys resident on the device) the same words."""
    import ctypes as C

    from suf_b200 import _lib

    oracle.prg_init(prg_state)
    rng = np.random.default_rng(900 + kind + n)
    x = signed_fixed(rng, n, 40)
    r_in, descs, keys = trunc_material(oracle, kind, 12, 17 + n)
    xhat = x + np.uint64(r_in)
    dx = to_dev(torch_cuda, xhat)
    out = [torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda") for _ in (0, 1)]
    pd = [to_product_desc(descs[p]) for p in (0, 1)]
    karr = [[np.ascontiguousarray(k, dtype=np.uint8) for k in keys[p]] for p in (0, 1)]
    ptrs = [(C.c_void_p * 4)(*[k.ctypes.data for k in karr[p]], *([None] * (4 - len(karr[p])))) for p in (0, 1)]
    sizes = [(C.c_size_t * 4)(*[k.size for k in karr[p]], *([0] * (4 - len(karr[p])))) for p in (0, 1)]
    _lib.check(_lib.lib().sufb200_trunc_bundle_eval_pair(
        ctx.h, C.byref(pd[0]), C.cast(ptrs[0], C.c_void_p), C.cast(sizes[0], C.c_void_p), C.byref(pd[1]),
        C.cast(ptrs[1], C.c_void_p), C.cast(sizes[1], C.c_void_p), dx.data_ptr(), n, out[0].data_ptr(),
        out[1].data_ptr(), None))
    ctx.sync()
    for p in (0, 1):
        assert (from_dev(out[p]) == oracle_trunc_eval(oracle, descs[p], keys[p], xhat)).all(), p
    # the same bundles with their keys resident on the device (no host copy;
    # the layer's capturable path), at odd device offsets
    dkeys = [[to_dev(torch_cuda, np.concatenate([np.zeros(3, np.uint8), k]))[3:] for k in karr[p]] for p in (0, 1)]
    dptrs = [(C.c_void_p * 4)(*[k.data_ptr() for k in dkeys[p]], *([None] * (4 - len(dkeys[p])))) for p in (0, 1)]
    out2 = [torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda") for _ in (0, 1)]
    _lib.check(_lib.lib().sufb200_trunc_bundle_eval_pair_dev(
        ctx.h, C.byref(pd[0]), C.cast(dptrs[0], C.c_void_p), C.cast(sizes[0], C.c_void_p), C.byref(pd[1]),
        C.cast(dptrs[1], C.c_void_p), C.cast(sizes[1], C.c_void_p), dx.data_ptr(), n, out2[0].data_ptr(),
        out2[1].data_ptr(), None))
    ctx.sync()
    for p in (0, 1):
        assert (from_dev(out2[p]) == from_dev(out[p])).all(), p


@pytest.mark.parametrize("lens", [[5, 0, 20_000, 1, 37], [300] * 61 + [0, 17_000]])
def test_jobs_bucket_matches_per_job(ctx, torch_cuda, oracle, prg_state, lens):
    """sufb200_trunc_bundle_eval_jobs over a bucket of jobs sharing one key
    (ragged, empty, more than one gather launch): each job's result equals the
    oracle's evaluation of that job alone."""
    import ctypes as C

    from suf_b200 import _lib

    oracle.prg_init(prg_state)
    rng = np.random.default_rng(sum(lens))
    r_in, descs, keys = trunc_material(oracle, KIND_GAPARS, 12, 33)
    xs = [signed_fixed(rng, n, 40) + np.uint64(r_in) for n in lens]
    dx = [to_dev(torch_cuda, x) if x.size else torch_cuda.zeros(1, dtype=torch_cuda.int64, device="cuda") for x in xs]
    dy = [torch_cuda.full((max(n, 1),), -1, dtype=torch_cuda.int64, device="cuda") for n in lens]
    pd = to_product_desc(descs[0])
    karr = [np.ascontiguousarray(k, dtype=np.uint8) for k in keys[0]]
    ptrs = (C.c_void_p * 4)(*[k.ctypes.data for k in karr], *([None] * (4 - len(karr))))
    sizes = (C.c_size_t * 4)(*[k.size for k in karr], *([0] * (4 - len(karr))))
    J = len(lens)
    xp = (C.c_void_p * J)(*[t.data_ptr() for t in dx])
    yp = (C.c_void_p * J)(*[t.data_ptr() for t in dy])
    ns = (C.c_size_t * J)(*lens)
    _lib.check(_lib.lib().sufb200_trunc_bundle_eval_jobs(ctx.h, C.byref(pd), C.cast(ptrs, C.c_void_p),
                                                         C.cast(sizes, C.c_void_p), C.cast(xp, C.c_void_p),
                                                         C.cast(ns, C.c_void_p), C.cast(yp, C.c_void_p), J, None))
    ctx.sync()
    for j, n in enumerate(lens):
        if n:
            assert (from_dev(dy[j])[:n] == oracle_trunc_eval(oracle, descs[0], keys[0], xs[j])).all(), j
        else:
            assert int(dy[j].cpu()[0]) == -1  # untouched


def _elem_desc(shape, words_row):
    """The oracle descriptor of one per-element gate: the shape's kind, f,
    party and slot widths, the element's words and plan."""
    from oracle.oracle import TruncDesc as OrcDesc

    d = OrcDesc()
    for name in ("kind", "frac_bits", "party", "nq"):
        setattr(d, name, getattr(shape, name))
    for q in range(4):
        d.q_bits[q] = shape.q_bits[q]
    d.carry_w, d.sign_w, d.haty, d.r_hi, d.m = (int(v) for v in words_row[:5])
    plan = int(words_row[5])
    idx = [(plan >> (4 * j)) & 0xF for j in range(5)]
    d.carry_a, d.carry_b, d.sign_a, d.sign_b, d.wrap_q = (-1 if v == 0xF else v for v in idx)
    return d


@pytest.mark.parametrize("kind,f,n", [(KIND_ARS, 16, 4096), (KIND_TR, 12, 16384), (KIND_GAPARS, 12, 16384)])
def test_per_element_bundles_bit_exact(ctx, torch_cuda, oracle, prg_state, kind, f, n):
    """Per-element masks (SUF_PER_ELEMENT_MASKS=1): every element has its own
    gate and keys.  Each party's shares equal the oracle's per-element
    composite eval + postproc word for word, and y0 + y1 is the truncation;
    the f = 12 cases hold elements whose gate has no carry queries (r_low =
    0), which the slot layout marks absent.  The level-major key layout
    (sufb200_elem_keys_to_soa) gives the same words."""
    from suf_b200.engine import Context, host_mt19937_64, myl7_key_bytes
    from tests.helpers import ONE_LE

    oracle.prg_init(prg_state)
    r_in, s0, s1, w0, w1, th = Context.trunc_gen_elem(kind, f, 77, n)
    nq = int(s0.nq)
    if f == 12:
        assert ((r_in & np.uint64((1 << f) - 1)) == 0).any()  # the carry-free elements are exercised
    seeds = host_mt19937_64(0xE1E1, 4 * n * nq).view(np.uint8).reshape(nq, n, 2, 16)
    keys = []
    for q in range(nq):
        k0, k1 = ctx.myl7_gen_batch(0, int(s0.q_bits[q]), th[:, q], ONE_LE, np.ascontiguousarray(seeds[q, :, 0]),
                                    np.ascontiguousarray(seeds[q, :, 1]))
        keys.append((k0, k1))
    rng = np.random.default_rng(5)
    x = signed_fixed(rng, n, 40)
    xhat = x + r_in
    dx = to_dev(torch_cuda, xhat)
    ys = []
    for p, shape, words in ((0, s0, w0), (1, s1, w1)):
        kb = [myl7_key_bytes(int(shape.q_bits[q]), 8) for q in range(nq)]
        dk = [to_dev(torch_cuda, keys[q][p].ravel()) for q in range(nq)]
        db = torch_cuda.zeros(3 * n, dtype=torch_cuda.int64, device="cuda")
        dy = ctx.trunc_bundle_eval_elem(shape, dk, kb, to_dev(torch_cuda, words.ravel()), dx, d_bools=db)
        ctx.sync()
        got = from_dev(dy)
        # the same keys in the level-major layout: the same words
        soa = [ctx.elem_keys_to_soa(int(shape.q_bits[q]), p, dk[q], n) for q in range(nq)]
        db2 = torch_cuda.zeros(3 * n, dtype=torch_cuda.int64, device="cuda")
        dy2 = ctx.trunc_bundle_eval_elem_soa(shape, soa, to_dev(torch_cuda, words.ravel()), dx, d_bools=db2)
        ctx.sync()
        assert (from_dev(dy2) == got).all() and (from_dev(db2) == from_dev(db)).all(), p
        pred = np.stack([oracle.myl7_eval(0, keys[q][p], kb[q], False, xhat, 8).view(np.uint64).ravel()
                         for q in range(nq)])
        exp = np.array([oracle.trunc_combine(_elem_desc(shape, words[i]), xhat[i:i + 1], pred[:, i].copy())[0]
                        for i in range(n)], dtype=np.uint64)
        assert (got == exp).all(), int((got != exp).sum())
        ys.append(got)
    want = (x >> np.uint64(f)) if kind == KIND_TR else (x.view(np.int64) >> f).view(np.uint64)
    assert ((ys[0] + ys[1]) == want).all()


def test_per_element_soa_flags_a_bad_key_header(ctx, torch_cuda):
    """A per-element key whose header does not match its slot is flagged when
    the keys are rearranged (sufb200_ctx_sync reports it) and that element's
    query evaluates to 0; the context stays usable."""
    from suf_b200 import SufB200Error
    from suf_b200.engine import Context, host_mt19937_64
    from tests.helpers import ONE_LE

    n = 64
    r_in, s0, s1, w0, w1, th = Context.trunc_gen_elem(KIND_GAPARS, 12, 5, n)
    seeds = host_mt19937_64(0xBAD, 4 * n).view(np.uint8).reshape(n, 2, 16)
    k0, _ = ctx.myl7_gen_batch(0, 12, th[:, 0], ONE_LE, np.ascontiguousarray(seeds[:, 0]),
                               np.ascontiguousarray(seeds[:, 1]))
    k0 = k0.copy()
    k0[7, 2] ^= 1  # element 7: the party byte of its header
    soa = ctx.elem_keys_to_soa(12, 0, to_dev(torch_cuda, k0.ravel()), n)
    with pytest.raises(SufB200Error):
        ctx.sync()
    ctx.sync()  # the status was cleared
    assert soa.numel() == n * (25 * 12 + 24)


@pytest.mark.parametrize("f,n", [(12, 20_000), (15, 99_072), (12, 128), (12, 1_536), (3, 1_000), (16, 5_001)])
def test_pair_tables_entry_matches(ctx, torch_cuda, oracle, prg_state, f, n):
    """sufb200_trunc_tables_dev (each party's full-domain tables of the GapARS
    carries, made apart from x^) + sufb200_trunc_bundle_eval_pair_tables_dev
    give the words of sufb200_trunc_bundle_eval_pair_dev, at element-level
    and row-level batch sizes."""
    import ctypes as C

    from suf_b200 import _lib

    oracle.prg_init(prg_state)
    rng = np.random.default_rng(31 + f + n)
    x = signed_fixed(rng, n, 30)
    r_in, descs, keys = trunc_material(oracle, KIND_GAPARS, f, 5 + n)
    xhat = x + np.uint64(r_in)
    dx = to_dev(torch_cuda, xhat)
    pd = [to_product_desc(descs[p]) for p in (0, 1)]
    dk = [[to_dev(torch_cuda, np.ascontiguousarray(k, dtype=np.uint8)) for k in keys[p]] for p in (0, 1)]
    ptrs = [(C.c_void_p * 4)(*[k.data_ptr() for k in dk[p]], *([None] * (4 - len(dk[p])))) for p in (0, 1)]
    sizes = [(C.c_size_t * 4)(*[k.numel() for k in dk[p]], *([0] * (4 - len(dk[p])))) for p in (0, 1)]
    L = _lib.lib()
    side = [(C.byref(pd[p]), C.cast(ptrs[p], C.c_void_p), C.cast(sizes[p], C.c_void_p)) for p in (0, 1)]
    ref = [torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda") for _ in (0, 1)]
    _lib.check(L.sufb200_trunc_bundle_eval_pair_dev(ctx.h, *side[0], *side[1], dx.data_ptr(), n, ref[0].data_ptr(),
                                                    ref[1].data_ptr(), None))
    tabs = []
    for p in (0, 1):
        nbytes = int(L.sufb200_trunc_tables_bytes(C.byref(pd[p])))
        assert nbytes > 0
        tabs.append(torch_cuda.empty(nbytes, dtype=torch_cuda.uint8, device="cuda"))
        _lib.check(L.sufb200_trunc_tables_dev(ctx.h, *side[p], tabs[p].data_ptr(), nbytes, None))
    out = [torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda") for _ in (0, 1)]
    _lib.check(L.sufb200_trunc_bundle_eval_pair_tables_dev(ctx.h, *side[0], tabs[0].data_ptr(), *side[1],
                                                           tabs[1].data_ptr(), dx.data_ptr(), n, out[0].data_ptr(),
                                                           out[1].data_ptr(), None))
    ctx.sync()
    for p in (0, 1):
        assert (from_dev(out[p]) == from_dev(ref[p])).all(), p
    assert ((from_dev(out[0]) + from_dev(out[1])) == (x.view(np.int64) >> f).view(np.uint64)).all()


def test_tables_reject_wide_queries(ctx, torch_cuda, oracle, prg_state):
    """A bundle with a query wider than 16 bits has no tables: size 0 and
    SUFB200_ERR_UNSUPPORTED from both tables entries."""
    import ctypes as C

    from suf_b200 import SufB200Error, _lib

    oracle.prg_init(prg_state)
    _, descs, keys = trunc_material(oracle, KIND_GAPARS, 24, 9)
    pd = [to_product_desc(descs[p]) for p in (0, 1)]
    dk = [[to_dev(torch_cuda, np.ascontiguousarray(k, dtype=np.uint8)) for k in keys[p]] for p in (0, 1)]
    ptrs = [(C.c_void_p * 4)(*[k.data_ptr() for k in dk[p]], *([None] * (4 - len(dk[p])))) for p in (0, 1)]
    sizes = [(C.c_size_t * 4)(*[k.numel() for k in dk[p]], *([0] * (4 - len(dk[p])))) for p in (0, 1)]
    L = _lib.lib()
    assert int(L.sufb200_trunc_tables_bytes(C.byref(pd[0]))) == 0
    buf = torch_cuda.empty(1 << 20, dtype=torch_cuda.uint8, device="cuda")
    side = [(C.byref(pd[p]), C.cast(ptrs[p], C.c_void_p), C.cast(sizes[p], C.c_void_p)) for p in (0, 1)]
    with pytest.raises(SufB200Error):
        _lib.check(L.sufb200_trunc_tables_dev(ctx.h, *side[0], buf.data_ptr(), buf.numel(), None))
    dx = to_dev(torch_cuda, np.zeros(8, dtype=np.uint64))
    with pytest.raises(SufB200Error):
        _lib.check(L.sufb200_trunc_bundle_eval_pair_tables_dev(ctx.h, *side[0], buf.data_ptr(), *side[1],
                                                               buf.data_ptr(), dx.data_ptr(), 8, dx.data_ptr(),
                                                               dx.data_ptr(), None))
