"""GPU parity: elementwise / row ring kernels against the oracle
(launch_* semantics of include/runtime/cuda_primitives.hpp)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tests.conftest import from_dev, rand_u64, to_dev

pytestmark = pytest.mark.gpu


def _p(t):
    return int(t.data_ptr()) if t is not None else None


class Keep:
    """Holds device tensors until the kernels that read them have run (a
    tensor freed before its kernel executes returns its memory to the caching
    allocator, which may hand it to the next upload)."""

    def __init__(self, torch):
        self.torch = torch
        self.held = []

    def dev(self, a):
        t = to_dev(self.torch, a)
        self.held.append(t)
        return _p(t)


@pytest.fixture(scope="module")
def L():
    from suf_b200 import _lib

    return _lib


def test_beaver_mul_and_aos(ctx, torch_cuda, oracle, L):
    rng = np.random.default_rng(1234)
    n = 100_003
    a, b, c, d, e = (rand_u64(rng, n) for _ in range(5))
    dv = [to_dev(torch_cuda, v) for v in (a, b, c, d, e)]
    for party in (0, 1):
        out = torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda")
        L.check(L.lib().sufb200_beaver_mul(party, *[_p(t) for t in dv], _p(out), n, None))
        tri = to_dev(torch_cuda, np.stack([a, b, c], axis=1).ravel())
        out2 = torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda")
        L.check(L.lib().sufb200_beaver_mul_aos(party, _p(tri), _p(dv[3]), _p(dv[4]), _p(out2), n, None))
        exp = oracle.beaver_mul(party, a, b, c, d, e)
        assert (from_dev(out) == exp).all() and (from_dev(out2) == exp).all()


def test_horner_cubic(ctx, torch_cuda, oracle, L):
    rng = np.random.default_rng(1234)
    n = 65_537
    vs = [rand_u64(rng, n) for _ in range(5)]
    dv = [to_dev(torch_cuda, v) for v in vs]
    out = torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda")
    L.check(L.lib().sufb200_horner_cubic(*[_p(t) for t in dv], _p(out), n, None))
    assert (from_dev(out) == oracle.horner_cubic(*vs)).all()


def _postproc_ref(party, gap, f, rhi, m, hatx, base, carry, sign, wrap):
    """launch_trunc_postproc_kernel, cuda/cuda_primitives.cu:179-252 (numpy)."""
    with np.errstate(over="ignore"):
        y = base.copy()
        if gap:
            hb = hatx + np.uint64(1 << 62)
            top = (hb >> np.uint64(f)) if party == 0 else np.zeros_like(hb)
            y = y + top - np.uint64(rhi) - carry
            y = np.where((hb >> np.uint64(63)) == 0, y + np.uint64(m), y)
            if party == 0:
                y = y - np.uint64(1 << (62 - f))
            return y
        if party == 0:
            y = y + (hatx >> np.uint64(f))
        y = y - np.uint64(rhi) - carry
        y = y + wrap * np.uint64(1 << (64 - f))
        y = y + sign * np.uint64((2**64 - 1) ^ ((1 << (64 - f)) - 1))
        return y


@pytest.mark.parametrize("gap", [0, 1])
def test_trunc_postproc(ctx, torch_cuda, L, gap):
    rng = np.random.default_rng(4321)
    n = 10_000
    hatx, base = rand_u64(rng, n), rand_u64(rng, n)
    bools = rng.integers(0, 2, (n, 3), dtype=np.uint64)
    arith = np.stack([rand_u64(rng, n), base], axis=1)
    f, rhi, m = 12, int(rand_u64(rng, 1)[0]), int(rand_u64(rng, 1)[0])
    k = Keep(torch_cuda)
    for party in (0, 1):
        out = torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda")
        L.check(L.lib().sufb200_trunc_postproc(party, gap, f, C.c_uint64(rhi), C.c_uint64(m), k.dev(hatx),
                                               k.dev(arith.ravel()), 2, 1, k.dev(bools.ravel()), 3, 0, 1, 2, _p(out), n,
                                               None))
        exp = _postproc_ref(party, gap, f, rhi, m, hatx, base, bools[:, 0], bools[:, 1], bools[:, 2])
        assert (from_dev(out) == exp).all()


def test_row_reductions(ctx, torch_cuda, oracle, L):
    rng = np.random.default_rng(4)
    rows, cols = 1536, 128  # softmax: 12 heads x 128 rows, causal lengths
    mat = rand_u64(rng, rows * cols).reshape(rows, cols)
    valid = np.array([(r % 128) + 1 for r in range(rows)], dtype=np.int32)
    dmat = to_dev(torch_cuda, mat.ravel())
    dval = torch_cuda.from_numpy(valid).cuda()
    out = torch_cuda.empty(rows, dtype=torch_cuda.int64, device="cuda")
    L.check(L.lib().sufb200_row_sum(_p(dmat), rows, cols, _p(dval), _p(out), None))
    assert (from_dev(out) == oracle.row_sum(mat, valid)).all()
    L.check(L.lib().sufb200_row_sum(_p(dmat), rows, cols, None, _p(out), None))
    assert (from_dev(out) == oracle.row_sum(mat)).all()
    mean = rand_u64(rng, rows)
    k = Keep(torch_cuda)
    L.check(L.lib().sufb200_row_variance(_p(dmat), k.dev(mean), rows, cols, _p(dval), _p(out), None))
    assert (from_dev(out) == oracle.row_variance(mat, mean, valid)).all()
    offs = np.concatenate([[0], np.cumsum(valid)]).astype(np.int32)
    vals = np.concatenate([mat[r, : valid[r]] for r in range(rows)])
    L.check(L.lib().sufb200_row_sum_ragged(k.dev(vals), k.dev(offs), rows, _p(out), None))
    assert (from_dev(out) == oracle.row_sum(mat, valid)).all()
    ln = rand_u64(rng, 128 * 768).reshape(128, 768)  # LayerNorm rows
    out2 = torch_cuda.empty(128, dtype=torch_cuda.int64, device="cuda")
    L.check(L.lib().sufb200_row_sum(k.dev(ln.ravel()), 128, 768, None, _p(out2), None))
    assert (from_dev(out2) == oracle.row_sum(ln)).all()


def test_row_broadcast_mul(ctx, torch_cuda, L):
    rng = np.random.default_rng(5)
    rows, cols = 1536, 128
    A, C_, d = (rand_u64(rng, rows * cols) for _ in range(3))
    B, e = rand_u64(rng, rows), rand_u64(rng, rows)
    valid = np.array([(r % 128) + 1 for r in range(rows)], dtype=np.int32)
    out = torch_cuda.empty(rows * cols, dtype=torch_cuda.int64, device="cuda")
    k = Keep(torch_cuda)
    ptrs = [k.dev(v) for v in (A, B, C_, d, e)]
    dval = k.dev(valid)
    for party in (0, 1):
        L.check(L.lib().sufb200_row_broadcast_mul(party, *ptrs, rows, cols, dval, _p(out), None))
        r = np.repeat(np.arange(rows), cols)
        with np.errstate(over="ignore"):
            exp = C_ + d * B[r] + e[r] * A + (d * e[r] if party == 0 else 0)
        exp = np.where(np.tile(np.arange(cols), rows) < valid[r], exp, 0).astype(np.uint64)
        assert (from_dev(out) == exp).all()


@pytest.mark.parametrize("eff_bits", [1, 7, 13, 37, 56, 63, 64])
def test_eff_bits_pack_unpack_and_open(ctx, torch_cuda, oracle, L, eff_bits):
    rng = np.random.default_rng(eff_bits)
    n = 10_007
    xs = rand_u64(rng, n)
    words = (n * eff_bits + 63) // 64
    dp = torch_cuda.zeros(words, dtype=torch_cuda.int64, device="cuda")
    k = Keep(torch_cuda)
    L.check(L.lib().sufb200_pack_eff_bits(k.dev(xs), eff_bits, _p(dp), n, None))
    assert (from_dev(dp) == oracle.pack_eff_bits(xs, eff_bits)).all()
    du = torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda")
    L.check(L.lib().sufb200_unpack_eff_bits(_p(dp), eff_bits, _p(du), n, None))
    mask = np.uint64((1 << eff_bits) - 1 if eff_bits < 64 else 2**64 - 1)
    assert (from_dev(du) == (xs & mask)).all()
    local = rand_u64(rng, n)
    L.check(L.lib().sufb200_unpack_add_mod(k.dev(local), _p(dp), eff_bits, _p(du), n, eff_bits, None))
    assert (from_dev(du) == ((local + (xs & mask)) & mask)).all()


def _scaled(acc, has_scale, c, sh):
    """beaver_scaled_acc (cuda/cuda_primitives.cu:391-417) on Python ints."""
    if not has_scale:
        return acc
    a = acc - (1 << 64) if acc >= 1 << 63 else acc
    prod = a * c
    return ((prod >> sh) if sh > 0 else prod) & (2**64 - 1)


@pytest.mark.parametrize("trans", [0, 1])
@pytest.mark.parametrize("scale", [(0, 0, 0), (1, 4096, 12), (1, -77, 0), (1, 3, 70)])
def test_beaver_matmul2d(ctx, torch_cuda, L, trans, scale):
    """Attention shapes: QK^T 12 x (128x64 . 64x128), ragged edges 37x29x45."""
    rng = np.random.default_rng(31 + trans)
    has_scale, mul_const, mul_shift = scale
    for batches, M, K, N in ((12, 128, 64, 128), (3, 37, 29, 45)):
        D = rand_u64(rng, batches * M * K).reshape(batches, M, K)
        E = rand_u64(rng, batches * K * N).reshape(batches, K, N)
        A = rand_u64(rng, M * K).reshape(M, K)
        B = rand_u64(rng, K * N).reshape(K, N)
        Cm = rand_u64(rng, M * N).reshape(M, N)
        Et = np.ascontiguousarray(E.transpose(0, 2, 1)) if trans else E
        Bt = np.ascontiguousarray(B.T) if trans else B
        k = Keep(torch_cuda)
        out = torch_cuda.empty(batches * M * N, dtype=torch_cuda.int64, device="cuda")
        for party in (0, 1):
            L.check(L.lib().sufb200_beaver_matmul2d(party, k.dev(D.ravel()), k.dev(Et.ravel()), k.dev(A.ravel()),
                                                    k.dev(Bt.ravel()), k.dev(Cm.ravel()), batches, M, K, N, trans,
                                                    has_scale, mul_const, mul_shift, _p(out), None))
            got = from_dev(out).reshape(batches, M, N)
            with np.errstate(over="ignore"):
                acc = Cm[None] + D @ B[None] + A[None] @ E + ((D @ E) if party == 0 else 0)
            if has_scale:
                exp = np.vectorize(lambda v: _scaled(int(v), 1, mul_const, mul_shift), otypes=[np.uint64])(acc)
            else:
                exp = acc
            assert (got == exp).all()


def test_row_mean_signed_opens_shift(ctx, torch_cuda, oracle, L):
    rng = np.random.default_rng(8)
    rows, cols = 128, 768
    mat = rand_u64(rng, rows * cols).reshape(rows, cols)
    valid = rng.integers(0, cols + 1, rows).astype(np.int32)
    k = Keep(torch_cuda)
    out = torch_cuda.empty(rows, dtype=torch_cuda.int64, device="cuda")
    L.check(L.lib().sufb200_row_mean(k.dev(mat.ravel()), rows, cols, k.dev(valid), _p(out), None))
    sums = oracle.row_sum(mat, valid)
    exp = np.array([int(s) // int(v) if v > 0 else 0 for s, v in zip(sums, valid)], dtype=np.uint64)
    assert (from_dev(out) == exp).all()
    n = 10_001
    a, b = rand_u64(rng, n), rand_u64(rng, n)
    for ring in (37, 50, 64):
        o = torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda")
        L.check(L.lib().sufb200_open_add_to_signed(k.dev(a), k.dev(b), _p(o), n, ring, None))
        m = (1 << ring) - 1
        exp = np.array([((int(x) + int(y)) & m) - ((1 << ring) if ((int(x) + int(y)) & m) >> (ring - 1) else 0)
                        for x, y in zip(a, b)], dtype=np.int64).view(np.uint64)
        assert (from_dev(o) == exp).all()
        packed = oracle.pack_eff_bits(b, ring)
        L.check(L.lib().sufb200_unpack_add_to_signed(k.dev(a), k.dev(packed), ring, _p(o), n, ring, None))
        bm = b & np.uint64(m)
        exp2 = np.array([((int(x) + int(y)) & m) - ((1 << ring) if ((int(x) + int(y)) & m) >> (ring - 1) else 0)
                         for x, y in zip(a, bm)], dtype=np.int64).view(np.uint64)
        assert (from_dev(o) == exp2).all()
    for f in (0, 12, 63, 64):
        o = torch_cuda.empty(n, dtype=torch_cuda.int64, device="cuda")
        L.check(L.lib().sufb200_trunc_shift(k.dev(a), _p(o), f, n, None))
        exp = a if f == 0 else (np.zeros_like(a) if f >= 64 else a >> np.uint64(f))
        assert (from_dev(o) == exp).all()
