"""GPU parity: exact Z_2^64 matmuls on the tensor cores (ring_gemm_tc.cu,
tcgen05 kind::i8 with 8-bit limbs) -- the public-weight matmul against numpy's
wrapping uint64 product, and the Beaver matmul against the CUDA-core
sufb200_beaver_matmul2d (pinned to cuda/cuda_primitives.cu:391-628), bit for
bit, on ragged and full-size shapes and at the worst-case depth."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tests.conftest import from_dev, rand_u64
from tests.test_gpu_primitives import L, Keep, _p  # noqa: F401  (L: the library fixture)

pytestmark = pytest.mark.gpu


def _public(ctx, L, k, X, W, bias, trans):
    batch, M, K = X.shape
    N = W.shape[0] if trans else W.shape[1]
    out = k.torch.empty(batch * M * N, dtype=k.torch.int64, device="cuda")
    L.check(L.lib().sufb200_ring_matmul(ctx.h, k.dev(X.ravel()), k.dev(W.ravel()),
                                        k.dev(bias) if bias is not None else None, _p(out), batch, M, K, N, trans,
                                        None))
    ctx.sync()
    return from_dev(out).reshape(batch, M, N)


@pytest.mark.parametrize("trans", [0, 1])
@pytest.mark.parametrize("shape", [(1, 1, 1, 1), (2, 129, 33, 65), (1, 300, 31, 200), (3, 128, 768, 192),
                                   (1, 64, 1000, 130)])
def test_public_weight_matmul(ctx, torch_cuda, L, trans, shape):
    batch, M, K, N = shape
    rng = np.random.default_rng(sum(shape) + trans)
    X = rand_u64(rng, batch * M * K).reshape(batch, M, K)
    W = rand_u64(rng, K * N).reshape(K, N)
    bias = rand_u64(rng, N)
    k = Keep(torch_cuda)
    got = _public(ctx, L, k, X, np.ascontiguousarray(W.T) if trans else W, bias, trans)
    with np.errstate(over="ignore"):
        exp = X @ W[None] + bias[None, None, :]
    assert (got == exp).all()


def test_public_weight_matmul_worst_case_depth(ctx, torch_cuda, L):
    """All-ones words at the maximum depth 8192: every limb diagonal at its
    largest sum."""
    M, K, N = 130, 8192, 70
    X = np.full((1, M, K), 2**64 - 1, dtype=np.uint64)
    W = np.full((K, N), 2**64 - 1, dtype=np.uint64)
    k = Keep(torch_cuda)
    got = _public(ctx, L, k, X, W, None, 0)
    assert (got == np.uint64(K)).all()  # (-1)(-1) K = K mod 2^64


@pytest.mark.parametrize("trans", [0, 1])
@pytest.mark.parametrize("scale", [(0, 0, 0), (1, 4096, 12), (1, -77, 0), (1, 3, 70)])
def test_beaver_matmul_tc_matches_cuda_core(ctx, torch_cuda, L, trans, scale):
    """configs[4] shapes (FFN1 128x768x3072, attention 12 x 128x64x128) and
    ragged edges: identical to the CUDA-core kernel for both parties."""
    rng = np.random.default_rng(57 + trans)
    has_scale, mul_const, mul_shift = scale
    for batches, M, K, N in ((1, 128, 768, 3072), (12, 128, 64, 128), (3, 37, 29, 45), (2, 200, 4096, 40)):
        D = rand_u64(rng, batches * M * K)
        E = rand_u64(rng, batches * K * N)
        A = rand_u64(rng, M * K)
        B = rand_u64(rng, K * N)
        Cm = rand_u64(rng, M * N)
        k = Keep(torch_cuda)
        args = [k.dev(D), k.dev(E), k.dev(A), k.dev(B), k.dev(Cm)]
        ref = torch_cuda.empty(batches * M * N, dtype=torch_cuda.int64, device="cuda")
        out = torch_cuda.empty_like(ref)
        for party in (0, 1):
            L.check(L.lib().sufb200_beaver_matmul2d(party, *args, batches, M, K, N, trans, has_scale, mul_const,
                                                    mul_shift, _p(ref), None))
            L.check(L.lib().sufb200_beaver_matmul2d_tc(ctx.h, party, *args, batches, M, K, N, trans, has_scale,
                                                       C.c_int64(mul_const), mul_shift, _p(out), None))
            ctx.sync()
            assert (from_dev(out) == from_dev(ref)).all(), (batches, M, K, N, party)


def test_beaver_matmul_tc_layer_shapes(ctx, torch_cuda, L):
    """The four Beaver matmuls of a configs[4] layer (QKV, O, FFN1, FFN2),
    whose contractions split into clusters of 3, 8, 2 and 9 CTAs (the last
    one a non-portable cluster size): identical to the CUDA-core kernel."""
    rng = np.random.default_rng(91)
    for M, K, N in ((128, 768, 2304), (128, 768, 768), (128, 768, 3072), (128, 3072, 768)):
        D, E, A, B = (rand_u64(rng, n) for n in (M * K, K * N, M * K, K * N))
        Cm = rand_u64(rng, M * N)
        k = Keep(torch_cuda)
        args = [k.dev(D), k.dev(E), k.dev(A), k.dev(B), k.dev(Cm)]
        ref = torch_cuda.empty(M * N, dtype=torch_cuda.int64, device="cuda")
        out = torch_cuda.empty_like(ref)
        for party in (0, 1):
            L.check(L.lib().sufb200_beaver_matmul2d(party, *args, 1, M, K, N, 0, 1, 4096, 12, _p(ref), None))
            L.check(L.lib().sufb200_beaver_matmul2d_tc(ctx.h, party, *args, 1, M, K, N, 0, 1, C.c_int64(4096), 12,
                                                       _p(out), None))
            ctx.sync()
            assert (from_dev(out) == from_dev(ref)).all(), (M, K, N, party)


def test_ring_matmul_rejects(ctx, torch_cuda, L):
    from suf_b200 import _lib

    k = Keep(torch_cuda)
    x = k.dev(np.zeros(16, dtype=np.uint64))
    assert L.lib().sufb200_ring_matmul(ctx.h, x, x, None, x, 1, 1, 8193, 1, 0, None) == _lib.ERR_UNSUPPORTED
    assert L.lib().sufb200_beaver_matmul2d_tc(ctx.h, 0, x, x, x, x, x, 1, 1, 4097, 1, 0, 0, C.c_int64(0), 0, x,
                                              None) == _lib.ERR_UNSUPPORTED
    assert L.lib().sufb200_ring_matmul(ctx.h, x + 4, x, None, x, 1, 1, 8, 1, 0, None) == _lib.ERR_INVALID
