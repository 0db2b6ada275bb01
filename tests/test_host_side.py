"""CPU tests of the product library's host side: exports, dealer keygen,
key builders and the CPU build of the device AES engine / walk."""
from __future__ import annotations

import ctypes as C
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle.oracle import GROUP_ADD, GROUP_XOR, KIND_ARS, KIND_GAPARS, KIND_TR
from tests.helpers import seeds_for

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def built():
    from suf_b200.build import build

    return build()


def header_functions() -> list[str]:
    txt = (ROOT / "include" / "sufb200.h").read_text()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(sufb200_\w+)\s*\(", txt)))


def test_library_exports_every_header_symbol(built):
    lib = C.CDLL(str(built))
    names = header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    from suf_b200 import _lib

    assert sorted(_lib.exported_symbols()) == names


def test_missing_library_fails_loudly(tmp_path):
    from suf_b200 import _lib

    with pytest.raises(FileNotFoundError):
        _lib.load(tmp_path / "libsufb200.so")


@pytest.fixture(scope="module")
def host_ctx(built, prg_state):
    from suf_b200.engine import Context

    import suf_b200._lib as L

    h = C.c_void_p()
    L.check(L.lib().sufb200_ctx_create(-1, C.byref(h)))
    ctx = Context.__new__(Context)
    ctx._L = L.lib()
    ctx.h = h
    ctx.device = -1
    ctx.prg_init(prg_state)
    yield ctx
    ctx.close()


def test_host_only_context_rejects_evaluation(host_ctx):
    from suf_b200 import SufB200Error

    import suf_b200._lib as L

    rc = L.lib().sufb200_myl7_dcf_eval(host_ctx.h, 0, 64, None, 2152, 1, None, 1, 8, None, None)
    assert rc == L.ERR_UNSUPPORTED
    with pytest.raises(SufB200Error):
        L.check(rc)


@pytest.mark.parametrize("group", [GROUP_ADD, GROUP_XOR])
def test_product_keygen_matches_oracle(oracle, prg_state, host_ctx, group):
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(5)
    for in_bits, plen in ((1, 8), (9, 1), (16, 8), (64, 8), (64, 20)):
        alpha = int(rng.integers(0, 2**63)) & ((1 << in_bits) - 1)
        payload = rng.integers(0, 256, plen, dtype=np.uint8).tobytes()
        nch = (plen + 15) // 16
        s0, s1 = rng.integers(0, 256, (2, 16 * nch), dtype=np.uint8)
        a0, a1 = host_ctx.myl7_gen(group, in_bits, alpha, payload, s0, s1)
        b0, b1 = oracle.myl7_gen(group, in_bits, alpha, payload, s0, s1)
        assert (a0 == b0).all() and (a1 == b1).all()


def test_product_batch_keygen(oracle, prg_state, host_ctx):
    oracle.prg_init(prg_state)
    n = 37
    alphas = oracle.mt64(1, n)
    s0, s1 = seeds_for(1, n, oracle)
    k0, k1 = host_ctx.myl7_gen_batch(GROUP_ADD, 64, alphas, (1).to_bytes(8, "little"), s0, s1)
    for i in (0, 17, n - 1):
        b0, b1 = oracle.myl7_gen(GROUP_ADD, 64, int(alphas[i]), (1).to_bytes(8, "little"), s0[i], s1[i])
        assert (k0[i] == b0).all() and (k1[i] == b1).all()


@pytest.mark.parametrize("kind", [KIND_TR, KIND_ARS, KIND_GAPARS])
@pytest.mark.parametrize("f", [4, 12, 16])
def test_product_trunc_dealer_matches_oracle(oracle, kind, f):
    from suf_b200.engine import Context

    for seed in (1, 2, 12345):
        r_a, p0, p1, thetas = Context.trunc_gen(kind, f, seed)
        r_b, o0, o1 = oracle.trunc_gen(kind, f, seed)
        assert r_a == r_b
        for p, o in ((p0, o0), (p1, o1)):
            for name in ("kind", "frac_bits", "party", "nq", "carry_a", "carry_b", "sign_a", "sign_b", "wrap_q",
                         "carry_w", "sign_w", "haty", "r_hi", "m"):
                assert getattr(p, name) == getattr(o, name), name
            assert list(p.q_bits) == list(o.q_bits)
        assert [int(t) for t in thetas[: o0.nq]] == [int(t) for t in o0.q_theta[: o0.nq]]


def test_product_key_builders_match_oracle(oracle):
    from suf_b200 import engine as E

    assert (E.thr_dcf_key(6, 5, b"\xaa") == oracle.thr_dcf_key(6, 5, b"\xaa")).all()
    for nid, tweak in ((1, 0), (2, 7), (12345, 3)):
        assert (E.seed_from_id(nid, tweak) == oracle.seed_from_id(nid, tweak)).all()
    seed = oracle.seed_from_id(4, 0)
    thr = [60, 5, 12, 33, 48]
    assert (E.packed_lt_key(1, 4, 6, thr, seed) == oracle.packed_key(1, 4, 6, thr, seed)).all()
    cuts, pay = [0, 20, 40, 64], [100, 200, 300, 400, 500, 600]
    assert (E.interval_lut_key(0, 5, 6, 2, cuts, pay, seed) == oracle.interval_key(0, 5, 6, 2, cuts, pay,
                                                                                     seed)).all()


def test_host_mt19937_64_matches_oracle(oracle):
    from suf_b200.engine import host_mt19937_64

    assert (host_mt19937_64(1, 1000) == oracle.mt64(1, 1000)).all()


# ---- CPU build of the device AES engine and walk (table layout, selectors) ----

@pytest.fixture(scope="module")
def emu(tmp_path_factory):
    out = tmp_path_factory.mktemp("emu") / "libemu.so"
    subprocess.run(["g++", "-std=c++17", "-O1", "-fPIC", "-shared", "-I/usr/local/cuda/include", "-o", str(out),
                    str(ROOT / "tests" / "hostemu" / "emu_shim.cpp")], check=True)
    E = C.CDLL(str(out))
    E.emu_dcf_eval.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_uint64, C.c_int, C.POINTER(C.c_uint64)]
    E.emu_frontier.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint32,
                               C.c_void_p]
    E.emu_walk_prefix.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_uint32, C.c_uint64, C.c_void_p]
    E.emu_make_plan.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_int, C.c_uint32, C.c_void_p, C.c_void_p,
                                C.c_void_p]
    E.emu_plan_index.argtypes = [C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint64, C.c_int]
    E.emu_plan_index.restype = C.c_uint32
    return E


def test_emulated_engine_aes_and_prg(emu, oracle, prg_state):
    p = lambda a: a.ctypes.data  # noqa: E731
    emu.emu_prg_init(C.c_void_p(p(prg_state)))
    rng = np.random.default_rng(9)
    for lane in range(32):
        key = rng.integers(0, 256, 16, dtype=np.uint8)
        blk = rng.integers(0, 256, 16, dtype=np.uint8)
        out = np.zeros(16, np.uint8)
        emu.emu_aes(C.c_void_p(p(key)), C.c_void_p(p(blk)), lane, C.c_void_p(p(out)))
        assert (out == oracle.aes_ecb(key.tobytes(), blk)[0]).all()
        seed = rng.integers(0, 256, 16, dtype=np.uint8)
        seed[15] &= 0x7F
        for xb in (0, 1):
            A = np.zeros(16, np.uint8)
            B = np.zeros(8, np.uint8)
            emu.emu_prg_level(C.c_void_p(p(seed)), xb, lane, C.c_void_p(p(A)), C.c_void_p(p(B)))
            ka = prg_state[32 * xb: 32 * xb + 16].tobytes()
            kb = prg_state[32 * xb + 16: 32 * xb + 32].tobytes()
            assert (A == (oracle.aes_ecb(ka, seed)[0] ^ seed)).all()
            assert (B == (oracle.aes_ecb(kb, seed)[0] ^ seed)[:8]).all()


@pytest.mark.parametrize("group", [GROUP_ADD, GROUP_XOR])
def test_emulated_walk_matches_oracle(emu, oracle, prg_state, group):
    emu.emu_prg_init(C.c_void_p(prg_state.ctypes.data))
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(13 + group)
    for nb in (1, 5, 16, 64):
        alpha = int(rng.integers(0, 2**63)) & ((1 << nb) - 1)
        s0, s1 = rng.integers(0, 256, (2, 16), dtype=np.uint8)
        k0, k1 = oracle.myl7_gen(group, nb, alpha, rng.integers(0, 256, 8, dtype=np.uint8).tobytes(), s0, s1)
        xs = rng.integers(0, 2**63, 40, dtype=np.uint64)
        xs[0] = alpha
        for k in (k0, k1):
            ref = oracle.myl7_eval(group, k, k.size, True, xs, 8).view(np.uint64).ravel()
            for i, x in enumerate(xs):
                v = C.c_uint64()
                emu.emu_dcf_eval(group, k.ctypes.data, nb, C.c_uint64(int(x)), i % 32, C.byref(v))
                assert v.value == int(ref[i])


# ---- shared-prefix plan and frontier traversal (prefix.cuh) on the CPU ----

def _plan(emu, pivot, mn, mx, n, kmax):
    d, c, f = C.c_uint32(), C.c_uint32(), C.c_uint64()
    emu.emu_make_plan(C.c_uint64(pivot), C.c_uint64((mn + 2**63) % 2**64), C.c_uint64((mx + 2**63) % 2**64),
                      n, kmax, C.byref(d), C.byref(c), C.byref(f))
    return d.value, c.value, f.value


def test_plan_matches_brute_force(emu):
    """make_plan picks the deepest D whose distinct D-bit prefixes over the
    window fit kmax, and plan_index maps them one-to-one onto 0 .. count-1
    (windows that wrap around 2^n, constant batches, full coverage)."""
    emu.emu_plan_index.restype = C.c_uint32
    rng = np.random.default_rng(21)
    for trial in range(600):
        n = int(rng.choice([6, 9, 12]))
        M = 1 << n
        pivot = int(rng.integers(0, 2**63)) * 2 + int(rng.integers(0, 2))
        width = int(rng.integers(0, min(M, 1 << int(rng.integers(0, n + 1)))))
        if trial % 50 == 0:
            width = 0
        mn = -int(rng.integers(0, width + 1))
        mx = mn + width
        kmax = int(rng.integers(1, 80))
        d, c, f = _plan(emu, pivot, mn, mx, n, kmax)
        vals = [((pivot + o) % 2**64) % M for o in range(mn, mx + 1)]
        best = (0, 1)
        for dd in range(n, 0, -1):
            pres = {v >> (n - dd) for v in vals}
            if len(pres) <= kmax:
                best = (dd, len(pres))
                break
        assert (d, c) == best, (n, pivot, mn, mx, kmax)
        if d:
            idx = {}
            for v in vals:
                i = emu.emu_plan_index(d, c, C.c_uint64(f), C.c_uint64(v), n)
                assert i < c
                assert idx.setdefault(v >> (n - d), i) == i
            assert len(set(idx.values())) == len(idx)


@pytest.mark.parametrize("group", [GROUP_ADD, GROUP_XOR])
def test_frontier_traversal_matches_prefix_walks(emu, oracle, prg_state, group):
    """The frontier pass (subtree roots + depth-first expansion) stores, in
    every slot exactly once, the state a walk of that slot's prefix from the
    root reaches (the output itself at depth n)."""
    emu.emu_prg_init(C.c_void_p(prg_state.ctypes.data))
    oracle.prg_init(prg_state)
    rng = np.random.default_rng(31 + group)
    heights = set()
    for n, trials in ((10, 12), (16, 10), (64, 6)):
        for trial in range(trials):
            alpha = int(rng.integers(0, 2**63)) & ((1 << n) - 1)
            s0, s1 = rng.integers(0, 256, (2, 16), dtype=np.uint8)
            k0, _ = oracle.myl7_gen(group, n, alpha, rng.integers(0, 256, 8, dtype=np.uint8).tobytes(), s0, s1)
            pivot = int(rng.integers(0, 2**63)) * 2
            span = int(rng.integers(0, min(n, 60)))
            width = int(rng.integers(0, 1 << span)) if span else 0
            if trial == 0:
                width = (1 << n) - 1 if n < 64 else 2**64 - 1  # the whole space
            mn = -int(rng.integers(0, width + 1)) if width < 2**62 else -(width // 2)
            if trial == 1:  # a window across 0 = 2^n
                pivot, width = 2**64 - 3, 1 << min(n - 3, 40)
                mn = -(width // 2)
            mx = mn + width
            kmax = int(rng.choice([1, 7, 40, 300])) if trial != 1 else 300
            d, c, f = _plan(emu, pivot, mn, mx, n, kmax)
            for min_roots in (1, 3, 16384):
                out = np.zeros((c, 4), dtype=np.uint64)
                h = emu.emu_frontier(group, k0.ctypes.data, n, d, c, C.c_uint64(f), min_roots, out.ctypes.data)
                heights.add(h)
                assert ((out[:, 3] >> np.uint64(32)) == 1).all(), (n, d, c, f, h)
                for slot in range(c):
                    e = np.zeros(4, dtype=np.uint64)
                    pre = (f + slot) % (1 << d) if d < 64 else (f + slot) % 2**64
                    emu.emu_walk_prefix(group, k0.ctypes.data, n, d, C.c_uint64(pre), e.ctypes.data)
                    got = out[slot].copy()
                    got[3] &= np.uint64(0xFFFFFFFF)
                    assert (got == e).all(), (n, d, c, f, h, slot)
    assert max(heights) >= 3 and 0 in heights


# ---- paired-GPU open: host-side checks (no GPU) ----

def test_open_rejects_host_only_context_and_null_comm():
    import ctypes as C

    from suf_b200 import _lib
    from suf_b200.engine import Context

    ctx = Context(-1)
    try:
        h = C.c_void_p()
        uid = (C.c_uint8 * 128)()
        rc = _lib.lib().sufb200_open_comm_create(ctx.h, C.cast(uid, C.c_void_p), 2, 0, 5.0, C.byref(h))
        assert rc == _lib.ERR_INVALID and not h.value
        assert b"GPU" in _lib.lib().sufb200_last_error()
        rc = _lib.lib().sufb200_open_exchange(None, 1, None, 4, 64, 64, 0, None, None)
        assert rc == _lib.ERR_INVALID
    finally:
        ctx.close()


def test_open_unique_id_after_torch():
    """The id comes from the NCCL the process already holds (torch's, when
    torch is imported first): two ids, 128 bytes each, differ."""
    code = ("import torch, sys; sys.path.insert(0, %r); from suf_b200.engine import open_unique_id; "
            "a = open_unique_id(); b = open_unique_id(); assert len(a) == len(b) == 128 and a != b; print('ok')"
            % str(ROOT))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]


# ---- the limb identity behind the tensor-core ring matmul (ring_gemm_tc.cu) ----

def _limb_product(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    """x @ y mod 2^64 the way the kernel forms it: byte planes, the 36 limb
    products with i + j <= 7 summed per diagonal in a wrapping 32-bit
    accumulator, then sum_s (P_s mod 2^32) << 8s mod 2^64."""
    xb = [((x >> np.uint64(8 * i)) & np.uint64(0xFF)).astype(np.int64) for i in range(8)]
    yb = [((y >> np.uint64(8 * j)) & np.uint64(0xFF)).astype(np.int64) for j in range(8)]
    out = np.zeros((x.shape[0], y.shape[1]), dtype=np.uint64)
    for s in range(8):
        p = sum(xb[i] @ yb[s - i] for i in range(s + 1))  # exact in int64 here
        out += (p.astype(np.uint64) & np.uint64(0xFFFFFFFF)) << np.uint64(8 * s)
    return out


def _exact_product(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    xo, yo = x.astype(object), y.astype(object)
    return np.array((xo @ yo) % (1 << 64), dtype=np.uint64)


@pytest.mark.parametrize("k", [1, 31, 32, 300, 8192])
def test_limb_identity_is_exact(k):
    """Worst case (all bytes 0xFF) and random words: the diagonal sums that
    survive the shift fit the 32-bit accumulator up to depth 8192."""
    rng = np.random.default_rng(k)
    for x, y in ((np.full((3, k), 2**64 - 1, dtype=np.uint64), np.full((k, 4), 2**64 - 1, dtype=np.uint64)),
                 (rng.integers(0, 2**63, (3, k), dtype=np.uint64) * np.uint64(2) + np.uint64(1),
                  rng.integers(0, 2**63, (k, 4), dtype=np.uint64) * np.uint64(3))):
        assert (_limb_product(x, y) == _exact_product(x, y)).all()
    worst = 4 * 8192 * 255 * 255  # diagonal s = 3 at the maximum depth
    assert worst < 2**31


# The twelve MMAs of one step of ring_gemm_tc.cu: (TMEM column, x plane,
# first y plane of the operand, N).  Operand y_b.. of width N covers the
# planes b .. b + N/64 - 1, and product (i, j) lands on column 64 (i + j).
def _ring_gemm_schedule():
    sched = [(0, 0, 0, 256), (256, 0, 4, 256)]
    sched += [(64 * i, i, 0, 256 if i <= 4 else 64 * (8 - i)) for i in range(1, 8)]
    sched += [(64 * (i + 4), i, 4, 256 - 64 * i) for i in range(1, 4)]
    return sched


def test_ring_gemm_schedule_covers_every_limb_pair_once():
    src = (Path(__file__).resolve().parents[1] / "suf_b200" / "csrc" / "ring_gemm_tc.cu").read_text()
    for pat in (r"umma_i8\(dt\[0\], as\[0\], bs\[0\], idesc_n\(256\), accumulate\)",
                r"umma_i8\(dt\[4\], as\[0\], bs\[4\], idesc_n\(256\), accumulate\)",
                r"for \(int i = 1; i < 8; i\+\+\) umma_i8\(dt\[i\], as\[i\], bs\[0\], idesc_n\(i <= 4 \? 256 : 64 \* \(8 - i\)\), 1u\)",
                r"for \(int i = 1; i < 4; i\+\+\) umma_i8\(dt\[i \+ 4\], as\[i\], bs\[4\], idesc_n\(256 - 64 \* i\), 1u\)"):
        assert re.search(pat, src), pat
    sched = _ring_gemm_schedule()
    assert len(sched) == 12
    seen = {}
    for col, i, b, n in sched:
        assert n % 16 == 0 and 16 <= n <= 256 and col + n <= 512 and b * 64 + n <= 512
        for q in range(n // 64):
            j = b + q
            assert col + 64 * q == 64 * (i + j)  # lands on diagonal i + j
            seen[(i, j)] = seen.get((i, j), 0) + 1
    assert seen == {(i, j): 1 for i in range(8) for j in range(8) if i + j <= 7}
    # the two MMAs that start from zero on the first step cover all 512 columns
    assert sorted((c, c + n) for c, _, _, n in sched[:2]) == [(0, 256), (256, 512)]


def test_ring_gemm_schedule_product_is_exact():
    """Numpy emulation of the twelve MMAs (u8 planes, wrapping int32
    columns) folded as the epilogue does, against the exact product."""
    rng = np.random.default_rng(12)
    M, K, N = 5, 96, 3
    x = rng.integers(0, 2**63, (M, K), dtype=np.uint64) * np.uint64(2) + np.uint64(1)
    y = rng.integers(0, 2**63, (K, N), dtype=np.uint64) * np.uint64(3)
    xp = [((x >> np.uint64(8 * i)) & np.uint64(255)).astype(np.int64) for i in range(8)]
    yp = [((y >> np.uint64(8 * j)) & np.uint64(255)).astype(np.int64) for j in range(8)]
    tmem = np.zeros((M, 8, N), dtype=np.int64)  # column block s of width N stands for 64 columns
    for col, i, b, n in _ring_gemm_schedule():
        for q in range(n // 64):
            tmem[:, col // 64 + q] = (tmem[:, col // 64 + q] + xp[i] @ yp[b + q]) % 2**32
    acc = np.zeros((M, N), dtype=np.uint64)
    with np.errstate(over="ignore"):
        for s in range(8):
            acc += tmem[:, s].astype(np.uint64) << np.uint64(8 * s)
    assert (acc == _exact_product(x, y)).all()


def test_bench_reference_dealer_matches_product_dealer():
    """bench.py's reference arm deals the configs[1] bundle with the oracle's
    truncation dealer and the reference's own dcf_gen (no product library);
    its material must equal the product dealer's byte for byte, so both arms
    evaluate the same keys."""
    import bench
    from oracle.oracle import RefMyl7
    from suf_b200.engine import Context

    if not RefMyl7.available():
        pytest.skip("oracle/_ref not built")
    ctx = Context(-1)
    try:
        ctx.prg_init(bench.prg_state())
        r1, d1, k1 = bench.dealer(ctx)
    finally:
        ctx.close()
    r2, d2, k2 = bench.ref_dealer()
    assert r1 == r2
    assert (bench.ref_prg_state() == bench.prg_state()).all()
    for p in (0, 1):
        for f in ("kind", "frac_bits", "party", "nq", "carry_a", "carry_b", "sign_a", "sign_b", "wrap_q", "carry_w",
                  "sign_w", "haty", "r_hi", "m"):
            assert getattr(d1[p], f) == getattr(d2[p], f), f
        assert len(k1[p]) == len(k2[p])
        for a, b in zip(k1[p], k2[p]):
            assert a.tobytes() == b.tobytes()


def test_bench_masked_shares_open_to_xhat():
    """The bench step opens x^ from the parties' masked shares."""
    import bench

    xh = np.arange(1000, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    m0, m1 = bench.masked_shares(xh, 3)
    assert ((m0 + m1) == xh).all()
    assert not (m0 == xh).all()


def test_per_element_dealer_matches_oracle_gates():
    """sufb200_trunc_gen_elem: element i is the oracle's trunc_gen(kind, f,
    seed + i * 0x9E3779B97F4A7C15) -- same mask, thresholds in the fixed
    slots, descriptor words -- for every kind, carry-free elements included."""
    from oracle.oracle import Oracle
    from suf_b200.engine import Context

    orc = Oracle()
    for kind, f in ((KIND_ARS, 16), (KIND_TR, 12), (KIND_GAPARS, 12)):
        n = 8192
        r, s0, s1, w0, w1, th = Context.trunc_gen_elem(kind, f, 77, n)
        assert s0.nq == {KIND_ARS: 4, KIND_TR: 3, KIND_GAPARS: 2}[kind]
        for i in [*range(0, n, 97), *np.flatnonzero((r & np.uint64((1 << f) - 1)) == 0).tolist()]:
            ro, d0, d1 = orc.trunc_gen(kind, f, (77 + i * 0x9E3779B97F4A7C15) & (2**64 - 1))
            assert ro == int(r[i])
            for q in range(d0.nq):
                assert int(d0.q_theta[q]) == int(th[i, q]) and d0.q_bits[q] == s0.q_bits[q]
            for q in range(d0.nq, s0.nq):  # carry-free element: threshold 0 in the f-bit slots
                assert int(th[i, q]) == 0
            plan = int(w0[i, 5])
            idx = [(plan >> (4 * j)) & 0xF for j in range(5)]
            assert [(-1 if v == 0xF else v) for v in idx] == [d0.carry_a, d0.carry_b, d0.sign_a, d0.sign_b, d0.wrap_q]
            for d, w in ((d0, w0), (d1, w1)):
                assert [d.carry_w, d.sign_w, d.haty, d.r_hi, d.m] == [int(v) for v in w[i, :5]]


def test_ctypes_mirrors_match_the_c_structs(tmp_path):
    """The Python mirrors of the C-ABI structs (TruncDesc, SoftmaxParty,
    LayerNormParty) have the C header's size and field offsets: a mismatch
    would hand the library shifted fields."""
    import ctypes as C

    from suf_b200._lib import TruncDesc
    from suf_b200.softmax import LayerNormParty, SoftmaxParty

    fields = {
        "sufb200_trunc_desc": (TruncDesc, ["frac_bits", "q_bits", "carry_a", "wrap_q", "carry_w", "haty", "m"]),
        "sufb200_softmax_party": (SoftmaxParty, ["recip_rin", "d_recip_lut", "d_row_c", "trunc", "trunc_rin",
                                                 "trunc_keys", "trunc_key_bytes", "trunc_keys_device",
                                                 "trunc_tables", "trunc_ready"]),
        "sufb200_layernorm_party": (LayerNormParty, ["d_rsqrt_lut", "d_norm_c", "trunc", "trunc_rin", "trunc_keys",
                                                     "trunc_key_bytes", "trunc_keys_device", "trunc_tables",
                                                     "trunc_ready"]),
    }
    src = ['#include <stdio.h>', '#include <stddef.h>', '#include "sufb200.h"', "int main(void) {"]
    for name, (_, fs) in fields.items():
        src.append(f'  printf("{name} %zu\\n", sizeof({name}));')
        for f in fs:
            src.append(f'  printf("{name}.{f} %zu\\n", offsetof({name}, {f}));')
    src.append("  return 0; }")
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    root = Path(__file__).resolve().parents[1]
    subprocess.run(["gcc", "-std=c11", f"-I{root / 'include'}", "-I/usr/local/cuda/include", str(c), "-o", str(exe)],
                   check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                        text=True).stdout.splitlines())
    for name, (cls, fs) in fields.items():
        assert int(got[name]) == C.sizeof(cls), name
        for f in fs:
            assert int(got[f"{name}.{f}"]) == getattr(cls, f).offset, f"{name}.{f}"
