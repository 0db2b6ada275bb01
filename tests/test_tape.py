"""Composite tapes of truncation gates against the reference's own writer
(tests/golden/trunc_tapes.npz, made by tests/golden/make_tape_fixture.py from
gates::composite_gen_trunc_gate + gates::composite_write_tapes,
include/gates/composite_fss.hpp:645-833, 2458-2610):

- sufb200_trunc_read_tape loads each reference tape into the same bundle
  descriptor this engine's dealer deals for that (kind, f, seed), and finds
  the keys;
- sufb200_trunc_write_tapes, given those keys, writes both tapes byte for
  byte;
- damaged or mismatched tapes are refused.
Host code only (no GPU)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from suf_b200 import SufB200Error
from suf_b200.engine import Context

GOLDEN = Path(__file__).resolve().parent / "golden" / "trunc_tapes.npz"
FIELDS = ["kind", "frac_bits", "party", "nq", "carry_a", "carry_b", "sign_a", "sign_b", "wrap_q", "carry_w",
          "sign_w", "haty", "r_hi", "m"]


def _cases():
    z = np.load(GOLDEN)
    meta = z["meta"]
    return [(int(m[0]), int(m[1]), int(m[2]), int(m[3]), int(m[4]), int(m[5]), z[f"tape0_{i}"].tobytes(),
             z[f"tape1_{i}"].tobytes()) for i, m in enumerate(meta)]


CASES = _cases()


def _same_desc(a, b) -> bool:
    return all(getattr(a, f) == getattr(b, f) for f in FIELDS) and list(a.q_bits) == list(b.q_bits)


@pytest.mark.parametrize("case", CASES, ids=[f"k{c[0]}-f{c[1]}-s{c[2]}" for c in CASES])
def test_reference_tape_reads_into_the_dealt_descriptor_and_writes_back(case):
    kind, f, seed, r_in, bit_order, nkeys, tape0, tape1 = case
    r, d0, d1, thetas = Context.trunc_gen(kind, f, seed)
    assert r == r_in
    keys = []
    shares = []
    for p, (tape, want) in enumerate(((tape0, d0), (tape1, d1))):
        d, k, share = Context.trunc_read_tape(tape, kind, r_in, p)
        assert _same_desc(d, want), p
        assert len(k) == nkeys == int(want.nq)
        keys.append(k)
        shares.append(share)
    assert (shares[0] + shares[1]) % 2**64 == r_in
    t0, t1 = Context.trunc_write_tapes(kind, f, seed, keys[0], keys[1], bit_order=bit_order)
    assert t0 == tape0 and t1 == tape1


def test_damaged_or_mismatched_tapes_are_refused():
    kind, f, seed, r_in, _, _, tape0, _ = next(c for c in CASES if c[0] == 1 and c[1] == 12)
    with pytest.raises(SufB200Error):
        Context.trunc_read_tape(tape0[:-1], kind, r_in, 0)  # truncated
    with pytest.raises(SufB200Error):
        Context.trunc_read_tape(tape0 + b"\0", kind, r_in, 0)  # trailing bytes
    with pytest.raises(SufB200Error):
        Context.trunc_read_tape(tape0, kind, r_in ^ 1, 0)  # another mask: r_low differs
    with pytest.raises(SufB200Error):
        Context.trunc_read_tape(tape0, 2, r_in, 0)  # another kind: query count differs
    bad = bytearray(tape0)
    bad[8] = 1  # a per-element r_in vector
    with pytest.raises(SufB200Error):
        Context.trunc_read_tape(bytes(bad), kind, r_in, 0)


def test_writer_checks_its_keys():
    kind, f, seed = 1, 12, 1
    r, d0, d1, thetas = Context.trunc_gen(kind, f, seed)
    keys = [np.zeros(8 + 32 + 33 * int(d0.q_bits[q]), dtype=np.uint8) for q in range(int(d0.nq))]
    Context.trunc_write_tapes(kind, f, seed, keys, keys)
    with pytest.raises(SufB200Error):
        Context.trunc_write_tapes(kind, f, seed, keys[:-1], keys[:-1])  # a query missing
    with pytest.raises(SufB200Error):
        Context.trunc_write_tapes(kind, f, seed, keys[:-1] + [keys[-1][:-1]], keys)  # short key


GOLDEN_MUL = 0x9E3779B97F4A7C15


@pytest.mark.gpu
@pytest.mark.parametrize("kind,f", [(0, 12), (1, 1), (1, 12), (2, 1)])
def test_per_element_tapes_on_the_device(ctx, torch_cuda, kind, f):
    """sufb200_trunc_write_tapes_elem: element i's device-written tape equals
    the host writer's tape of element i's gate (trunc_gen(kind, f, seed +
    i * 0x9E3779B97F4A7C15) with element i's keys from the slots), for both
    parties, carry-free elements included, and reads back into the element's
    descriptor."""
    from suf_b200.engine import host_mt19937_64, myl7_key_bytes
    from tests.conftest import to_dev
    from tests.helpers import ONE_LE

    n, seed = 1500, 91
    r_in, s0, s1, w0, w1, th = Context.trunc_gen_elem(kind, f, seed, n)
    nq = int(s0.nq)
    share0 = Context.trunc_gen_elem_rin_shares(kind, f, seed, n)
    seeds = host_mt19937_64(0x7A7E, 4 * n * nq).view(np.uint8).reshape(nq, n, 2, 16)
    keys = [ctx.myl7_gen_batch(0, int(s0.q_bits[q]), th[:, q], ONE_LE, np.ascontiguousarray(seeds[q, :, 0]),
                               np.ascontiguousarray(seeds[q, :, 1])) for q in range(nq)]
    kb = [myl7_key_bytes(int(s0.q_bits[q]), 8) for q in range(nq)]
    tapes = []
    for p, shape, words in ((0, s0, w0), (1, s1, w1)):
        dk = [to_dev(torch_cuda, keys[q][p].ravel()) for q in range(nq)]
        share = share0 if p == 0 else r_in - share0
        out, lens = ctx.trunc_write_tapes_elem(shape, dk, kb, to_dev(torch_cuda, words.ravel()),
                                               to_dev(torch_cuda, r_in), to_dev(torch_cuda, share))
        ctx.sync()
        tapes.append((out.cpu().numpy(), lens.cpu().numpy()))
    carry_free = 0
    for i in range(n):
        si = (seed + i * GOLDEN_MUL) % 2**64
        r, d0, d1, _ = Context.trunc_gen(kind, f, si)
        assert r == int(r_in[i])
        nqi = int(d0.nq)
        carry_free += int(d0.carry_a < 0 and f > 0)
        ki = [[keys[q][p][i] for q in range(nqi)] for p in range(2)]
        want = Context.trunc_write_tapes(kind, f, si, ki[0], ki[1])
        for p in range(2):
            buf, lens = tapes[p]
            got = buf[i, :lens[i]].tobytes()
            assert got == want[p], (i, p)
        d, _, sh = Context.trunc_read_tape(want[1], kind, r, 1)
        assert int(d.haty) == int(w1[i, 2]) and int(d.r_hi) == int(w1[i, 3]) and sh == (int(r_in[i]) - int(share0[i])) % 2**64
    if f == 1:
        assert carry_free > 0
