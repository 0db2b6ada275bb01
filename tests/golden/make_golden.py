"""Regenerate the golden fixtures in tests/golden/ (run in a checkout that has
the reference checkout, found by oracle.reference_root(): $SUF_REFERENCE or
BASELINE.json's reference_path, and oracle/_ref built).

* myl7_{add,xor}.npz -- key pairs made by the reference's own dcf_gen
  (oracle/_ref, third_party/myl7_fss/src/dcf.c) from fixed seeds, and both
  parties' outputs from the reference adapter's eval_dcf
  (include/proto/myl7_fss_backend.hpp:215-256).
* aes_ctr.json -- the KAT shape of src/demo/test_cuda_prg.cpp:22-112 (key
  bytes = mt19937_64(12345)() & 0xFF, little-endian counter blocks), with the
  ciphertexts from OpenSSL through the `cryptography` package, plus the
  FIPS-197 Appendix C.1 example.
* ref_vectors.json -- the fixed inputs and expected reconstructions of the
  reference's GPU-backend tests (src/demo/test_pfss_gpu.cpp:54-72,
  src/demo/test_cuda_packed_pfss.cpp:33-179,
  src/demo/test_cuda_trunc_gapars.cpp:57-153).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def mt64(seed: int, n: int) -> list[int]:
    from oracle.oracle import Oracle

    return [int(v) for v in Oracle().mt64(seed, n)]


def make_myl7(group: int, name: str, payload_len: int) -> None:
    from oracle.oracle import RefMyl7

    ref = RefMyl7(group)
    state = np.frombuffer(np.array(mt64(0xC0FFEE, 16), dtype=np.uint64).tobytes(), dtype=np.uint8).copy()
    ref.prg_init(state)
    rng = np.random.default_rng(20240601 + group)
    rec = {"prg_state": state}
    cases = []
    for ci, in_bits in enumerate((1, 6, 16, 37, 64)):
        alpha = int(rng.integers(0, 2**62)) & ((1 << in_bits) - 1)
        payload = rng.integers(0, 256, payload_len, dtype=np.uint8).tobytes()
        s0 = rng.integers(0, 256, 16, dtype=np.uint8)
        s1 = rng.integers(0, 256, 16, dtype=np.uint8)
        k0, k1 = ref.gen_seeded(in_bits, alpha, payload, s0, s1)
        xs = (rng.integers(0, 2**63, 24, dtype=np.uint64) * np.uint64(2)) & np.uint64((1 << in_bits) - 1)
        xs[:4] = [alpha, (alpha - 1) % (1 << in_bits), 0, (1 << in_bits) - 1]
        o0 = ref.adapter_eval(in_bits, k0, k0.size, True, xs, payload_len)
        o1 = ref.adapter_eval(in_bits, k1, k1.size, True, xs, payload_len)
        rec[f"c{ci}_meta"] = np.array([in_bits, alpha, payload_len], dtype=np.uint64)
        rec[f"c{ci}_payload"] = np.frombuffer(payload, dtype=np.uint8).copy()
        rec[f"c{ci}_seed0"] = s0
        rec[f"c{ci}_seed1"] = s1
        rec[f"c{ci}_key0"] = k0
        rec[f"c{ci}_key1"] = k1
        rec[f"c{ci}_xs"] = xs
        rec[f"c{ci}_out0"] = o0
        rec[f"c{ci}_out1"] = o1
        cases.append(ci)
    rec["cases"] = np.array(cases, dtype=np.int64)
    np.savez_compressed(HERE / name, **rec)


def make_aes() -> None:
    from cryptography.hazmat.primitives.ciphers import Cipher, algorithms, modes

    key = bytes(v & 0xFF for v in mt64(12345, 16))
    enc = Cipher(algorithms.AES(key), modes.ECB()).encryptor()
    blocks = []
    for i in list(range(8)) + [1023]:
        pt = i.to_bytes(8, "little") + bytes(8)
        blocks.append({"ctr": i, "ct": enc.update(pt).hex()})
    out = {
        "test_cuda_prg_key": key.hex(),
        "test_cuda_prg_blocks": blocks,
        "fips197_c1": {"key": bytes(range(16)).hex(), "pt": "00112233445566778899aabbccddeeff",
                       "ct": "69c4e0d86a7b0430d8cdb78070b4c55a"},
    }
    (HERE / "aes_ctr.json").write_text(json.dumps(out, indent=1) + "\n")


def make_ref_vectors() -> None:
    thr = [5, 12, 33, 48, 60]
    xs_p = [0, 15, 63]
    packed_expect = [sum(1 << j for j, t in enumerate(thr) if x < t) for x in xs_p]
    cuts = [0, 20, 40, 64]
    pay = [100, 200, 300, 400, 500, 600]
    xs_l = [0, 25, 50]
    lut_expect = []
    for x in xs_l:
        iv = 0 if x < 20 else (1 if x < 40 else 2)
        lut_expect.append(pay[2 * iv: 2 * iv + 2])
    plain = [16, -8, 3, -1]
    out = {
        "dcf_threshold": {"source": "src/demo/test_pfss_gpu.cpp:54-72", "in_bits": 6, "alpha": 5,
                          "payload": [0xAA], "xs": [3, 5, 7], "party0_expect": [0xAA, 0, 0]},
        "interval_small": {"source": "src/demo/test_pfss_gpu.cpp:75-120", "in_bits": 6, "out_words": 1,
                           "cutpoints": [0, 32, 64], "payload": [10, 20], "xs": [0, 15, 40], "expect": [10, 10, 20]},
        "packed": {"source": "src/demo/test_cuda_packed_pfss.cpp:33-63", "in_bits": 6, "thresholds": thr,
                   "xs": xs_p, "expect": packed_expect},
        "interval": {"source": "src/demo/test_cuda_packed_pfss.cpp:103-140", "in_bits": 6, "out_words": 2,
                     "cutpoints": cuts, "payload": pay, "xs": xs_l, "expect": lut_expect},
        "trunc": {"source": "src/demo/test_cuda_trunc_gapars.cpp:57-153, src/demo/test_pfss_gpu.cpp:124-204",
                  "plain": plain, "frac_bits": 4, "seeds": [1, 2, 12345],
                  "expect_ars": [v >> 4 for v in plain]},
    }
    (HERE / "ref_vectors.json").write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    from oracle.oracle import GROUP_ADD, GROUP_XOR

    make_myl7(GROUP_ADD, "myl7_add.npz", 8)
    make_myl7(GROUP_XOR, "myl7_xor.npz", 1)
    make_aes()
    make_ref_vectors()
    print("golden fixtures written to", HERE)
