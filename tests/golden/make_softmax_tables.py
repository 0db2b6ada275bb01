"""Writes the configs[4] softmax fixtures from the reference's own code (run
here, where the reference checkout and oracle/_ref are built):
  suf_b200/tables/softmax_suf_f12.json -- the nExp / reciprocal SUF tables
                              the reference builds (oracle/_ref/softmax_tables
                              12); the device block's dealer reads them
  suf_b200/tables/layer_suf_f12.json -- the ReLU (row max) and 256-segment
                              constant GeLU SUF tables of the device layer
                              (oracle/_ref/softmax_tables 12 layer)
  softmax_ref_h1_l64.npz   -- a causal 64 x 64 block (seed 4): the input t and
                              the reference's own reconstruction of the
                              SoftmaxBlockTask output on its CPU backend
                              (oracle/_ref/ref_softmax_drive --dump)
  layernorm_ref_r32_c64.npz -- a 32 x 64 LayerNorm block (x ~ N(0, 1) at f = 12,
                              seed 4): x and the reference's own reconstruction
                              of runtime::LayerNormTask on its CPU backend run
                              as the protocol (SUF_FORCE_PFSS=1; without it the
                              task computes a plaintext LayerNorm instead)
Usage: python tests/golden/make_softmax_tables.py"""
from __future__ import annotations

import os
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = HERE.parents[1] / "oracle" / "_ref"


def main() -> None:
    js = subprocess.run([str(REF / "softmax_tables"), "12"], check=True, capture_output=True, text=True).stdout
    (HERE.parents[1] / "suf_b200" / "tables" / "softmax_suf_f12.json").write_text(js)
    js = subprocess.run([str(REF / "softmax_tables"), "12", "layer"], check=True, capture_output=True,
                        text=True).stdout
    (HERE.parents[1] / "suf_b200" / "tables" / "layer_suf_f12.json").write_text(js)
    with tempfile.TemporaryDirectory() as d:
        out = Path(d) / "dump.bin"
        subprocess.run([str(REF / "ref_softmax_drive"), "--heads=1", "--len=64", "--reps=1", f"--dump={out}"],
                       capture_output=True, text=True)
        raw = np.fromfile(out, dtype=np.uint64)
    n = raw.size // 2
    np.savez_compressed(HERE / "softmax_ref_h1_l64.npz", t=raw[:n], y=raw[n:], heads=1, len=64, seed=4)
    with tempfile.TemporaryDirectory() as d:
        out = Path(d) / "dump.bin"
        env = dict(os.environ, SUF_FORCE_PFSS="1")
        subprocess.run([str(REF / "ref_softmax_drive"), "--block=ln", "--rows=32", "--cols=64", "--reps=1",
                        f"--dump={out}"], capture_output=True, text=True, env=env)
        raw = np.fromfile(out, dtype=np.uint64)
    n = raw.size // 2
    np.savez_compressed(HERE / "layernorm_ref_r32_c64.npz", x=raw[:n], y=raw[n:], rows=32, cols=64, seed=4)


if __name__ == "__main__":
    main()
