"""The drop-in C++ adapter (proto::SufB200Backend).

CPU: it compiles against the mirror of the reference interfaces and, when the
reference checkout is present, against the reference's own proto/ headers
(the type-level proof that make_real_gpu_backend() can return it).
GPU: tests/cpp/test_backend.cpp runs the reference's GPU-backend test
scenarios through the adapter.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

import pytest

from oracle.oracle import reference_root

ROOT = Path(__file__).resolve().parents[1]
REF = reference_root() or Path("/nonexistent")
CUDA_INC = "/usr/local/cuda/include"
FLAGS = ["-std=c++17", f"-I{ROOT / 'include'}", f"-I{ROOT / 'suf_b200' / 'host'}", f"-I{CUDA_INC}"]


def test_adapter_compiles_against_mirror():
    subprocess.run(["g++", *FLAGS, "-fsyntax-only", str(ROOT / "suf_b200" / "host" / "make_backend.cpp")], check=True)


def test_paired_open_handle_compiles(tmp_path):
    src = tmp_path / "open_tu.cpp"
    src.write_text('#include "sufb200_open.hpp"\n'
                   'int f(sufb200_ctx c, cudaStream_t s, const uint64_t* a, uint64_t* b) {\n'
                   '  sufb200::PairedOpen o(c, sufb200::PairedOpen::unique_id(), 2, 0, 1);\n'
                   '  o.exchange(a, 8, sufb200::PairedOpen::eff_bits_for_ring(37), 37, true, b, s);\n'
                   '  return sufb200::PairedOpen::eff_bits_for_ring(64); }\n')
    subprocess.run(["g++", *FLAGS, "-fsyntax-only", str(src)], check=True)


@pytest.mark.skipif(not (REF / "include" / "proto" / "backend_gpu.hpp").exists(), reason="reference checkout absent")
def test_adapter_compiles_against_reference_headers():
    subprocess.run(["g++", *FLAGS, "-DSUFB200_WITH_REFERENCE_PROTO", "-DSUF_HAVE_CUDA", f"-I{REF / 'include'}",
                    "-fsyntax-only", str(ROOT / "suf_b200" / "host" / "make_backend.cpp")], check=True)


@pytest.mark.gpu
def test_reference_backend_scenarios_through_adapter(tmp_path, torch_cuda):
    from suf_b200.build import build

    lib = build()
    exe = tmp_path / "test_backend"
    subprocess.run(["g++", *FLAGS, "-O1", str(ROOT / "tests" / "cpp" / "test_backend.cpp"), "-o", str(exe),
                    f"-L{lib.parent}", "-lsufb200", "-L/usr/local/cuda/lib64", "-lcudart",
                    f"-Wl,-rpath,{lib.parent}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip().endswith("OK")
