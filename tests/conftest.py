"""Shared fixtures.  Markers: `gpu` = needs a B200 (parity tests proper)."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build_oracle

    lib = ROOT / "oracle" / "liboracle.so"
    src = ROOT / "oracle" / "suf_oracle.c"
    if not lib.exists() or lib.stat().st_mtime < src.stat().st_mtime:
        build_oracle()
    return Oracle()


@pytest.fixture(scope="session")
def prg_state():
    """Fixed PRG state (8 AES keys, the reference build's kBlocks = 8)."""
    from suf_b200.engine import host_mt19937_64

    return host_mt19937_64(0x5EED_0001, 16).view(np.uint8).copy()


@pytest.fixture(scope="session")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device in this environment")
    return torch


@pytest.fixture(scope="session")
def ctx(torch_cuda, prg_state):
    """Engine context on cuda:0 with the fixed PRG installed.  A missing
    libsufb200.so raises (no fallback)."""
    from suf_b200.engine import Context

    torch_cuda.cuda.init()
    c = Context(0)
    c.prg_init(prg_state)
    yield c
    c.close()


def rand_u64(rng: np.random.Generator, n: int) -> np.ndarray:
    return rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)


def to_dev(torch, a: np.ndarray):
    """numpy (any dtype) -> CUDA tensor holding the same bytes."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint64:
        return torch.from_numpy(a.view(np.int64)).cuda()
    return torch.from_numpy(a).cuda()


def from_dev(t, dtype=np.uint64) -> np.ndarray:
    return t.cpu().numpy().view(dtype)
