"""configs[4] through the reference's own runtime: nn::SoftmaxBlockTask (nExp
cubic gate, ragged row sums, reciprocal with one Newton step, row-broadcast
Beaver product, probability truncation) run by the reference's phase
executor for both parties, once on its CPU backend (proto::ReferenceBackend)
and once on the B200 engine behind proto::make_real_gpu_backend with the
reference's GPU switches on (oracle/_ref/ref_softmax_drive, built from the
reference sources by oracle/Makefile).  The reconstructed probabilities must
be identical, with the reference's GPU switches on and off."""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import pytest

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
DRIVE = REF / "ref_softmax_drive"
_skip = pytest.mark.skipif(not DRIVE.exists(), reason="oracle/_ref/ref_softmax_drive not built (needs the reference checkout)")


def _run(args, timeout=1200):
    r = subprocess.run([str(DRIVE), *args], capture_output=True, text=True, timeout=timeout)
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert line, (r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    return r.returncode, json.loads(line[-1])


@_skip
def test_reference_softmax_cpu_leg_is_a_softmax():
    """Without a GPU the driver still runs the reference CPU leg: a small causal
    block whose reconstruction is within the reference's approximation error
    of the double-precision softmax."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("covered by the GPU test")
    rc, j = _run(["--heads=1", "--len=32", "--reps=1"])
    assert rc == 3 and j["active"] == 32 * 33 // 2
    assert j["ref_max_err_vs_double"] < 0.03


@pytest.mark.gpu
@_skip
@pytest.mark.parametrize("switches", [1, 0])
def test_reference_softmax_block_identical_on_b200(torch_cuda, switches):
    rc, j = _run(["--heads=12", "--len=128", "--reps=2", f"--switches={switches}"])
    print(json.dumps(j))
    assert rc == 0 and j["identical"] and j["mismatches"] == 0, j
    assert j["active"] == 99072 and j["max_err_vs_double"] < 0.03
