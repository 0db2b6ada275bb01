"""Build recipe for libsufb200.so (the CUDA kernels + C ABI), in-tree.

``python -m suf_b200.build`` (or ``build()`` from Python) compiles every
source under ``suf_b200/csrc`` with nvcc for sm_100a only and links the shared
library next to this file, so it travels with the repository snapshot.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libsufb200.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fopenmp,-O3", "--use_fast_math"]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC or put /usr/local/cuda/bin on PATH")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + [INCLUDE / "sufb200.h", Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool, ptxas_info: bool) -> str:
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if ptxas_info and src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"]
    if src.suffix == ".cpp":
        cmd = [nvcc, "-x", "cu", *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return r.stderr if ptxas_info else ""


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile the library if any source changed; return its path.  Sources
    compile in parallel; an object is rebuilt when its source, a shared
    header or this recipe is newer than it."""
    from concurrent.futures import ThreadPoolExecutor

    if not force and not _stale():
        return LIB
    nvcc = _nvcc()
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    shared = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + [INCLUDE / "sufb200.h", Path(__file__)]
    t_shared = max(p.stat().st_mtime for p in shared)
    jobs = []
    objs = []
    for src in sources():
        obj = objdir / (src.name + ".o")
        objs.append(str(obj))
        if force or ptxas_info or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, t_shared):
            jobs.append((src, obj))
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for err in ex.map(lambda j: _compile(nvcc, j[0], j[1], verbose, ptxas_info), jobs):
            if err:
                print(err, file=sys.stderr)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fopenmp", "-o", str(tmp), *objs, "-lgomp", "-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
