"""Build recipe of the LeanInfer B200 CUDA library (sm_100a only).

Compiles every ``csrc/*.cu`` translation unit with nvcc for
``-gencode arch=compute_100a,code=sm_100a`` and links them into
``leaninfer_b200/libleaninfer_cuda.so`` in the source tree (the built file is
not committed, but travels with the tree). Objects go to ``_build/``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libleaninfer_cuda.so"
BUILD = ROOT / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-DGGML_USE_CUDA", "-diag-suppress", "177", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the LeanInfer B200 library cannot be built")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps_mtime() -> float:
    files = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h"))
    return max(f.stat().st_mtime for f in files)


def up_to_date() -> bool:
    return LIB.exists() and LIB.stat().st_mtime >= _deps_mtime()


def _compile(src: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, ptxas_verbose: bool = False, verbose: bool = False) -> Path:
    """Compile (if stale) and return the path of the shared library."""
    if not force and up_to_date():
        return LIB
    BUILD.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_verbose), sources()))
    if verbose or ptxas_verbose:
        for obj, log in results:
            if log.strip():
                print(f"--- {obj.name}\n{log}", file=sys.stderr)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *[str(o) for o, _ in results],
           "-lcudart", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, ptxas_verbose="-v" in sys.argv, verbose=True)
    print(p)
