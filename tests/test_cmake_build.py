"""The committed CMake target (leaninfer-cuda.cmake, the counterpart of the
reference's cuda/leaninfer-cuda.cmake:25-56) configures and builds the
static library `leaninfer_cuda` for sm_100a only, and a C program links
against it the way the `llama` target would. CPU only: nvcc cross-compiles,
nothing is launched."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from conftest import ROOT

PROG = r"""
#include <stdio.h>
#include "leaninfer-cuda.h"
int main(void) {
    li_deltanet_layer L = {0};
    L.hidden = 4096; L.n_k_heads = 16; L.n_v_heads = 32; L.head_dim = 128; L.conv_kernel = 4;
    L.w_in_type = LI_WTYPE_Q4_K; L.w_out_type = LI_WTYPE_Q4_K;
    printf("%zu %zu\n", li_row_bytes(LI_WTYPE_Q4_K, 4096), li_deltanet_layer_workspace_size(&L, 64));
    return 0;
}
"""


def _cmake() -> str | None:
    return shutil.which("cmake")


@pytest.mark.skipif(_cmake() is None, reason="cmake not installed")
def test_cmake_builds_the_static_target_for_sm_100a(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not found")
    bdir = tmp_path / "build"
    r = subprocess.run([_cmake(), "-S", str(ROOT), "-B", str(bdir), f"-DCMAKE_CUDA_COMPILER={nvcc}"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    flags = (bdir / "CMakeFiles" / "leaninfer_cuda.dir" / "flags.make").read_text()
    assert "arch=compute_100a,code=[sm_100a]" in flags, flags      # sm_100a and nothing else
    r = subprocess.run([_cmake(), "--build", str(bdir), "-j", str(os.cpu_count() or 4)],
                       capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    lib = bdir / "libleaninfer_cuda.a"
    assert lib.exists()
    src = tmp_path / "prog.c"
    src.write_text(PROG)
    exe = tmp_path / "prog"
    cudalib = "/usr/local/cuda/lib64"
    r = subprocess.run(["gcc", "-std=c99", "-DGGML_USE_CUDA", f"-I{ROOT / 'include'}", str(src), str(lib),
                        f"-L{cudalib}", "-lcudart", "-lstdc++", "-lm", "-ldl", "-lpthread", "-lrt",
                        f"-Wl,-rpath,{cudalib}", "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    row, ws = (int(v) for v in out.stdout.split())
    assert row == 16 * 144 and ws > 0
