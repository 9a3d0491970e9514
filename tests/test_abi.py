"""The C ABI: header shape, exported symbols and host-side argument checks
(CPU only: nothing here launches a kernel)."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "leaninfer-cuda.h"


def _cuda_branch() -> str:
    text = HEADER.read_text()
    start = text.index("#if defined(GGML_USE_CUDA) || defined(GGML_USE_CUBLAS)")
    end = text.index("#else  /* no CUDA")
    return text[start:end]


def declared_functions() -> list[str]:
    body = re.sub(r"/\*.*?\*/", "", _cuda_branch(), flags=re.S)
    return re.findall(r"\b(li_[a-z0-9_]+)\s*\(", body)


REFERENCE_ENTRIES = [
    "li_launch_fused_rms_norm_matmul_f32", "li_launch_fused_rms_norm_swiglu_f32",
    "li_launch_fused_rms_norm_swiglu_f16", "li_launch_fused_rms_norm_silu_gate_f32",
    "li_launch_fused_deltanet_recurrent_out_f32",
]


@pytest.fixture(scope="module")
def lib():
    from leaninfer_b200 import build, _lib
    build.build()
    return _lib.load()


def test_header_keeps_reference_entries_and_dual_shape():
    names = declared_functions()
    for n in REFERENCE_ENTRIES + ["li_launch_fused_rms_norm_qkv_f32"]:
        assert n in names
    text = HEADER.read_text()
    # stub branch keeps static no-op versions of the reference entries
    stubs = text[text.index("#else  /* no CUDA"):]
    for n in REFERENCE_ENTRIES:
        assert f"static inline void {n}(" in stubs


def test_library_exports_every_declared_symbol(lib):
    for n in declared_functions():
        assert hasattr(lib, n), f"{n} declared in include/leaninfer-cuda.h but not exported"


def test_binding_covers_header(lib):
    from leaninfer_b200 import _lib
    assert set(declared_functions()) <= set(_lib.exported_names())


def test_header_compiles_as_c_without_cuda(tmp_path):
    import subprocess
    src = tmp_path / "t.c"
    src.write_text('#include "leaninfer-cuda.h"\nint main(void){li_launch_fused_rms_norm_matmul_f32(0,0,0,0,0,0,0.f,0);'
                   'return li_get_last_error() == LI_ERR_NO_CUDA ? 0 : 1;}\n')
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{ROOT/'include'}", str(src), "-o",
                        str(tmp_path / "t")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert subprocess.run([str(tmp_path / "t")]).returncode == 0


def test_row_bytes(lib):
    assert lib.li_row_bytes(8, 2048) == 64 * 34
    assert lib.li_row_bytes(12, 4096) == 16 * 144
    assert lib.li_row_bytes(12, 100) == 0
    assert lib.li_row_bytes(0, 7) == 28
    assert lib.li_row_bytes(99, 256) == 0


def test_argument_checks_reject_before_launch(lib):
    """Bad arguments are rejected on the host: no CUDA call happens, so these
    run without a GPU."""
    c = ctypes
    # null pointers
    assert lib.li_launch_rms_norm_matmul_q(12, None, None, None, None, 4096, 8, 1, 1e-6, None) == 2001
    # unsupported weight type
    x = c.c_void_p(16)
    assert lib.li_launch_rms_norm_matmul_q(3, x, None, x, x, 4096, 8, 1, 1e-6, None) == 2003
    # misaligned weights
    assert lib.li_launch_rms_norm_matmul_q(12, x, None, c.c_void_p(18), x, 4096, 8, 1, 1e-6, None) == 2005
    # K not a multiple of 256 (bulk-copied rows must be 16-byte multiples)
    assert lib.li_launch_rms_norm_matmul_q(8, x, None, x, x, 96, 8, 1, 1e-6, None) == 2002
    # empty work is a successful no-op
    assert lib.li_launch_rms_norm_matmul_q(12, x, None, x, x, 4096, 0, 1, 1e-6, None) == 0
    assert lib.li_launch_rms_norm_matmul_q(12, x, None, x, x, 4096, 8, 0, 1e-6, None) == 0
    # FFN without workspace
    assert lib.li_launch_fused_ffn_q(12, x, x, x, x, x, x, 4096, 512, 1, 1e-6, None, 0, None) == 2004
    # recurrence: unsupported head_dim
    assert lib.li_launch_deltanet_recurrent_f32(x, x, x, x, x, x, x, x, 96, 1, 4, 1, 0, 1, 96, 96, 384,
                                                None) == 2003
    # legacy void entry records its error for li_get_last_error (and clears it)
    lib.li_launch_fused_deltanet_recurrent_out_f32(x, x, x, x, x, x, x, x, x, 96, 1, 4, 1, 0, 1, 16, 96, 96,
                                                   384, None)
    assert lib.li_get_last_error() == 2003
    assert lib.li_get_last_error() == 0
    # the bounded-wait diagnostic takes 1 us .. 1 s
    assert lib.li_selftest_bounded_wait(0, None, None) == 2001
    assert lib.li_selftest_bounded_wait(1000001, None, None) == 2001


def test_layer_workspace_size(lib):
    from leaninfer_b200._lib import DeltaNetLayer
    L = DeltaNetLayer(hidden=4096, n_k_heads=16, n_v_heads=32, head_dim=128, conv_kernel=4)
    NI = 2 * 16 * 128 + 2 * 32 * 128 + 64
    need = lib.li_deltanet_layer_workspace_size(ctypes.byref(L), 64)
    assert need >= (NI + 32 * 128) * 64 * 4
    assert need % 256 == 0


def test_layer_projection_path_by_shape(lib):
    """The layer's projections are SIMT GEMVs up to 3 sequences when both
    projection shapes suit the few-row kernel (Q4_K, K = 4096: 2 units per
    lane), tensor-core GEMMs from 4 on; the workspace (proj + og fp32 for the
    SIMT path, plus the f16 operands for the tensor path) shows the choice
    without a GPU."""
    from leaninfer_b200._lib import DeltaNetLayer

    def al(v):
        return (v + 255) // 256 * 256

    L = DeltaNetLayer(hidden=4096, n_k_heads=16, n_v_heads=32, head_dim=128, conv_kernel=4,
                      w_in_type=12, w_out_type=12)
    NI = 2 * 16 * 128 + 2 * 32 * 128 + 64
    for B in (1, 2, 3):
        assert lib.li_deltanet_layer_workspace_size(ctypes.byref(L), B) == al(NI * B * 4) + al(4096 * B * 4)
    for B in (4, 8, 64):
        assert lib.li_deltanet_layer_workspace_size(ctypes.byref(L), B) > al(NI * B * 4) + al(4096 * B * 4)
    # hidden 1024 with Q4_K: K is not a multiple of 32 units of 64 weights, so
    # 3 sequences already take the tensor cores
    L2 = DeltaNetLayer(hidden=1024, n_k_heads=4, n_v_heads=8, head_dim=128, conv_kernel=4,
                       w_in_type=12, w_out_type=12)
    NI2 = 2 * 4 * 128 + 2 * 8 * 128 + 16
    assert lib.li_deltanet_layer_workspace_size(ctypes.byref(L2), 2) == al(NI2 * 2 * 4) + al(1024 * 2 * 4)
    assert lib.li_deltanet_layer_workspace_size(ctypes.byref(L2), 3) > al(NI2 * 3 * 4) + al(1024 * 3 * 4)


def test_f16_state_layer_entry_checks_before_launch(lib):
    """The fp16-state layer entry applies the fp32 entry's host checks."""
    from leaninfer_b200._lib import DeltaNetLayer
    c = ctypes
    p = c.c_void_p(256)
    L = DeltaNetLayer(hidden=1024, n_k_heads=4, n_v_heads=8, head_dim=128, conv_kernel=4, w_in_type=12,
                      w_out_type=12, w_in=256, conv_w=256, a_log=256, dt_bias=256, norm_w=256, w_out=256)
    f = lib.li_launch_deltanet_layer_decode_f16state
    ws = lib.li_deltanet_layer_workspace_size(c.byref(L), 2)
    assert f(c.byref(L), p, p, p, None, 2, p, ws, None) == 2001                   # no state
    assert f(c.byref(L), p, p, p, c.c_void_p(258), 2, p, ws, None) == 2005        # misaligned state
    assert f(c.byref(L), p, p, p, p, 2, None, 0, None) == 2004                    # no workspace
    assert f(c.byref(L), p, p, p, p, 0, p, ws, None) == 0                         # no sequences: no-op
    L.head_dim = 64
    assert f(c.byref(L), p, p, p, p, 2, p, ws, None) == 2003                      # head_dim not built
