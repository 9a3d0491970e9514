"""A C host program (gcc, C99) built against include/*.h and linked to
libleaninfer_cuda.so, as a ggml build would link it, calling the host-side
functions that need no GPU: row sizes, the layer workspace size through the
layer descriptor and through a ggml node, and node checks."""
from __future__ import annotations

import os
import subprocess

import pytest

from conftest import ROOT

SRC = r"""
#include <stdio.h>
#include <string.h>
#include "leaninfer-ggml.h"

static void f32(li_ggml_tensor *t, long n0, long n1, long n2, long n3) {
    memset(t, 0, sizeof(*t));
    t->type = LI_GGML_TYPE_F32;
    t->ne[0] = n0; t->ne[1] = n1; t->ne[2] = n2; t->ne[3] = n3;
    t->nb[0] = 4; t->nb[1] = 4 * n0; t->nb[2] = t->nb[1] * n1; t->nb[3] = t->nb[2] * n2;
    t->data = (void *)256;
}

static void q4k(li_ggml_tensor *t, long k, long n) {
    memset(t, 0, sizeof(*t));
    t->type = LI_GGML_TYPE_Q4_K;
    t->ne[0] = k; t->ne[1] = n; t->ne[2] = 1; t->ne[3] = 1;
    t->nb[0] = 144; t->nb[1] = li_row_bytes(LI_WTYPE_Q4_K, k); t->nb[2] = t->nb[1] * n; t->nb[3] = t->nb[2];
    t->data = (void *)256;
}

int main(void) {
    const int hidden = 4096, Hk = 16, Hv = 32, D = 128, B = 8;
    const int C = 2 * Hk * D + Hv * D, NI = C + Hv * D + 2 * Hv;
    li_deltanet_layer L;
    memset(&L, 0, sizeof(L));
    L.hidden = hidden; L.n_k_heads = Hk; L.n_v_heads = Hv; L.head_dim = D; L.conv_kernel = 4;
    L.w_in_type = LI_WTYPE_Q4_K; L.w_out_type = LI_WTYPE_Q4_K;
    const size_t ws_layer = li_deltanet_layer_workspace_size(&L, B);

    li_ggml_tensor y, x, cs, st, win, cw, alog, dtb, nw, wout;
    f32(&y, hidden, B, 1, 1); f32(&x, hidden, B, 1, 1); f32(&cs, 3, C, B, 1); f32(&st, D, D, Hv, B);
    q4k(&win, hidden, NI); f32(&cw, 4, C, 1, 1); f32(&alog, Hv, 1, 1, 1); f32(&dtb, Hv, 1, 1, 1);
    f32(&nw, D, 1, 1, 1); q4k(&wout, Hv * D, hidden);
    y.op = LI_GGML_OP_DELTANET_DECODE;
    li_ggml_tensor *srcs[9] = {&x, &cs, &st, &win, &cw, &alog, &dtb, &nw, &wout};
    for (int i = 0; i < 9; ++i) y.src[i] = srcs[i];
    y.op_params[0] = Hk;
    const size_t ws_node = li_ggml_workspace_size(&y);

    win.ne[1] = NI - 1;                                /* a wrong in-projection */
    const int bad_shape = li_ggml_compute_forward(&y, NULL, 0, NULL);
    y.op = 77;
    const int bad_op = li_ggml_compute_forward(&y, NULL, 0, NULL);
    printf("%zu %zu %zu %d %d\n", li_row_bytes(LI_WTYPE_Q8_0, 4096), ws_layer, ws_node, bad_shape, bad_op);
    return 0;
}
"""


def test_c_program_links_and_calls_the_host_api(tmp_path):
    from leaninfer_b200 import _lib, build
    build.build()
    lib = _lib.LIB_PATH
    src = tmp_path / "host.c"
    src.write_text(SRC)
    exe = tmp_path / "host"
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-DGGML_USE_CUDA", f"-I{ROOT / 'include'}", str(src),
                        "-o", str(exe), f"-L{lib.parent}", "-lleaninfer_cuda", f"-Wl,-rpath,{lib.parent}"],
                       capture_output=True, text=True)
    if r.returncode and "cannot find -lleaninfer_cuda" in r.stderr:
        pytest.skip("library not built")
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, env={**os.environ}, timeout=120)
    assert out.returncode == 0, out.stderr
    row, ws_layer, ws_node, bad_shape, bad_op = (int(v) for v in out.stdout.split())
    assert row == 4096 // 32 * 34
    assert ws_layer > 0 and ws_node == ws_layer
    assert bad_shape == 2002 and bad_op == 2003


def _declared_names(text: str) -> set[str]:
    import re
    return set(re.findall(r"^(?:int|size_t|void)\s+(li_\w+)\(", text, flags=re.M))


def _stub_names(text: str) -> set[str]:
    import re
    return set(re.findall(r"^static inline (?:int|size_t|void)\s+(li_\w+)\(", text, flags=re.M))


def test_every_declared_entry_has_a_no_cuda_stub():
    """The headers keep the reference's dual shape (reference
    cuda/leaninfer-cuda.h:16, :54-76) for every entry: each function declared
    for CUDA builds has a static inline stand-in for builds without it."""
    for name in ("leaninfer-cuda.h", "leaninfer-ggml.h"):
        text = (ROOT / "include" / name).read_text()
        decl, stubs = _declared_names(text), _stub_names(text)
        assert decl, name
        assert decl == stubs, (name, sorted(decl ^ stubs))


NO_CUDA_SRC = r"""
#include <stdio.h>
#include "leaninfer-ggml.h"

int main(void) {
    int bad = 0;
    float f = 0.f;
    li_deltanet_layer L = {0};
    li_ggml_tensor node = {0};
    /* the reference entries are no-ops and report LI_ERR_NO_CUDA */
    li_launch_fused_rms_norm_matmul_f32(&f, &f, &f, &f, 1, 1, 1e-6f, NULL);
    li_launch_fused_rms_norm_swiglu_f32(&f, &f, &f, &f, &f, 1, 1, 1e-6f, NULL);
    li_launch_fused_rms_norm_swiglu_f16(&f, &f, &f, &f, &f, 1, 1, 1e-6f, NULL);
    li_launch_fused_rms_norm_silu_gate_f32(&f, &f, &f, &f, 1, 1, 1e-6f, NULL);
    li_launch_fused_deltanet_recurrent_out_f32(&f, &f, &f, &f, &f, &f, &f, &f, &f, 128, 1, 1, 1, 0, 1, 1,
                                               0, 0, 0, NULL);
    li_launch_fused_rms_norm_qkv_f32(&f, &f, NULL, NULL, 1, 1, 1e-6f, NULL);
    bad += li_get_last_error() != LI_ERR_NO_CUDA;
    /* the additive entries return LI_ERR_NO_CUDA, size queries 0 */
    bad += li_device_status() != LI_ERR_NO_CUDA;
    bad += li_row_bytes(LI_WTYPE_Q4_K, 4096) != 16 * 144;
    bad += li_launch_dequantize(LI_WTYPE_Q8_0, &f, &f, 32, NULL) != LI_ERR_NO_CUDA;
    bad += li_launch_rms_norm_matmul_q(LI_WTYPE_Q8_0, &f, &f, &f, &f, 32, 1, 1, 1e-6f, NULL) != LI_ERR_NO_CUDA;
    bad += li_launch_fused_rms_norm_qkv_q(LI_WTYPE_Q8_0, &f, &f, &f, &f, &f, &f, &f, &f, 32, 1, 1, 1, 1, 1e-6f,
                                          NULL) != LI_ERR_NO_CUDA;
    bad += li_launch_fused_rms_norm_swiglu_q(LI_WTYPE_Q8_0, &f, &f, &f, &f, &f, 32, 1, 1, 1e-6f, NULL)
           != LI_ERR_NO_CUDA;
    bad += li_fused_ffn_workspace_size(32, 32, 1) != 0;
    bad += li_launch_fused_ffn_q(LI_WTYPE_Q8_0, &f, &f, &f, &f, &f, &f, 32, 32, 1, 1e-6f, NULL, 0, NULL)
           != LI_ERR_NO_CUDA;
    bad += li_launch_deltanet_recurrent_f32(&f, &f, &f, &f, &f, &f, &f, &f, 128, 1, 1, 1, 0, 1, 0, 0, 0, NULL)
           != LI_ERR_NO_CUDA;
    bad += li_deltanet_layer_workspace_size(&L, 1) != 0;
    bad += li_launch_deltanet_layer_decode(&L, &f, &f, &f, &f, 1, NULL, 0, NULL) != LI_ERR_NO_CUDA;
    bad += li_launch_deltanet_layer_decode_f16state(&L, &f, &f, &f, &f, 1, NULL, 0, NULL) != LI_ERR_NO_CUDA;
    bad += li_launch_deltanet_layer_decode_noalloc(&L, &f, &f, &f, &f, 1, NULL) != LI_ERR_NO_CUDA;
    bad += li_deltanet_chunk_prefill_workspace_size(64, 1, 128) != 0;
    bad += li_launch_deltanet_chunk_prefill_bf16(&f, &f, &f, &f, &f, &f, &f, 64, 1, 1, 128, 1.f, NULL, 0, NULL)
           != LI_ERR_NO_CUDA;
    bad += li_launch_gated_rmsnorm_bf16(&f, &f, &f, &f, 4, 1, 1e-6f, NULL) != LI_ERR_NO_CUDA;
    bad += li_launch_gemm_bf16_f32(&f, &f, &f, 128, 256, 64, NULL) != LI_ERR_NO_CUDA;
    bad += li_ggml_workspace_size(&node) != 0;
    bad += li_ggml_compute_forward(&node, NULL, 0, NULL) != LI_ERR_NO_CUDA;
    printf("%d\n", bad);
    return bad != 0;
}
"""


def test_c_program_without_cuda_compiles_against_the_stubs(tmp_path):
    """A C99 caller of every entry, compiled without GGML_USE_CUDA (a CPU-only
    ggml build), compiles, links with nothing and gets LI_ERR_NO_CUDA."""
    src = tmp_path / "nocuda.c"
    src.write_text(NO_CUDA_SRC)
    exe = tmp_path / "nocuda"
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}", str(src),
                        "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.strip() == "0", out.stdout + out.stderr
