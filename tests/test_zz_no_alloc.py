"""The layer decode entry for callers that cannot allocate device memory.

li_launch_deltanet_layer_decode_noalloc serves callers that have no way to
hand the layer a workspace (a ggml graph whose buffers were planned before
this op, a host runtime that owns every device allocation): its scratch is a
device array inside the library. These checks call it through the C ABI and
compare it with the workspace entry, li_launch_deltanet_layer_decode, on the
same inputs over two decode steps in a row (the array keeps the first call's
contents when the second starts), within the tolerance of the other GPU
parity tests. This file is collected last so a run that stops at the first
failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import assert_close, rng

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_noalloc_matches_workspace_entry_two_steps(cuda):
    """Batches 256, 64, 4, 3 and 1 in that order (every projection path:
    one-tile tensor-core GEMMs at 33-256 rows, X-stationary GEMMs at 4-32, the
    SIMT GEMVs up to 3), each for two no-allocation steps back to back on one
    stream, as consecutive layers would call it; so every call after the first
    finds the array holding a larger or equal batch's leftovers. y, the conv
    state and the recurrent state are compared with the workspace entry run
    on its own copies of the same inputs."""
    import torch
    from leaninfer_b200 import _lib, ops, synth

    lib = _lib.load()
    r = rng(2024)
    hidden, Hk, Hv = 4096, 16, 32
    w = synth.deltanet_layer(r, hidden=hidden, n_k_heads=Hk, n_v_heads=Hv, wtype=synth.Q4_K)
    layer = ops.DeltaNetLayerDecode(
        hidden=hidden, n_k_heads=Hk, n_v_heads=Hv, head_dim=128, w_in=_dev(w["w_in"], cuda),
        conv_w=_dev(w["conv_w"], cuda), a_log=_dev(w["a_log"], cuda), dt_bias=_dev(w["dt_bias"], cuda),
        norm_w=_dev(w["norm_w"], cuda), w_out=_dev(w["w_out"], cuda))
    stream = torch.cuda.current_stream().cuda_stream
    for B in (256, 64, 4, 3, 1):
        inp = synth.deltanet_inputs(r, B, w)
        # two independent copies of the states: one per entry
        cs_a, st_a = _dev(inp["conv_state"], cuda), _dev(inp["state"], cuda)
        cs_b, st_b = _dev(inp["conv_state"], cuda), _dev(inp["state"], cuda)
        ws = torch.empty(layer.workspace_bytes(B), device=cuda, dtype=torch.uint8)
        xs = [_dev((r.standard_normal((B, hidden)) * synth.DELTANET_X_SCALE).astype(np.float32), cuda)
              for _ in range(2)]
        y_a = [torch.empty(B, hidden, device=cuda) for _ in range(2)]
        y_b = [torch.empty(B, hidden, device=cuda) for _ in range(2)]
        for step in range(2):
            rc = lib.li_launch_deltanet_layer_decode(ctypes.byref(layer.L), xs[step].data_ptr(), y_a[step].data_ptr(),
                                                     cs_a.data_ptr(), st_a.data_ptr(), B, ws.data_ptr(),
                                                     ws.numel(), stream)
            assert rc == 0, (B, step, rc)
        torch.cuda.synchronize()
        for step in range(2):      # back to back, nothing in between
            rc = lib.li_launch_deltanet_layer_decode_noalloc(ctypes.byref(layer.L), xs[step].data_ptr(),
                                                             y_b[step].data_ptr(), cs_b.data_ptr(), st_b.data_ptr(),
                                                             B, stream)
            assert rc == 0, (B, step, rc)
        torch.cuda.synchronize()
        for step in range(2):
            assert_close(y_b[step].cpu().numpy(), y_a[step].cpu().numpy(), TOL, f"y B={B} step {step}")
        assert_close(cs_b.cpu().numpy(), cs_a.cpu().numpy(), TOL, f"conv state B={B}")
        assert_close(st_b.cpu().numpy(), st_a.cpu().numpy(), TOL, f"state B={B}")
        del st_a, st_b, ws
    assert lib.li_device_status() == 0


def test_noalloc_rejects_batches_beyond_the_scratch(cuda):
    from leaninfer_b200 import _lib
    from leaninfer_b200._lib import DeltaNetLayer

    lib = _lib.load()
    L = DeltaNetLayer(hidden=4096, n_k_heads=16, n_v_heads=32, head_dim=128, conv_kernel=4)
    L.w_in_type = L.w_out_type = 12   # Q4_K
    # every batch of the tensor-core path (up to 256 sequences) of this shape
    # fits in the 32 MiB array; 600 sequences do not
    assert max(lib.li_deltanet_layer_workspace_size(ctypes.byref(L), b) for b in range(1, 257)) <= 32 << 20
    assert lib.li_deltanet_layer_workspace_size(ctypes.byref(L), 600) > 32 << 20
    p = ctypes.c_void_p(256)
    assert lib.li_launch_deltanet_layer_decode_noalloc(ctypes.byref(L), p, p, p, p, 600, None) == 2008
