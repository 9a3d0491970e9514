"""bench.py's reference arm (the oracle port on the host cores) runs without a
GPU: one JSON line per run with the keys the measurement contract names, for
each workload."""
from __future__ import annotations

import json
import subprocess
import sys

import pytest

from conftest import ROOT


@pytest.mark.parametrize("args", [["--batch", "2"], ["--workload", "qkv"], ["--workload", "ffn", "--batch", "1"],
                                  ["--workload", "layerffn", "--batch", "2"],
                                  ["--workload", "stack", "--layers", "4", "--ctx", "512"]])
def test_reference_arm_prints_one_contract_line(args):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3", *args], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]


def test_traffic_constant_matches_the_committed_capture():
    """roofline.traffic of the default line is the per-step DRAM traffic of
    the committed ncu summary (its table's per-launch bytes, summed per step
    and averaged), so the number can be recomputed from profiles/."""
    import re
    import bench
    text = (ROOT / "profiles" / "layer_decode_q4k_b64_traffic.md").read_text()
    rows = re.findall(r"^\| (\d) \| [^|]+ \| ([\d,]+) \| ([\d,]+) \|", text, flags=re.M)
    assert len(rows) == 8
    per = [int(a.replace(",", "")) + int(b.replace(",", "")) for _, a, b in rows]
    steps = [sum(per[0:4]), sum(per[4:8])]
    mean = sum(steps) // 2
    assert f"traffic_bytes_per_step_mean: {mean}" in text
    assert bench.NCU_TRAFFIC[64] == mean


def test_reference_gpu_arm_without_gpu_reports_unavailable():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "refgpu",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(ln) for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and "unavailable" in lines[0]


def test_stack_launch_count_and_bytes():
    """The stack's kernel count per step and algorithmic bytes (64 layers,
    256 sequences, context 4096 on one GPU: about 162 GB, the figure the
    workload's definition gives)."""
    import bench
    by = bench.stack_bytes(64, 256, 4096, 1)
    assert 150e9 < by["total"] < 170e9
    assert bench.stack_bytes(64, 32, 4096, 8)["weights"] < by["weights"]
    # the residual adds ride on the output projections; a sharded FFN adds
    # its reduce-scattered result with one kernel
    assert bench.stack_launches(64, 256, 1) == 48 * (4 + 4) + 16 * (2 + 3 + 2 + 4)
    # 32 sequences per GPU: X-stationary projections (prep, GEMM, reduce)
    assert bench.stack_launches(64, 32, 8) == 48 * (6 + 4 + 1) + 16 * (3 + 3 + 3 + 4 + 1)


def test_layerffn_bytes_and_launches():
    """The DeltaNet+FFN layer's algorithmic bytes are the layer's plus the
    FFN's weights (about 84.9 MB of Q4_K) and the residual stream; its kernel
    count per step is the layer's and the FFN's (their output projections add
    into the residual stream)."""
    import bench
    ffn_w = 2 * bench.q4k_bytes(12288, 4096) + bench.q4k_bytes(4096, 12288)
    assert 84e6 < ffn_w < 86e6
    assert bench.layerffn_bytes(64) == bench.algorithmic_bytes(64) + ffn_w + 4096 * 4 + 64 * 4096 * 4 * 2
    assert bench.layerffn_launches(64) == 4 + 4
    assert bench.layerffn_launches(1) == 3 + 2
