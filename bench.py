"""Benchmark of the fused DeltaNet decode layer (one token per sequence).

Workload: a Gated DeltaNet layer with hidden 4096, 16 k-heads, 32 v-heads,
head_dim 128, Q4_K in-projection 4096 -> 12352 and out-projection 4096 ->
4096, width-4 causal conv, fp32 recurrent state [B, 32, 128, 128]; B
independent sequences per GPU (default 64). A step is one decode step of the
layer for the B sequences: li_launch_deltanet_layer_decode (in-projection +
conv, recurrence + gated RMSNorm, out-projection). Inputs are seeded
synthetic (random-code Q4_K weights, see leaninfer_b200/synth.py).

Multi-GPU: one process per GPU (torchrun); sequences shard across ranks with
no data-path communication (weak scaling: B sequences per rank); the time is
the max over ranks of the CUDA-event time.

L2 hygiene: steps rotate over several independent layer instances (weights
and states) so that consecutive uses of one instance are separated by more
than 3x the L2 capacity of traffic.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl reference]

Other workloads (`--workload`): `layerffn` (the same layer followed by the
SwiGLU FFN 4096 -> 12288 -> 4096, each adding into the residual stream), `prefill` (one
8192-token chunked prefill + gated norm + bf16 out-projection), `qkv`
(RMSNorm + Q/K/V Q8_0 GEMV, K = 2048, one token), `ffn` (RMSNorm + SwiGLU FFN
4096 -> 12288 -> 4096, `--batch` rows, `--wtype` 12 = Q4_K or 8 = Q8_0),
`stack` (the 64-layer hybrid decode stack) and `refgpu` (the reference's own
kernels next to this library's entries).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, HK, HV, D = 4096, 16, 32, 128
CONV_CH = 2 * HK * D + HV * D
N_IN = CONV_CH + HV * D + 2 * HV
METRIC = "fused-layer decode tokens/s"

# DRAM bytes per step (dram__bytes_read.sum + dram__bytes_write.sum summed over
# the step's kernels), the mean of two steps of one ncu capture of this bench
# (profiles/layer_decode_q4k_b64_traffic.md); writes still in L2 when a kernel
# ends are not counted by ncu.
NCU_TRAFFIC = {64: 265_305_216}
UNIT = "tokens/s"


# Batch rows from which the layer's projections run on the tensor cores (up
# to 3 rows they are SIMT GEMVs at this layer shape), and up to which they use
# the X-stationary kernel (each projection is then a GEMM launch plus a reduce
# launch).
TC_MIN_ROWS, TCX_MAX_ROWS = 4, 32


def kernels_per_step(batch: int) -> int:
    if batch < TC_MIN_ROWS:
        return 3      # in-projection GEMV, recurrence, out-projection GEMV
    if batch <= TCX_MAX_ROWS:
        return 6      # x prep, in-projection GEMM + reduce, recurrence, out-projection GEMM + reduce
    # x prep, in-projection GEMM (one CTA per 128-row tile: 97 tiles, no K
    # split, the conv epilogue inside), recurrence, out-projection GEMM
    return 4


def algorithmic_bytes(batch: int, state_bytes: int = 4) -> int:
    """Bytes a step must move at least once: both weight matrices (Q4_K), the
    conv weights, and per sequence the recurrent state (state_bytes per
    element) and conv state read and written plus x in and y out."""
    w_in = N_IN * (HIDDEN // 256) * 144
    w_out = HIDDEN * (HV * D // 256) * 144
    conv_w = CONV_CH * 4 * 4
    small = (2 * HV + D) * 4
    per_seq = HV * D * D * state_bytes * 2 + CONV_CH * 3 * 4 * 2 + HIDDEN * 4 * 2
    return w_in + w_out + conv_w + small + batch * per_seq


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# --------------------------------------------------------------------------
# clocks sampled during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows: list[tuple[float, list[str]]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [c.strip() for c in line.split(",")]))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float, t1: float) -> dict:
        rows = [r for t, r in self.rows if t0 <= t <= t1] or [r for _, r in self.rows]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[3:7]) if v.lower().startswith("active")})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------
# timed replays: the steps of the rotating instances chained in CUDA graphs
# --------------------------------------------------------------------------
def chained_graphs(insts: list, launch, steps: int):
    """One graph holding every instance's step in rotation order and one with
    the first steps % len(insts) of them, so `steps` steps replay as whole
    chains (a model replays its layers the same way) with no host launch
    between consecutive steps. Returns a function that runs the steps."""
    import torch

    def capture(items):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for it in items:
                launch(it)
        return g
    n = len(insts)
    full = capture(insts)
    rem = steps % n
    part = capture(insts[:rem]) if rem else None
    torch.cuda.synchronize()

    def run():
        for _ in range(steps // n):
            full.replay()
        if part is not None:
            part.replay()
    return run


def pipelined_e2e(n_inst: int, steps: int, copy_in, replay, copy_out) -> float:
    """End-to-end milliseconds of `steps` steps over the rotating instances,
    each step copying its input in from pinned host memory (copy_in(j)),
    running (replay(j)) and copying its result out (copy_out(j)), as a serving
    loop double-buffers them: host-to-device copies on one stream,
    device-to-host copies on another, the steps on the current stream, so the
    copies of one step overlap the computation of its neighbours. Instance j's
    input goes in once its previous result is out (the result may live in the
    input buffer), the step waits for its input, its result goes out after
    it. The CUDA-event interval covers every copy."""
    import torch
    stream = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ready = [torch.cuda.Event() for _ in range(n_inst)]     # input j copied in
    done = [torch.cuda.Event() for _ in range(n_inst)]      # step on instance j finished
    out = [torch.cuda.Event() for _ in range(n_inst)]       # result j copied out

    def one(i: int):
        j = i % n_inst
        with torch.cuda.stream(h2d):
            if i >= n_inst:
                h2d.wait_event(out[j])
            copy_in(j)
            ready[j].record(h2d)
        stream.wait_event(ready[j])
        replay(j)
        done[j].record(stream)
        with torch.cuda.stream(d2h):
            d2h.wait_event(done[j])
            copy_out(j)
            out[j].record(d2h)

    for i in range(min(3, steps)):
        one(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    h2d.wait_event(e0)
    d2h.wait_event(e0)
    for i in range(steps):
        one(i)
    stream.wait_stream(h2d)
    stream.wait_stream(d2h)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------
def build_instances(dev, batch: int, n_inst: int, seed: int, state_dtype=None):
    import torch
    from leaninfer_b200 import ops, synth
    insts = []
    for i in range(n_inst):
        r = np.random.Generator(np.random.PCG64(seed * 1000 + i))
        w = synth.deltanet_layer(r, hidden=HIDDEN, n_k_heads=HK, n_v_heads=HV, head_dim=D, wtype=synth.Q4_K)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        layer = ops.DeltaNetLayerDecode(hidden=HIDDEN, n_k_heads=HK, n_v_heads=HV, head_dim=D, w_in=t(w["w_in"]),
                                        conv_w=t(w["conv_w"]), a_log=t(w["a_log"]), dt_bias=t(w["dt_bias"]),
                                        norm_w=t(w["norm_w"]), w_out=t(w["w_out"]))
        inp = synth.deltanet_inputs(r, batch, w)
        state = torch.empty(batch, HV, D, D, device=dev, dtype=state_dtype or torch.float32)
        # state ~ N(0, 0.02), drawn on the device (268 MB per instance at B=64)
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1000 + i)
        state.normal_(0.0, 0.02, generator=g)
        insts.append(dict(layer=layer, x=t(inp["x"]), y=torch.empty(batch, HIDDEN, device=dev),
                          conv_state=t(inp["conv_state"]), state=state,
                          ws=torch.empty(layer.workspace_bytes(batch), device=dev, dtype=torch.uint8)))
    return insts


def run_ours(args, rank: int, world: int, dist) -> dict | None:
    import torch
    from leaninfer_b200 import ops
    from leaninfer_b200.shard import max_over_ranks, shard_bounds
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    # weak scaling: a global batch of batch x world sequences, one contiguous
    # shard of `batch` sequences per rank, no data exchange during a step
    _, B = shard_bounds(args.batch * world, world, rank)
    sbytes = 2 if args.state == "f16" else 4
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    per_inst = algorithmic_bytes(B, sbytes)
    n_inst = max(2, math.ceil(3 * l2 / per_inst) + 1)
    insts = build_instances(dev, B, n_inst, seed=rank + 1,
                            state_dtype=torch.float16 if sbytes == 2 else torch.float32)
    stream = torch.cuda.current_stream()

    def launch(it):
        it["layer"].step(it["x"], it["y"], it["conv_state"], it["state"], workspace=it["ws"])

    # One CUDA graph per instance holds the step's three launches (the ABI is
    # capture-safe: no allocation, no synchronisation); one eager call per
    # instance first fills the library's launch-attribute caches.
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for it in insts:
            launch(it)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    for it in insts:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            launch(it)
        it["graph"] = g
    torch.cuda.synchronize()

    def step(i: int):
        insts[i % n_inst]["graph"].replay()

    timed = chained_graphs(insts, launch, args.steps)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    sampler = ClockSampler(dev.index)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t_wall0 = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    timed()
    e1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    sampler.stop()
    clocks = sampler.summary(t_wall0, t_wall1)
    status = ops.device_status()
    if status:
        raise RuntimeError(f"device status {status} after the timed region")

    # e2e through the public entry with host buffers: pinned x in, y out each step
    hx = [torch.empty(B, HIDDEN, pin_memory=True) for _ in range(n_inst)]
    hy = [torch.empty(B, HIDDEN, pin_memory=True) for _ in range(n_inst)]
    for i in range(n_inst):
        hx[i].copy_(insts[i]["x"].cpu())
    e_steps = max(1, min(args.steps, 200))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e2e_ms = pipelined_e2e(n_inst, e_steps, lambda j: insts[j]["x"].copy_(hx[j], non_blocking=True),
                           lambda j: insts[j]["graph"].replay(),
                           lambda j: hy[j].copy_(insts[j]["y"], non_blocking=True))
    if dist:
        dist.barrier()

    ms, e2e_ms = max_over_ranks([ms, e2e_ms], dist, device=dev)
    if rank != 0:
        return None

    peaks = measured_peaks()
    step_s = ms / 1e3 / args.steps
    achieved = algorithmic_bytes(B, sbytes) / step_s / 1e9
    value = world * B * args.steps / (ms / 1e3)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (Q4_K weights" + (", f16 recurrent state)" if sbytes == 2 else ")"), "data": "synthetic",
        "config": {"workload": "deltanet_layer_decode_q4k" + ("_f16state" if sbytes == 2 else ""),
                   "batch_per_gpu": B, "global_batch": B * world,
                   "hidden": HIDDEN, "k_heads": HK, "v_heads": HV, "head_dim": D, "weights": "Q4_K",
                   "parallelism": f"sequence-sharded x{world}, no collectives",
                   "l2": f"inputs larger than L2: rotating {n_inst} layer instances of {per_inst / 1e6:.1f} MB"},
        "roofline": {"bound": "hbm", "kernel": "deltanet layer decode step: " + (
                         "x prep + tcgen05 in-projection (+ conv finish) + recurrence + tcgen05 out-projection"
                         if B >= TC_MIN_ROWS else
                         "in-projection GEMV + recurrence + out-projection GEMV") + " (PDL-chained)",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "algorithmic_bytes_per_step": algorithmic_bytes(B, sbytes),
                     "traffic": args.traffic if args.traffic is not None else
                     (NCU_TRAFFIC.get(B) if sbytes == 4 else None)},
        "e2e": {"value": round(world * B * e_steps / (e2e_ms / 1e3), 1), "unit": UNIT,
                "h2d_bytes_per_step": B * HIDDEN * 4, "d2h_bytes_per_step": B * HIDDEN * 4},
        "gpu_launches": kernels_per_step(B) * args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(B, args.cpu_steps)
    return line


# --------------------------------------------------------------------------
# CPU legs: the oracle (the C restatement of the path) on the host cores
# --------------------------------------------------------------------------
def cpu_oracle():
    """The oracle for the timed CPU legs: rebuilt with -march=native for this
    host when the compiler allows (else the portable build)."""
    from oracle import oracle
    native = oracle.use_native()
    return oracle, ("-O3 -march=native" if native else "-O3 -march=x86-64-v3")


def cpu_baseline(batch: int, steps: int) -> dict:
    """The layer step on the host cores in ggml's CPU arithmetic (q8_K
    activations, integer dots for the Q4_K projections; the recurrence in
    double), all threads."""
    from leaninfer_b200 import synth
    oracle, flags = cpu_oracle()
    r = np.random.Generator(np.random.PCG64(7))
    w = synth.deltanet_layer(r, hidden=HIDDEN, n_k_heads=HK, n_v_heads=HV, head_dim=D, wtype=synth.Q4_K)
    L, keep = oracle.make_layer(w)
    inp = synth.deltanet_inputs(r, batch, w)
    cs, st = inp["conv_state"], inp["state"]
    oracle.deltanet_layer_decode_q8act(L, keep, inp["x"], cs, st)        # warm-up
    t0 = time.perf_counter()
    for _ in range(steps):
        oracle.deltanet_layer_decode_q8act(L, keep, inp["x"], cs, st)
    dt = time.perf_counter() - t0
    return {"value": round(batch * steps / dt, 2), "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{steps} decode steps of the same layer at batch {batch} (oracle/li_oracle.c built {flags}: "
                      f"projections with ggml-style q8_K activations and integer dots, recurrence in double; "
                      f"{oracle.num_threads()} host threads)",
            "seconds": round(dt, 3)}


# --------------------------------------------------------------------------
# chunked prefill workload (one sequence; replicas only across GPUs)
# --------------------------------------------------------------------------
PF_T, PF_HK, PF_HV, PF_D, PF_HIDDEN = 8192, 16, 32, 128, 4096
# algorithmic FLOPs of one sequence: chunked gated delta rule (per v-head and
# chunk of 64: 5 C x C x D products, 3 C x D x D, the C^3/3 triangular
# solve) + the 4096 x 4096 out-projection
PF_FLOPS = PF_HV * (PF_T // 64) * (5 * 2 * 64 * 64 * 128 + 3 * 2 * 64 * 128 * 128 + 2 * 64 ** 3 // 3) + \
    2 * PF_T * PF_HIDDEN * PF_HV * PF_D


def run_prefill(args, rank: int, world: int, dist) -> dict | None:
    """One step = one 8192-token sequence through the chunked WY prefill
    (bf16 q/k/v, fp32 state), the bf16 gated RMSNorm and the bf16 4096x4096
    out-projection. Each rank runs its own sequences (independent replicas)."""
    import torch
    from leaninfer_b200 import _lib, ops
    from leaninfer_b200.shard import max_over_ranks
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    T, Hk, Hv, Dh = PF_T, PF_HK, PF_HV, PF_D
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(T, Hk, Dh, device=dev, generator=g), dim=-1).bfloat16()
    k = nrm(torch.randn(T, Hk, Dh, device=dev, generator=g), dim=-1).bfloat16()
    v = torch.randn(T, Hv, Dh, device=dev, generator=g).bfloat16()
    beta = torch.sigmoid(torch.randn(T, Hv, device=dev, generator=g))
    gl = -torch.nn.functional.softplus(torch.randn(T, Hv, device=dev, generator=g)) * \
        torch.exp(0.5 * torch.randn(T, Hv, device=dev, generator=g))
    z = torch.randn(T, Hv * Dh, device=dev, generator=g)
    gamma = torch.rand(Dh, device=dev, generator=g) + 0.5
    w_out = (0.02 * torch.randn(PF_HIDDEN, Hv * Dh, device=dev, generator=g)).bfloat16()
    state0 = 0.02 * torch.randn(Hv, Dh, Dh, device=dev, generator=g)
    states = [state0.clone() for _ in range(2)]
    ws = torch.empty(int(_lib.load().li_deltanet_chunk_prefill_workspace_size(T, Hv, Dh)), device=dev,
                     dtype=torch.uint8)
    o = torch.empty(T, Hv, Dh, device=dev)
    y = torch.empty(T, PF_HIDDEN, device=dev)
    scale = Dh ** -0.5

    def step(i: int):
        ops.deltanet_chunk_prefill_bf16(q, k, v, gl, beta, states[i % 2], scale, workspace=ws, out=o)
        og = ops.gated_rmsnorm_bf16(o.view(T * Hv, Dh), z.view(T * Hv, Dh), gamma)
        ops.gemm_bf16(og.view(T, Hv * Dh), w_out, out=y)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    sampler = ClockSampler(dev.index)
    sampler.start()
    time.sleep(0.3)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    ms = e0.elapsed_time(e1)
    sampler.stop()
    # e2e: q, k, v, g, beta, z from pinned host memory, y back, every step
    hin = [t.cpu().pin_memory() for t in (q, k, v, gl, beta, z)]
    hy = torch.empty(T, PF_HIDDEN, pin_memory=True)
    e_steps = max(1, min(args.steps, 5))
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(e_steps):
        for dst, src in zip((q, k, v, gl, beta, z), hin):
            dst.copy_(src, non_blocking=True)
        step(i)
        hy.copy_(y, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    status = ops.device_status()
    if status:
        raise RuntimeError(f"device status {status} after the timed region")
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], dist, device=dev)
    if rank != 0:
        return None
    peaks = measured_peaks()
    step_s = ms / 1e3 / args.steps
    achieved = PF_FLOPS / step_s / 1e12
    h2d = sum(t.numel() * t.element_size() for t in hin)
    line = {
        "metric": "chunked prefill tokens/s", "value": round(world * T * args.steps / (ms / 1e3), 1),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (fp32 accumulation and state)", "data": "synthetic",
        "config": {"workload": "deltanet_chunk_prefill_bf16", "tokens_per_sequence": T, "chunk": 64,
                   "k_heads": Hk, "v_heads": Hv, "head_dim": Dh, "out_proj": "bf16 4096x4096",
                   "parallelism": f"replicas x{world} (one sequence per step per GPU)",
                   "l2": "working set per step (q/k/v/z/o/y/workspace, ~1 GB) larger than L2"},
        "roofline": {"bound": "tensor", "kernel": "prefill step: chunk prep + chunk state + gated norm + bf16 GEMM",
                     "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(achieved / peaks["bf16_tflops"], 4), "peak_source": peaks["source"],
                     "algorithmic_flops_per_step": PF_FLOPS, "traffic": None},
        "e2e": {"value": round(world * T * e_steps / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": T * PF_HIDDEN * 4},
        "gpu_launches": 4 * args.steps,
        "clocks": sampler.summary(t_wall0, t_wall1),
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_prefill()
    return line


def cpu_baseline_prefill() -> dict:
    """The oracle's token-by-token recurrence (double precision, all host
    threads over the heads) on the first 256 tokens of a sequence; the
    out-projection is not in the sample."""
    oracle, flags = cpu_oracle()
    r = np.random.Generator(np.random.PCG64(11))
    n = 256

    def bf16(a):
        u = np.ascontiguousarray(a, np.float32).view(np.uint32)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    q = bf16(r.standard_normal((n, PF_HK, PF_D)) / np.sqrt(PF_D))
    k = bf16(r.standard_normal((n, PF_HK, PF_D)) / np.sqrt(PF_D))
    v = bf16(r.standard_normal((n, PF_HV, PF_D)))
    g = (-np.log1p(np.exp(r.standard_normal((n, PF_HV))))).astype(np.float32)
    beta = (1 / (1 + np.exp(-r.standard_normal((n, PF_HV))))).astype(np.float32)
    st = np.zeros((PF_HV, PF_D, PF_D), np.float32)
    t0 = time.perf_counter()
    oracle.gdr_prefill(q, k, v, g, beta, st, PF_D ** -0.5)
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 2), "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{n} tokens of the chunk recurrence, 32 v-heads (oracle/li_oracle.c built {flags}, token by token, "
                      f"double precision, {oracle.num_threads()} host threads; out-projection not included)",
            "seconds": round(dt, 3)}


# --------------------------------------------------------------------------
# quantized GEMV workloads: RMSNorm + Q/K/V (Q8_0, one token) and the SwiGLU
# FFN (gate/up + down, Q4_K or Q8_0, B rows)
# --------------------------------------------------------------------------
QKV_K, QKV_N = 2048, (2048, 512, 512)
FFN_K, FFN_N = 4096, 12288


def gemv_bytes(kind: str, wtype: int, rows: int) -> int:
    """Algorithmic bytes per step: every weight byte once, gamma, x in and
    the outputs out."""
    from leaninfer_b200 import _lib
    rb = lambda n, k: n * int(_lib.load().li_row_bytes(wtype, k))
    if kind == "qkv":
        return sum(rb(n, QKV_K) for n in QKV_N) + 4 * QKV_K * (rows + 1) + 4 * rows * sum(QKV_N)
    return 2 * rb(FFN_N, FFN_K) + rb(FFN_K, FFN_N) + 4 * FFN_K * (2 * rows + 1)


# rows from which li_launch_fused_ffn_q runs on the tensor cores
FFN_TC_MIN_ROWS = 3


def gemv_launches(kind: str, rows: int) -> int:
    if kind == "qkv":
        return 1                                  # one GEMV over the three weight segments
    if rows < FFN_TC_MIN_ROWS:
        return 2                                  # gate/up GEMV + down GEMV
    return 6 if rows <= TCX_MAX_ROWS else 4      # prep + GEMM (+ reduce) per projection


def run_gemv(args, rank: int, world: int, dist) -> dict | None:
    """qkv: li_launch_fused_rms_norm_qkv_q, K = 2048 -> 2048 / 512 / 512, Q8_0,
    one token per step (rows = 1). ffn: li_launch_fused_ffn_q, 4096 -> 12288
    -> 4096 (gate/up + down), `--wtype` Q4_K (12) or Q8_0 (8), `--batch` rows.
    Steps replay one CUDA graph per weight instance and rotate over enough
    instances that consecutive uses of one are separated by more than 3x the
    L2 capacity of traffic."""
    import torch
    from leaninfer_b200 import _lib, ops, synth
    from leaninfer_b200.shard import max_over_ranks
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    kind = args.workload
    wtype = synth.Q8_0 if kind == "qkv" else args.wtype
    rows = 1 if kind == "qkv" else args.batch
    lib = _lib.load()
    per = gemv_bytes(kind, wtype, rows)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    n_inst = max(2, math.ceil(3 * l2 / per) + 1)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    K = QKV_K if kind == "qkv" else FFN_K
    insts = []
    for i in range(n_inst):
        r = np.random.Generator(np.random.PCG64((rank + 1) * 1000 + i))
        it = dict(x=t(r.standard_normal((rows, K)).astype(np.float32)),
                  gamma=t(r.uniform(0.5, 1.5, K).astype(np.float32)))
        if kind == "qkv":
            it["W"] = [t(synth.random_weights(r, wtype, n, K)) for n in QKV_N]
            it["out"] = [torch.empty(rows, n, device=dev) for n in QKV_N]
        else:
            it["W"] = [t(synth.random_weights(r, wtype, FFN_N, K)), t(synth.random_weights(r, wtype, FFN_N, K)),
                       t(synth.random_weights(r, wtype, K, FFN_N))]
            it["y"] = torch.empty(rows, K, device=dev)
            it["ws"] = torch.empty(int(lib.li_fused_ffn_workspace_size(K, FFN_N, rows)), device=dev,
                                   dtype=torch.uint8)
        insts.append(it)
    p = ops._p

    def launch(it):
        s = ops._stream()
        if kind == "qkv":
            rc = lib.li_launch_fused_rms_norm_qkv_q(wtype, p(it["x"]), p(it["gamma"]), *(p(w) for w in it["W"]),
                                                     *(p(o) for o in it["out"]), K, *QKV_N, rows, 1e-6, s)
        else:
            rc = lib.li_launch_fused_ffn_q(wtype, p(it["x"]), p(it["gamma"]), *(p(w) for w in it["W"]),
                                           p(it["y"]), K, FFN_N, rows, 1e-6, p(it["ws"]), it["ws"].numel(), s)
        if rc:
            raise RuntimeError(f"{kind} launch failed: {rc}")

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for it in insts:
            launch(it)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    for it in insts:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            launch(it)
        it["graph"] = g
    torch.cuda.synchronize()
    timed = chained_graphs(insts, launch, args.steps)
    for i in range(args.warmup):
        insts[i % n_inst]["graph"].replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    sampler = ClockSampler(dev.index)
    sampler.start()
    time.sleep(0.3)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    e0.record(stream)
    timed()
    e1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    ms = e0.elapsed_time(e1)
    sampler.stop()
    # e2e: x from pinned host memory, the outputs back, every step
    outs = (lambda it: it["out"]) if kind == "qkv" else (lambda it: [it["y"]])
    hx = [it["x"].cpu().pin_memory() for it in insts]
    ho = [[o.cpu().pin_memory() for o in outs(it)] for it in insts]
    e_steps = max(1, min(args.steps, 200))

    def copy_out(j: int):
        for h, o in zip(ho[j], outs(insts[j])):
            h.copy_(o, non_blocking=True)

    torch.cuda.synchronize()
    e2e_ms = pipelined_e2e(n_inst, e_steps, lambda j: insts[j]["x"].copy_(hx[j], non_blocking=True),
                           lambda j: insts[j]["graph"].replay(), copy_out)
    status = ops.device_status()
    if status:
        raise RuntimeError(f"device status {status} after the timed region")
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], dist, device=dev)
    if rank != 0:
        return None
    peaks = measured_peaks()
    step_s = ms / 1e3 / args.steps
    achieved = per / step_s / 1e9
    wname = "Q8_0" if wtype == synth.Q8_0 else "Q4_K"
    out_bytes = sum(o.numel() * 4 for o in outs(insts[0]))
    line = {
        "metric": "tokens/s", "value": round(world * rows * args.steps / (ms / 1e3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": f"f32 ({wname} weights)",
        "data": "synthetic",
        "config": {"workload": "rms_norm_qkv_q8_0" if kind == "qkv" else f"ffn_{wname.lower()}",
                   "rows_per_gpu": rows, "K": K, "N": list(QKV_N) if kind == "qkv" else [FFN_N, FFN_N, FFN_K],
                   "weights": wname, "parallelism": f"replicas x{world}, no collectives",
                   "l2": f"inputs larger than L2: rotating {n_inst} weight instances of {per / 1e6:.1f} MB"},
        "roofline": {"bound": "hbm", "kernel": "RMSNorm + Q/K/V GEMV" if kind == "qkv" else
                     "RMSNorm + SwiGLU gate/up + down projection",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "algorithmic_bytes_per_step": per, "traffic": None},
        "e2e": {"value": round(world * rows * e_steps / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": rows * K * 4, "d2h_bytes_per_step": out_bytes},
        "gpu_launches": gemv_launches(kind, rows) * args.steps,
        "clocks": sampler.summary(t_wall0, t_wall1),
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_gemv(kind, wtype, rows)
    return line


def cpu_baseline_gemv(kind: str, wtype: int, rows: int) -> dict:
    """The oracle in ggml's CPU arithmetic (quantized activations, integer
    dots), all threads, on the same shapes: one step of the qkv workload, one
    row of the FFN. For the FFN also the reference's own single-thread fp32
    CPU function (cpu_rms_norm_swiglu, cuda/benchmark_fused.cu:99-121) at the
    gate/up shape, when it was built (oracle/_ref)."""
    from leaninfer_b200 import synth
    oracle, flags = cpu_oracle()
    r = np.random.Generator(np.random.PCG64(13))
    K = QKV_K if kind == "qkv" else FFN_K
    x = r.standard_normal((1, K)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
    if kind == "qkv":
        Ws = [synth.random_weights(r, wtype, n, K) for n in QKV_N]
        t0 = time.perf_counter()
        for w, n in zip(Ws, QKV_N):
            oracle.rms_norm_matmul_q8act(wtype, x, gamma, w, n, 1e-6)
    else:
        Wg, Wu = synth.random_weights(r, wtype, FFN_N, K), synth.random_weights(r, wtype, FFN_N, K)
        Wd = synth.random_weights(r, wtype, K, FFN_N)
        t0 = time.perf_counter()
        oracle.ffn_q8act(wtype, x, gamma, Wg, Wu, Wd, FFN_N, 1e-6)
    dt = time.perf_counter() - t0
    out = {"value": round(1 / dt, 2), "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
           "sample": f"one row of the {kind} workload (oracle/li_oracle.c built {flags}: ggml-style quantized "
                     f"activations and integer dots, {oracle.num_threads()} host threads)", "seconds": round(dt, 3)}
    if kind == "ffn" and oracle.REF_BENCH.exists():
        Wgf = (0.02 * r.standard_normal((FFN_N, K))).astype(np.float32)
        Wuf = (0.02 * r.standard_normal((FFN_N, K))).astype(np.float32)
        t0 = time.perf_counter()
        oracle.ref_cpu_rms_norm_swiglu(x[0], gamma, Wgf, Wuf, 1e-6)
        t_ref = time.perf_counter() - t0
        out["reference_literal"] = {
            "value": round(1 / t_ref, 2), "unit": "rows/s (gate/up only, fp32 weights)", "cores": 1,
            "sample": "the reference's cpu_rms_norm_swiglu (cuda/benchmark_fused.cu:99-121) compiled from its "
                      "sources, one row at K=4096 N=12288 with fp32 weights", "seconds": round(t_ref, 3)}
    return out


# --------------------------------------------------------------------------
# hybrid decode stack (Qwen3.5-27B-like): 48 Gated DeltaNet + 16 gated
# attention layers (3:1), SwiGLU FFN after each, 256 sequences over N GPUs
# --------------------------------------------------------------------------
ST_HIDDEN, ST_HK, ST_HV, ST_D = 5120, 16, 48, 128
ST_HQ, ST_HKV, ST_ROPE, ST_FFN = 40, 8, 64, 17408
ST_CONV = 2 * ST_HK * ST_D + ST_HV * ST_D
ST_NI = ST_CONV + ST_HV * ST_D + 2 * ST_HV
ST_NP = 2 * ST_HQ * ST_D + 2 * ST_HKV * ST_D


def q4k_bytes(rows: int, k: int) -> int:
    return rows * (k // 256) * 144


def stack_bytes(n_layers: int, batch: int, ctx: int, tp: int) -> dict:
    """Algorithmic bytes of one stack step on one GPU holding `batch`
    sequences: every weight byte once (FFN shards when tp > 1), per sequence
    the DeltaNet state and conv state read and written, the KV cache read (and
    the new token's row written), x in and out of every layer."""
    n_attn = n_layers // 4
    n_dn = n_layers - n_attn
    dn_w = q4k_bytes(ST_NI, ST_HIDDEN) + q4k_bytes(ST_HIDDEN, ST_HV * ST_D) + ST_CONV * 16 + (2 * ST_HV + ST_D + ST_HIDDEN) * 4
    at_w = q4k_bytes(ST_NP, ST_HIDDEN) + q4k_bytes(ST_HIDDEN, ST_HQ * ST_D) + (2 * ST_D + ST_HIDDEN) * 4
    ffn_w = (2 * q4k_bytes(ST_FFN, ST_HIDDEN) + q4k_bytes(ST_HIDDEN, ST_FFN)) // tp + ST_HIDDEN * 4
    per_seq = n_dn * (ST_HV * ST_D * ST_D * 4 * 2 + ST_CONV * 3 * 4 * 2) + \
        n_attn * (ctx * ST_HKV * ST_D * 2 * 2 + ST_HKV * ST_D * 2 * 2) + n_layers * 2 * (ST_HIDDEN * 4 * 2)
    weights = n_dn * dn_w + n_attn * at_w + n_layers * ffn_w
    return {"weights": weights, "per_seq": per_seq, "total": weights + batch * per_seq}


def build_stack(dev, batch: int, n_layers: int, ctx: int, tp: int, tp_rank: int, seed: int = 1):
    """The stack's layers on the device, weights drawn per layer from a
    generator seeded by the layer index (the same on every rank, so FFN shards
    of different ranks are slices of one set of weights)."""
    import torch
    from leaninfer_b200.stack import random_q4_k_device
    from leaninfer_b200.tp_ffn import ffn_split
    layers = []
    for li in range(n_layers):
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 100000 + li)
        u = lambda *shape: torch.rand(*shape, device=dev, generator=g)
        q4 = lambda n, k: random_q4_k_device(n, k, dev, g)
        attn = li % 4 == 3
        if not attn:
            l = dict(kind="deltanet", hidden=ST_HIDDEN, n_k_heads=ST_HK, n_v_heads=ST_HV, head_dim=ST_D, wtype=12,
                     w_in=q4(ST_NI, ST_HIDDEN), w_out=q4(ST_HIDDEN, ST_HV * ST_D),
                     conv_w=0.1 * torch.randn(ST_CONV, 4, device=dev, generator=g),
                     a_log=0.5 * torch.randn(ST_HV, device=dev, generator=g), dt_bias=torch.zeros(ST_HV, device=dev),
                     norm_w=u(ST_D) + 0.5, in_norm_w=(u(ST_HIDDEN) + 0.5) / 128.0,
                     conv_state=torch.zeros(batch, ST_CONV, 3, device=dev),
                     state=0.02 * torch.randn(batch, ST_HV, ST_D, ST_D, device=dev, generator=g))
        else:
            kc = torch.randn(batch, ctx, ST_HKV, ST_D, device=dev, generator=g).half()
            vc = torch.randn(batch, ctx, ST_HKV, ST_D, device=dev, generator=g).half()
            l = dict(kind="attn", hidden=ST_HIDDEN, n_q_heads=ST_HQ, n_kv_heads=ST_HKV, head_dim=ST_D,
                     rope_dim=ST_ROPE, rope_theta=1e7, wtype=12, w_in=q4(ST_NP, ST_HIDDEN),
                     w_out=q4(ST_HIDDEN, ST_HQ * ST_D), in_norm_w=(u(ST_HIDDEN) + 0.5) / 128.0,
                     q_norm_w=u(ST_D) + 0.5, k_norm_w=u(ST_D) + 0.5, k_cache=kc, v_cache=vc)
        wg, wu, wd = q4(ST_FFN, ST_HIDDEN), q4(ST_FFN, ST_HIDDEN), q4(ST_HIDDEN, ST_FFN)
        n0, n1 = ffn_split(ST_FFN, 12, tp, tp_rank) if tp > 1 else (0, ST_FFN)
        if tp > 1:
            wg, wu = wg[n0:n1].contiguous(), wu[n0:n1].contiguous()
            wd = wd[:, n0 // 256 * 144:n1 // 256 * 144].contiguous()
        l["ffn"] = dict(wtype=12, hidden=ST_HIDDEN, n_inner=n1 - n0, norm_w=(u(ST_HIDDEN) + 0.5) / 128.0,
                        w_gate=wg, w_up=wu, w_down=wd)
        layers.append(l)
    return layers


def run_stack(args, rank: int, world: int, dist) -> dict | None:
    """One step = one token for every sequence through the whole stack.
    Sequences shard across ranks (strong scaling: args.batch in total);
    with --tp-ffn the FFN weights are also split across the ranks (NCCL
    all-gather + reduce-scatter inside li_launch_ffn_q_tp)."""
    import ctypes

    import torch
    from leaninfer_b200 import _lib, ops
    from leaninfer_b200.shard import max_over_ranks, shard_bounds
    from leaninfer_b200.stack import HybridStackDecode
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    lib = _lib.load()
    tp = world if (args.tp_ffn and world > 1) else 1
    if tp > 1 and args.batch % world:
        raise ValueError("--tp-ffn needs the same number of sequences on every rank")
    _, B = shard_bounds(args.batch, world, rank)
    comm = None
    if tp > 1:
        uid = ctypes.create_string_buffer(128)
        if rank == 0 and lib.li_nccl_get_unique_id(uid) != 0:
            raise RuntimeError("li_nccl_get_unique_id failed")
        obj = [bytes(uid.raw)]
        dist.broadcast_object_list(obj, src=0)
        uid = ctypes.create_string_buffer(obj[0], 128)
        c = ctypes.c_void_p()
        rc = lib.li_nccl_comm_init_rank(ctypes.byref(c), tp, uid, rank)
        if rc:
            raise RuntimeError(f"li_nccl_comm_init_rank: {rc}")
        comm = c.value
    layers = build_stack(dev, B, args.layers, args.ctx, tp, rank)
    stack = HybridStackDecode(layers, n_seqs=B, max_ctx=args.ctx, tp_comm=comm, tp_nranks=tp)
    x = torch.randn(B, ST_HIDDEN, device=dev)
    pos = torch.full((B,), args.ctx - 1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    stack.step(x, pos)                       # eager call: fills the launch-attribute caches
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            stack.step(x, pos)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    sampler = ClockSampler(dev.index)
    sampler.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    ms = e0.elapsed_time(e1)
    sampler.stop()
    # e2e: x from pinned host memory in, the residual stream out, every step
    hx = x.cpu().pin_memory()
    hy = torch.empty_like(hx).pin_memory()
    e_steps = max(1, min(args.steps, 10))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0.record(stream)
    for _ in range(e_steps):
        x.copy_(hx, non_blocking=True)
        graph.replay()
        hy.copy_(x, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    status = ops.device_status()
    if status:
        raise RuntimeError(f"device status {status} after the timed region")
    del graph
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    if comm:
        lib.li_nccl_comm_destroy(ctypes.c_void_p(comm))
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], dist, device=dev)
    if rank != 0:
        return None
    peaks = measured_peaks()
    step_s = ms / 1e3 / args.steps
    by = stack_bytes(args.layers, B, args.ctx, tp)
    achieved = by["total"] / step_s / 1e9
    line = {
        "metric": "hybrid-stack decode tokens/s", "value": round(args.batch * args.steps / (ms / 1e3), 1),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (Q4_K weights, fp16 KV cache)", "data": "synthetic",
        "config": {"workload": "hybrid_stack_decode", "layers": args.layers,
                   "pattern": "3 Gated DeltaNet : 1 gated attention, SwiGLU FFN after each",
                   "global_batch": args.batch, "batch_per_gpu": B, "hidden": ST_HIDDEN,
                   "deltanet": {"k_heads": ST_HK, "v_heads": ST_HV, "head_dim": ST_D},
                   "attention": {"q_heads": ST_HQ, "kv_heads": ST_HKV, "head_dim": ST_D, "rope_dim": ST_ROPE,
                                 "context": args.ctx},
                   "ffn": ST_FFN, "weights": "Q4_K",
                   "parallelism": f"sequence-sharded x{world}" + (f", FFN 2-D sharded x{tp} (NCCL)" if tp > 1 else
                                                                  ", weights replicated"),
                   "l2": f"{by['total'] / 1e9:.1f} GB moved per step per GPU, far beyond L2"},
        "roofline": {"bound": "hbm", "kernel": "whole stack step (one CUDA graph)", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"], "algorithmic_bytes_per_step": by["total"], "traffic": None},
        "e2e": {"value": round(args.batch * e_steps / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": B * ST_HIDDEN * 4, "d2h_bytes_per_step": B * ST_HIDDEN * 4},
        "gpu_launches": stack_launches(args.layers, B, tp) * args.steps,
        "clocks": sampler.summary(t_wall0, t_wall1),
    }
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline_stack(args.layers, args.ctx)
    return line


def cpu_baseline_stack(n_layers: int, ctx: int) -> dict:
    """The oracle on the host cores: one DeltaNet layer step, one attention
    layer step (a cache of `ctx` tokens) and one FFN, each for one sequence at
    the stack's shapes, timed and combined as the stack composes them
    (tokens/s of one sequence = 1 / (48 t_deltanet + 16 t_attention + 64 t_ffn)
    for 64 layers)."""
    from leaninfer_b200 import synth
    oracle, flags = cpu_oracle()
    r = np.random.Generator(np.random.PCG64(17))
    w = synth.deltanet_layer(r, hidden=ST_HIDDEN, n_k_heads=ST_HK, n_v_heads=ST_HV, head_dim=ST_D, wtype=12)
    L, keep = oracle.make_layer(w)
    inp = synth.deltanet_inputs(r, 1, w)
    t0 = time.perf_counter()
    oracle.deltanet_layer_decode(L, keep, inp["x"], inp["conv_state"], inp["state"])
    t_dn = time.perf_counter() - t0
    wa = synth.attn_layer(r, hidden=ST_HIDDEN, n_q_heads=ST_HQ, n_kv_heads=ST_HKV, rope_dim=ST_ROPE, wtype=12)
    La, keepa = oracle.make_attn_layer(wa)
    ia = synth.attn_inputs(r, 1, wa, ctx)
    t0 = time.perf_counter()
    oracle.attn_layer_decode(La, keepa, ia["x"], ia["k_cache"], ia["v_cache"], ia["pos"])
    t_at = time.perf_counter() - t0
    Wg, Wu = synth.random_q4_k(r, ST_FFN, ST_HIDDEN), synth.random_q4_k(r, ST_FFN, ST_HIDDEN)
    Wd = synth.random_q4_k(r, ST_HIDDEN, ST_FFN)
    x = r.standard_normal((1, ST_HIDDEN)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, ST_HIDDEN).astype(np.float32)
    t0 = time.perf_counter()
    oracle.ffn(12, x, gamma, Wg, Wu, Wd, ST_FFN)
    t_ffn = time.perf_counter() - t0
    n_attn = n_layers // 4
    per_token = (n_layers - n_attn) * t_dn + n_attn * t_at + n_layers * t_ffn
    return {"value": round(1.0 / per_token, 4), "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"one sequence: one DeltaNet layer ({t_dn * 1e3:.1f} ms), one attention layer over {ctx} "
                      f"cached tokens ({t_at * 1e3:.1f} ms) and one FFN ({t_ffn * 1e3:.1f} ms) of the oracle "
                      f"(oracle/li_oracle.c built {flags}, double accumulation, {oracle.num_threads()} host threads), composed "
                      f"for {n_layers} layers", "seconds": round(t_dn + t_at + t_ffn, 3)}


# --------------------------------------------------------------------------
# DeltaNet + FFN decode layer: the headline's Gated DeltaNet layer followed by
# the SwiGLU FFN 4096 -> 12288 -> 4096 (Q4_K), a residual add after each, one
# li_launch_stack_decode call per step
# --------------------------------------------------------------------------
LF_METRIC = "deltanet+ffn layer decode tokens/s"


def layerffn_bytes(batch: int) -> int:
    """Algorithmic bytes of one DeltaNet+FFN layer step: the DeltaNet layer's
    (algorithmic_bytes: weights, states, x in and y out), the FFN's Q4_K
    weights and norm weights once, and per sequence the residual stream into
    and out of the FFN sub-layer."""
    ffn_w = 2 * q4k_bytes(FFN_N, FFN_K) + q4k_bytes(FFN_K, FFN_N) + FFN_K * 4
    return algorithmic_bytes(batch) + ffn_w + batch * HIDDEN * 4 * 2


def layerffn_launches(batch: int) -> int:
    """Kernels of the library per step: the DeltaNet layer's and the FFN's
    (the residual adds ride on their output projections)."""
    return kernels_per_step(batch) + gemv_launches("ffn", batch)


def build_layerffn(dev, batch: int, n_inst: int, seed: int) -> list:
    """Independent one-layer stacks (weights drawn on the device with the
    synth distributions: random-code Q4_K blocks; states N(0, 0.02))."""
    import torch
    from leaninfer_b200.stack import HybridStackDecode, random_q4_k_device
    insts = []
    for i in range(n_inst):
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1000 + i)
        u = lambda *shape: torch.rand(*shape, device=dev, generator=g)
        q4 = lambda n, k: random_q4_k_device(n, k, dev, g)
        l = dict(kind="deltanet", hidden=HIDDEN, n_k_heads=HK, n_v_heads=HV, head_dim=D, wtype=12,
                 w_in=q4(N_IN, HIDDEN), w_out=q4(HIDDEN, HV * D),
                 conv_w=0.1 * torch.randn(CONV_CH, 4, device=dev, generator=g),
                 a_log=0.5 * torch.randn(HV, device=dev, generator=g), dt_bias=torch.zeros(HV, device=dev),
                 norm_w=u(D) + 0.5, in_norm_w=(u(HIDDEN) + 0.5) / 128.0,
                 conv_state=0.1 * torch.randn(batch, CONV_CH, 3, device=dev, generator=g),
                 state=0.02 * torch.randn(batch, HV, D, D, device=dev, generator=g))
        l["ffn"] = dict(wtype=12, hidden=HIDDEN, n_inner=FFN_N, norm_w=(u(HIDDEN) + 0.5) / 128.0,
                        w_gate=q4(FFN_N, HIDDEN), w_up=q4(FFN_N, HIDDEN), w_down=q4(HIDDEN, FFN_N))
        stack = HybridStackDecode([l], n_seqs=batch, max_ctx=1)
        insts.append(dict(layer=l, stack=stack, x=torch.randn(batch, HIDDEN, device=dev, generator=g),
                          pos=torch.zeros(batch, dtype=torch.int32, device=dev)))
    return insts


def run_layerffn(args, rank: int, world: int, dist) -> dict | None:
    """One step = one token for each of the B sequences of this rank through
    the DeltaNet+FFN layer (x += deltanet(x); x += ffn(x)). Sequences shard
    across ranks with no data-path communication (weak scaling); steps rotate
    over layer instances so that consecutive uses of one are separated by more
    than 3x the L2 capacity of traffic."""
    import torch
    from leaninfer_b200 import ops
    from leaninfer_b200.shard import max_over_ranks, shard_bounds
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    _, B = shard_bounds(args.batch * world, world, rank)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    per_inst = layerffn_bytes(B)
    n_inst = max(2, math.ceil(3 * l2 / per_inst) + 1)
    insts = build_layerffn(dev, B, n_inst, seed=rank + 1)
    stream = torch.cuda.current_stream()

    def launch(it):
        it["stack"].step(it["x"], it["pos"])

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for it in insts:
            launch(it)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    for it in insts:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            launch(it)
        it["graph"] = g
    torch.cuda.synchronize()
    timed = chained_graphs(insts, launch, args.steps)
    for i in range(args.warmup):
        insts[i % n_inst]["graph"].replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    sampler = ClockSampler(dev.index)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t_wall0 = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    timed()
    e1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    ms = e0.elapsed_time(e1)
    sampler.stop()
    clocks = sampler.summary(t_wall0, t_wall1)
    status = ops.device_status()
    if status:
        raise RuntimeError(f"device status {status} after the timed region")
    # e2e: each step's x from pinned host memory in and the residual stream out
    hx = [it["x"].cpu().pin_memory() for it in insts]
    hy = [torch.empty_like(h).pin_memory() for h in hx]
    e_steps = max(1, min(args.steps, 200))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e2e_ms = pipelined_e2e(n_inst, e_steps, lambda j: insts[j]["x"].copy_(hx[j], non_blocking=True),
                           lambda j: insts[j]["graph"].replay(),
                           lambda j: hy[j].copy_(insts[j]["x"], non_blocking=True))
    if dist:
        dist.barrier()
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], dist, device=dev)
    if rank != 0:
        return None
    peaks = measured_peaks()
    step_s = ms / 1e3 / args.steps
    achieved = layerffn_bytes(B) / step_s / 1e9
    line = {
        "metric": LF_METRIC, "value": round(world * B * args.steps / (ms / 1e3), 1), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (Q4_K weights)",
        "data": "synthetic",
        "config": {"workload": "deltanet_ffn_layer_decode_q4k", "batch_per_gpu": B, "global_batch": B * world,
                   "hidden": HIDDEN, "k_heads": HK, "v_heads": HV, "head_dim": D, "ffn": FFN_N, "weights": "Q4_K",
                   "parallelism": f"sequence-sharded x{world}, no collectives",
                   "l2": f"inputs larger than L2: rotating {n_inst} layer instances of {per_inst / 1e6:.1f} MB"},
        "roofline": {"bound": "hbm", "kernel": "DeltaNet layer (prep, in-projection, recurrence, out-projection "
                                                "adding into the residual stream) + SwiGLU FFN (prep, gate/up, prep, "
                                                "down adding into the residual stream), one li_launch_stack_decode "
                                                "call",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "algorithmic_bytes_per_step": layerffn_bytes(B), "traffic": None},
        "e2e": {"value": round(world * B * e_steps / (e2e_ms / 1e3), 1), "unit": UNIT,
                "h2d_bytes_per_step": B * HIDDEN * 4, "d2h_bytes_per_step": B * HIDDEN * 4},
        "gpu_launches": layerffn_launches(B) * args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline_layerffn(B, args.cpu_steps)
    return line


def cpu_baseline_layerffn(batch: int, steps: int) -> dict:
    """The DeltaNet+FFN layer on the host cores in ggml's CPU arithmetic
    (q8_K activations and integer dots for every Q4_K projection, the
    recurrence in double), all threads, `steps` steps at `batch` sequences."""
    from leaninfer_b200 import synth
    oracle, flags = cpu_oracle()
    r = np.random.Generator(np.random.PCG64(11))
    w = synth.deltanet_layer(r, hidden=HIDDEN, n_k_heads=HK, n_v_heads=HV, head_dim=D, wtype=synth.Q4_K)
    L, keep = oracle.make_layer(w)
    inp = synth.deltanet_inputs(r, batch, w)
    Wg, Wu = synth.random_q4_k(r, FFN_N, HIDDEN), synth.random_q4_k(r, FFN_N, HIDDEN)
    Wd = synth.random_q4_k(r, HIDDEN, FFN_N)
    gamma = r.uniform(0.5, 1.5, HIDDEN).astype(np.float32) / 128.0
    cs, st = inp["conv_state"], inp["state"]

    def step(x):
        x = x + oracle.deltanet_layer_decode_q8act(L, keep, x, cs, st)
        return (x + oracle.ffn_q8act(12, x, gamma, Wg, Wu, Wd, FFN_N)).astype(np.float32)
    x = step(inp["x"])                   # warm-up
    t0 = time.perf_counter()
    for _ in range(steps):
        x = step(x)
    dt = time.perf_counter() - t0
    return {"value": round(batch * steps / dt, 2), "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{steps} steps of the DeltaNet+FFN layer at batch {batch} (oracle/li_oracle.c built {flags}: "
                      f"projections with ggml-style q8_K activations and integer dots, recurrence in double; "
                      f"{oracle.num_threads()} host threads)", "seconds": round(dt, 3)}


def stack_launches(n_layers: int, batch: int, tp: int) -> int:
    """Kernels of the library per stack step (NCCL's own kernels not counted):
    per layer the mixer's and the FFN's; the residual adds ride on their
    output projections, except after a sharded FFN (one add kernel)."""
    def proj(rows):   # one projection: SIMT GEMV, or prep + GEMM (+ reduce for the X-stationary kernel)
        return 1 if rows < TC_MIN_ROWS else (3 if rows <= TCX_MAX_ROWS else 2)
    n_attn = n_layers // 4
    dn = kernels_per_step(batch)
    at = proj(batch) + 3 + proj(batch)
    ffn = gemv_launches("ffn", batch * tp)
    add = 1 if tp > 1 else 0
    return (n_layers - n_attn) * (dn + ffn + add) + n_attn * (at + ffn + add)


# --------------------------------------------------------------------------
# the reference's own GPU kernels next to this library's entries, same box
# --------------------------------------------------------------------------
# fp32 RMSNorm + SwiGLU shapes of the reference benchmark
# (cuda/benchmark_fused.cu:144-148): Qwen2.5-0.5B, Qwen3.5-9B, Qwen3-14B
REF_SWIGLU_SHAPES = [("Qwen2.5-0.5B", 896, 4864), ("Qwen3.5-9B", 3584, 18944), ("Qwen3-14B", 5120, 17408)]


def run_refgpu(args, impl: str) -> dict:
    """Times the fp32 RMSNorm + SwiGLU entry at the reference benchmark's
    three shapes and the recurrence + out-projection entry at the decode
    layer's shape (64 sequences, 32 v-heads, head_dim 128, hidden 4096, one
    token), all through li_launch_* with the same arguments: impl "ours" calls
    this library, impl "reference" the reference's kernels built from its
    sources (oracle/_ref/libliref_gpu.so). Timing as the reference benchmark
    (cuda/benchmark_fused.cu:126-137: warm-up, then back-to-back launches), but
    with CUDA events; weight copies rotate so that the working set of
    consecutive launches exceeds 3x the L2."""
    import ctypes

    import torch
    if not torch.cuda.is_available():
        return {"impl": impl, "unavailable": "no CUDA device: the reference's kernels need a GPU"}
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    if impl == "reference":
        from oracle import oracle
        if not oracle.REF_GPU.exists():
            return {"impl": "reference", "unavailable": "the reference's kernels were not built (oracle/_ref)"}
        lib = ctypes.CDLL(str(oracle.REF_GPU))
    else:
        from leaninfer_b200 import _lib
        lib = _lib.load()
    c_p, c_i, c_f, c_64, c_sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int64, ctypes.c_size_t
    sw = lib.li_launch_fused_rms_norm_swiglu_f32
    sw.argtypes = [c_p] * 5 + [c_i, c_i, c_f, c_p]
    sw.restype = None
    rec = lib.li_launch_fused_deltanet_recurrent_out_f32
    rec.argtypes = [c_p] * 9 + [c_64] * 4 + [c_i, c_64, c_64, c_sz, c_sz, c_sz, c_p]
    rec.restype = None
    stream = torch.cuda.current_stream()
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    peaks = measured_peaks()
    cases = {}
    g = torch.Generator(device=dev)
    g.manual_seed(31)

    def timed(fn, n_copies, iters):
        for i in range(3):
            fn(i % n_copies)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(iters):
            fn(i % n_copies)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters * 1e3     # us per launch

    for name, K, N in REF_SWIGLU_SHAPES:
        wbytes = 2 * N * K * 4
        n_copies = max(1, math.ceil(3 * l2 / wbytes) + 1) if wbytes < 3 * l2 else 1
        Ws = [(0.02 * torch.randn(N, K, device=dev, generator=g), 0.02 * torch.randn(N, K, device=dev, generator=g))
              for _ in range(n_copies)]
        x = torch.randn(K, device=dev, generator=g)
        gamma = torch.rand(K, device=dev, generator=g) + 0.5
        h = torch.empty(N, device=dev)
        fn = lambda i: sw(x.data_ptr(), gamma.data_ptr(), Ws[i][0].data_ptr(), Ws[i][1].data_ptr(), h.data_ptr(),
                          K, N, 1e-5, stream.cuda_stream)
        us = timed(fn, n_copies, 50)
        by = wbytes + 2 * K * 4 + N * 4
        cases[f"swiglu_f32 {name} K={K} N={N}"] = {"us": round(us, 2), "GB/s": round(by / us / 1e3, 1),
                                                   "frac": round(by / us / 1e3 / peaks["hbm_gbs"], 4)}
        del Ws
    # recurrence + out-projection, decode layer shape, one token
    B, H, gqa, D, hidden = 64, 32, 2, 128, 4096
    q = torch.randn(B, H // gqa, 1, D, device=dev, generator=g)
    k = torch.nn.functional.normalize(torch.randn(B, H // gqa, 1, D, device=dev, generator=g), dim=-1)
    v = torch.randn(B, H, 1, D, device=dev, generator=g)
    gg = -torch.rand(B, 1, H, device=dev, generator=g)
    beta = torch.randn(B, 1, H, device=dev, generator=g)
    states = [0.02 * torch.randn(B, H, D, D, device=dev, generator=g) for _ in range(2)]
    W = 0.02 * torch.randn(hidden, H * D, device=dev, generator=g)
    dsts = [torch.empty(B * H * D + B * H * D * D, device=dev) for _ in range(2)]
    proj = torch.empty(hidden, device=dev)
    fn = lambda i: rec(q.data_ptr(), k.data_ptr(), v.data_ptr(), gg.data_ptr(), beta.data_ptr(), states[i].data_ptr(),
                       W.data_ptr(), dsts[i].data_ptr(), proj.data_ptr(), D, 1, H, gqa, 0, B, hidden, D, D, D * H,
                       stream.cuda_stream)
    us = timed(fn, 2, 50)
    by = 2 * B * H * D * D * 4 + hidden * H * D * 4 + B * H * D * 4 * 3 + B * H * D * 4
    cases[f"recurrent_out_f32 B={B} H={H} D={D} hidden={hidden}"] = {
        "us": round(us, 2), "GB/s": round(by / us / 1e3, 1), "frac": round(by / us / 1e3 / peaks["hbm_gbs"], 4)}
    big = cases[f"swiglu_f32 Qwen3-14B K=5120 N=17408"]
    line = {"metric": "fp32 RMSNorm+SwiGLU GB/s (Qwen3-14B shape)", "value": big["GB/s"], "unit": "GB/s",
            "n_gpus": 1, "steps": 50, "warmup": 3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "reference_kernel_shapes", "cases": cases,
                       "l2": "weight copies rotate: consecutive launches touch more than 3x the L2"},
            "roofline": {"bound": "hbm", "kernel": "li_launch_fused_rms_norm_swiglu_f32 at K=5120 N=17408",
                         "achieved": big["GB/s"], "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": big["frac"],
                         "peak_source": peaks["source"], "traffic": None},
            "e2e": {"value": big["GB/s"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 50 * 4 if impl == "ours" else 0}
    if impl == "reference":
        line["impl"] = "reference"
        line["note"] = "the reference's CUDA kernels (cuda/leaninfer-fused-{ffn,deltanet}.cu) built unchanged " \
                       "for sm_100a; its recurrence's projection sums D/32 of the terms per head (less work)"
    return line


def run_reference(args, rank: int) -> dict | None:
    """The reference's CPU path for the workload (the oracle port: ggml's CPU
    ops are not vendored), on the host cores with all threads; rank 0 only."""
    if rank != 0:
        return None
    if args.workload == "refgpu":
        return run_refgpu(args, "reference")
    if args.workload != "decode":
        if args.workload == "stack":
            cb = cpu_baseline_stack(args.layers, args.ctx)
            cfg = {"workload": "hybrid_stack_decode", "layers": args.layers, "global_batch": args.batch,
                   "context": args.ctx, "rows_timed": 1}
            cfg["note"] = "the reference's ggml CPU ops are not vendored; its CPU path is the C oracle port"
            return {"impl": "reference", "metric": "hybrid-stack decode tokens/s", "value": cb["value"],
                    "unit": cb["unit"], "n_gpus": 0, "steps": args.steps, "warmup": args.warmup,
                    "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                    "dtype": "f64 accumulation", "data": "synthetic", "config": cfg,
                    "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                    "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0}}
        if args.workload == "layerffn":
            cb = cpu_baseline_layerffn(args.batch, max(1, min(args.steps, 4)))
            return {"impl": "reference", "metric": LF_METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": 0,
                    "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "f64 accumulation (Q4_K weights)", "data": "synthetic",
                    "config": {"workload": "deltanet_ffn_layer_decode_q4k", "batch_per_gpu": args.batch,
                               "hidden": HIDDEN, "k_heads": HK, "v_heads": HV, "head_dim": D, "ffn": FFN_N,
                               "weights": "Q4_K",
                               "note": "the reference's ggml CPU ops are not vendored; its CPU path is the C "
                                       "oracle port"},
                    "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                    "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        if args.workload == "prefill":
            cb, metric, cfg = cpu_baseline_prefill(), "chunked prefill tokens/s", {
                "workload": "deltanet_chunk_prefill_bf16", "tokens_per_sequence": PF_T, "chunk": 64}
        else:
            wtype = 8 if args.workload == "qkv" else args.wtype
            cb, metric = cpu_baseline_gemv(args.workload, wtype, 1), "tokens/s"
            cfg = {"workload": "rms_norm_qkv_q8_0" if args.workload == "qkv" else
                   f"ffn_{'q8_0' if wtype == 8 else 'q4_k'}", "rows_timed": 1}
        cfg["note"] = "the reference's ggml CPU ops are not vendored; its CPU path is the C oracle port"
        return {"impl": "reference", "metric": metric, "value": cb["value"], "unit": cb["unit"], "n_gpus": 0,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f64 accumulation", "data": "synthetic", "config": cfg,
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    cb = cpu_baseline(args.batch, max(1, args.steps if args.steps <= 8 else 8))
    return {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64 accumulation (Q4_K weights)", "data": "synthetic",
            "config": {"workload": "deltanet_layer_decode_q4k", "batch_per_gpu": args.batch, "hidden": HIDDEN,
                       "k_heads": HK, "v_heads": HV, "head_dim": D, "weights": "Q4_K",
                       "note": "the reference's ggml CPU ops are not vendored; its CPU path is the C oracle port"},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    # 5000 decode steps at B = 64 are ~0.5 s of timed work: several clock samples (100 ms apart)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU (decode, default 64; ffn rows, default 64); stack: sequences in total "
                         "(default 256)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-steps", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--traffic", type=float, default=None, help="ncu DRAM bytes per step, if captured")
    ap.add_argument("--layers", type=int, default=64, help="stack: layers (3 DeltaNet : 1 attention)")
    ap.add_argument("--ctx", type=int, default=4096, help="stack: attention context (KV cache length)")
    ap.add_argument("--tp-ffn", action="store_true", help="stack: shard the FFN weights across the GPUs (NCCL)")
    ap.add_argument("--workload", choices=["decode", "layerffn", "prefill", "qkv", "ffn", "stack", "refgpu"],
                    default="decode",
                    help="decode: the fused DeltaNet layer decode step (the headline); layerffn: that layer "
                         "followed by the SwiGLU FFN 4096 -> 12288 -> 4096, residual adds after each; prefill: one "
                         "8192-token chunked prefill + gated norm + bf16 out-projection; qkv: RMSNorm + Q/K/V Q8_0 "
                         "GEMV (K=2048, one token); ffn: RMSNorm + SwiGLU FFN 4096 -> 12288 -> 4096 (--batch "
                         "rows, --wtype)")
    ap.add_argument("--wtype", type=int, choices=[8, 12], default=12, help="ffn weights: 12 = Q4_K, 8 = Q8_0")
    ap.add_argument("--state", choices=["f32", "f16"], default="f32",
                    help="decode: recurrent state storage (f16 = li_launch_deltanet_layer_decode_f16state)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.batch is None:
        args.batch = 256 if args.workload == "stack" else 64
    if args.workload == "stack" and "--steps" not in sys.argv:
        args.steps = 20          # about 1 s of timed work on one GPU (a step is ~50 ms there)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank)
        if line:
            print(json.dumps(line), flush=True)
        return

    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dist = tdist
    from leaninfer_b200 import _lib, build
    if not _lib.LIB_PATH.exists():
        if rank == 0:
            build.build()
        if dist:
            dist.barrier()
    _lib.load()
    try:
        if args.workload == "prefill":
            line = run_prefill(args, rank, world, dist)
        elif args.workload == "stack":
            line = run_stack(args, rank, world, dist)
        elif args.workload == "layerffn":
            line = run_layerffn(args, rank, world, dist)
        elif args.workload == "refgpu":
            line = run_refgpu(args, "ours") if rank == 0 else None
        elif args.workload in ("qkv", "ffn"):
            line = run_gemv(args, rank, world, dist)
        else:
            line = run_ours(args, rank, world, dist)
    finally:
        if dist:
            dist.destroy_process_group()
    if line:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
