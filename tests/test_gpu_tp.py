"""The two-way sharded SwiGLU FFN over NCCL (li_launch_ffn_q_tp) on two GPUs
against the oracle's unsharded FFN: each rank holds its block-aligned share
of the inner dimension (W_gate / W_up rows, the matching W_down columns,
leaninfer_b200.tp_ffn.shard_ffn) and its own rows of x; after the
all-gather, the local products and the reduce-scatter, its rows of y must
equal the full FFN of its rows within 1e-3 normwise (the partial sums of the
two shards meet in fp32). The communicator is made by the library's own
entries (li_nccl_get_unique_id / li_nccl_comm_init_rank), the unique id sent
through a gloo group. Runs only where two GPUs are visible."""
from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, rows, wtype, q):
    import ctypes
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    import torch
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        from leaninfer_b200 import _lib, synth
        from leaninfer_b200.tp_ffn import shard_ffn
        from oracle import oracle
        lib = _lib.load()
        uid = ctypes.create_string_buffer(128)
        if rank == 0:
            assert lib.li_nccl_get_unique_id(uid) == 0
        obj = [bytes(uid.raw)]
        dist.broadcast_object_list(obj, src=0)
        uid = ctypes.create_string_buffer(obj[0], 128)
        comm = ctypes.c_void_p()
        assert lib.li_nccl_comm_init_rank(ctypes.byref(comm), world, uid, rank) == 0
        r = np.random.Generator(np.random.PCG64(4242))
        K, N = 4096, 12288
        Wg, Wu = synth.random_weights(r, wtype, N, K), synth.random_weights(r, wtype, N, K)
        Wd = synth.random_weights(r, wtype, K, N)
        gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
        x_all = r.standard_normal((world * rows, K)).astype(np.float32)
        dev = torch.device("cuda", rank)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        sh = shard_ffn(Wg, Wu, Wd, wtype, K, N, world, rank, to=t)
        x = t(x_all[rank * rows:(rank + 1) * rows])
        y = torch.empty(rows, K, device=dev)
        ws = torch.empty(int(lib.li_ffn_tp_workspace_size(K, sh.n_local, rows, world)), dtype=torch.uint8, device=dev)
        for _ in range(2):   # twice: the second call reuses the communicator and workspace
            rc = lib.li_launch_ffn_q_tp(wtype, x.data_ptr(), t(gamma).data_ptr(), sh.Wg.data_ptr(), sh.Wu.data_ptr(),
                                        sh.Wd.data_ptr(), y.data_ptr(), K, sh.n_local, rows, 1e-6, comm, world,
                                        ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
            assert rc == 0, rc
        torch.cuda.synchronize()
        ref = oracle.ffn(wtype, x_all[rank * rows:(rank + 1) * rows], gamma, Wg, Wu, Wd, N)
        got = y.cpu().numpy()
        err = float(np.abs(got - ref).max() / np.abs(ref).max())
        assert lib.li_device_status() == 0
        assert lib.li_nccl_comm_destroy(comm) == 0
        dist.destroy_process_group()
        q.put((rank, err, None))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("rows,wtype", [(32, 12), (2, 12), (16, 8)])
def test_ffn_tp_two_gpus(cuda, rows, wtype):
    import multiprocessing as mp
    import socket
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(rk, 2, port, rows, wtype, q)) for rk in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, err, exc in sorted(res):
        assert exc is None, f"rank {rank}: {exc}"
        assert err <= 1e-3, f"rank {rank}: normwise error {err:.3e}"
