"""Sequence sharding on two ranks (gloo, CPU): each rank runs its
contiguous shard of a global batch through the layer decode (the oracle
restatement stands in for the device here; nothing launches a kernel), the
shards gathered in rank order equal the unsharded run bit for bit (sequences
are independent), and the timing reduction takes the maximum over ranks."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from leaninfer_b200.shard import max_over_ranks, shard_bounds


def test_shard_bounds_cover_the_batch():
    for n in (0, 1, 5, 64, 257):
        for w in (1, 2, 3, 8):
            got = [shard_bounds(n, w, r) for r in range(w)]
            assert sum(c for _, c in got) == n
            assert all(got[r][0] == sum(c for _, c in got[:r]) for r in range(w))
            assert max(c for _, c in got) - min(c for _, c in got) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, n_seqs: int, out_dir: str):
    import torch
    import torch.distributed as dist
    from leaninfer_b200 import synth
    from oracle import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = np.random.Generator(np.random.PCG64(77))
        w = synth.deltanet_layer(r, hidden=512, n_k_heads=2, n_v_heads=4, wtype=synth.Q8_0)   # replicated
        inp = synth.deltanet_inputs(r, n_seqs, w)
        x = (r.standard_normal((n_seqs, 512)) * synth.DELTANET_X_SCALE).astype(np.float32)
        first, count = shard_bounds(n_seqs, world, rank)
        L, keep = oracle.make_layer(w)
        cs = np.ascontiguousarray(inp["conv_state"][first:first + count])
        st = np.ascontiguousarray(inp["state"][first:first + count])
        y = oracle.deltanet_layer_decode(L, keep, x[first:first + count], cs, st) if count else \
            np.zeros((0, 512), np.float32)
        # gather the shards (padded to the largest) for the check on rank 0
        cmax = shard_bounds(n_seqs, world, 0)[1]
        pad = np.zeros((cmax, 512), np.float32)
        pad[:count] = y
        bufs = [torch.zeros(cmax, 512) for _ in range(world)]
        dist.all_gather(bufs, torch.from_numpy(pad))
        t = max_over_ranks([1.0 + rank, 5.0 - rank], dist)
        if rank == 0:
            parts = [bufs[q][:shard_bounds(n_seqs, world, q)[1]].numpy() for q in range(world)]
            np.save(os.path.join(out_dir, "y_sharded.npy"), np.concatenate(parts))
            np.save(os.path.join(out_dir, "tmax.npy"), np.array(t))
    finally:
        dist.destroy_process_group()


def test_two_ranks_match_unsharded(tmp_path):
    import torch.multiprocessing as mp
    from leaninfer_b200 import synth
    from oracle import oracle
    n_seqs, world = 5, 2
    mp.spawn(_worker, args=(world, _free_port(), n_seqs, str(tmp_path)), nprocs=world, join=True)
    r = np.random.Generator(np.random.PCG64(77))
    w = synth.deltanet_layer(r, hidden=512, n_k_heads=2, n_v_heads=4, wtype=synth.Q8_0)
    inp = synth.deltanet_inputs(r, n_seqs, w)
    x = (r.standard_normal((n_seqs, 512)) * synth.DELTANET_X_SCALE).astype(np.float32)
    L, keep = oracle.make_layer(w)
    y_ref = oracle.deltanet_layer_decode(L, keep, x, inp["conv_state"].copy(), inp["state"].copy())
    y = np.load(tmp_path / "y_sharded.npy")
    assert np.array_equal(y, y_ref)
    assert list(np.load(tmp_path / "tmax.npy")) == [2.0, 5.0]
