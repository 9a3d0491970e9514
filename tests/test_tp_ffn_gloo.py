"""Two-dimensional FFN sharding (leaninfer_b200/tp_ffn.py) on CPU: the
block-aligned splits and weight slices reassemble the full matrices, two
gloo ranks (the oracle standing in for the device products) produce the
unsharded FFN's output for their sequences, and a rank that leaves between
steps ends the other rank's next step with an error instead of a hang."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from leaninfer_b200 import synth
from leaninfer_b200.tp_ffn import BLOCK, ffn_split, shard_ffn, slice_down


@pytest.mark.parametrize("wtype", [8, 12])
@pytest.mark.parametrize("world", [1, 2, 3])
def test_splits_and_slices_reassemble(wtype, world):
    r = np.random.Generator(np.random.PCG64(5))
    K, N = 512, 1024
    Wg, Wu = synth.random_weights(r, wtype, N, K), synth.random_weights(r, wtype, N, K)
    Wd = synth.random_weights(r, wtype, K, N)
    blk = BLOCK[wtype][0]
    ranges = [ffn_split(N, wtype, world, q) for q in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == N
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    assert all(n0 % blk == 0 and n1 % blk == 0 for n0, n1 in ranges)
    shards = [shard_ffn(Wg, Wu, Wd, wtype, K, N, world, q) for q in range(world)]
    assert np.array_equal(np.concatenate([s.Wg for s in shards]), Wg)
    assert np.array_equal(np.concatenate([s.Wu for s in shards]), Wu)
    assert np.array_equal(np.concatenate([s.Wd for s in shards], axis=1), Wd)
    assert np.array_equal(slice_down(Wd, wtype, 0, N), Wd)
    with pytest.raises(ValueError):
        ffn_split(N + 1, wtype, world, 0)
    # more ranks than blocks: refused before any collective could start
    with pytest.raises(ValueError):
        ffn_split(N, wtype, N // blk + 1, 0)


class OracleCompute:
    """The local products on the oracle (torch tensors in and out)."""

    def __init__(self, wtype):
        self.wtype = wtype

    def swiglu(self, x, gamma, Wg, Wu, n_local):
        import torch
        from oracle import oracle
        return torch.from_numpy(oracle.rms_norm_swiglu(self.wtype, x.numpy(), gamma.numpy(), Wg, Wu, n_local))

    def down(self, h, Wd, K):
        import torch
        from oracle import oracle
        return torch.from_numpy(oracle.rms_norm_matmul(self.wtype, h.numpy(), None, Wd, K))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(wtype, K, N, n_total):
    r = np.random.Generator(np.random.PCG64(41))
    Wg, Wu = synth.random_weights(r, wtype, N, K), synth.random_weights(r, wtype, N, K)
    Wd = synth.random_weights(r, wtype, K, N)
    gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
    x = r.standard_normal((n_total, K)).astype(np.float32)
    return Wg, Wu, Wd, gamma, x


def _worker(rank, world, port, wtype, K, N, n_total, out_dir):
    import torch
    import torch.distributed as dist
    from leaninfer_b200.shard import shard_bounds
    from leaninfer_b200.tp_ffn import tp_ffn_forward
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        Wg, Wu, Wd, gamma, x = _weights(wtype, K, N, n_total)
        shard = shard_ffn(Wg, Wu, Wd, wtype, K, N, world, rank)
        first, count = shard_bounds(n_total, world, rank)
        y = tp_ffn_forward(torch.from_numpy(x[first:first + count]), torch.from_numpy(gamma), shard, dist,
                           n_total, OracleCompute(wtype))
        assert y.shape == (count, K)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("wtype", [8, 12])
def test_two_ranks_match_unsharded_ffn(tmp_path, wtype):
    import torch.multiprocessing as mp
    from oracle import oracle
    K, N, n_total, world = 256, 1024, 5, 2
    mp.spawn(_worker, args=(world, _free_port(), wtype, K, N, n_total, str(tmp_path)), nprocs=world, join=True)
    y = np.concatenate([np.load(tmp_path / f"y{q}.npy") for q in range(world)])
    Wg, Wu, Wd, gamma, x = _weights(wtype, K, N, n_total)
    y_ref = oracle.ffn(wtype, x, gamma, Wg, Wu, Wd, N, 1e-6)
    err = np.abs(y - y_ref).max() / np.abs(y_ref).max()
    assert err <= 1e-5, err     # partial sums over the two halves of N meet in fp32


def _worker_leaves(rank, world, port, out_dir):
    """Rank 1 leaves after the rendezvous, before the step's collectives;
    rank 0's step must end with an error inside the group's timeout."""
    import datetime
    import time

    import torch
    import torch.distributed as dist
    from leaninfer_b200.tp_ffn import tp_ffn_forward
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        return                      # gone between steps: no collective of this rank in flight
    K, N, wtype, n_total = 256, 1024, 8, 4
    Wg, Wu, Wd, gamma, x = _weights(wtype, K, N, n_total)
    shard = shard_ffn(Wg, Wu, Wd, wtype, K, N, world, rank)
    t0 = time.time()
    try:
        tp_ffn_forward(torch.from_numpy(x[:2]), torch.from_numpy(gamma), shard, dist, n_total, OracleCompute(wtype))
        outcome = "completed"
    except Exception as e:          # the backend reports the lost peer or the timeout
        outcome = f"error {type(e).__name__}"
    with open(os.path.join(out_dir, "outcome.txt"), "w") as f:
        f.write(f"{outcome} {time.time() - t0:.1f}")


def test_lost_rank_ends_the_step_with_an_error(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker_leaves, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    outcome, seconds = (tmp_path / "outcome.txt").read_text().rsplit(" ", 1)
    assert outcome.startswith("error"), outcome
    assert float(seconds) < 60
