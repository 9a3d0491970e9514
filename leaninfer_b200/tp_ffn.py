"""Two-dimensional sharding of the SwiGLU FFN across ranks.

Sequence sharding alone replicates every weight on every GPU; for a stack
whose weights dominate the step, the wide FFN is split as well: the inner
dimension N (12288 at hidden 4096) is cut into contiguous, block-aligned
ranges, one per rank. Rank r holds rows [n0, n1) of W_gate and W_up
(column-parallel: it computes h[:, n0:n1]) and the matching slice of every
row of W_down (row-parallel: it computes a partial y over its part of N).
A step on the sequence-sharded activations is

    x_all = all_gather(x_local)                       # [B, K], every rank
    h_r   = silu(rmsnorm(x_all) Wg_r^T) * (rmsnorm(x_all) Wu_r^T)
    y_r   = h_r Wd_r^T                                # partial sums over N_r
    y_local = reduce_scatter(y_r)                     # back to this rank's sequences

Quantized rows slice on block boundaries only (Q4_K: 256 values, Q8_0: 32),
so the split points are multiples of the block size; a row's slice is a
contiguous byte range of it. The local products run on the library's
entries (li_launch_fused_rms_norm_swiglu_q, li_launch_rms_norm_matmul_q) or,
in the CPU tests, on the oracle; the collectives are torch.distributed's
(NCCL on GPUs; gloo, which has no reduce-scatter, takes all-reduce + slice).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .shard import shard_bounds

BLOCK = {8: (32, 34), 12: (256, 144)}   # ggml type -> (values, bytes) per block


def ffn_split(N: int, wtype: int, world: int, rank: int) -> tuple[int, int]:
    """(n0, n1): rank's block-aligned range of the inner dimension N."""
    blk = BLOCK[wtype][0]
    if N % blk:
        raise ValueError(f"N = {N} is not a multiple of the {blk}-value block")
    if world > N // blk:
        # a rank with an empty range would call the entries with N = 0 and fail
        # between the collectives, leaving the other ranks waiting in them
        raise ValueError(f"{world} ranks cannot each take a block of the {N // blk} blocks of N = {N}")
    b0, nb = shard_bounds(N // blk, world, rank)
    return b0 * blk, (b0 + nb) * blk


def slice_down(Wd: np.ndarray, wtype: int, n0: int, n1: int) -> np.ndarray:
    """Columns [n0, n1) of every row of the quantized down matrix [K rows,
    N values] (raw blocks, [K, row_bytes]): a contiguous byte range per row."""
    blk, size = BLOCK[wtype]
    return np.ascontiguousarray(Wd[:, n0 // blk * size:n1 // blk * size])


@dataclass
class FFNShard:
    wtype: int
    K: int            # model width
    N: int            # full inner width
    n0: int
    n1: int
    Wg: object        # [n1 - n0, K row bytes]
    Wu: object
    Wd: object        # [K, (n1 - n0) row bytes]

    @property
    def n_local(self) -> int:
        return self.n1 - self.n0


def shard_ffn(Wg: np.ndarray, Wu: np.ndarray, Wd: np.ndarray, wtype: int, K: int, N: int, world: int,
              rank: int, to=lambda a: a) -> FFNShard:
    """Rank's share of the FFN weights (raw ggml blocks); `to` places each
    slice (e.g. onto the rank's GPU)."""
    n0, n1 = ffn_split(N, wtype, world, rank)
    return FFNShard(wtype, K, N, n0, n1, to(np.ascontiguousarray(Wg[n0:n1])), to(np.ascontiguousarray(Wu[n0:n1])),
                    to(slice_down(Wd, wtype, n0, n1)))


def _gather_rows(x_local, dist, counts):
    """All-gather of sequence shards with unequal counts (padded to the
    largest, then trimmed), in rank order."""
    import torch
    world = dist.get_world_size()
    cmax = max(counts)
    pad = torch.zeros((cmax,) + tuple(x_local.shape[1:]), dtype=x_local.dtype, device=x_local.device)
    pad[:x_local.shape[0]] = x_local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad)
    return torch.cat([bufs[q][:counts[q]] for q in range(world)])


def _reduce_scatter_rows(y_partial, dist, counts, rank):
    """Sum of every rank's partial y, each rank keeping its own sequences."""
    import torch
    if dist.get_backend() == "nccl":
        world = dist.get_world_size()
        cmax = max(counts)
        firsts = np.cumsum([0] + list(counts[:-1]))
        pad = torch.zeros((world * cmax,) + tuple(y_partial.shape[1:]), dtype=y_partial.dtype,
                          device=y_partial.device)
        for q in range(world):
            pad[q * cmax:q * cmax + counts[q]] = y_partial[firsts[q]:firsts[q] + counts[q]]
        out = torch.empty((cmax,) + tuple(y_partial.shape[1:]), dtype=y_partial.dtype, device=y_partial.device)
        dist.reduce_scatter_tensor(out, pad)
        return out[:counts[rank]]
    y = y_partial.clone()
    dist.all_reduce(y)
    first = int(sum(counts[:rank]))
    return y[first:first + counts[rank]]


def tp_ffn_forward(x_local, gamma, shard: FFNShard, dist, n_total: int, compute) -> object:
    """y for this rank's sequences (x_local = its contiguous shard of
    n_total sequences, torch [count, K]). `compute` supplies
    swiglu(x, gamma, Wg, Wu, n_local) -> h and down(h, Wd, K) -> y_partial on
    torch tensors (the library's entries on a GPU)."""
    world, rank = dist.get_world_size(), dist.get_rank()
    counts = [shard_bounds(n_total, world, q)[1] for q in range(world)]
    x_all = _gather_rows(x_local, dist, counts)
    h = compute.swiglu(x_all, gamma, shard.Wg, shard.Wu, shard.n_local)
    y_partial = compute.down(h, shard.Wd, shard.K)
    return _reduce_scatter_rows(y_partial, dist, counts, rank)


class DeviceCompute:
    """The local products on the library's entries (CUDA tensors)."""

    def __init__(self, wtype: int, eps: float = 1e-6):
        self.wtype, self.eps = wtype, eps

    def swiglu(self, x, gamma, Wg, Wu, n_local):
        from . import ops
        return ops.rms_norm_swiglu_q(self.wtype, x, gamma, Wg, Wu, n_local, self.eps)

    def down(self, h, Wd, K):
        from . import ops
        return ops.rms_norm_matmul_q(self.wtype, h.contiguous(), None, Wd, K)
