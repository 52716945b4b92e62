"""Tensor-parallel N-split of a W4A16 AWQ projection across ranks.

Reference analog: the column interleave of the Anvil-Q2 GEMV banks
(anvil-q2/rtl/anvil_q2_gemv_lane.sv:117,187) -- every bank owns a slice of the
output columns and sees the whole activation vector.  Here rank r of W owns the
contiguous output columns [r N/W, (r+1) N/W): qweight[:, r W8/W : (r+1) W8/W]
(W8 = N/8 packed words per row), the same words of qzeros, scales[:, cols] and
bias[cols].  x is replicated; each rank computes its slice with the single-GPU
kernels, and one all-gather (NCCL on GPUs) assembles y.

The exchange is the only collective: ranks share no partial sums (the K
reduction is complete inside each rank), so results are bit-identical to the
single-GPU call on the same slice of columns.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def column_range(N: int, rank: int, world: int):
    """Output columns owned by `rank`; N / world must be a multiple of 8 (whole packed words)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank outside the process group")
    if N % (8 * world):
        raise ValueError(f"N={N} does not split into {world} slices of whole 8-column words")
    n = N // world
    return rank * n, (rank + 1) * n


def shard_awq(qweight, qzeros, scales, bias, rank: int, world: int):
    """The rank's column slice of one AWQ projection (views, made contiguous)."""
    W8 = qweight.shape[1]
    c0, c1 = column_range(W8 * 8, rank, world)
    w0, w1 = c0 // 8, c1 // 8
    part = (qweight[:, w0:w1].contiguous(), qzeros[:, w0:w1].contiguous(), scales[:, c0:c1].contiguous(),
            None if bias is None else bias[c0:c1].contiguous())
    return part


def gather_columns(y_local, world: int, group=None):
    """[M, N/W] on every rank -> [M, N] on every rank, columns in rank order (all-gather)."""
    M, n = y_local.shape
    stacked = torch.empty((world * M, n), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(stacked, y_local.contiguous(), group=group)
    return stacked.view(world, M, n).permute(1, 0, 2).reshape(M, world * n)


class TPLinear:
    """One projection split across the ranks of a process group.

    ``compute(x, qweight, qzeros, scales, bias, group) -> y`` is the per-rank
    kernel (``ops.gemm`` by default; tests on CPU ranks substitute the oracle).
    """

    def __init__(self, qweight, qzeros, scales, bias=None, group_size: int = 128, process_group=None,
                 compute=None):
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self.N = qweight.shape[1] * 8
        self.group_size = group_size
        self.shard = shard_awq(qweight, qzeros, scales, bias, self.rank, self.world)
        if compute is None:
            from . import ops
            compute = ops.gemm
        self.compute = compute

    def local(self, x):
        """This rank's [M, N/W] slice of y = x W (+ bias)."""
        return self.compute(x, *self.shard, self.group_size)

    def __call__(self, x):
        x2 = x.unsqueeze(0) if x.dim() == 1 else x
        y = gather_columns(self.local(x2), self.world, self.pg)
        return y.view(self.N) if x.dim() == 1 else y
