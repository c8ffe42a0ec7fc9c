"""Tensor parallelism with sequence parallelism over a pair of GPUs.

The residual stream is split along tokens: TP rank r holds tokens
[r*T/tp, (r+1)*T/tp) of every microbatch.  Column-parallel projections
(QKV, and the expert block, whose experts are split over the pair: EP = TP,
ETP = 1) consume the all-gathered activation; row-parallel projections
(attention output, expert combine) produce partial sums that are
reduce-scattered back to the token split.  In backward, all-gather and
reduce-scatter swap roles.  This is Megatron's TP + SP with EP laid over the
TP group -- the layout the reference runs inside each replica
(shift_full/train.py:201-216, sequence_parallel off there), on one box.

``TPComm`` implements the two collectives.  ``backend="nccl"`` uses the TP
process group; ``backend="peer"`` uses symmetric peer buffers and the
peer-memory kernels (gathered halves are written straight into the peer's
buffer; reduce-scatter adds the peer's partial half in a fixed rank order).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class TPComm:
    def __init__(self, group, rank: int, size: int, device):
        self.group = group
        self.rank = rank
        self.size = size
        self.device = torch.device(device)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """[T/tp, H] -> [T, H] (rank order)."""
        if self.size == 1:
            return x
        out = torch.empty((x.shape[0] * self.size,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        """[T, H] partial sums -> [T/tp, H] of the sum."""
        if self.size == 1:
            return x
        out = torch.empty((x.shape[0] // self.size,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
        return out

    def all_reduce_(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(x, group=self.group)
        return x

    def local_rows(self, x: torch.Tensor) -> torch.Tensor:
        n = x.shape[0] // self.size
        return x[self.rank * n:(self.rank + 1) * n]
