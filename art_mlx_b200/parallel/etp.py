"""Expert tensor parallelism (ETP): each expert's FFN split over the ranks of
an ETP group.

Reference behaviour: Megatron expert-TP with the expert LoRA following the
expert weight sharding and its own gradient-sync domain
(``src/art/megatron/training/finalize_grads.py:38-52``,
``src/art/megatron/lora.py:209-229``).

Layout: the job's ``world = ep x etp`` ranks are split into consecutive ETP
groups of ``etp`` ranks; the ranks of one ETP group own the same experts and
rank ``j`` of the group holds intermediate columns ``[j*F/etp, (j+1)*F/etp)``
of each (gate/up column-sharded, down row-sharded).  The expert-parallel
group of a rank is the set of ranks with the same ``j`` (stride ``etp``).

One MoE layer:
  1. the ETP group all-gathers its tokens, routing weights and expert ids, so
     every member holds the group's whole token set;
  2. expert parallelism dispatches them inside the EP group, each member's
     experts compute their F-slice, and the combine returns partial outputs
     (sum over the slice only);
  3. a reduce-scatter over the ETP group sums the slices and hands every rank
     the outputs of its own tokens.
The all-gather and the reduce-scatter are autograd pairs (backward: reduce-
scatter, all-gather), so input, routing-weight and replicated-LoRA gradients
arrive as sums over the slices.  LoRA factors stay full-size in every rank's
flat store: the sharded ones (B of gate/up, A of down) get gradients only in
the rank's slice, the replicated ones (A of gate/up, B of down) get the
rank's partial sum, and the job-wide gradient reduction completes both.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import mutation
from .cp import CPContext, gather
from .topology import shard_subgroup


class ETPContext:
    def __init__(self, group: dist.ProcessGroup | None, size: int, device: torch.device) -> None:
        self.size = size
        self.comm = CPContext(shard_subgroup(group, size), device, transport="nccl")
        self.rank = self.comm.rank

    def slice(self, F: int) -> tuple[int, int]:
        """(first column, width) of this rank's share of an intermediate size F."""
        if F % self.size != 0:
            raise ValueError(f"expert intermediate size {F} is not divisible by etp={self.size}")
        w = F // self.size
        return self.rank * w, w

    def gather(self, x: torch.Tensor) -> torch.Tensor:
        """Differentiable all-gather over the ETP group (backward: reduce-scatter)."""
        return gather(x.contiguous(), self.comm)

    def gather_nograd(self, x: torch.Tensor) -> torch.Tensor:
        return self.comm.all_gather(x.contiguous())

    def reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        """Differentiable reduce-scatter over the ETP group (backward: all-gather)."""
        if mutation.active("etp_skip_reduce_scatter"):
            rows = x.shape[0] // self.size
            return x[self.rank * rows : (self.rank + 1) * rows]
        return _ReduceScatter.apply(x.contiguous(), self.comm)


class _ReduceScatter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm):
        ctx.comm = comm
        return comm.reduce_scatter(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.comm.all_gather(g.contiguous()), None
