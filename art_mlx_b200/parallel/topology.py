"""Process-group layout of one training job.

Ranks are arranged ``dp x shard`` where ``shard`` is the tensor-parallel or
the context-parallel size (the two split a packed row in different ways and
are not combined): ranks ``[k*shard, (k+1)*shard)`` form one shard group and
process the same rows; the ``dp`` groups process different rows.  Gradients
of the (replicated, full-size) LoRA factors are summed over every rank of the
job, which also completes the tensor-parallel gradient sync.  Expert
parallelism spans the whole job.

Mirrors the topology surface of the reference
(``src/art/types.py:33-39``, ``src/art/megatron/provider.py:60-63``):
``dp = world / (tp * cp * pp)``.
"""

from __future__ import annotations

import torch.distributed as dist


def group_ranks(group: dist.ProcessGroup | None) -> list[int]:
    if group is None or group == dist.group.WORLD:
        return list(range(dist.get_world_size()))
    return list(dist.get_process_group_ranks(group))


def shard_subgroup(group: dist.ProcessGroup | None, size: int) -> dist.ProcessGroup | None:
    """Collective over ``group``: split it into consecutive blocks of ``size``
    ranks and return the block that holds this rank (``group`` itself when
    the block is the whole group)."""
    ranks = group_ranks(group)
    if size == len(ranks):
        return group
    if len(ranks) % size != 0:
        raise ValueError(f"shard size {size} does not divide the {len(ranks)} ranks")
    me = dist.get_rank()
    mine = None
    for k in range(0, len(ranks), size):
        block = ranks[k : k + size]
        g = dist.new_group(block)  # every rank creates every block, in order
        if me in block:
            mine = g
    return mine


def strided_subgroup(group: dist.ProcessGroup | None, stride: int) -> dist.ProcessGroup | None:
    """Collective over ``group``: split it into ``stride`` groups of ranks
    ``{j, j + stride, j + 2*stride, ...}`` and return the one that holds this
    rank (the ranks that share a position inside their consecutive block of
    ``stride``)."""
    ranks = group_ranks(group)
    if len(ranks) % stride != 0:
        raise ValueError(f"stride {stride} does not divide the {len(ranks)} ranks")
    if stride == 1:
        return group
    me = dist.get_rank()
    mine = None
    for j in range(stride):
        members = ranks[j::stride]
        g = dist.new_group(members)
        if me in members:
            mine = g
    return mine
