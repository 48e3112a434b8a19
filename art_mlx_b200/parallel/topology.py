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


def default_topology(cfg, world: int, row_tokens: int | None = None, gpu_bytes: int = 180 << 30,
                     tokens_per_rank: int = 16384) -> dict[str, int]:
    """The layout a job gets when the caller names none.

    The reference puts every GPU into context parallelism (or tensor
    parallelism for families without CP) and expert parallelism over all
    GPUs for MoE models (``src/art/megatron/provider.py:371-385``).  On
    180 GB B200s most LoRA jobs fit one GPU per replica, and data
    parallelism then moves the least data per token, so the policy here is:

    * MoE: expert parallelism over every GPU (the experts are the memory);
    * the bf16 base weights plus a working margin exceed one GPU: tensor
      parallelism over the smallest power of two that fits;
    * packed rows longer than ``tokens_per_rank``: context parallelism over
      the smallest power of two that brings a row slice under it (rows are
      not split otherwise), for families whose layers support it;
    * the remaining factor is data parallelism.
    Returns ``{"dp", "tp", "cp", "ep", "etp"}``."""
    from ..models.registry import get_model_support

    spec = get_model_support(cfg, allow_unvalidated_arch=True)
    H, L, V = cfg.hidden_size, cfg.num_hidden_layers, cfg.vocab_size
    if cfg.is_moe:
        F = cfg.moe_intermediate_size
        mlp = 3 * H * F * cfg.num_experts + 3 * H * cfg.shared_expert_intermediate_size
    else:
        mlp = 3 * H * cfg.intermediate_size
    attn = H * (cfg.q_size * (2 if cfg.attn_output_gate else 1) + 2 * cfg.kv_size) + cfg.q_size * H
    weight_bytes = 2 * (L * (attn + mlp) + 2 * V * H)
    tp = cp = 1
    ep = world if cfg.is_moe else 1
    if not cfg.is_moe:
        while tp < world and weight_bytes / tp > 0.6 * gpu_bytes:
            tp *= 2
        if tp > 1 and "tp" not in spec.supports:
            raise ValueError(f"{spec.key}: the base weights do not fit one GPU and the family has no tensor parallelism")
    if row_tokens is not None and "cp" in spec.supports and tp == 1:
        while cp < world and row_tokens / cp > tokens_per_rank:
            cp *= 2
    if world % (tp * cp):
        raise ValueError(f"tp={tp} x cp={cp} does not divide {world} GPUs")
    return {"dp": world // (tp * cp), "tp": tp, "cp": cp, "ep": ep, "etp": 1}
