"""LoRA adapter layouts of MoE experts.

This package trains and saves expert adapters per expert, under the keys
vLLM's LoRA loader reads::

    ....mlp.experts.{e}.gate_proj.lora_A.weight   [r, hidden]
    ....mlp.experts.{e}.gate_proj.lora_B.weight   [F, r]
    ....mlp.experts.{e}.up_proj.lora_{A,B}.weight
    ....mlp.experts.{e}.down_proj.lora_A.weight   [r, F]
    ....mlp.experts.{e}.down_proj.lora_B.weight   [hidden, r]

with ``"experts"`` among the adapter config's ``target_modules``.  Trainers
that adapt the fused expert parameters (PEFT ``target_parameters``, as the
reference's Megatron path does, ``src/art/megatron/model_support/handlers/
qwen3_moe.py:95-236``) write one fused block per layer instead::

    ....mlp.experts.base_layer.lora_{A,B}.weight   (gate/up, all experts)
    ....mlp.experts.lora_{A,B}.weight              (down, all experts)

in one of two arrangements (below).  :func:`expand_fused_moe_lora` turns
either into the per-expert keys, so such adapters can be resumed or forked
here and served by vLLM; gate and up then share their A factor.
"""

from __future__ import annotations

import re
from typing import Any

import torch

_FUSED_KEY = re.compile(r"^(?P<prefix>.*\.mlp\.experts)\.(?:(?P<base>base_layer)\.)?(?P<lora>lora_[AB])\.weight$")
_EXPERT_KEY = re.compile(r"^.*\.mlp\.experts\.\d+\.(?:gate_proj|up_proj|down_proj)\.lora_[AB]\.weight$")


def moe_adapter_config(config: dict[str, Any]) -> dict[str, Any]:
    """Adapter config of an MoE model: ``experts`` among the target modules."""
    out = dict(config)
    targets = list(out.get("target_modules") or [])
    if "experts" not in targets:
        targets.append("experts")
    out["target_modules"] = targets
    return out


def has_fused_moe_lora(tensors: dict[str, torch.Tensor]) -> bool:
    return any(_FUSED_KEY.match(k) for k in tensors)


def _by_expert(packed: torch.Tensor, experts: int, rank: int) -> torch.Tensor:
    """``[out, rank * experts]`` with rank-major columns (column ``j * E + e``
    holds rank ``j`` of expert ``e``) -> ``[experts, out, rank]``."""
    return packed.reshape(packed.shape[0], rank, experts).permute(2, 0, 1)


def _expand_block(prefix: str, gu_a: torch.Tensor, gu_b: torch.Tensor, d_a: torch.Tensor, d_b: torch.Tensor,
                  rank: int) -> dict[str, torch.Tensor]:
    if any(t.ndim != 2 for t in (gu_a, gu_b, d_a, d_b)):
        raise ValueError(f"{prefix}: fused expert LoRA factors must be 2-D")
    if gu_a.shape[0] % rank:
        raise ValueError(f"{prefix}: gate/up lora_A rows {gu_a.shape[0]} not a multiple of rank {rank}")
    E = gu_a.shape[0] // rank
    cols = E * rank
    out: dict[str, torch.Tensor] = {}
    c = lambda t: t.clone().contiguous()  # noqa: E731
    if gu_b.shape[1] == cols and d_b.shape[1] == cols and gu_a.shape[1] == 2 * d_b.shape[0] \
            and tuple(d_a.shape) == (cols, gu_b.shape[0]):
        # transposed arrangement: gu_a [E r, 2F] holds the gate/up B factors
        # (rows per expert), gu_b [H, E r] the shared A (columns per expert),
        # d_a [E r, H] the down B, d_b [F, E r] the down A
        F = d_b.shape[0]
        for e in range(E):
            rows = slice(e * rank, (e + 1) * rank)
            p = f"{prefix}.{e}"
            a_shared = gu_b[:, rows].t()
            out[f"{p}.gate_proj.lora_A.weight"] = c(a_shared)
            out[f"{p}.up_proj.lora_A.weight"] = c(a_shared)
            out[f"{p}.gate_proj.lora_B.weight"] = c(gu_a[rows, :F].t())
            out[f"{p}.up_proj.lora_B.weight"] = c(gu_a[rows, F:].t())
            out[f"{p}.down_proj.lora_A.weight"] = c(d_b[:, rows].t())
            out[f"{p}.down_proj.lora_B.weight"] = c(d_a[rows].t())
        return out
    # PEFT target_parameters arrangement: A factors stacked by expert
    # (gu_a [E r, H], d_a [E r, F]), B factors packed rank-major
    # (gu_b [2F, r E] with gate rows then up rows, d_b [H, r E])
    if gu_b.shape[0] % 2 or gu_b.shape[1] != cols or d_b.shape[1] != cols or tuple(d_a.shape) != (cols, gu_b.shape[0] // 2):
        raise ValueError(f"{prefix}: fused expert LoRA shapes {[tuple(t.shape) for t in (gu_a, gu_b, d_a, d_b)]} "
                         f"match neither arrangement at rank {rank}")
    F = gu_b.shape[0] // 2
    gub, db = _by_expert(gu_b, E, rank), _by_expert(d_b, E, rank)
    for e in range(E):
        rows = slice(e * rank, (e + 1) * rank)
        p = f"{prefix}.{e}"
        out[f"{p}.gate_proj.lora_A.weight"] = c(gu_a[rows])
        out[f"{p}.up_proj.lora_A.weight"] = c(gu_a[rows])
        out[f"{p}.gate_proj.lora_B.weight"] = c(gub[e, :F])
        out[f"{p}.up_proj.lora_B.weight"] = c(gub[e, F:])
        out[f"{p}.down_proj.lora_A.weight"] = c(d_a[rows])
        out[f"{p}.down_proj.lora_B.weight"] = c(db[e])
    return out


def expand_fused_moe_lora(tensors: dict[str, torch.Tensor], rank: int) -> dict[str, torch.Tensor]:
    """Per-expert adapter tensors from fused expert blocks (other keys kept)."""
    blocks: dict[str, dict[str, torch.Tensor]] = {}
    for k, t in tensors.items():
        m = _FUSED_KEY.match(k)
        if m:
            blocks.setdefault(m.group("prefix"), {})[("base." if m.group("base") else "") + m.group("lora")] = t
    out = {k: t for k, t in tensors.items() if not _FUSED_KEY.match(k)}
    for prefix, b in blocks.items():
        try:
            gu_a, gu_b, d_a, d_b = b["base.lora_A"], b["base.lora_B"], b["lora_A"], b["lora_B"]
        except KeyError as exc:
            raise ValueError(f"incomplete fused expert LoRA block {prefix}") from exc
        for k, t in _expand_block(prefix, gu_a, gu_b, d_a, d_b, rank).items():
            if k in out:
                raise ValueError(f"duplicate adapter tensor {k}")
            out[k] = t
    return out
