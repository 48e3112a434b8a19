"""Gated DeltaNet linear-attention layer (Qwen3-Next style hybrid models)."""

from __future__ import annotations

from .config import LoRASpec, ModelConfig
from .lora import peft_key


def gdn_lora_specs(cfg: ModelConfig, i: int, spec: LoRASpec) -> list[tuple[str, tuple[int, ...], str]]:
    return []


class GatedDeltaNet:
    def __init__(self, cfg: ModelConfig, i, gen, dev, dt, store, spec) -> None:
        raise NotImplementedError("gated DeltaNet layers are not available yet")
