"""Base weights from a local Hugging Face checkpoint directory
(``config.json`` + ``*.safetensors`` shards).

The reference loads base weights through Unsloth / Megatron-Bridge
(``src/art/megatron/runtime/bridge_runtime.py:240`` ``load_unique_hf_keys_once``);
here each shard is read once with safetensors and copied into the fused
layout of :class:`DecoderLM` (q/k/v and gate/up concatenated).  Without a
directory the model keeps its seeded random init (benchmarks, tests).
"""

from __future__ import annotations

import glob
import os

import torch


def has_weights(path: str) -> bool:
    return os.path.isdir(path) and bool(glob.glob(os.path.join(path, "*.safetensors")))


def load_state_dict(path: str, device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    sd: dict[str, torch.Tensor] = {}
    for f in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
        sd.update(load_file(f, device=str(device)))
    return sd


def maybe_load_base_weights(model, base_model: str) -> bool:
    """Load ``base_model``'s weights into ``model`` when it names a local
    checkpoint directory; returns whether weights were loaded."""
    if not has_weights(base_model):
        return False
    model.load_hf_state_dict(load_state_dict(base_model))
    return True
