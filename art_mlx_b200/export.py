"""Merged-weight export: fold a LoRA adapter into base weights.

The MLX fork exports trained adapters by merging them into the base model
(``src/art/mlx/export.py:159`` ``merge_adapters``) and the Megatron path
streams merged weights to the rollout server
(``src/art/megatron/weights/merged_weight_export.py:135``).  Here
:func:`merge_lora_into_state_dict` applies ``W += (alpha / r) * B @ A`` to
every Hugging Face weight an adapter targets (PEFT key names), and
:func:`export_merged` writes the merged model as ``model.safetensors`` plus
a ``config.json``, loadable by this framework (``models.weights``) or any
Hugging Face reader.  Gated DeltaNet and expert LoRA keys are merged the
same way (their PEFT keys name the HF weight directly).
"""

from __future__ import annotations

import json
import os
import re
from typing import Any

import torch

_PEFT = re.compile(r"^base_model\.model\.(.+)\.lora_([AB])\.weight$")


def merge_lora_into_state_dict(base: dict[str, torch.Tensor], adapter: dict[str, torch.Tensor],
                               scale: float, dtype: torch.dtype | None = None) -> dict[str, torch.Tensor]:
    """A new state dict with every targeted ``{module}.weight`` merged
    (fp32 arithmetic, result in ``dtype`` or the base weight's dtype)."""
    pairs: dict[str, dict[str, torch.Tensor]] = {}
    for k, v in adapter.items():
        m = _PEFT.match(k)
        if m:
            pairs.setdefault(m.group(1), {})[m.group(2)] = v
    out = dict(base)
    for module, ab in pairs.items():
        if "A" not in ab or "B" not in ab:
            raise ValueError(f"{module}: adapter has only one LoRA factor")
        key = module + ".weight"
        if key not in base:
            raise KeyError(f"adapter targets {key}, which the base weights do not have")
        w = base[key]
        delta = ab["B"].float().to(w.device) @ ab["A"].float().to(w.device)
        out[key] = (w.float() + scale * delta).to(dtype or w.dtype)
    return out


def export_merged(model: Any, adapter_dir: str, out_dir: str, hf_config: dict[str, Any] | None = None) -> str:
    """Merge the adapter at ``adapter_dir`` into ``model``'s base weights and
    write ``out_dir/model.safetensors`` (+ ``config.json``)."""
    from safetensors.torch import load_file, save_file

    from .runtime.checkpoint import load_adapter_config

    cfg = load_adapter_config(adapter_dir)
    scale = float(cfg["lora_alpha"]) / float(cfg["r"])
    adapter = load_file(os.path.join(adapter_dir, "adapter_model.safetensors"))
    base = {k: v.detach().to("cpu") for k, v in model.hf_state_dict().items()}
    merged = merge_lora_into_state_dict(base, adapter, scale)
    os.makedirs(out_dir, exist_ok=True)
    save_file({k: v.contiguous() for k, v in merged.items()}, os.path.join(out_dir, "model.safetensors"))
    mc = model.cfg
    hf = hf_config or {
        "model_type": mc.family, "vocab_size": mc.vocab_size, "hidden_size": mc.hidden_size,
        "num_hidden_layers": mc.num_hidden_layers, "num_attention_heads": mc.num_attention_heads,
        "num_key_value_heads": mc.num_key_value_heads, "head_dim": mc.head_dim,
        "intermediate_size": mc.intermediate_size, "rms_norm_eps": mc.rms_norm_eps, "rope_theta": mc.rope_theta,
        "tie_word_embeddings": mc.tie_word_embeddings,
    }
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(hf, f, indent=2)
    return out_dir
