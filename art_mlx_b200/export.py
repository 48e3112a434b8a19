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


# ---------------------------------------------------------------------------
# GGUF and Hugging Face Hub (MLX fork: ``src/art/mlx/export.py:54,199``)
# ---------------------------------------------------------------------------
_GGUF_ARCH = {"qwen2": "qwen2", "qwen3": "qwen3", "llama": "llama", "mistral": "llama"}
_GGUF_LAYER = {
    "input_layernorm.weight": "attn_norm.weight",
    "post_attention_layernorm.weight": "ffn_norm.weight",
    "self_attn.q_proj.weight": "attn_q.weight", "self_attn.k_proj.weight": "attn_k.weight",
    "self_attn.v_proj.weight": "attn_v.weight", "self_attn.o_proj.weight": "attn_output.weight",
    "self_attn.q_proj.bias": "attn_q.bias", "self_attn.k_proj.bias": "attn_k.bias",
    "self_attn.v_proj.bias": "attn_v.bias",
    "self_attn.q_norm.weight": "attn_q_norm.weight", "self_attn.k_norm.weight": "attn_k_norm.weight",
    "mlp.gate_proj.weight": "ffn_gate.weight", "mlp.up_proj.weight": "ffn_up.weight",
    "mlp.down_proj.weight": "ffn_down.weight",
}


def _interleave_rope_rows(w: torch.Tensor, heads: int) -> torch.Tensor:
    """Rows of a q/k projection from the rotate-half RoPE layout (first half
    of each head, then the second) to the pairwise-interleaved layout that
    GGML's Llama RoPE rotates: row ``(h, i, j)`` -> ``(h, j, i)`` for the
    half ``i`` and offset ``j`` inside a head."""
    out_f = w.shape[0]
    return (w.reshape(heads, 2, out_f // heads // 2, *w.shape[1:]).swapaxes(1, 2).reshape(w.shape))


def convert_to_gguf(model_dir: str, out_path: str, dtype: str = "f16") -> str:
    """Write a dense checkpoint directory (``config.json`` + safetensors, e.g.
    the output of :func:`export_merged`) as one GGUF file for llama.cpp-style
    runtimes: tensors under GGUF names, the architecture's hyper-parameters
    as metadata; weights in ``f16``, ``bf16`` or ``f32`` (1-D norms and
    biases stay f32)."""
    import gguf

    from .models.weights import load_state_dict

    with open(os.path.join(model_dir, "config.json")) as f:
        hf = json.load(f)
    family = hf.get("model_type")
    arch = _GGUF_ARCH.get(family)
    if arch is None:
        raise ValueError(f"GGUF export supports {sorted(_GGUF_ARCH)} checkpoints, not {family!r}")
    sd = load_state_dict(model_dir)
    heads, kv = int(hf["num_attention_heads"]), int(hf.get("num_key_value_heads", hf["num_attention_heads"]))
    hidden = int(hf["hidden_size"])
    rp = hf.get("rope_parameters") or {}
    w = gguf.GGUFWriter(out_path, arch)
    w.add_name(os.path.basename(os.path.normpath(model_dir)))
    w.add_context_length(int(hf.get("max_position_embeddings", 32768)))
    w.add_embedding_length(hidden)
    w.add_block_count(int(hf["num_hidden_layers"]))
    w.add_feed_forward_length(int(hf["intermediate_size"]))
    w.add_head_count(heads)
    w.add_head_count_kv(kv)
    w.add_key_length(int(hf.get("head_dim") or hidden // heads))
    w.add_value_length(int(hf.get("head_dim") or hidden // heads))
    w.add_rope_freq_base(float(hf.get("rope_theta", rp.get("rope_theta", 10000.0))))
    w.add_layer_norm_rms_eps(float(hf.get("rms_norm_eps", 1e-6)))
    np_dt = {"f16": "float16", "bf16": "float32", "f32": "float32"}[dtype]
    for name, t in sorted(sd.items()):
        if name == "model.embed_tokens.weight":
            gname = "token_embd.weight"
        elif name == "model.norm.weight":
            gname = "output_norm.weight"
        elif name == "lm_head.weight":
            gname = "output.weight"
        else:
            m = re.match(r"model\.layers\.(\d+)\.(.+)$", name)
            if m is None or m.group(2) not in _GGUF_LAYER:
                raise ValueError(f"no GGUF name for {name}")
            gname = f"blk.{m.group(1)}.{_GGUF_LAYER[m.group(2)]}"
        t = t.float()
        if arch == "llama" and gname.endswith(("attn_q.weight", "attn_k.weight")):
            t = _interleave_rope_rows(t, heads if "attn_q" in gname else kv)
        arr = t.numpy()
        if t.dim() > 1:
            if dtype == "bf16":
                w.add_tensor(gname, t.to(torch.bfloat16).view(torch.int16).numpy(),
                             raw_dtype=gguf.GGMLQuantizationType.BF16, raw_shape=arr.shape)
                continue
            arr = arr.astype(np_dt)
        w.add_tensor(gname, arr)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return out_path


def push_to_hub(model_dir: str, repo_id: str, *, token: str | None = None, private: bool = True,
                commit_message: str = "Upload model", api: Any = None) -> str:
    """Create (if needed) the Hub repository ``repo_id`` and upload the
    directory (a merged model, a PEFT adapter checkpoint or a GGUF file's
    folder); returns the repository URL."""
    if api is None:
        from huggingface_hub import HfApi

        api = HfApi(token=token)
    url = api.create_repo(repo_id=repo_id, private=private, exist_ok=True)
    api.upload_folder(folder_path=model_dir, repo_id=repo_id, commit_message=commit_message)
    return str(url)
