"""Model architecture configs and the named presets.

The presets are the architectures of the benchmark configurations: a tiny
Qwen3-style decoder, Qwen2.5-7B, Qwen3-30B-A3B (MoE), a Qwen3-Next-style
hybrid (gated DeltaNet + full attention + MoE) and Qwen3-32B.  Field names
follow the Hugging Face config keys so an HF ``config.json`` maps directly
(:meth:`ModelConfig.from_hf_dict`).
"""

from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, replace
from typing import Any, Literal


@dataclass(frozen=True)
class ModelConfig:
    name: str
    family: str  # the checkpoint's model_type: qwen2, qwen3, qwen3_moe, qwen3_next, llama, mistral, gpt_oss
    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position_embeddings: int = 131072
    attention_bias: bool = False  # Qwen2: bias on q/k/v
    qk_norm: bool = False  # Qwen3: RMSNorm over head_dim on q and k
    tie_word_embeddings: bool = False
    sliding_window: int | None = None
    # RoPE frequency scaling of the checkpoint (sorted (key, value) pairs of
    # its rope_scaling / rope_parameters; empty = plain RoPE)
    rope_scaling: tuple = ()
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    shared_expert_intermediate_size: int = 0
    # hybrid linear attention (gated DeltaNet)
    full_attention_interval: int = 0  # every k-th layer is full attention; 0 = all full
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 0
    linear_value_head_dim: int = 0
    linear_conv_kernel_dim: int = 4
    linear_chunk_size: int = 64
    attn_output_gate: bool = False
    # per-layer kinds of transformers-5 configs ("full_attention",
    # "sliding_attention", "linear_attention"); empty = from the fields above
    layer_types: tuple = ()
    # GPT-OSS: learned per-head attention sinks, bias on o_proj, router and
    # expert biases, clamped GLU experts ((up + 1) * g * sigmoid(alpha g))
    attn_sinks: bool = False
    o_bias: bool = False
    router_bias: bool = False
    expert_bias: bool = False
    expert_act: str = "swiglu"  # or "clamped_glu"
    glu_alpha: float = 1.702
    glu_limit: float = 7.0
    # Qwen3-Next / Qwen3.5: RoPE on the first rotary_dim dims of a head only
    # (0: all), RMSNorm weights stored as offsets from one, gated DeltaNet
    # projections stored split (in_proj_qkv / z / b / a) instead of grouped
    rotary_dim: int = 0
    norm_zero_centered: bool = False
    gdn_split_proj: bool = False
    # family-specific settings as sorted (key, value) pairs (Gemma-4: global
    # head size and kv heads, key = value attention, kv sharing, per-layer
    # inputs, the MoE block, logit soft-capping, per-kind RoPE)
    extra: tuple = ()

    @property
    def ex(self) -> dict[str, Any]:
        return dict(self.extra)

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def layer_kind(self, i: int) -> Literal["attention", "linear_attention"]:
        if self.layer_types:
            return "linear_attention" if self.layer_types[i] == "linear_attention" else "attention"
        if self.full_attention_interval and (i + 1) % self.full_attention_interval != 0:
            return "linear_attention"
        return "attention"

    def layer_window(self, i: int) -> int:
        """Sliding-window size of layer ``i`` (0: full attention)."""
        if self.layer_types and self.layer_types[i] == "sliding_attention" and self.sliding_window:
            return int(self.sliding_window)
        return 0

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    def scaled(self, **kw: Any) -> "ModelConfig":
        return replace(self, **kw)

    @classmethod
    def from_hf_dict(cls, d: dict[str, Any], name: str = "custom") -> "ModelConfig":
        if "model_type" not in d:
            raise ValueError("config.json has no model_type: the architecture cannot be identified")
        # the family is the checkpoint's own model_type: an architecture the
        # registry does not know is refused there, never trained as another one
        family = str(d["model_type"])
        if isinstance(d.get("text_config"), dict):  # multimodal wrappers: the language model's config
            d = {**d["text_config"], "model_type": d["text_config"].get("model_type", family)}
            family = str(d["model_type"])
        heads = d["num_attention_heads"]
        # transformers 5 nests the RoPE base and scaling in rope_parameters;
        # hub checkpoints keep rope_theta / rope_scaling at the top level
        rp = dict(d.get("rope_parameters") or {})
        rs = dict(d.get("rope_scaling") or {})
        theta = d.get("rope_theta", rp.get("rope_theta", 1e6))
        scaling = {k: v for k, v in {**rp, **rs}.items() if k != "rope_theta"}
        if (scaling.get("rope_type") or scaling.get("type") or "default") == "default":
            scaling = {}
        aliases = {"qwen3_5_text": "qwen3_5", "qwen3_5_moe_text": "qwen3_5_moe", "gemma4_text": "gemma4"}
        family = aliases.get(family, family)
        if family == "gemma4":
            return _gemma4_config(d, name)
        num_experts = d.get("num_experts", d.get("num_local_experts", 0)) or 0
        gpt_oss = family == "gpt_oss"
        hybrid = family in ("qwen3_next", "qwen3_5", "qwen3_5_moe")
        layer_types = tuple(d.get("layer_types") or ())
        prf = float(d.get("partial_rotary_factor", rp.get("partial_rotary_factor", 1.0)) or 1.0)
        head_dim = d.get("head_dim") or d["hidden_size"] // heads
        return cls(
            name=name,
            family=family,  # type: ignore[arg-type]
            vocab_size=d["vocab_size"],
            hidden_size=d["hidden_size"],
            num_hidden_layers=d["num_hidden_layers"],
            num_attention_heads=heads,
            num_key_value_heads=d.get("num_key_value_heads", heads),
            head_dim=head_dim,
            intermediate_size=d.get("intermediate_size", 0),
            rms_norm_eps=d.get("rms_norm_eps", 1e-6),
            rope_theta=float(theta),
            rope_scaling=tuple(sorted((k, v) for k, v in scaling.items() if not isinstance(v, (list, dict)))),
            attention_bias=family == "qwen2" or d.get("attention_bias", False),
            qk_norm=family in ("qwen3", "qwen3_moe") or hybrid,
            tie_word_embeddings=d.get("tie_word_embeddings", False),
            num_experts=num_experts,
            num_experts_per_tok=d.get("num_experts_per_tok", 0),
            moe_intermediate_size=d.get("moe_intermediate_size", 0) or (d.get("intermediate_size", 0) if gpt_oss else 0),
            norm_topk_prob=d.get("norm_topk_prob", True),
            shared_expert_intermediate_size=d.get("shared_expert_intermediate_size", 0),
            full_attention_interval=d.get("full_attention_interval", 0),
            linear_num_key_heads=d.get("linear_num_key_heads", 0),
            linear_num_value_heads=d.get("linear_num_value_heads", 0),
            linear_key_head_dim=d.get("linear_key_head_dim", 0),
            linear_value_head_dim=d.get("linear_value_head_dim", 0),
            linear_conv_kernel_dim=d.get("linear_conv_kernel_dim", 4),
            sliding_window=d.get("sliding_window") if any(t == "sliding_attention" for t in layer_types) else None,
            layer_types=layer_types,
            attn_sinks=gpt_oss,
            o_bias=gpt_oss and bool(d.get("attention_bias", True)),
            router_bias=gpt_oss,
            expert_bias=gpt_oss,
            expert_act="clamped_glu" if gpt_oss else "swiglu",
            glu_alpha=float(d.get("swiglu_alpha", 1.702)) if gpt_oss else 1.702,
            glu_limit=float(d.get("swiglu_limit", 7.0)) if gpt_oss else 7.0,
            attn_output_gate=hybrid and bool(d.get("attn_output_gate", True)),
            rotary_dim=int(head_dim * prf) if prf < 1.0 else 0,
            norm_zero_centered=hybrid,
            gdn_split_proj=family in ("qwen3_5", "qwen3_5_moe"),
        )


def _gemma4_config(d: dict[str, Any], name: str) -> ModelConfig:
    """Gemma-4 text model: sliding / full attention layers with their own head
    sizes and RoPE, the family's settings kept in ``extra`` (its experts run
    beside the dense MLP and are not routed through the MoE machinery of the
    other families, so ``num_experts`` stays 0)."""
    heads = d["num_attention_heads"]
    L = d["num_hidden_layers"]
    layer_types = tuple(d.get("layer_types") or
                        ["sliding_attention" if (i + 1) % 6 else "full_attention" for i in range(L)])
    rp = dict(d.get("rope_parameters") or {})
    sl = dict(rp.get("sliding_attention") or {"rope_type": "default", "rope_theta": 10_000.0})
    fu = dict(rp.get("full_attention") or {"rope_type": "proportional", "partial_rotary_factor": 0.25,
                                           "rope_theta": 1_000_000.0})
    head_dim = d.get("head_dim") or d["hidden_size"] // heads
    extra = {
        "hidden_activation": d.get("hidden_activation", "gelu_pytorch_tanh"),
        "global_head_dim": int(d.get("global_head_dim") or head_dim),
        "num_global_key_value_heads": int(d.get("num_global_key_value_heads") or d.get("num_key_value_heads", heads)),
        "attention_k_eq_v": bool(d.get("attention_k_eq_v", False)),
        "num_kv_shared_layers": int(d.get("num_kv_shared_layers", 0) or 0),
        "hidden_size_per_layer_input": int(d.get("hidden_size_per_layer_input", 0) or 0),
        "vocab_size_per_layer_input": int(d.get("vocab_size_per_layer_input", d["vocab_size"]) or d["vocab_size"]),
        "use_double_wide_mlp": bool(d.get("use_double_wide_mlp", False)),
        "enable_moe_block": bool(d.get("enable_moe_block", False)),
        "moe_num_experts": int(d.get("num_experts", 0) or 0),
        "moe_top_k": int(d.get("top_k_experts", 0) or 0),
        "moe_intermediate_size": int(d.get("moe_intermediate_size", 0) or 0),
        "final_logit_softcapping": float(d["final_logit_softcapping"]) if d.get("final_logit_softcapping") else 0.0,
        "rope_sliding_theta": float(sl.get("rope_theta", 10_000.0)),
        "rope_sliding_type": str(sl.get("rope_type", "default")),
        "rope_full_theta": float(fu.get("rope_theta", 1_000_000.0)),
        "rope_full_type": str(fu.get("rope_type", "default")),
        "rope_full_partial": float(fu.get("partial_rotary_factor", 1.0)),
        "rope_full_factor": float(fu.get("factor", 1.0)),
        "rope_sliding_factor": float(sl.get("factor", 1.0)),
    }
    return ModelConfig(
        name=name, family="gemma4", vocab_size=d["vocab_size"], hidden_size=d["hidden_size"], num_hidden_layers=L,
        num_attention_heads=heads, num_key_value_heads=d.get("num_key_value_heads", heads), head_dim=head_dim,
        intermediate_size=d.get("intermediate_size", 0), rms_norm_eps=d.get("rms_norm_eps", 1e-6),
        rope_theta=extra["rope_sliding_theta"], max_position_embeddings=d.get("max_position_embeddings", 131072),
        attention_bias=bool(d.get("attention_bias", False)), qk_norm=True,
        tie_word_embeddings=bool(d.get("tie_word_embeddings", True)), sliding_window=d.get("sliding_window"),
        layer_types=layer_types, extra=tuple(sorted(extra.items())),
    )


PRESETS: dict[str, ModelConfig] = {
    "tiny-qwen3": ModelConfig(
        name="tiny-qwen3",
        family="qwen3",
        vocab_size=1024,
        hidden_size=256,
        num_hidden_layers=4,
        num_attention_heads=4,
        num_key_value_heads=2,
        head_dim=64,
        intermediate_size=704,
        qk_norm=True,
    ),
    # head_dim 128 (the GPU attention kernels' head size) at test scale
    "small-qwen3": ModelConfig(
        name="small-qwen3",
        family="qwen3",
        vocab_size=2048,
        hidden_size=512,
        num_hidden_layers=4,
        num_attention_heads=4,
        num_key_value_heads=2,
        head_dim=128,
        intermediate_size=1024,
        qk_norm=True,
    ),
    "qwen2.5-7b": ModelConfig(
        name="qwen2.5-7b",
        family="qwen2",
        vocab_size=152064,
        hidden_size=3584,
        num_hidden_layers=28,
        num_attention_heads=28,
        num_key_value_heads=4,
        head_dim=128,
        intermediate_size=18944,
        attention_bias=True,
    ),
    "qwen3-30b-a3b": ModelConfig(
        name="qwen3-30b-a3b",
        family="qwen3_moe",
        vocab_size=151936,
        hidden_size=2048,
        num_hidden_layers=48,
        num_attention_heads=32,
        num_key_value_heads=4,
        head_dim=128,
        intermediate_size=6144,
        qk_norm=True,
        num_experts=128,
        num_experts_per_tok=8,
        moe_intermediate_size=768,
    ),
    "qwen3-next-hybrid": ModelConfig(
        name="qwen3-next-hybrid",
        family="qwen3_next",
        vocab_size=151936,
        hidden_size=2048,
        num_hidden_layers=48,
        num_attention_heads=16,
        num_key_value_heads=2,
        head_dim=128,
        intermediate_size=5120,
        qk_norm=True,
        num_experts=512,
        num_experts_per_tok=10,
        moe_intermediate_size=512,
        shared_expert_intermediate_size=512,
        full_attention_interval=4,
        linear_num_key_heads=16,
        linear_num_value_heads=16,
        linear_key_head_dim=128,
        linear_value_head_dim=128,
        attn_output_gate=True,
    ),
    "qwen3-32b": ModelConfig(
        name="qwen3-32b",
        family="qwen3",
        vocab_size=151936,
        hidden_size=5120,
        num_hidden_layers=64,
        num_attention_heads=64,
        num_key_value_heads=8,
        head_dim=128,
        intermediate_size=25600,
        qk_norm=True,
    ),
}

# Hugging Face ids that map onto a preset shape (weights are random-init here).
HF_ALIASES = {
    "Qwen/Qwen2.5-7B-Instruct": "qwen2.5-7b",
    "Qwen/Qwen2.5-7B": "qwen2.5-7b",
    "Qwen/Qwen3-30B-A3B": "qwen3-30b-a3b",
    "Qwen/Qwen3-30B-A3B-Instruct-2507": "qwen3-30b-a3b",
    "Qwen/Qwen3-Next-80B-A3B-Instruct": "qwen3-next-hybrid",
    "Qwen/Qwen3-32B": "qwen3-32b",
}


def get_config(name: str) -> ModelConfig:
    """A preset by name or Hugging Face id, or the ``config.json`` of a local
    checkpoint directory."""
    cj = os.path.join(name, "config.json")
    if os.path.isdir(name) and os.path.exists(cj):
        with open(cj) as f:
            return ModelConfig.from_hf_dict(json.load(f), name=os.path.basename(os.path.normpath(name)))
    key = HF_ALIASES.get(name, name)
    if key not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[key]


@dataclass(frozen=True)
class LoRASpec:
    r: int = 8
    alpha: int = 16
    target_modules: tuple[str, ...] = (
        "q_proj",
        "k_proj",
        "v_proj",
        "o_proj",
        "gate_proj",
        "up_proj",
        "down_proj",
    )
    # MoE experts carry LoRA on their gate/up/down; the GDN in/out projections
    # on ``in_proj_qkvz``/``in_proj_ba``/``out_proj`` when targeted.
    expert_targets: tuple[str, ...] = ("gate_proj", "up_proj", "down_proj")

    @property
    def scale(self) -> float:
        return self.alpha / self.r

    @classmethod
    def from_peft(cls, d: dict[str, Any]) -> "LoRASpec":
        return cls(
            r=int(d.get("r", 8)),
            alpha=int(d.get("lora_alpha", 16)),
            target_modules=tuple(d.get("target_modules") or cls.target_modules),
        )

