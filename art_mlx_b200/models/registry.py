"""Model-support registry: which architectures the trainer knows, their
default LoRA targets and which parallel modes and features they support.

Role of the reference ``src/art/megatron/model_support/spec.py:92``
(``ModelSupportSpec``), ``registry.py`` and the per-family handlers: the
backend resolves ``base_model`` (a preset name, a Hugging Face id or a local
checkpoint directory) to a family, refuses unknown families unless
``allow_unvalidated_arch`` is set, and takes the family's default LoRA
targets.  Families are described by data here, since every supported family
runs through the same :class:`DecoderLM` layers.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .config import ModelConfig, get_config


@dataclass(frozen=True)
class ModelSupportSpec:
    key: str  # family name (ModelConfig.family)
    hf_model_types: tuple[str, ...]
    default_target_modules: tuple[str, ...]
    is_moe: bool = False
    linear_attention: bool = False
    supports: frozenset[str] = field(default_factory=frozenset)  # "dp", "tp", "cp", "ep", "generate"


_DENSE = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
_REGISTRY: dict[str, ModelSupportSpec] = {}


def register_model_support(spec: ModelSupportSpec) -> None:
    _REGISTRY[spec.key] = spec


for _spec in (
    ModelSupportSpec("qwen2", ("qwen2",), _DENSE, supports=frozenset({"dp", "tp", "cp", "generate"})),
    ModelSupportSpec("qwen3", ("qwen3",), _DENSE, supports=frozenset({"dp", "tp", "cp", "generate"})),
    ModelSupportSpec("qwen3_moe", ("qwen3_moe",), _DENSE, is_moe=True,
                     supports=frozenset({"dp", "ep", "cp", "generate"})),
    ModelSupportSpec("qwen3_next", ("qwen3_next",), _DENSE + ("in_proj_qkvz", "out_proj"), is_moe=True,
                     linear_attention=True, supports=frozenset({"dp", "ep", "cp"})),
    # Qwen3.5 (reference model_support/handlers/qwen3_5.py): the Qwen3-Next
    # hybrid with split gated-DeltaNet projections; dense and MoE variants
    ModelSupportSpec("qwen3_5", ("qwen3_5", "qwen3_5_text"),
                     _DENSE + ("in_proj_qkv", "in_proj_z", "out_proj"), linear_attention=True,
                     supports=frozenset({"dp", "cp"})),
    ModelSupportSpec("qwen3_5_moe", ("qwen3_5_moe", "qwen3_5_moe_text"),
                     _DENSE + ("in_proj_qkv", "in_proj_z", "out_proj"), is_moe=True, linear_attention=True,
                     supports=frozenset({"dp", "ep", "cp"})),
    # the default dense decoder (reference: model_support/handlers/default_dense.py): Llama-style
    # checkpoints run through the same layers (no q/k norm, optional q/k/v bias, RoPE scaling)
    ModelSupportSpec("llama", ("llama",), _DENSE, supports=frozenset({"dp", "tp", "cp", "generate"})),
    ModelSupportSpec("mistral", ("mistral",), _DENSE, supports=frozenset({"dp", "tp", "cp", "generate"})),
    # GPT-OSS (reference model_support/registry.py GPT_OSS_MOE_SPEC): attention
    # sinks, sliding-window layers, biased projections and clamped-GLU experts
    # on the data-parallel path (the expert-parallel exchange runs plain SwiGLU
    # experts; the decode kernel has no sinks or windows)
    ModelSupportSpec("gpt_oss", ("gpt_oss",), _DENSE, is_moe=True, supports=frozenset({"dp"})),
    # Gemma-4 dense / MoE (reference model_support/handlers/gemma4.py): sandwich
    # norms, sliding / full layers with their own head sizes, key = value
    # attention, kv-shared layers, per-layer inputs, soft-capped logits; its
    # expert block runs beside the dense MLP on every rank (models/gemma4.py)
    ModelSupportSpec("gemma4", ("gemma4", "gemma4_text"), _DENSE, supports=frozenset({"dp"})),
):
    register_model_support(_spec)


def registered_families() -> list[str]:
    return sorted(_REGISTRY)


def get_model_support(base_model: str | ModelConfig, allow_unvalidated_arch: bool = False) -> ModelSupportSpec:
    cfg = base_model if isinstance(base_model, ModelConfig) else get_config(base_model)
    spec = _REGISTRY.get(cfg.family)
    if spec is None:
        if not allow_unvalidated_arch:
            raise ValueError(f"model family {cfg.family!r} is not supported (known: {registered_families()}); "
                             "pass allow_unvalidated_arch=True to try it anyway")
        return ModelSupportSpec(cfg.family, (cfg.family,), _DENSE)
    return spec


def check_parallelism(spec: ModelSupportSpec, *, tp: int = 1, cp: int = 1, ep: bool = False, etp: int = 1) -> None:
    for mode, on in (("tp", tp > 1), ("cp", cp > 1), ("ep", ep or etp > 1)):
        if on and mode not in spec.supports:
            raise ValueError(f"{spec.key} does not support {mode} parallelism (supported: {sorted(spec.supports)})")
