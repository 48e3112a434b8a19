"""Parity of :class:`DecoderLM` with Hugging Face transformers.

For each supported family a tiny random model is built with transformers,
saved with ``save_pretrained`` (safetensors + config.json), loaded through
this package's own path (``get_config(dir)`` + ``maybe_load_base_weights``)
and run on the same tokens: the logits must agree in fp32.  This is the
oracle for the architectures (reference counterpart: the HF-parity suites of
``tests/integration/megatron/model_support/``) and checks the checkpoint
loader against real HF checkpoints.
"""

import pytest
import torch

transformers = pytest.importorskip("transformers")

from art_mlx_b200.models.config import LoRASpec, get_config  # noqa: E402
from art_mlx_b200.models.transformer import DecoderLM  # noqa: E402
from art_mlx_b200.models.weights import maybe_load_base_weights  # noqa: E402
from art_mlx_b200.ops import fused  # noqa: E402


def _tiny(kind: str):
    common = dict(vocab_size=512, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, max_position_embeddings=512, rms_norm_eps=1e-6, rope_theta=10000.0,
                  tie_word_embeddings=False)
    if kind == "qwen2":
        return transformers.Qwen2Config(intermediate_size=96, **common)
    if kind == "qwen3":
        return transformers.Qwen3Config(intermediate_size=96, head_dim=16, **common)
    if kind == "qwen3_moe":
        return transformers.Qwen3MoeConfig(intermediate_size=96, head_dim=16, moe_intermediate_size=32,
                                           num_experts=4, num_experts_per_tok=2, norm_topk_prob=True,
                                           decoder_sparse_step=1, mlp_only_layers=[], **common)
    if kind == "llama":
        return transformers.LlamaConfig(intermediate_size=96, head_dim=16, **common)
    if kind == "gpt_oss":
        # sinks, a sliding window on alternate layers (shorter than the
        # sequence), biases everywhere, clamped GLU experts, YaRN RoPE
        c = dict(common, num_hidden_layers=4, rope_theta=150000.0)
        return transformers.GptOssConfig(
            intermediate_size=48, head_dim=16, num_local_experts=4, num_experts_per_tok=2, sliding_window=8,
            layer_types=["sliding_attention", "full_attention"] * 2,
            rope_parameters={"rope_type": "yarn", "factor": 4.0, "beta_fast": 32.0, "beta_slow": 1.0,
                             "truncate": False, "original_max_position_embeddings": 64, "rope_theta": 150000.0},
            **{k: v for k, v in c.items() if k != "rope_theta"})
    hybrid = dict(common, num_hidden_layers=4, linear_num_key_heads=2, linear_num_value_heads=4,
                  linear_key_head_dim=16, linear_value_head_dim=16,
                  layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"])
    if kind == "qwen3_next":  # gated DeltaNet + gated attention with partial RoPE + MoE with a shared expert
        return transformers.Qwen3NextConfig(intermediate_size=96, head_dim=16, moe_intermediate_size=32,
                                            num_experts=4, num_experts_per_tok=2,
                                            shared_expert_intermediate_size=32, **hybrid)
    if kind == "qwen3_5":
        from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig

        return Qwen3_5TextConfig(intermediate_size=96, head_dim=16, **hybrid)
    if kind == "qwen3_5_moe":
        from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig

        return Qwen3_5MoeTextConfig(head_dim=16, moe_intermediate_size=32, num_experts=4, num_experts_per_tok=2,
                                    shared_expert_intermediate_size=32, **hybrid)
    raise KeyError(kind)


def _logits_ours(path: str, tokens: torch.Tensor) -> torch.Tensor:
    cfg = get_config(path)
    m = DecoderLM(cfg, LoRASpec(r=4, alpha=8), "cpu", seed=5)
    assert maybe_load_base_weights(m, path)
    m.lora_enabled = False
    T = tokens.numel()
    meta = fused.AttnMeta.build(torch.arange(T), torch.full((T,), T, dtype=torch.int32), torch.device("cpu"))
    with torch.no_grad():
        h = m.forward(tokens, meta, {})
    return h.float() @ m.lm_head.float().t()


@pytest.mark.parametrize("kind", ["qwen2", "qwen3", "qwen3_moe", "llama", "gpt_oss", "qwen3_next", "qwen3_5",
                                  "qwen3_5_moe"])
def test_logits_match_transformers(kind, tmp_path):
    torch.manual_seed(0)
    hf_cfg = _tiny(kind)
    model = transformers.AutoModelForCausalLM.from_config(hf_cfg).float().eval()
    with torch.no_grad():  # non-trivial norm weights, biases and sinks (HF initialises them to 1 / 0)
        for name, p in model.named_parameters():
            if "norm" in name or "bias" in name or "sinks" in name:
                p.add_(0.1 * torch.randn_like(p))
            if kind == "gpt_oss" and "experts" in name and "bias" not in name:
                p.normal_(0, 0.5)  # large enough that the GLU clamp (limit 7) is active somewhere
    model.save_pretrained(tmp_path)
    tokens = torch.randint(0, hf_cfg.vocab_size, (37,))
    with torch.no_grad():
        ref = model(tokens.unsqueeze(0)).logits[0].float()
    ours = _logits_ours(str(tmp_path), tokens)
    err = (ours - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-4, f"{kind}: max relative logit error {err}"


def _tiny_gemma4():
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig

    # every Gemma-4 feature at once: sliding (window shorter than the sequence)
    # and full layers with different head sizes, key = value attention on the
    # full layers, the last two layers sharing keys / values, per-layer inputs,
    # double-wide MLPs on the shared layers, the expert block, soft-capping
    return Gemma4TextConfig(
        vocab_size=512, hidden_size=64, intermediate_size=48, num_hidden_layers=6, num_attention_heads=4,
        num_key_value_heads=2, head_dim=16, global_head_dim=32, num_global_key_value_heads=1, attention_k_eq_v=True,
        num_kv_shared_layers=2, hidden_size_per_layer_input=8, vocab_size_per_layer_input=512,
        use_double_wide_mlp=True, enable_moe_block=True, num_experts=4, top_k_experts=2, moe_intermediate_size=24,
        final_logit_softcapping=30.0, sliding_window=8, layer_types=["sliding_attention", "full_attention"] * 3,
        max_position_embeddings=512, tie_word_embeddings=True)


def test_gemma4_logits_match_transformers(tmp_path):
    from art_mlx_b200.models.gemma4 import Gemma4LM

    torch.manual_seed(0)
    hf_cfg = _tiny_gemma4()
    model = transformers.AutoModelForCausalLM.from_config(hf_cfg).float().eval()
    with torch.no_grad():  # non-trivial norms, router scales and layer scalars (HF initialises them to 1)
        for name, p in model.named_parameters():
            if "norm" in name or "scale" in name:
                p.add_(0.1 * torch.randn_like(p))
        for name, b in model.named_buffers():
            if "layer_scalar" in name:
                b.add_(0.1 * torch.randn_like(b))
    model.save_pretrained(tmp_path)
    tokens = torch.randint(0, hf_cfg.vocab_size, (37,))
    with torch.no_grad():  # use_cache: the kv-shared layers read their source layer's keys / values
        ref = model(tokens.unsqueeze(0), use_cache=True).logits[0].float()
    cfg = get_config(str(tmp_path))
    assert cfg.family == "gemma4" and not cfg.is_moe
    m = Gemma4LM(cfg, LoRASpec(r=4, alpha=8), "cpu", seed=5)
    assert maybe_load_base_weights(m, str(tmp_path))
    m.lora_enabled = False
    T = tokens.numel()
    meta = fused.AttnMeta.build(torch.arange(T), torch.full((T,), T, dtype=torch.int32), torch.device("cpu"))
    with torch.no_grad():
        h = m.forward(tokens, meta, {})
        lp, _ = m.token_logprobs_hidden(h, tokens, entropy=False)
    z = torch.tanh((h.float() @ m.lm_head.float().t()) / 30.0) * 30.0
    err = (z - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-4, f"gemma4: max relative logit error {err}"
    ref_lp = torch.log_softmax(ref, -1).gather(-1, tokens.unsqueeze(-1)).squeeze(-1)
    assert torch.allclose(lp, ref_lp, atol=1e-4)
