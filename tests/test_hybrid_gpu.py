"""A Qwen3-Next checkpoint (gated DeltaNet layers, gated attention with
partial RoPE, zero-centred norms, MoE with a shared expert) loaded from its
Hugging Face files into a GPU trainer (bf16, fused kernels: the RoPE kernels
read q / k through the partial-rotary permutation) and a CPU fp32 trainer:
one GRPO micro step per packed row, loss and LoRA gradients agree."""

import random

import pytest
import torch

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def test_qwen3_next_checkpoint_step_matches_cpu_fp32(cuda, tmp_path):
    transformers = pytest.importorskip("transformers")
    from art_mlx_b200.models.config import LoRASpec, get_config
    from art_mlx_b200.models.weights import load_state_dict
    from art_mlx_b200.preprocessing.pack import packed_tensors_from_tokenized_results
    from art_mlx_b200.preprocessing.synthetic import synthetic_groups
    from art_mlx_b200.preprocessing.tokenize import tokenize_trajectory_groups
    from art_mlx_b200.runtime.trainer import GRPOTrainer, stage_row

    hf = transformers.Qwen3NextConfig(
        vocab_size=2048, hidden_size=256, num_hidden_layers=4, num_attention_heads=2, num_key_value_heads=1,
        head_dim=128, intermediate_size=256, moe_intermediate_size=128, num_experts=4, num_experts_per_tok=2,
        shared_expert_intermediate_size=128, linear_num_key_heads=2, linear_num_value_heads=4,
        linear_key_head_dim=128, linear_value_head_dim=128, partial_rotary_factor=0.25,
        layer_types=["linear_attention", "full_attention", "linear_attention", "full_attention"],
        max_position_embeddings=4096, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = transformers.AutoModelForCausalLM.from_config(hf).float().eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.add_(0.1 * torch.randn_like(p))
    model.save_pretrained(tmp_path)
    cfg = get_config(str(tmp_path))
    assert cfg.rotary_dim == 32 and cfg.attn_output_gate and cfg.norm_zero_centered
    sd = load_state_dict(str(tmp_path))
    lora = LoRASpec(r=8, alpha=16)
    tg = GRPOTrainer(cfg, lora, cuda, seed=0)
    tc = GRPOTrainer(cfg, lora, "cpu", seed=0)
    tg.model.load_hf_state_dict(sd)
    tc.model.load_hf_state_dict(sd)
    g = torch.Generator().manual_seed(0)
    vals = torch.randn(tc.store.numel, generator=g) * 0.02
    tc.store.master.copy_(vals)
    tc.store.sync_compute()
    tg.store.master.copy_(vals.to(cuda))
    tg.store.sync_compute()
    groups = synthetic_groups(num_groups=2, rollouts_per_group=4, prompt_len=100, completion_len=40,
                              vocab_size=2048, seed=3)
    res = list(tokenize_trajectory_groups(None, groups, False, True, rng=random.Random(0)))
    packed = packed_tensors_from_tokenized_results(res, 1024, rng=random.Random(0))
    from art_mlx_b200.runtime.trainer import _route_counts

    total = float(packed["assistant_mask"][:, 1:].sum())
    for row in range(packed["tokens"].shape[0]):
        mg = stage_row(packed, row, cuda, conv_width=cfg.linear_conv_kernel_dim, linear_layers=True)
        mc = stage_row(packed, row, torch.device("cpu"), conv_width=cfg.linear_conv_kernel_dim, linear_layers=True)
        # the CPU model's expert choices replayed on both (routing replay): near-tied
        # router logits must not pick different experts in bf16 and fp32
        rec: dict = {}
        with torch.no_grad():
            tc.model.forward(mc.tokens, mc.meta, {"record_routes": rec, "group_ids": mc.group_ids,
                                                  "parent_ids": mc.parent_ids})
        routes = torch.stack([rec[i] for i in sorted(rec)], dim=1)
        mc.routes, mg.routes = routes, routes.to(cuda)
        mc.route_counts = mg.route_counts = _route_counts(routes)
        og = tg.micro_step(mg, {}, total)
        oc = tc.micro_step(mc, {}, total)
        assert abs(float(og["loss"]) - float(oc["loss"])) < 2e-2 * max(1.0, abs(float(oc["loss"])))
    torch.cuda.synchronize()
    from art_mlx_b200.ops import native

    assert native.lib().tc_error_code() == 0
    gg, gc = tg.store.grad.cpu(), tc.store.grad
    parts: dict = {"attention": [], "linear_attn": [], "experts": []}
    for name, e in tc.store.entries.items():
        part = "experts" if ".experts." in name else ("linear_attn" if ".linear_attn." in name else "attention")
        parts[part].append(slice(e.offset, e.offset + e.numel))
    errs = {k: rel_err(torch.cat([gg[s] for s in v]), torch.cat([gc[s] for s in v])) for k, v in parts.items() if v}
    assert all(v < 5e-2 for v in errs.values()), errs
