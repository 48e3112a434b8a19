"""GPT-OSS layers on the GPU (bf16, tcgen05 attention with sinks and a
sliding window on 64-wide heads, clamped-GLU experts with biases on the
grouped tcgen05 GEMM) against the same model in fp32 on the CPU: one GRPO
micro step per packed row, loss and LoRA gradients."""

import random

import pytest
import torch

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def test_gpt_oss_step_matches_cpu_fp32(cuda):
    from art_mlx_b200.models.config import LoRASpec, ModelConfig
    from art_mlx_b200.preprocessing.pack import packed_tensors_from_tokenized_results
    from art_mlx_b200.preprocessing.synthetic import synthetic_groups
    from art_mlx_b200.preprocessing.tokenize import tokenize_trajectory_groups
    from art_mlx_b200.runtime.trainer import GRPOTrainer, stage_row

    cfg = ModelConfig(
        name="small-gpt-oss", family="gpt_oss", vocab_size=2048, hidden_size=256, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, intermediate_size=256, attention_bias=True,
        rope_theta=150000.0, num_experts=4, num_experts_per_tok=2, moe_intermediate_size=256,
        sliding_window=32, layer_types=("sliding_attention", "full_attention"), attn_sinks=True, o_bias=True,
        router_bias=True, expert_bias=True, expert_act="clamped_glu",
        rope_scaling=(("beta_fast", 32.0), ("beta_slow", 1.0), ("factor", 4.0),
                      ("original_max_position_embeddings", 128), ("rope_type", "yarn"), ("truncate", False)),
    )
    groups = synthetic_groups(num_groups=2, rollouts_per_group=4, prompt_len=100, completion_len=40,
                              vocab_size=2048, seed=3)
    res = list(tokenize_trajectory_groups(None, groups, False, True, rng=random.Random(0)))
    packed = packed_tensors_from_tokenized_results(res, 1024, rng=random.Random(0))
    lora = LoRASpec(r=8, alpha=16)
    tg = GRPOTrainer(cfg, lora, cuda, seed=0)
    tc = GRPOTrainer(cfg, lora, "cpu", seed=0)
    cp = lambda dst, src: dst.copy_(src.float().cpu())  # noqa: E731
    for lg, lc in zip(tg.model.layers, tc.model.layers):
        for name in ("in_norm", "post_norm", "qkv_w", "qkv_b", "o_w", "o_b", "sinks"):
            cp(getattr(lc, name), getattr(lg, name))
        mg, mc = lg.moe, lc.moe
        for a, b in ((mc.router_w, mg.router_w), (mc.router_b, mg.router_b), (mc.gu_w_t, mg.gu_w_t),
                     (mc.down_w_t, mg.down_w_t), (mc.params.gu_b, mg.params.gu_b),
                     (mc.params.down_b, mg.params.down_b)):
            cp(a, b)
        with torch.no_grad():
            # some gate / up values beyond the clamp limit, and a router whose
            # choices do not hinge on bf16 rounding (bias steps of 1 between experts)
            mc.gu_w_t.mul_(10.0)
            mg.gu_w_t.copy_(mc.gu_w_t.to(mg.gu_w_t.dtype))
            mc.router_b.copy_(torch.tensor([2.0, 1.0, 0.0, -1.0]))
            mg.router_b.copy_(mc.router_b.to(mg.router_b.dtype))
        lg.sinks.normal_(0.0, 1.0)
        cp(lc.sinks, lg.sinks)
    for name in ("embed", "lm_head", "final_norm"):
        cp(getattr(tc.model, name), getattr(tg.model, name))
    g = torch.Generator().manual_seed(0)
    vals = torch.randn(tc.store.numel, generator=g) * 0.02
    tc.store.master.copy_(vals)
    tc.store.sync_compute()
    tg.store.master.copy_(vals.to(cuda))
    tg.store.sync_compute()
    total = float(packed["assistant_mask"][:, 1:].sum())
    for row in range(packed["tokens"].shape[0]):
        og = tg.micro_step(stage_row(packed, row, cuda), {}, total)
        oc = tc.micro_step(stage_row(packed, row, torch.device("cpu")), {}, total)
        assert abs(float(og["loss"]) - float(oc["loss"])) < 2e-2 * max(1.0, abs(float(oc["loss"])))
    torch.cuda.synchronize()
    from art_mlx_b200.ops import native

    assert native.lib().tc_error_code() == 0
    gg, gc = tg.store.grad.cpu(), tc.store.grad
    parts = {"attention": [], "experts": []}
    for name, e in tc.store.entries.items():
        parts["experts" if ".experts." in name else "attention"].append(slice(e.offset, e.offset + e.numel))
    errs = {k: rel_err(torch.cat([gg[s] for s in v]), torch.cat([gc[s] for s in v])) for k, v in parts.items()}
    assert errs["attention"] < 5e-2 and errs["experts"] < 5e-2, errs
