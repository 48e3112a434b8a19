"""MoE adapter layouts: per-expert keys (what this package writes and vLLM
reads, with ``experts`` in the target modules) and the two fused arrangements
of expert blocks that ``target_parameters`` trainers write, expanded back."""

import json

import torch

from art_mlx_b200.models.adapter_formats import expand_fused_moe_lora, has_fused_moe_lora, moe_adapter_config

P = "base_model.model.model.layers.0.mlp.experts"


def _per_expert(E=3, r=4, H=10, F=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(E, r, H, generator=g)  # gate and up share A in the fused layouts
    Bg, Bu = torch.randn(E, F, r, generator=g), torch.randn(E, F, r, generator=g)
    Ad, Bd = torch.randn(E, r, F, generator=g), torch.randn(E, H, r, generator=g)
    return A, Bg, Bu, Ad, Bd


def _check(out, A, Bg, Bu, Ad, Bd):
    E = A.shape[0]
    for e in range(E):
        p = f"{P}.{e}"
        assert torch.equal(out[f"{p}.gate_proj.lora_A.weight"], A[e])
        assert torch.equal(out[f"{p}.up_proj.lora_A.weight"], A[e])
        assert torch.equal(out[f"{p}.gate_proj.lora_B.weight"], Bg[e])
        assert torch.equal(out[f"{p}.up_proj.lora_B.weight"], Bu[e])
        assert torch.equal(out[f"{p}.down_proj.lora_A.weight"], Ad[e])
        assert torch.equal(out[f"{p}.down_proj.lora_B.weight"], Bd[e])


def _pack_rank_major(B):  # [E, out, r] -> [out, r * E], column j * E + e
    E, O, r = B.shape
    return B.permute(1, 2, 0).reshape(O, r * E)


def test_target_parameters_arrangement_expands():
    A, Bg, Bu, Ad, Bd = _per_expert()
    E, r = A.shape[0], A.shape[1]
    fused = {
        f"{P}.base_layer.lora_A.weight": A.reshape(E * r, -1),
        f"{P}.base_layer.lora_B.weight": _pack_rank_major(torch.cat([Bg, Bu], dim=1)),
        f"{P}.lora_A.weight": Ad.reshape(E * r, -1),
        f"{P}.lora_B.weight": _pack_rank_major(Bd),
        "other.lora_A.weight": torch.ones(2, 2),
    }
    assert has_fused_moe_lora(fused)
    out = expand_fused_moe_lora(fused, r)
    _check(out, A, Bg, Bu, Ad, Bd)
    assert torch.equal(out["other.lora_A.weight"], torch.ones(2, 2)) and not has_fused_moe_lora(out)


def test_transposed_arrangement_expands():
    A, Bg, Bu, Ad, Bd = _per_expert(H=14, F=5)
    E, r = A.shape[0], A.shape[1]
    fused = {
        f"{P}.base_layer.lora_A.weight": torch.cat([Bg, Bu], dim=1).transpose(1, 2).reshape(E * r, -1),  # [E r, 2F]
        f"{P}.base_layer.lora_B.weight": A.transpose(1, 2).permute(1, 0, 2).reshape(A.shape[2], E * r),  # [H, E r]
        f"{P}.lora_A.weight": Bd.transpose(1, 2).reshape(E * r, -1),  # [E r, H]
        f"{P}.lora_B.weight": Ad.transpose(1, 2).permute(1, 0, 2).reshape(Ad.shape[2], E * r),  # [F, E r]
    }
    _check(expand_fused_moe_lora(fused, r), A, Bg, Bu, Ad, Bd)


def test_moe_checkpoint_config_lists_experts(tmp_path):
    from art_mlx_b200.models.config import LoRASpec
    from art_mlx_b200.models.lora import LoRAStore
    from art_mlx_b200.runtime.checkpoint import save_adapter

    st = LoRAStore([(f"{P}.0.gate_proj.lora_A.weight", (4, 10), "A")], "cpu", torch.float32)
    save_adapter(str(tmp_path / "ck"), st, "base", LoRASpec(r=4, alpha=8))
    cfg = json.load(open(tmp_path / "ck" / "adapter_config.json"))
    assert "experts" in cfg["target_modules"]
    assert moe_adapter_config(cfg) == cfg
