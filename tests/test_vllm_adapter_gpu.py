"""The adapters this package publishes load through vLLM's own LoRA loader
(PEFT config validation, key parsing, tensor shapes): dense and MoE
(per-expert) checkpoints.  GPU-marked because vLLM's loader pins host memory,
which needs a driver; the tensors themselves are loaded on the CPU."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _load(path: str, expected: set[str]):
    vllm_lora = pytest.importorskip("vllm.lora.lora_model")
    from vllm.lora.peft_helper import PEFTHelper

    ph = PEFTHelper.from_local_dir(path, max_position_embeddings=4096)
    return vllm_lora.LoRAModel.from_local_checkpoint(path, expected, ph, device="cpu", dtype=torch.float32)


@pytest.mark.parametrize("moe", [False, True])
def test_vllm_loads_published_adapter(cuda, tmp_path, moe):
    from art_mlx_b200.models.config import LoRASpec, ModelConfig
    from art_mlx_b200.models.transformer import DecoderLM
    from art_mlx_b200.runtime.checkpoint import save_adapter

    kw = dict(num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32) if moe else {}
    cfg = ModelConfig(name="t", family="qwen3_moe" if moe else "qwen3", vocab_size=256, hidden_size=64,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                      intermediate_size=96, qk_norm=True, **kw)
    m = DecoderLM(cfg, LoRASpec(r=4, alpha=8), "cpu", seed=0)
    m.store.master.normal_()
    path = str(tmp_path / "ck")
    save_adapter(path, m.store, "Qwen/Qwen3-0.6B", m.lora_spec)
    expected = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "experts"}
    if moe:  # vLLM checks an expert module by its suffix from ".experts" on
        expected |= {f"experts.{e}.{p}" for e in range(4) for p in ("gate_proj", "up_proj", "down_proj")}
    lm = _load(path, expected)
    assert lm.rank == 4
    n_modules = len({k.rsplit(".lora_", 1)[0] for k in m.store.entries})
    assert len(lm.loras) == n_modules
    for name, w in lm.loras.items():
        key = f"base_model.model.{name}.lora_A.weight"
        e = m.store.entries[key]
        assert tuple(w.lora_a.shape) in {tuple(e.shape), tuple(reversed(e.shape))}  # layout per vLLM version
