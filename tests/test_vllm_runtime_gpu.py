"""vLLM as the rollout engine: the managed vLLM OpenAI server starts on a
tiny random Qwen3 checkpoint (saved with transformers; token-id prompts, no
tokenizer), hot-loads an adapter this package published, and its greedy
completion with the adapter differs from the base model's."""

import asyncio

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_vllm_serves_published_adapter(cuda, tmp_path):
    transformers = pytest.importorskip("transformers")
    pytest.importorskip("vllm")
    import httpx

    from art_mlx_b200.models.config import LoRASpec, get_config
    from art_mlx_b200.models.transformer import DecoderLM
    from art_mlx_b200.runtime.checkpoint import save_adapter
    from art_mlx_b200.runtime.vllm_runtime import ManagedVllmRuntime, VllmRuntimeConfig

    hf = transformers.Qwen3Config(vocab_size=1024, hidden_size=256, num_hidden_layers=2, num_attention_heads=2,
                                  num_key_value_heads=1, head_dim=128, intermediate_size=512,
                                  max_position_embeddings=1024, tie_word_embeddings=False)
    torch.manual_seed(0)
    transformers.AutoModelForCausalLM.from_config(hf).to(torch.bfloat16).save_pretrained(tmp_path / "base")
    cfg = get_config(str(tmp_path / "base"))
    m = DecoderLM(cfg, LoRASpec(r=8, alpha=16), "cpu", seed=0)
    m.store.master.normal_(0, 0.5)  # a visible adapter
    save_adapter(str(tmp_path / "ck"), m.store, str(tmp_path / "base"), m.lora_spec)
    rt = ManagedVllmRuntime(
        VllmRuntimeConfig(base_model=str(tmp_path / "base"), served_model_name="agent", max_lora_rank=8,
                          skip_tokenizer=True,
                          engine_args={"enforce_eager": True, "max_model_len": 512, "gpu_memory_utilization": 0.2,
                                       "dtype": "bfloat16"}),
        log_path=str(tmp_path / "vllm.log"))

    async def go():
        url = await rt.start(timeout_s=600)
        await rt.load_lora("agent@1", str(tmp_path / "ck"))
        prompt = list(range(5, 37))
        out = {}
        async with httpx.AsyncClient(timeout=120) as c:
            for name in ("agent", "agent@1"):
                r = await c.post(url + "/completions", json={"model": name, "prompt": prompt, "max_tokens": 16,
                                                             "temperature": 0.0, "return_token_ids": True})
                assert r.status_code == 200, r.text
                ch = r.json()["choices"][0]
                out[name] = ch.get("token_ids") or ch.get("text")
        return out

    try:
        out = asyncio.run(go())
    except Exception:
        print(open(tmp_path / "vllm.log").read()[-4000:])
        raise
    finally:
        rt.close()
    assert out["agent"] and out["agent@1"] and out["agent"] != out["agent@1"]
