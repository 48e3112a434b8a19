"""Merged export: the merged base model without LoRA equals the adapted model."""

import asyncio

import torch

import art_mlx_b200 as art
from art_mlx_b200.backends.local import LocalBackend
from art_mlx_b200.export import export_merged
from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.models.transformer import DecoderLM
from art_mlx_b200.models.weights import maybe_load_base_weights
from art_mlx_b200.ops import fused
from art_mlx_b200.preprocessing.synthetic import synthetic_groups


def test_export_merged_matches_adapter(tmp_path):
    async def go():
        backend = LocalBackend(path=str(tmp_path / "art"), device="cpu")
        model = art.TrainableModel(name="m", project="p", base_model="tiny-qwen3",
                                   _internal_config={"peft_args": {"r": 4, "lora_alpha": 8}})
        await model.register(backend)
        groups = synthetic_groups(num_groups=2, rollouts_per_group=4, prompt_len=16, completion_len=8,
                                  vocab_size=1024, seed=0)
        res = await backend.train(model, groups, learning_rate=5e-2)  # big step: a visible adapter
        return backend._get_trainer(model).model, res.checkpoint_path

    trained, ck = asyncio.run(go())
    out = export_merged(trained, ck, str(tmp_path / "merged"))
    merged = DecoderLM(get_config(out), LoRASpec(r=4, alpha=8), "cpu", seed=123)
    assert maybe_load_base_weights(merged, out)
    merged.lora_enabled = False
    T = 20
    meta = fused.AttnMeta.build(torch.arange(T), torch.full((T,), T, dtype=torch.int32), torch.device("cpu"))
    toks = torch.randint(0, 1024, (T,))
    with torch.no_grad():
        a = trained.forward(toks, meta, {})
        b = merged.forward(toks, meta, {})
    assert (a - b).abs().max() < 1e-4
    trained.lora_enabled = False
    with torch.no_grad():
        c = trained.forward(toks, meta, {})
    trained.lora_enabled = True
    assert (a - c).abs().max() > 1e-3  # the adapter mattered


def test_gguf_export_roundtrip(tmp_path):
    import pytest

    gguf = pytest.importorskip("gguf")
    transformers = pytest.importorskip("transformers")
    from art_mlx_b200.export import convert_to_gguf

    cfg = transformers.Qwen3Config(vocab_size=256, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                                   num_key_value_heads=2, head_dim=16, intermediate_size=96,
                                   tie_word_embeddings=False)
    m = transformers.AutoModelForCausalLM.from_config(cfg).float()
    m.save_pretrained(tmp_path / "hf")
    out = convert_to_gguf(str(tmp_path / "hf"), str(tmp_path / "m.gguf"), dtype="f32")
    r = gguf.GGUFReader(out)
    names = {t.name: t for t in r.tensors}
    assert {"token_embd.weight", "output.weight", "output_norm.weight", "blk.1.attn_q_norm.weight",
            "blk.0.ffn_down.weight"} <= set(names)
    q = names["blk.0.attn_q.weight"]
    ref = m.model.layers[0].self_attn.q_proj.weight.detach().numpy()
    assert tuple(reversed(q.shape.tolist())) == ref.shape or tuple(q.shape.tolist()) == ref.shape
    assert abs(q.data.reshape(ref.shape) - ref).max() < 1e-6
    arch = bytes(r.fields["general.architecture"].parts[-1]).decode()
    assert arch == "qwen3"


def test_push_to_hub_uses_the_hub_api(tmp_path):
    from art_mlx_b200.export import push_to_hub

    calls = []

    class FakeApi:
        def create_repo(self, **kw):
            calls.append(("create", kw))
            return "https://huggingface.co/me/m"

        def upload_folder(self, **kw):
            calls.append(("upload", kw))

    (tmp_path / "adapter_config.json").write_text("{}")
    url = push_to_hub(str(tmp_path), "me/m", api=FakeApi())
    assert url.endswith("me/m") and calls[0][1]["private"] is True and calls[1][1]["folder_path"] == str(tmp_path)
