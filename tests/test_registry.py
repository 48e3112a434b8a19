import pytest

from art_mlx_b200.models.config import get_config
from art_mlx_b200.models.registry import check_parallelism, get_model_support, registered_families


def test_registry_resolves_presets_and_hf_ids():
    assert get_model_support("Qwen/Qwen2.5-7B-Instruct").key == "qwen2"
    s = get_model_support("qwen3-30b-a3b")
    assert s.is_moe and "ep" in s.supports
    assert get_model_support("qwen3-next-hybrid").linear_attention
    assert set(registered_families()) >= {"qwen2", "qwen3", "qwen3_moe", "qwen3_next"}
    with pytest.raises(ValueError, match="does not support tp"):
        check_parallelism(get_model_support("qwen3-30b-a3b"), tp=2)
    assert get_model_support(get_config("tiny-qwen3").scaled(family="llama")).key == "llama"
    cfg = get_config("tiny-qwen3").scaled(family="gpt_neox")
    with pytest.raises(ValueError, match="not supported"):
        get_model_support(cfg)
    assert get_model_support(cfg, allow_unvalidated_arch=True).key == "gpt_neox"


def test_unknown_hf_model_type_is_refused(tmp_path):
    import json

    d = tmp_path / "ckpt"
    d.mkdir()
    (d / "config.json").write_text(json.dumps({
        "model_type": "some_new_arch", "vocab_size": 64, "hidden_size": 32, "num_hidden_layers": 1,
        "num_attention_heads": 2, "intermediate_size": 64}))
    cfg = get_config(str(d))
    assert cfg.family == "some_new_arch"  # never silently mapped to another family
    with pytest.raises(ValueError, match="not supported"):
        get_model_support(str(d))
    (d / "config.json").write_text(json.dumps({"vocab_size": 64}))
    with pytest.raises(ValueError, match="model_type"):
        get_config(str(d))


def test_default_topology_policy():
    from art_mlx_b200.models.config import get_config
    from art_mlx_b200.parallel.topology import default_topology

    # dense 7B fits one GPU: data parallel; a long row turns on context parallelism
    assert default_topology(get_config("qwen2.5-7b"), 8) == {"dp": 8, "tp": 1, "cp": 1, "ep": 1, "etp": 1}
    assert default_topology(get_config("qwen2.5-7b"), 8, row_tokens=65536)["cp"] == 4
    # MoE: experts over every GPU
    assert default_topology(get_config("qwen3-30b-a3b"), 8)["ep"] == 8
    # a model whose bf16 weights exceed the budget of one GPU: tensor parallel
    assert default_topology(get_config("qwen3-32b"), 8, gpu_bytes=40 << 30)["tp"] == 4
