"""Public API end to end on CPU: TrainableModel + LocalBackend (config 1)."""

import asyncio
import os

import torch

import art_mlx_b200 as art
from art_mlx_b200.backends.local import LocalBackend
from art_mlx_b200.preprocessing.synthetic import synthetic_groups
from art_mlx_b200.runtime.checkpoint import load_adapter_config


def _model():
    return art.TrainableModel(
        name="tiny", project="p", base_model="tiny-qwen3",
        _internal_config={"peft_args": {"r": 8, "lora_alpha": 16}},
    )


def _groups(seed=0):
    return synthetic_groups(num_groups=4, rollouts_per_group=8, prompt_len=32, completion_len=16,
                            vocab_size=1024, seed=seed)


def test_register_train_checkpoint_resume(tmp_path):
    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu")
        model = _model()
        await model.register(backend)
        assert model.inference_model_name == "tiny@0"
        assert await model.get_step() == 0
        res = await backend.train(model, _groups(), learning_rate=1e-4, loss_fn="ppo", epsilon=0.2)
        assert res.step == 1
        assert os.path.exists(os.path.join(res.checkpoint_path, "adapter_model.safetensors"))
        cfg = load_adapter_config(res.checkpoint_path)
        assert cfg["r"] == 8 and cfg["lora_alpha"] == 16 and cfg["base_model_name_or_path"] == "tiny-qwen3"
        assert res.metrics["data/step_trainer_tokens"] == 4 * 8 * 16
        assert res.metrics["loss/grad_norm"] > 0
        assert model.get_inference_name() == "tiny@1"
        # PEFT key names
        from safetensors.torch import load_file

        sd = load_file(os.path.join(res.checkpoint_path, "adapter_model.safetensors"))
        assert "base_model.model.model.layers.0.self_attn.q_proj.lora_A.weight" in sd
        assert sd["base_model.model.model.layers.3.mlp.down_proj.lora_B.weight"].shape == (256, 8)
        # resume on a fresh backend continues from step 1 with the same weights
        backend2 = LocalBackend(path=str(tmp_path), device="cpu")
        model2 = _model()
        await model2.register(backend2)
        t1 = backend._get_trainer(model).store.master
        t2 = backend2._get_trainer(model2).store.master
        assert torch.equal(t1, t2)
        res2 = await backend2.train(model2, _groups(1), learning_rate=1e-4)
        assert res2.step == 2

    asyncio.run(go())


def test_step_advances_when_nothing_is_trainable(tmp_path):
    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu")
        model = _model()
        await model.register(backend)
        groups = _groups()
        for g in groups:
            for t in g:
                t.reward = 1.0  # zero advantages everywhere
        res = await backend.train(model, groups, learning_rate=1e-4)
        assert res.step == 1
        assert res.metrics["data/step_trainer_tokens"] == 0.0

    asyncio.run(go())


def test_log_and_delete_checkpoints(tmp_path):
    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu")
        model = _model()
        await model.register(backend)
        for i in range(3):
            groups = _groups(i)
            res = await backend.train(model, groups, learning_rate=1e-4)
            await model.log(groups, split="val", metrics={"reward": float(-i)}, step=res.step)
        await model.delete_checkpoints("val/reward")
        steps = sorted(os.listdir(os.path.join(str(tmp_path), "p/models/tiny/checkpoints")))
        assert steps == ["0001", "0003"]  # best (val/reward highest at step 1) and latest

    asyncio.run(go())


def test_openai_client_requests_token_ids(tmp_path):
    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu")
        model = _model()
        await model.register(backend)
        client = model.openai_client()
        assert client._extra == {"return_token_ids": True, "return_tokens_as_token_ids": True}

    asyncio.run(go())


def test_grad_accumulation_sequences_splits_the_call(tmp_path):
    """grad_accumulation_sequences=1: one optimizer step per packed row,
    equal to calling train once per row."""
    import random

    from art_mlx_b200.preprocessing.pack import packed_tensors_from_tokenized_results, select_rows
    from art_mlx_b200.preprocessing.tokenize import tokenize_trajectory_groups

    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu")
        model = _model()
        await model.register(backend)
        res = await backend.train(model, _groups(), learning_rate=1e-4, grad_accumulation_sequences=1,
                                  packed_sequence_length=128)
        return backend._get_trainer(model).store.master.clone(), res.metrics["data/step_num_gradient_steps"]

    multi, nsteps = asyncio.run(go())
    # the same rows, one train_step each, on a fresh trainer
    from art_mlx_b200.models.config import LoRASpec, get_config
    from art_mlx_b200.runtime.trainer import GRPOTrainer

    res = list(tokenize_trajectory_groups(None, _groups(), False, True, rng=random.Random(0)))
    packed = packed_tensors_from_tokenized_results(res, 128, rng=random.Random(7))
    tr = GRPOTrainer(get_config("tiny-qwen3"), LoRASpec(r=8, alpha=16), "cpu", seed=0)
    for r in range(int(packed["tokens"].shape[0])):
        tr.train_step(select_rows(packed, [r]), 1e-4, {})
    assert nsteps == packed["tokens"].shape[0] > 1
    assert torch.allclose(multi, tr.store.master, atol=1e-6)


def test_pinned_inference_step_and_leases(tmp_path):
    from art_mlx_b200.adapter_leases import pin_inference_step

    async def go():
        backend = LocalBackend(path=str(tmp_path), device="cpu")
        model = _model()
        await model.register(backend)
        for s in range(3):
            await backend.train(model, _groups(s), learning_rate=1e-4)
        assert model.get_inference_name() == "tiny@3"
        async with pin_inference_step("tiny", 1):
            assert model.get_inference_name() == "tiny@1"
            async with backend.adapter_leases(model).lease(1):
                await backend._delete_checkpoint_files(model, [3])
        assert model.get_inference_name() == "tiny@3"
        ck = os.path.join(str(tmp_path), "p", "models", "tiny", "checkpoints")
        assert sorted(os.listdir(ck)) == ["0001", "0003"]

    asyncio.run(go())
