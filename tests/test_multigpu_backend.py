"""MultiGPUBackend end to end on CPU: a persistent 2-rank gloo worker group
driven by job files, compared with the in-process LocalBackend; job errors
and a rank that exits between steps surface as client errors."""

import asyncio
import os

import pytest
import torch
from safetensors.torch import load_file

import art_mlx_b200 as art
from art_mlx_b200.backends.local import LocalBackend
from art_mlx_b200.backends.multigpu import MultiGPUBackend
from art_mlx_b200.preprocessing.synthetic import synthetic_groups
from art_mlx_b200.runtime import jobs as J


def _model(name="mg"):
    return art.TrainableModel(name=name, project="p", base_model="tiny-qwen3",
                              _internal_config={"peft_args": {"r": 8, "lora_alpha": 16}})


def _groups(seed=0):
    return synthetic_groups(num_groups=4, rollouts_per_group=4, prompt_len=24, completion_len=12,
                            vocab_size=1024, seed=seed)


def _adapter(res):
    return load_file(os.path.join(res.checkpoint_path, "adapter_model.safetensors"))


@pytest.mark.timeout(600)
def test_multigpu_backend_matches_local(tmp_path):
    async def go():
        mg = MultiGPUBackend(path=str(tmp_path / "mg"), num_gpus=2, device="cpu", worker_timeout_s=120)
        lo = LocalBackend(path=str(tmp_path / "lo"), device="cpu")
        try:
            m1, m2 = _model(), _model()
            await m1.register(mg)
            await m2.register(lo)
            for seed in (0, 1):
                r1 = await mg.train(m1, _groups(seed), learning_rate=1e-4)
                r2 = await lo.train(m2, _groups(seed), learning_rate=1e-4)
                assert r1.step == r2.step == seed + 1
                assert abs(r1.metrics["loss/train"] - r2.metrics["loss/train"]) < 1e-5
            a1, a2 = _adapter(r1), _adapter(r2)
            for k in a2:
                torch.testing.assert_close(a1[k], a2[k], atol=1e-6, rtol=1e-5)
            # a job that fails on every rank is reported, and the group restarts
            g = mg._groups[m1.name]
            path = J.next_job_path(g.jobs_dir)
            bad = J.TrainJob(packed_dir=str(tmp_path / "missing"), num_sequences=1, sequence_length=128,
                             checkpoint_dir=str(tmp_path / "no-adapter"), output_dir=None, base_model="tiny-qwen3",
                             learning_rate=1e-4, log_path=path[:-5] + ".log")
            J.write_job(bad, path)
            with pytest.raises(RuntimeError, match="worker job failed"):
                async for _ in J.stream_job(bad, path, process=g.proc):
                    pass
            g.proc.wait(timeout=120)
            r3 = await mg.train(m1, _groups(2), learning_rate=1e-4)
            assert r3.step == 3
        finally:
            await mg.close()

    asyncio.run(go())


@pytest.mark.timeout(600)
def test_multigpu_backend_rank_exit_is_detected(tmp_path, monkeypatch):
    monkeypatch.setenv("ART_B200_WORKER_EXIT", "1:train")
    async def go():
        mg = MultiGPUBackend(path=str(tmp_path), num_gpus=2, device="cpu", worker_timeout_s=30)
        try:
            m = _model("exit")
            await m.register(mg)
            with pytest.raises(RuntimeError, match="exited|stopped beating"):
                await mg.train(m, _groups(), learning_rate=1e-4)
        finally:
            await mg.close()

    asyncio.run(go())


@pytest.mark.timeout(600)
def test_multigpu_backend_context_parallel(tmp_path):
    """cp=2: both ranks split every packed row; same result as one process."""
    async def go():
        mg = MultiGPUBackend(path=str(tmp_path / "mg"), num_gpus=2, device="cpu",
                             topology={"tp": 1, "cp": 2, "ep": 1})
        lo = LocalBackend(path=str(tmp_path / "lo"), device="cpu")
        try:
            m1, m2 = _model("cp"), _model("cp")
            await m1.register(mg)
            await m2.register(lo)
            r1 = await mg.train(m1, _groups(), learning_rate=1e-4)
            r2 = await lo.train(m2, _groups(), learning_rate=1e-4)
            assert abs(r1.metrics["loss/train"] - r2.metrics["loss/train"]) < 1e-5
            a1, a2 = _adapter(r1), _adapter(r2)
            for k in a2:
                torch.testing.assert_close(a1[k], a2[k], atol=1e-6, rtol=1e-5)
        finally:
            await mg.close()

    asyncio.run(go())


@pytest.mark.gpu
@pytest.mark.timeout(900)
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multigpu_backend_two_gpus(tmp_path, monkeypatch):
    """Persistent NCCL worker group (fused peer-memory DP optimizer) through
    the public API; matches the in-process single-GPU LocalBackend."""
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")

    async def go():
        mg = MultiGPUBackend(path=str(tmp_path / "mg"), num_gpus=2, device="cuda")
        lo = LocalBackend(path=str(tmp_path / "lo"), device="cuda:0")
        try:
            m1 = art.TrainableModel(name="g", project="p", base_model="small-qwen3",
                                    _internal_config={"peft_args": {"r": 8, "lora_alpha": 16}})
            m2 = art.TrainableModel(name="g", project="p", base_model="small-qwen3",
                                    _internal_config={"peft_args": {"r": 8, "lora_alpha": 16}})
            await m1.register(mg)
            await m2.register(lo)
            groups = synthetic_groups(num_groups=4, rollouts_per_group=4, prompt_len=96, completion_len=48,
                                      vocab_size=2048, seed=3)
            r1 = await mg.train(m1, groups, learning_rate=1e-4)
            r2 = await lo.train(m2, groups, learning_rate=1e-4)
            assert r1.step == r2.step == 1
            assert abs(r1.metrics["loss/train"] - r2.metrics["loss/train"]) < 1e-2 * max(1.0, abs(r2.metrics["loss/train"]))
            a1, a2 = _adapter(r1), _adapter(r2)
            num = sum(float((a1[k].float() - a2[k].float()).norm() ** 2) for k in a2) ** 0.5
            den = sum(float(a2[k].float().norm() ** 2) for k in a2) ** 0.5
            assert num / den < 1e-2
        finally:
            await mg.close()

    asyncio.run(go())
