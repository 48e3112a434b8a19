"""Client utilities: retry, dataset iteration, concurrency limits, SFT
schedules / file streaming, and the S3 layout through a fake ``aws`` CLI
(an executable on PATH that maps ``s3://`` URIs onto a local directory)."""

import asyncio
import json
import math
import os
import stat
import sys

import pytest

from art_mlx_b200.utils.iterate_dataset import iterate_dataset
from art_mlx_b200.utils.limit_concurrency import limit_concurrency
from art_mlx_b200.utils.retry import retry
from art_mlx_b200.utils.sft import (create_lr_schedule, create_sft_dataset_iterator, get_file_row_count,
                                    iterate_file)


def test_retry_sync_and_async():
    calls, seen = [], []

    @retry(max_attempts=3, delay=0.001, on_retry=lambda e, n: seen.append(n))
    def flaky():
        calls.append(1)
        if len(calls) < 3:
            raise ValueError("x")
        return "ok"

    assert flaky() == "ok" and len(calls) == 3 and seen == [1, 2]

    @retry(max_attempts=2, delay=0.001, exceptions=(KeyError,))
    async def always():
        raise KeyError("k")

    with pytest.raises(KeyError):
        asyncio.run(always())

    @retry(max_attempts=5, delay=0.001, exceptions=(KeyError,))
    def other():
        calls.append(2)
        raise ValueError("not retried")

    n = len(calls)
    with pytest.raises(ValueError):
        other()
    assert len(calls) == n + 1


def test_iterate_dataset_is_deterministic_and_resumable():
    data = list(range(10))
    full = list(iterate_dataset(data, groups_per_step=3, num_epochs=2, use_tqdm=False))
    assert [b.step for b in full] == list(range(8))
    assert sorted(x for b in full[:4] for x in b.items) == data  # one epoch covers every item once
    assert full[4].epoch == 1 and full[4].epoch_step == 0
    resumed = list(iterate_dataset(data, groups_per_step=3, num_epochs=2, initial_step=5, use_tqdm=False))
    assert [b.items for b in resumed] == [b.items for b in full[5:]]


def test_limit_concurrency_caps_parallel_calls():
    active, peak = [0], [0]

    @limit_concurrency(2, derive_key=lambda k: k)
    async def work(k):
        active[0] += 1
        peak[0] = max(peak[0], active[0])
        await asyncio.sleep(0.01)
        active[0] -= 1

    async def go():
        await asyncio.gather(*[work("a") for _ in range(6)])

    asyncio.run(go())
    assert peak[0] == 2


def test_lr_schedules():
    lin = create_lr_schedule(10, 1.0, "linear", warmup_steps=2)
    assert lin[:2] == [0.5, 1.0] and lin[2] == 1.0 and abs(lin[-1]) < 1e-12
    cos = create_lr_schedule(5, 2.0, "cosine", min_lr=0.5)
    assert cos[0] == 2.0 and abs(cos[-1] - 0.5) < 1e-12 and abs(cos[2] - 1.25) < 1e-12
    assert create_lr_schedule(3, 1e-4, "constant") == [1e-4] * 3
    assert create_lr_schedule(0, 1.0) == []
    with pytest.raises(ValueError):
        create_lr_schedule(3, 1.0, "bogus")


def test_sft_dataset_chunks_slice_one_schedule():
    trajs = list(range(23))
    chunks = list(create_sft_dataset_iterator(trajs, chunk_size=2, epochs=2, batch_size=3, show_progress=False))
    total = math.ceil(23 / 3) * 2
    full = create_lr_schedule(total, 2e-4, "linear", int(total * 0.1))
    lrs = [lr for c in chunks for lr in c.config.learning_rate]
    assert lrs == full
    assert sum(len(c.trajectories) for c in chunks) == 46
    later = list(create_sft_dataset_iterator(trajs, chunk_size=2, epochs=2, batch_size=3, initial_step=4,
                                             show_progress=False))
    assert [c.step for c in later] == [c.step for c in chunks][2:]


def test_iterate_file_streams_every_row_each_epoch(tmp_path):
    p = tmp_path / "d.jsonl"
    rows = [{"messages": [{"role": "user", "content": str(i)}, {"role": "assistant", "content": "a"}]}
            for i in range(25)]
    p.write_text("\n".join(json.dumps(r) for r in rows) + "\n\n")
    assert get_file_row_count(str(p)) == 25
    got = [t.messages_and_choices[0]["content"] for t in iterate_file(str(p), epochs=2, shuffle_buffer_size=4)]
    assert len(got) == 50 and sorted(got[:25]) == sorted(str(i) for i in range(25))
    assert len(list(iterate_file(str(p), epochs=2, shuffle_buffer_size=4, initial_skip=30))) == 20
    with pytest.raises(ValueError):
        list(iterate_file(str(tmp_path / "x.json")))


_FAKE_AWS = r'''#!PYTHON
import os, shutil, sys
root = os.environ["FAKE_S3_ROOT"]
args = sys.argv[1:]
if args[:1] == ["--profile"]:
    args = args[2:]
def loc(u):
    return os.path.join(root, u[len("s3://"):]) if u.startswith("s3://") else u
if args[0] == "s3" and args[1] in ("sync", "cp"):
    pos = [a for a in args[2:] if not a.startswith("--")]
    ex = [args[i + 1] for i, a in enumerate(args) if a == "--exclude"]
    pos = [a for a in pos if a not in ex]
    src, dst = loc(pos[0]), loc(pos[1])
    if os.path.isfile(src):
        os.makedirs(os.path.dirname(dst), exist_ok=True); shutil.copy(src, dst)
    else:
        if not os.path.isdir(src):
            sys.exit(1)
        skip = tuple(e[:-2] for e in ex)
        for d, _, files in os.walk(src):
            rel = os.path.relpath(d, src)
            if rel.split(os.sep)[0] in skip:
                continue
            os.makedirs(os.path.join(dst, rel), exist_ok=True)
            for f in files:
                shutil.copy(os.path.join(d, f), os.path.join(dst, rel, f))
elif args[0] == "s3" and args[1] == "ls":
    d = loc(args[2])
    if not os.path.isdir(d):
        sys.exit(1)
    for n in sorted(os.listdir(d)):
        print(("                           PRE " + n + "/") if os.path.isdir(os.path.join(d, n)) else n)
elif args[0] == "s3" and args[1] == "presign":
    print("https://example.invalid/" + args[2][len("s3://"):])
else:
    sys.exit(2)
'''


@pytest.fixture()
def fake_aws(tmp_path, monkeypatch):
    bindir = tmp_path / "bin"
    bindir.mkdir()
    exe = bindir / "aws"
    exe.write_text(_FAKE_AWS.replace("#!PYTHON", "#!" + sys.executable))
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{bindir}{os.pathsep}{os.environ['PATH']}")
    monkeypatch.setenv("FAKE_S3_ROOT", str(tmp_path / "s3"))
    monkeypatch.setenv("BACKUP_BUCKET", "bkt")
    return tmp_path / "s3" / "bkt"


def test_s3_push_pull_latest_and_presign(fake_aws, tmp_path):
    from art_mlx_b200.utils import s3

    art = tmp_path / "art"
    mdir = art / "proj" / "models" / "m"
    for step in (1, 3):
        ck = mdir / "checkpoints" / f"{step:04d}"
        ck.mkdir(parents=True)
        (ck / "adapter_model.safetensors").write_bytes(b"w%d" % step)
    (mdir / "history.jsonl").write_text("{}\n")
    assert s3.build_s3_path(model_name="m", project="proj", step=3, prefix="/runs/") == \
        "s3://bkt/runs/proj/models/m/checkpoints/0003"

    async def go():
        await s3.push_model_to_s3("m", "proj", art_path=str(art))
        assert (fake_aws / "proj" / "models" / "m" / "checkpoints" / "0003" / "adapter_model.safetensors").exists()
        assert await s3.get_latest_checkpoint_step_from_s3("m", "proj") == 3
        assert await s3.get_checkpoint_step_not_after_from_s3("m", "proj", 2) == 1
        dst = await s3.pull_model_from_s3("m", "proj", step=1, art_path=str(tmp_path / "art2"))
        assert open(os.path.join(dst, "adapter_model.safetensors"), "rb").read() == b"w1"
        url = await s3.archive_and_presign_step_url("m", "proj", 3, art_path=str(art))
        assert url.endswith("proj/models/m/zipped-steps/0003.zip")
        assert (fake_aws / "proj" / "models" / "m" / "zipped-steps" / "0003.zip").exists()
        with pytest.raises(s3.S3SyncError):
            await s3.s3_sync(str(tmp_path / "missing"), "s3://bkt/x")

    asyncio.run(go())


def test_get_model_config_merges_defaults(tmp_path):
    from art_mlx_b200 import dev

    out = dev.get_model_config("qwen2.5-7b", str(tmp_path / "none"), {"engine_args": {"max_num_seqs": 8},
                                                                       "trainer_args": {"learning_rate": 1e-5}})
    assert out["engine_args"]["max_num_seqs"] == 8 and out["engine_args"]["enable_sleep_mode"] is True
    assert out["engine_args"]["max_model_len"] == out["init_args"]["max_seq_length"]
    assert out["trainer_args"]["learning_rate"] == 1e-5 and out["trainer_args"]["adam_beta2"] == 0.99
    assert "q_proj" in out["lora_config"]["target_modules"] and out["rollout_weights_mode"] == "lora"
    assert out["engine_args"]["lora_target_modules"] == out["lora_config"]["target_modules"]
    ck = tmp_path / "m" / "checkpoints" / "0003"
    ck.mkdir(parents=True)
    ded = dev.get_model_config("qwen2.5-7b", str(tmp_path / "m"), {"trainer_gpu_ids": [0], "inference_gpu_ids": [1],
                                                                   "engine_args": {"enable_sleep_mode": True}})
    assert ded["engine_args"]["enable_sleep_mode"] is False and ded["inference_gpu_ids"] == [1]
    assert ded["init_args"]["model_name"].endswith("0003")
    with pytest.raises(ValueError):
        dev.get_model_config("qwen2.5-7b", "", {"trainer_gpu_ids": [0], "inference_gpu_ids": [0]})
