"""Sharded AdamW state: with the fused data-parallel optimizer every rank
writes only its slice of the moments into the published checkpoint; loading
assembles the slices (and refuses an incomplete set)."""

import os

import torch

from art_mlx_b200.models.lora import LoRAStore
from art_mlx_b200.runtime.checkpoint import AsyncCheckpointWriter, load_optimizer_state


def _store() -> LoRAStore:
    st = LoRAStore([("a.lora_A.weight", (4, 40), "A"), ("a.lora_B.weight", (33, 4), "B")], "cpu", torch.float32)
    g = torch.Generator().manual_seed(0)
    st.exp_avg.copy_(torch.randn(st.numel, generator=g))
    st.exp_avg_sq.copy_(torch.rand(st.numel, generator=g))
    st.step = 7
    return st


def _shards(numel: int, world: int):
    per = (numel + world - 1) // world
    return [(r * per, max(0, min(per, numel - r * per))) for r in range(world)]


def test_shards_assemble_to_full_moments(tmp_path):
    st = _store()
    path = str(tmp_path / "0001")
    os.makedirs(path)
    w = AsyncCheckpointWriter()
    for r, (off, n) in enumerate(_shards(st.numel, 3)):
        w.submit_optimizer_shard(path, st, off, n, r, 3)
    w.close()
    opt = load_optimizer_state(path)
    assert opt is not None and opt["step"] == 7
    assert torch.equal(opt["exp_avg"], st.exp_avg)
    assert torch.equal(opt["exp_avg_sq"], st.exp_avg_sq)


def test_incomplete_shard_set_gives_no_moments(tmp_path):
    st = _store()
    path = str(tmp_path / "0002")
    os.makedirs(path)
    w = AsyncCheckpointWriter()
    off, n = _shards(st.numel, 2)[0]
    w.submit_optimizer_shard(path, st, off, n, 0, 2)
    w.close()
    assert load_optimizer_state(path) is None


def test_full_optimizer_file_still_preferred(tmp_path):
    st = _store()
    path = str(tmp_path / "0003")
    w = AsyncCheckpointWriter()
    w.submit(path, st, "base", __import__("art_mlx_b200.models.config", fromlist=["LoRASpec"]).LoRASpec(r=4, alpha=8))
    w.close()
    opt = load_optimizer_state(path)
    assert torch.equal(opt["exp_avg"], st.exp_avg) and opt["step"] == 7
