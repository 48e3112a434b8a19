"""Offloading a trainer's device state to pinned host memory and back."""

import pytest
import torch

from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.ops import fused
from art_mlx_b200.runtime.trainer import GRPOTrainer

pytestmark = pytest.mark.gpu


def test_offload_reload_roundtrip(cuda):
    tr = GRPOTrainer(get_config("small-qwen3"), LoRASpec(r=8, alpha=16), cuda, seed=0)
    T = 256
    meta = fused.AttnMeta.build(torch.arange(T), torch.full((T,), T, dtype=torch.int32), cuda)
    toks = torch.randint(0, 2048, (T,), device=cuda)
    with torch.no_grad():
        before = tr.model.forward(toks, meta, {}).clone()
    torch.cuda.synchronize()
    used = torch.cuda.memory_allocated()
    moved = tr.offload()
    torch.cuda.empty_cache()
    assert moved > 0 and torch.cuda.memory_allocated() < used - moved // 2
    tr.reload()
    with torch.no_grad():
        after = tr.model.forward(toks, meta, {})
    assert torch.equal(before, after)
