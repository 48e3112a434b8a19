"""Layer-wise weight streaming: training with the layers' base weights in
pinned host memory (two device slots) gives the step of the resident model
with activation recompute, dense and MoE."""

import os

import pytest
import torch

from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.runtime.trainer import GRPOTrainer
from test_distributed import CONFIGS, GPU_CFG, _packed, _shape


def test_streaming_needs_a_gpu_model():
    tr = GRPOTrainer(get_config("tiny-qwen3"), LoRASpec(r=4, alpha=8), "cpu", seed=0)
    with pytest.raises(RuntimeError):
        tr.model.enable_weight_streaming()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("name", ["dense", "moe-small"])
def test_streamed_step_matches_resident_step(name):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    cfg = GPU_CFG.scaled(num_hidden_layers=4) if name == "dense" else CONFIGS[name]
    dev = torch.device("cuda", 0)
    packed = _packed(*_shape("nccl", cfg))
    runs = []
    for stream in (False, True):
        tr = GRPOTrainer(cfg, LoRASpec(r=8, alpha=16), dev, seed=0, recompute=True, stream_weights=stream)
        for _ in range(2):
            m = tr.train_step(packed, 1e-3, {}).to_host()
        runs.append((tr.store.master.float().cpu(), m, tr.model.streamer))
    (m0, h0, _), (m1, h1, st) = runs
    err = (m0 - m1).norm() / m0.norm()
    assert err < 1e-4, err  # the attention backward's reduce-adds are order-dependent
    assert abs(h0["loss/train"] - h1["loss/train"]) < 1e-3 * max(1.0, abs(h0["loss/train"]))
    host = sum(h.numel() for h in st.host)
    assert st.bytes_copied >= 2 * host  # every layer came in for the forward and again for the backward
    assert st.resident_bytes() < host  # only two layers' worth of base weights on the device
