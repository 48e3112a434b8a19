"""Layer-wise weight streaming: training with the layers' base weights in
pinned host memory (two device slots) gives the step of the resident model
with activation recompute, dense and MoE."""

import os

import pytest
import torch

from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.runtime.trainer import GRPOTrainer
from test_distributed import CONFIGS, GPU_CFG, _packed, _shape


@pytest.mark.parametrize("name", ["tiny-qwen3", "moe-tiny"])
def test_base_tensors_exclude_the_adapter(name):
    """What a layer's host buffer would hold: its frozen matrices, never a
    view of the LoRA store nor the caches its bindings derive from the store
    (those change with every optimizer step)."""
    from art_mlx_b200.ops.fused import LoRABinding
    from art_mlx_b200.runtime.weight_stream import base_tensors

    cfg = CONFIGS.get(name) or get_config(name)
    tr = GRPOTrainer(cfg, LoRASpec(r=4, alpha=8), "cpu", seed=0)
    tr.train_step(_packed(*_shape("gloo", cfg)), 1e-3, {})  # fills the bindings' caches
    st = tr.store
    store_ptrs = {t.untyped_storage().data_ptr() for t in (st.master, st.compute, st.grad, st.exp_avg, st.exp_avg_sq)}
    layer = tr.model.layers[0]
    caches = set()
    for obj in vars(layer).values():
        for b in (obj if isinstance(obj, (list, tuple)) else [obj]):
            if isinstance(b, LoRABinding):
                caches |= {id(getattr(b, k, None)) for k in ("_bd", "_bd_s", "_at_s", "_bdt")}
    ts = base_tensors(tr.model, layer, "cpu")
    assert ts and not any(t.untyped_storage().data_ptr() in store_ptrs for t in ts)
    assert not any(id(t) in caches for t in ts)
    ids = {id(t) for t in ts}
    assert id(layer.qkv_w) in ids and id(layer.o_w) in ids
    if layer.moe is not None:
        assert id(layer.moe.gu_w_t) in ids and id(layer.moe.down_w_t) in ids and id(layer.moe.router_w) in ids
    else:
        assert id(layer.mlp.gu_w) in ids and id(layer.mlp.down_w) in ids


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
    for stream in (False, False, True):  # two resident runs: the run-to-run spread of the GPU step
        tr = GRPOTrainer(cfg, LoRASpec(r=8, alpha=16), dev, seed=0, recompute=True, stream_weights=stream)
        hs = [tr.train_step(packed, 1e-3, {}).to_host() for _ in range(2)]
        runs.append((tr.store.master.float().cpu(), hs, tr.model.streamer))
    (m0, h0, _), (m1, _, _), (m2, h2, st) = runs
    spread = (m0 - m1).norm() / m0.norm()  # order-dependent reduce-adds in the attention backward, through Adam
    err = (m0 - m2).norm() / m0.norm()
    assert err < 4 * spread + 1e-6, (err, spread)
    for a, b in zip(h0, h2):
        assert abs(a["loss/train"] - b["loss/train"]) < 1e-3 * max(1.0, abs(a["loss/train"]))
        assert abs(a["loss/grad_norm"] - b["loss/grad_norm"]) < 1e-3 * a["loss/grad_norm"]
    host = sum(h.numel() for h in st.host)
    if cfg.num_hidden_layers > len(st.slots):
        # the forward brought every layer in, the backward all but the two still resident
        assert st.bytes_copied >= 2 * host - 2 * max(h.numel() for h in st.host)
        assert st.resident_bytes() < host  # only two layers' worth of base weights on the device
    else:
        assert st.bytes_copied == host  # every layer fits the slots: each came in once
