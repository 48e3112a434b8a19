"""PEFT-format LoRA checkpoints, optimizer state and atomic publishing.

Format (what the rollout server loads, reference
``src/art/megatron/model_support/lora_disk.py:26-110`` and
``src/art/unsloth/service.py:66-108``):

``checkpoints/{step:04d}/adapter_model.safetensors`` — PEFT keys
``base_model.model.model.layers.{i}.self_attn.q_proj.lora_A.weight`` ...
``checkpoints/{step:04d}/adapter_config.json`` — PEFT ``LoraConfig``.
``checkpoints/{step:04d}/optimizer.pt`` — AdamW moments and step (resume).

A checkpoint is written into a staging directory and renamed into place, so
readers never observe a partial checkpoint (reference
``src/art/megatron/service.py:882-905``).
"""

from __future__ import annotations

import json
import os
import shutil
import uuid
from typing import Any

import torch
from safetensors.torch import load_file, save_file

from ..models.config import LoRASpec
from ..models.lora import LoRAStore


def adapter_config(base_model: str, spec: LoRASpec, **extra: Any) -> dict[str, Any]:
    cfg = {
        "base_model_name_or_path": base_model,
        "peft_type": "LORA",
        "task_type": "CAUSAL_LM",
        "r": spec.r,
        "lora_alpha": spec.alpha,
        "lora_dropout": 0.0,
        "target_modules": sorted(spec.target_modules),
        "bias": "none",
        "fan_in_fan_out": False,
        "inference_mode": True,
        "init_lora_weights": True,
        "use_rslora": False,
        "modules_to_save": None,
    }
    cfg.update(extra)
    return cfg


def snapshot_adapter(store: LoRAStore, optimizer_state: dict | None = None,
                     dtype: torch.dtype = torch.float32) -> tuple[dict[str, torch.Tensor], dict | None]:
    """Host copies of the adapter (and optimizer state) that later training
    steps do not touch, for writing now or in the background."""
    sd = store.state_dict(dtype)
    on_cpu = store.master.device.type == "cpu"
    if on_cpu:  # .cpu() of a host tensor is the tensor itself: copy
        sd = {k: v.clone() for k, v in sd.items()}
    opt = None
    if optimizer_state is not None:
        opt = {k: (v.detach().cpu().clone() if isinstance(v, torch.Tensor) else v) for k, v in optimizer_state.items()}
    return sd, opt


def write_adapter(path: str, sd: dict[str, torch.Tensor], base_model: str, spec: LoRASpec,
                  optimizer_state: dict | None = None) -> str:
    """Write a snapshot to ``path`` atomically (stage + rename)."""
    parent = os.path.dirname(os.path.abspath(path))
    os.makedirs(parent, exist_ok=True)
    stage = os.path.join(parent, f".staging-{uuid.uuid4().hex[:8]}")
    os.makedirs(stage)
    try:
        save_file(sd, os.path.join(stage, "adapter_model.safetensors"), metadata={"format": "pt"})
        with open(os.path.join(stage, "adapter_config.json"), "w") as f:
            json.dump(adapter_config(base_model, spec), f, indent=2)
        if optimizer_state is not None:
            torch.save(optimizer_state, os.path.join(stage, "optimizer.pt"))
        if os.path.exists(path):
            shutil.rmtree(path)
        os.replace(stage, path)
    except BaseException:
        shutil.rmtree(stage, ignore_errors=True)
        raise
    return path


def save_adapter(
    path: str,
    store: LoRAStore,
    base_model: str,
    spec: LoRASpec,
    optimizer_state: dict | None = None,
    dtype: torch.dtype = torch.float32,
) -> str:
    """Write a checkpoint to ``path`` atomically (stage + rename)."""
    sd = store.state_dict(dtype)
    return write_adapter(path, sd, base_model, spec, optimizer_state)


def _write_optimizer(path: str, optimizer_state: dict) -> None:
    tmp = os.path.join(path, f".optimizer-{uuid.uuid4().hex[:8]}.tmp")
    torch.save(optimizer_state, tmp)
    os.replace(tmp, os.path.join(path, "optimizer.pt"))


class AsyncCheckpointWriter:
    """Publishes the adapter of a step at once (the rollout side may load it
    immediately) and writes the optimizer state, which only a resume reads,
    on one background thread so that its file I/O overlaps the next step.
    Both files appear atomically (stage + rename); ``wait()`` returns once
    every submitted write is on disk and re-raises a write error."""

    def __init__(self) -> None:
        from concurrent.futures import ThreadPoolExecutor

        self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="ckpt-writer")
        self._pending: list = []

    def submit(self, path: str, store: LoRAStore, base_model: str, spec: LoRASpec,
               optimizer_state: dict | None = None) -> str:
        sd, opt = snapshot_adapter(store, optimizer_state)
        write_adapter(path, sd, base_model, spec, None)
        if opt is not None:
            self._pending.append(self._pool.submit(_write_optimizer, path, opt))
        return path

    def wait(self) -> None:
        pending, self._pending = self._pending, []
        for f in pending:
            f.result()

    def close(self) -> None:
        self.wait()
        self._pool.shutdown(wait=True)


def load_adapter(path: str, store: LoRAStore, strict: bool = True) -> dict | None:
    """Load adapter weights (and return the optimizer state if present)."""
    sd = load_file(os.path.join(path, "adapter_model.safetensors"))
    store.load_state_dict(sd, strict=strict)
    opt = os.path.join(path, "optimizer.pt")
    return torch.load(opt, map_location="cpu") if os.path.exists(opt) else None


def load_adapter_config(path: str) -> dict[str, Any]:
    with open(os.path.join(path, "adapter_config.json")) as f:
        return json.load(f)
