"""PEFT-format LoRA checkpoints, optimizer state and atomic publishing.

Format (what the rollout server loads, reference
``src/art/megatron/model_support/lora_disk.py:26-110`` and
``src/art/unsloth/service.py:66-108``):

``checkpoints/{step:04d}/adapter_model.safetensors`` — PEFT keys
``base_model.model.model.layers.{i}.self_attn.q_proj.lora_A.weight`` ...
``checkpoints/{step:04d}/adapter_config.json`` — PEFT ``LoraConfig``.
``checkpoints/{step:04d}/optimizer.pt`` — AdamW moments and step (resume);
with the sharded data-parallel optimizer instead one
``optimizer-shard-{rank:02d}-of-{world:02d}.pt`` per rank (its slice of the
flat moments, with the slice's offset), assembled again on load.

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


def _config_for(base_model: str, spec: LoRASpec, names) -> dict[str, Any]:
    """``adapter_config.json`` of an adapter with tensors ``names`` (MoE
    adapters list ``experts`` among the targets, as vLLM expects)."""
    from ..models.adapter_formats import moe_adapter_config

    cfg = adapter_config(base_model, spec)
    return moe_adapter_config(cfg) if any(".mlp.experts." in n for n in names) else cfg


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
            json.dump(_config_for(base_model, spec, sd), f, indent=2)
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
    _write_file(path, "optimizer.pt", optimizer_state)


def _write_file(path: str, name: str, obj: dict) -> None:
    tmp = os.path.join(path, f".{name}-{uuid.uuid4().hex[:8]}.tmp")
    torch.save(obj, tmp)
    os.replace(tmp, os.path.join(path, name))


def load_optimizer_state(path: str) -> dict | None:
    """The checkpoint's AdamW state: ``optimizer.pt``, or the per-rank shard
    files assembled into full flat moments (``None`` if absent or if a shard
    of the set is missing)."""
    full = os.path.join(path, "optimizer.pt")
    if os.path.exists(full):
        return torch.load(full, map_location="cpu")
    names = sorted(n for n in os.listdir(path) if n.startswith("optimizer-shard-") and n.endswith(".pt"))
    if not names:
        return None
    shards = [torch.load(os.path.join(path, n), map_location="cpu") for n in names]
    world = int(shards[0]["world"])
    if len(shards) != world or sorted(int(x["rank"]) for x in shards) != list(range(world)):
        return None  # an incomplete set (a writer did not finish): no moments
    total = int(shards[0]["total"])
    ea = torch.zeros(total, dtype=torch.float32)
    eq = torch.zeros(total, dtype=torch.float32)
    for x in shards:
        o, n = int(x["offset"]), int(x["numel"])
        ea[o : o + n] = x["exp_avg"]
        eq[o : o + n] = x["exp_avg_sq"]
    return {"exp_avg": ea, "exp_avg_sq": eq, "step": int(shards[0]["step"])}


class _PinnedSlot:
    """Host copy of a store's flat master weights and AdamW moments."""

    def __init__(self, numel: int, pin: bool) -> None:
        mk = lambda: torch.empty(numel, dtype=torch.float32, pin_memory=pin)  # noqa: E731
        self.master, self.exp_avg, self.exp_avg_sq = mk(), mk(), mk()
        self.pending = None  # the optimizer write still reading this slot


def write_safetensors_from_flat(path: str, flat: torch.Tensor, entries: dict,
                                metadata: dict[str, str] | None = None) -> None:
    """Write the entries of a flat fp32 host buffer as a safetensors file
    (8-byte little-endian header length, JSON header with dtype / shape /
    data offsets, then the raw tensor bytes) straight from the buffer: no
    per-tensor copies.  Tensors are stored in name order."""
    import struct

    header: dict[str, Any] = {"__metadata__": dict(metadata or {"format": "pt"})}
    names = sorted(entries)
    off = 0
    for name in names:
        e = entries[name]
        nbytes = e.numel * 4
        header[name] = {"dtype": "F32", "shape": list(e.shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((-len(hb)) % 8)
    arr = flat.numpy()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name in names:
            e = entries[name]
            f.write(memoryview(arr[e.offset : e.offset + e.numel]))


class AsyncCheckpointWriter:
    """Checkpoint publishing with the least work on the training path.

    ``submit`` snapshots the store's flat master weights and AdamW moments
    with one device-to-host copy each into pinned host memory (two slots
    alternate), publishes the adapter at once (``adapter_model.safetensors``
    written straight from the pinned buffer, ``adapter_config.json``, stage +
    rename), and writes ``optimizer.pt`` (read only by a resume) on one
    background thread.  ``wait()`` returns once every submitted write is on
    disk and re-raises a write error."""

    def __init__(self) -> None:
        from concurrent.futures import ThreadPoolExecutor

        self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="ckpt-writer")
        self._pending: list = []
        self._slots: list[_PinnedSlot] = []
        self._turn = 0

    def _slot(self, numel: int, pin: bool) -> _PinnedSlot:
        if not self._slots or self._slots[0].master.numel() != numel:
            self.wait()
            self._slots = [_PinnedSlot(numel, pin), _PinnedSlot(numel, pin)]
        slot = self._slots[self._turn]
        self._turn ^= 1
        if slot.pending is not None:
            slot.pending.result()
            slot.pending = None
        return slot

    def submit(self, path: str, store: LoRAStore, base_model: str, spec: LoRASpec,
               with_optimizer: bool = True) -> str:
        cuda = store.master.device.type == "cuda"
        slot = self._slot(store.numel, cuda)
        slot.master.copy_(store.master, non_blocking=cuda)
        if with_optimizer:
            slot.exp_avg.copy_(store.exp_avg, non_blocking=cuda)
            slot.exp_avg_sq.copy_(store.exp_avg_sq, non_blocking=cuda)
        if cuda:
            torch.cuda.current_stream(store.master.device).synchronize()
        parent = os.path.dirname(os.path.abspath(path))
        os.makedirs(parent, exist_ok=True)
        stage = os.path.join(parent, f".staging-{uuid.uuid4().hex[:8]}")
        os.makedirs(stage)
        try:
            write_safetensors_from_flat(os.path.join(stage, "adapter_model.safetensors"), slot.master,
                                        store.entries)
            with open(os.path.join(stage, "adapter_config.json"), "w") as f:
                json.dump(_config_for(base_model, spec, store.entries), f, indent=2)
            if os.path.exists(path):
                shutil.rmtree(path)
            os.replace(stage, path)
        except BaseException:
            shutil.rmtree(stage, ignore_errors=True)
            raise
        if with_optimizer:
            opt = {"exp_avg": slot.exp_avg, "exp_avg_sq": slot.exp_avg_sq, "step": store.step}
            fut = self._pool.submit(_write_optimizer, path, opt)
            slot.pending = fut
            self._pending.append(fut)
        return path

    def submit_optimizer_shard(self, path: str, store: LoRAStore, offset: int, numel: int, rank: int,
                               world: int) -> None:
        """Write this rank's slice of the AdamW moments into the published
        checkpoint ``path`` (one device-to-host copy of the slice, the file
        written on the background thread)."""
        if not os.path.isdir(path):
            raise FileNotFoundError(f"optimizer shard of rank {rank}: checkpoint directory {path} not published "
                                    "(every rank must share the model directory)")
        cuda = store.master.device.type == "cuda"
        # two pinned slots reused across steps (a pinned allocation per call
        # costs more than the copy)
        key = (numel, cuda)
        if getattr(self, "_shard_key", None) != key:
            self.wait()
            mk = lambda: torch.empty(numel, dtype=torch.float32, pin_memory=cuda)  # noqa: E731
            self._shard_slots = [(mk(), mk(), None), (mk(), mk(), None)]
            self._shard_key, self._shard_turn = key, 0
        ea, eq, pending = self._shard_slots[self._shard_turn]
        if pending is not None:
            pending.result()
        ea.copy_(store.exp_avg[offset : offset + numel], non_blocking=cuda)
        eq.copy_(store.exp_avg_sq[offset : offset + numel], non_blocking=cuda)
        if cuda:
            torch.cuda.current_stream(store.master.device).synchronize()
        shard = {"offset": offset, "numel": numel, "total": store.numel, "exp_avg": ea, "exp_avg_sq": eq,
                 "step": store.step, "rank": rank, "world": world}
        name = f"optimizer-shard-{rank:02d}-of-{world:02d}.pt"
        fut = self._pool.submit(_write_file, path, name, shard)
        self._shard_slots[self._shard_turn] = (ea, eq, fut)
        self._shard_turn ^= 1
        self._pending.append(fut)

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
    from ..models.adapter_formats import expand_fused_moe_lora, has_fused_moe_lora

    if has_fused_moe_lora(sd):  # fused expert blocks (PEFT target_parameters): per-expert keys
        sd = expand_fused_moe_lora(sd, int(load_adapter_config(path)["r"]))
    store.load_state_dict(sd, strict=strict)
    return load_optimizer_state(path)


def load_adapter_config(path: str) -> dict[str, Any]:
    with open(os.path.join(path, "adapter_config.json")) as f:
        return json.load(f)
