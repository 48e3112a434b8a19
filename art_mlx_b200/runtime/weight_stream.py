"""Layer-wise streaming of frozen base weights from pinned host memory.

Role of the reference's streaming weight offload
(``src/art/megatron/training/streaming_weight_offload.py:107``): a model
whose base weights do not fit next to its activations keeps every decoder
layer's frozen weights in pinned host memory and brings one layer at a time
into a small ring of device slots, prefetching the next layer on a copy
stream while the current one computes.

Design here: each layer's base tensors (everything the layer object reaches
on the device except the LoRA store's views) are packed once into one pinned
host buffer per layer; the device holds ``slots`` buffers of the largest
layer's size.  Bringing layer ``i`` in is one host-to-device copy into a slot
followed by re-pointing the layer's tensors at their offsets in that slot
(``Tensor.set_``, so every holder of a reference sees the new storage).  The
copy stream waits for the compute stream before it overwrites a slot (the
work already issued there may still read the evicted layer) and the compute
stream waits for the copy before it uses the layer.  Streaming needs
per-layer activation recompute: the backward runs each layer's forward
again, which brings the layer back, and the slot it occupies is not evicted
until the next layer is entered (by then its backward has been issued).
Prefetch follows the direction of the last two layers entered (ascending in
the forward, descending in the backward's recomputation).
"""

from __future__ import annotations

from typing import Any

import torch

from art_mlx_b200.ops.fused import LoRABinding


def _collect(obj: Any, skip: set[int], seen: set[int], out: list[torch.Tensor], dev_type: str = "cuda") -> None:
    """Append to ``out`` every tensor on ``dev_type`` reachable from ``obj``
    whose storage is not in ``skip``.  LoRA bindings are not entered: they
    hold views of the adapter store and caches derived from it, which change
    with every optimizer step and are not frozen weights."""
    if isinstance(obj, torch.Tensor):
        if obj.device.type == dev_type and id(obj) not in seen and obj.untyped_storage().data_ptr() not in skip:
            seen.add(id(obj))
            out.append(obj)
        return
    if isinstance(obj, LoRABinding):
        return
    if isinstance(obj, (list, tuple)):
        for x in obj:
            _collect(x, skip, seen, out, dev_type)
        return
    if isinstance(obj, dict):
        for x in obj.values():
            _collect(x, skip, seen, out, dev_type)
        return
    if hasattr(obj, "__dict__") and not isinstance(obj, (type, torch.nn.Module, torch.device)):
        for k, x in vars(obj).items():
            if k in ("ep", "etp", "cfg"):  # contexts shared by every layer stay where they are
                continue
            _collect(x, skip, seen, out, dev_type)


def base_tensors(model: Any, layer: Any, dev_type: str = "cuda") -> list[torch.Tensor]:
    """The frozen base tensors of one decoder layer: everything the layer
    reaches on the device except views of the model's LoRA store."""
    st = model.store
    held = (getattr(st, k, None) for k in ("master", "compute", "grad", "exp_avg", "exp_avg_sq"))
    skip = {t.untyped_storage().data_ptr() for t in held if isinstance(t, torch.Tensor)}
    out: list[torch.Tensor] = []
    _collect(layer, skip, set(), out, dev_type)
    return out


class LayerWeightStreamer:
    """Keeps ``model.layers``' base weights on the host and streams them in."""

    def __init__(self, model: Any, slots: int = 2) -> None:
        if slots < 2:
            raise ValueError("weight streaming needs at least two device slots (one in use, one prefetching)")
        dev = model.device
        if dev.type != "cuda":
            raise RuntimeError("weight streaming moves device weights; the model is on the CPU")
        self.model = model
        self.device = dev
        # per layer: (tensor, byte offset of its storage in the layer's buffer, storage offset, shape, stride)
        self.layers: list[list[tuple[torch.Tensor, int, int, tuple, tuple]]] = []
        self.host: list[torch.Tensor] = []
        biggest = 0
        for layer in model.layers:
            ts = base_tensors(model, layer)
            # one entry per storage: views of one storage move together
            by_storage: dict[int, list[torch.Tensor]] = {}
            for t in ts:
                by_storage.setdefault(t.untyped_storage().data_ptr(), []).append(t)
            entries, off = [], 0
            parts = []
            for ptr, views in by_storage.items():
                stor = views[0].untyped_storage()
                n = stor.nbytes()
                base = torch.empty(0, dtype=torch.uint8, device=dev).set_(stor)
                parts.append((base, off, n))
                for v in views:
                    entries.append((v, off, v.storage_offset(), tuple(v.shape), tuple(v.stride())))
                off += (n + 255) // 256 * 256
            host = torch.empty(off, dtype=torch.uint8, pin_memory=True)
            for base, o, n in parts:
                host[o : o + n].copy_(base)
            self.layers.append(entries)
            self.host.append(host)
            biggest = max(biggest, off)
        torch.cuda.synchronize(dev)
        self.slots = [torch.empty(biggest, dtype=torch.uint8, device=dev) for _ in range(slots)]
        self.slot_of: list[int | None] = [None] * len(model.layers)  # layer -> slot
        self.owner: list[int | None] = [None] * slots  # slot -> layer
        self.ready = [torch.cuda.Event() for _ in range(slots)]
        self.copy_stream = torch.cuda.Stream(dev)
        self.current: int | None = None
        self.bytes_copied = 0
        # the device copies of the base weights are dropped: every view
        # now points at a slot (or at nothing until its layer is brought in)
        for entries in self.layers:
            for t, *_ in entries:
                t.set_(torch.empty(0, dtype=t.dtype, device=dev))

    def _bring(self, i: int, avoid: set[int]) -> int:
        """Issue the copy of layer ``i`` into a free slot (not one in ``avoid``)."""
        if self.slot_of[i] is not None:
            return self.slot_of[i]
        cands = [s for s in range(len(self.slots)) if s not in avoid]
        # a slot nobody holds, else the one whose layer is furthest from i
        s = next((s for s in cands if self.owner[s] is None), None)
        if s is None:
            s = max(cands, key=lambda s: abs(self.owner[s] - i))
        old = self.owner[s]
        if old is not None:
            self.slot_of[old] = None
        compute = torch.cuda.current_stream(self.device)
        self.copy_stream.wait_stream(compute)  # work already issued may still read the evicted layer
        host = self.host[i]
        with torch.cuda.stream(self.copy_stream):
            self.slots[s][: host.numel()].copy_(host, non_blocking=True)
            self.ready[s].record(self.copy_stream)
        self.bytes_copied += host.numel()
        self.owner[s], self.slot_of[i] = i, s
        return s

    def _attach(self, i: int, s: int) -> None:
        stor = self.slots[s].untyped_storage()
        for t, off, soff, shape, stride in self.layers[i]:
            elem = t.element_size()
            t.set_(stor, off // elem + soff, shape, stride)

    def ensure(self, i: int) -> None:
        """Called on entry to layer ``i``: the layer is resident (waited for on
        the compute stream) and the next one in the current direction is on
        its way."""
        cur = None if self.current is None else self.slot_of[self.current]
        s = self._bring(i, set() if cur is None else {cur})
        self._attach(i, s)
        torch.cuda.current_stream(self.device).wait_event(self.ready[s])
        direction = 0 if self.current is None else (1 if i > self.current else -1)
        self.current = i
        nxt = i + (direction or 1)
        if 0 <= nxt < len(self.layers) and len(self.slots) > 1:
            self._bring(nxt, {s})

    def resident_bytes(self) -> int:
        return sum(x.numel() for x in self.slots)
