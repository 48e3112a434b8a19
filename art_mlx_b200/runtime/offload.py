"""Moving a trainer's device state to pinned host memory and back.

Role of the reference ``src/art/megatron/training/weight_offload.py:27``
(``WeightOffloadManager``, offload between jobs): when a trainer shares its
GPU with something else between steps (an external inference server, another
job), its base weights and LoRA/optimizer buffers move to pinned host memory
and come back before the next step.  Tensors are re-pointed in place
(``Tensor.set_``), so every module that holds a reference (layers, fused
views, the LoRA store's views) sees the restored storage without rebuilding
anything.  Host copies are pinned, so both directions run at full PCIe /
C2C speed, and one copy per tensor is issued (no batched-copy API).
"""

from __future__ import annotations

import torch


def _device_tensors(obj, seen: set[int], out: list[torch.Tensor]) -> None:
    if isinstance(obj, torch.Tensor):
        if obj.is_cuda and id(obj) not in seen:
            seen.add(id(obj))
            out.append(obj)
        return
    if isinstance(obj, (list, tuple)):
        for x in obj:
            _device_tensors(x, seen, out)
        return
    if isinstance(obj, dict):
        for x in obj.values():
            _device_tensors(x, seen, out)
        return
    if hasattr(obj, "__dict__") and not isinstance(obj, (type, torch.nn.Module)):
        for x in vars(obj).values():
            _device_tensors(x, seen, out)


class OffloadState:
    """Offloads the storages reachable from ``roots`` (e.g. the model and the
    optimizer); views share a storage and are restored with it."""

    def __init__(self, *roots) -> None:
        self.roots = roots
        self._host: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}  # storage ptr -> (base, host copy)
        self._views: list[tuple[torch.Tensor, int, tuple, tuple, int]] = []
        self.offloaded = False

    def offload(self) -> int:
        """Device -> pinned host; returns the bytes moved."""
        if self.offloaded:
            return 0
        tensors: list[torch.Tensor] = []
        seen: set[int] = set()
        for r in self.roots:
            _device_tensors(r, seen, tensors)
        moved = 0
        for t in tensors:
            st = t.untyped_storage()
            key = st.data_ptr()
            if key not in self._host:
                base = torch.empty(0, dtype=torch.uint8, device=t.device).set_(st)
                host = torch.empty(base.numel(), dtype=torch.uint8, pin_memory=True)
                host.copy_(base, non_blocking=True)
                self._host[key] = (base, host)
                moved += base.numel()
            self._views.append((t, key, tuple(t.shape), tuple(t.stride()), t.storage_offset()))
        torch.cuda.synchronize()
        # drop the device storages: every view now points at an empty placeholder
        for t, key, *_ in self._views:
            t.set_(torch.empty(0, dtype=t.dtype, device=t.device))
        for key, (base, host) in self._host.items():
            base.set_(torch.empty(0, dtype=torch.uint8, device=base.device))
        self.offloaded = True
        return moved

    def reload(self) -> None:
        """Pinned host -> fresh device storages; views re-attached in place."""
        if not self.offloaded:
            return
        storages: dict[int, torch.Tensor] = {}
        for key, (base, host) in self._host.items():
            dev = torch.empty(host.numel(), dtype=torch.uint8, device=base.device)
            dev.copy_(host, non_blocking=True)
            storages[key] = dev
        for t, key, shape, stride, offset in self._views:
            t.set_(storages[key].untyped_storage(), offset, shape, stride)
        torch.cuda.synchronize()
        self._host.clear()
        self._views.clear()
        self.offloaded = False
