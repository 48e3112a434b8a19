"""Flat LoRA parameter store and PEFT-format naming.

All LoRA factors of a model live in ONE contiguous fp32 master buffer with a
compute-dtype copy, one fp32 gradient buffer and the AdamW moments.  Every
per-module ``lora_A`` / ``lora_B`` tensor is a view into those buffers, so the
optimizer, gradient clipping and the data-parallel gradient exchange each run
as a single kernel over one buffer.

Initialisation follows PEFT (and the reference ``megatron/lora.py:529-538``):
``A`` Kaiming-uniform (a = sqrt(5)), ``B`` zero, scale ``alpha / r``.
Key names are PEFT's: ``base_model.model.model.layers.{i}.{self_attn|mlp}.
{proj}.lora_{A|B}.weight`` (experts: ``mlp.experts.{e}.{proj}``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

ALIGN = 64  # elements; keeps every view 256-byte aligned in the fp32 buffers


@dataclass(frozen=True)
class Entry:
    name: str
    shape: tuple[int, ...]
    offset: int
    kind: str  # "A" or "B"

    @property
    def numel(self) -> int:
        return math.prod(self.shape)


class LoRAStore:
    def __init__(
        self,
        specs: list[tuple[str, tuple[int, ...], str]],
        device: torch.device | str,
        compute_dtype: torch.dtype,
        compute_buf: torch.Tensor | None = None,
        grad_buf: torch.Tensor | None = None,
    ) -> None:
        """``compute_buf`` / ``grad_buf`` (optional) place the compute copy and
        the gradient in caller-provided memory (e.g. a peer-mapped arena)."""
        self.entries: dict[str, Entry] = {}
        off = 0
        for name, shape, kind in specs:
            self.entries[name] = Entry(name, tuple(shape), off, kind)
            off += (math.prod(shape) + ALIGN - 1) // ALIGN * ALIGN
        self.numel = off
        self.device = torch.device(device)
        self.compute_dtype = compute_dtype
        self.master = torch.zeros(off, dtype=torch.float32, device=self.device)
        if compute_buf is not None:
            assert compute_buf.numel() == off and compute_buf.dtype == compute_dtype
            self.compute = compute_buf
        else:
            self.compute = (
                self.master
                if compute_dtype == torch.float32
                else torch.zeros(off, dtype=compute_dtype, device=self.device)
            )
        if grad_buf is not None:
            assert grad_buf.numel() == off and grad_buf.dtype == torch.float32
            self.grad = grad_buf
        else:
            self.grad = torch.zeros(off, dtype=torch.float32, device=self.device)
        self.exp_avg = torch.zeros(off, dtype=torch.float32, device=self.device)
        self.exp_avg_sq = torch.zeros(off, dtype=torch.float32, device=self.device)
        self.version = 0  # bumped whenever the parameters change
        self.step = 0

    # ---- views -----------------------------------------------------------
    def _view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        e = self.entries[name]
        return buf[e.offset : e.offset + e.numel].view(e.shape)

    def param(self, name: str) -> torch.Tensor:
        return self._view(self.compute, name)

    def master_view(self, name: str) -> torch.Tensor:
        return self._view(self.master, name)

    def grad_view(self, name: str) -> torch.Tensor:
        return self._view(self.grad, name)

    def contiguous_span(self, names: list[str]) -> tuple[int, int]:
        """(offset, numel) if ``names`` are stored back to back without padding."""
        es = [self.entries[n] for n in names]
        for a, b in zip(es, es[1:]):
            if a.offset + a.numel != b.offset:
                raise ValueError("entries are not contiguous")
        return es[0].offset, sum(e.numel for e in es)

    # ---- init / sync -----------------------------------------------------
    def init_(self, seed: int) -> None:
        g = torch.Generator(device="cpu").manual_seed(seed)
        for e in self.entries.values():
            v = self.master_view(e.name)
            if e.kind == "A":
                fan_in = e.shape[-1]
                bound = math.sqrt(6.0 / ((1 + 5.0) * fan_in))  # kaiming_uniform(a=sqrt(5))
                v.copy_((torch.rand(e.shape, generator=g) * 2 - 1) * bound)
            else:
                v.zero_()
        self.sync_compute()

    @staticmethod
    def numel_for(specs: list[tuple[str, tuple[int, ...], str]]) -> int:
        return sum((math.prod(s) + ALIGN - 1) // ALIGN * ALIGN for _, s, _ in specs)

    def sync_compute(self) -> None:
        if self.compute is not self.master:
            self.compute.copy_(self.master)
        self.version += 1

    def zero_grad(self) -> None:
        self.grad.zero_()

    # ---- (de)serialisation -------------------------------------------------
    def state_dict(self, dtype: torch.dtype | None = None) -> dict[str, torch.Tensor]:
        out = {}
        for name in self.entries:
            t = self.master_view(name)
            out[name] = (t.to(dtype) if dtype is not None else t).detach().cpu().contiguous()
        return out

    def load_state_dict(self, sd: dict[str, torch.Tensor], strict: bool = True) -> None:
        missing = [n for n in self.entries if n not in sd]
        if strict and missing:
            raise KeyError(f"missing LoRA tensors: {missing[:5]}{'...' if len(missing) > 5 else ''}")
        for name, t in sd.items():
            if name not in self.entries:
                if strict:
                    raise KeyError(f"unexpected LoRA tensor {name}")
                continue
            dst = self.master_view(name)
            if tuple(t.shape) != tuple(dst.shape):
                raise ValueError(f"{name}: shape {tuple(t.shape)} != {tuple(dst.shape)}")
            dst.copy_(t.to(torch.float32))
        self.sync_compute()


def peft_key(layer: int, block: str, proj: str, ab: str, expert: int | None = None) -> str:
    """PEFT state-dict key of one LoRA factor."""
    mid = f"experts.{expert}.{proj}" if expert is not None else proj
    return f"base_model.model.model.layers.{layer}.{block}.{mid}.lora_{ab}.weight"
