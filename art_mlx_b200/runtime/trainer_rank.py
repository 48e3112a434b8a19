"""``TrainerRank``: a low-level, per-rank training API for custom objectives.

Role of the reference ``src/art/trainer_rank/__init__.py:504-1700``
(``TrainerRank``: named LoRA / checkpoint slots, ``forward_micro_batches``,
``dp_rank_forward``, ``dp_reduce``, ``optim_step``): the caller runs forward
passes that return per-token log-probabilities attached to autograd, builds
any loss from them, calls ``backward()`` (LoRA gradients accumulate into the
flat store), then reduces over data-parallel ranks and steps the optimizer.

Here it wraps a :class:`GRPOTrainer` (model, flat LoRA store, AdamW):

* ``forward(inputs)``: each :class:`ForwardInput` is one token sequence (or a
  packed prefix-tree row) and the positions whose next token is scored; the
  prefix-tree attention kernels run them, the LM head + log-softmax returns
  ``logprobs`` (and optionally the entropy) for the scored positions;
* slots: ``load_lora_slot(name, path)`` / ``save_lora_slot(name, dir)``,
  ``set_lora(name)`` and ``with push_lora(name):`` switch the adapter the
  forward uses (``None`` = the trainable live adapter, ``"base"`` = LoRA
  off); only the live adapter receives gradients;
* ``dp_reduce()`` sums gradients over the trainer's process group;
  ``optim_step(lr)`` runs the clipped AdamW (the fused reduce + update on
  GPUs when the trainer has one, which also covers the reduction).
"""

from __future__ import annotations

import contextlib
import os
from dataclasses import dataclass, field
from typing import Iterator, Sequence

import torch
import torch.distributed as dist

from ..ops import fused
from ..ops.fused import AttnMeta


@dataclass
class ForwardInput:
    tokens: Sequence[int]
    # positions t whose next token (tokens[t+1]) is scored; default: all but the last
    score_positions: Sequence[int] | None = None
    # prefix-tree rows: per-token group / parent ids (None: one plain sequence)
    group_ids: Sequence[int] | None = None
    parent_ids: Sequence[int] | None = None
    positions: Sequence[int] | None = None
    entropy: bool = False


@dataclass
class ForwardOutput:
    logprobs: torch.Tensor  # [n_scored], attached to autograd
    entropy: torch.Tensor | None = None
    targets: torch.Tensor = field(default_factory=lambda: torch.empty(0, dtype=torch.long))


class TrainerRank:
    def __init__(self, trainer) -> None:
        self.tr = trainer
        self.slots: dict[str, torch.Tensor] = {}
        self._active: str | None = None
        self._stack: list[str | None] = []

    # ------------------------------------------------------------------ slots
    def load_lora_slot(self, name: str, path: str) -> None:
        from safetensors.torch import load_file

        st = self.tr.store
        sd = load_file(os.path.join(path, "adapter_model.safetensors"))
        flat = torch.zeros_like(st.compute)
        for key, e in st.entries.items():
            if key in sd:
                flat[e.offset : e.offset + e.numel].copy_(sd[key].reshape(-1).to(flat.dtype))
        self.slots[name] = flat

    def snapshot_lora_slot(self, name: str) -> None:
        """The live adapter's current weights as a named (frozen) slot."""
        self.slots[name] = self.tr.store.compute.clone()

    def save_lora_slot(self, name: str | None, output_dir: str) -> None:
        """Write a slot (``None`` = the live adapter) as a PEFT checkpoint."""
        from .checkpoint import save_adapter

        st = self.tr.store
        if name is None:
            self.tr.prepare_checkpoint()
            save_adapter(output_dir, st, self.tr.model.cfg.name, self.tr.model.lora_spec, self.tr.optim.state_dict())
            return
        saved = st.master.clone()
        try:
            st.master.copy_(self.slots[name].float())
            save_adapter(output_dir, st, self.tr.model.cfg.name, self.tr.model.lora_spec, None)
        finally:
            st.master.copy_(saved)

    def set_lora(self, name: str | None) -> None:
        if name not in (None, "base") and name not in self.slots:
            raise KeyError(f"no LoRA slot named {name!r}")
        self._active = name

    @contextlib.contextmanager
    def push_lora(self, name: str | None) -> Iterator[None]:
        self._stack.append(self._active)
        self.set_lora(name)
        try:
            yield
        finally:
            self._active = self._stack.pop()

    @contextlib.contextmanager
    def _adapter(self) -> Iterator[None]:
        m, st = self.tr.model, self.tr.store
        name = self._active
        if name is None:
            yield
            return
        if name == "base":
            m.lora_enabled = False
            try:
                yield
            finally:
                m.lora_enabled = True
            return
        saved = st.compute.clone()
        st.compute.copy_(self.slots[name])
        st.version += 1
        try:
            yield
        finally:
            st.compute.copy_(saved)
            st.version += 1

    # ------------------------------------------------------------------ forward / backward
    def forward(self, inputs: Sequence[ForwardInput]) -> list[ForwardOutput]:
        """One forward per input; the outputs stay on the autograd graph while
        the live adapter is selected (frozen slots return detached values)."""
        from ..preprocessing.prefix_tree import visibility_ends

        dev = self.tr.device
        outs = []
        for inp in inputs:
            toks = torch.tensor(list(inp.tokens), dtype=torch.long)
            T = int(toks.numel())
            if inp.group_ids is not None:
                gid = torch.tensor(list(inp.group_ids)).view(1, T)
                pid = torch.tensor(list(inp.parent_ids)).view(1, T)
                kend = visibility_ends(gid, pid)[0]
            else:
                kend = torch.full((T,), T, dtype=torch.int32)
            pos = torch.tensor(list(inp.positions) if inp.positions is not None else list(range(T)))
            meta = AttnMeta.build(pos, kend, dev)
            sp = list(inp.score_positions) if inp.score_positions is not None else list(range(T - 1))
            sel = torch.tensor(sp, dtype=torch.long)
            targets = toks[sel + 1].to(dev)
            ctx = {"group_ids": None if inp.group_ids is None else torch.tensor(list(inp.group_ids)),
                   "parent_ids": None if inp.parent_ids is None else torch.tensor(list(inp.parent_ids))}
            grad = self._active is None and torch.is_grad_enabled()
            with self._adapter(), torch.set_grad_enabled(grad):
                h = self.tr.model.forward(toks.to(dev), meta, ctx)
                lp, ent = fused.lm_head_logprobs(h.index_select(0, sel.to(dev)), self.tr.model.lm_head, targets,
                                                 self.tr.logprob_chunk, inp.entropy)
            outs.append(ForwardOutput(logprobs=lp, entropy=ent, targets=targets))
        return outs

    def zero_grad(self) -> None:
        self.tr.store.grad.zero_()

    def dp_reduce(self) -> None:
        """Sum LoRA gradients over the trainer's ranks (not needed before
        ``optim_step`` when the fused data-parallel optimizer is in use)."""
        if self.tr.world > 1 and self.tr.grad_sync is None:
            dist.all_reduce(self.tr.store.grad, group=self.tr.group)

    def optim_step(self, learning_rate: float) -> float:
        """Clipped AdamW on the live adapter; returns the gradient norm."""
        tr = self.tr
        if tr.grad_sync is not None:
            tr.grad_sync.reduce_and_step(tr.optim, learning_rate)
        else:
            tr.optim.step(learning_rate)
        return float(tr.optim.grad_norm)
