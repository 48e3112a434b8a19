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
    # prefix-tree rows: per-token group / parent ids (None: one plain sequence).  The target of a
    # scored position is the next token of the ROW, so every branch must repeat the token its
    # first target is predicted from: pack with at most ``prompt_length - 1`` tokens shareable
    # (``prefix_tree_pack(..., shareable_lengths=[P - 1, ...])``), never the whole prompt
    group_ids: Sequence[int] | None = None
    parent_ids: Sequence[int] | None = None
    positions: Sequence[int] | None = None
    entropy: bool = False
    # extra outputs at the scored positions (reference ForwardInput.top_k /
    # logits / hidden_states): the k most likely next tokens with their
    # log-probabilities, the full logits, the final-normed hidden states
    top_k: int | None = None
    logits: bool = False
    hidden_states: bool = False


@dataclass(frozen=True)
class TopK:
    logprobs: torch.Tensor  # [n_scored, k] fp32, descending
    tokens: torch.Tensor  # [n_scored, k] int64


@dataclass
class ForwardOutput:
    logprobs: torch.Tensor  # [n_scored], attached to autograd
    entropy: torch.Tensor | None = None
    targets: torch.Tensor = field(default_factory=lambda: torch.empty(0, dtype=torch.long))
    top_k: TopK | None = None
    logits: torch.Tensor | None = None  # [n_scored, V], attached to autograd
    hidden_states: torch.Tensor | None = None  # [n_scored, hidden], attached to autograd


def top_k_logprobs(h: torch.Tensor, W: torch.Tensor, k: int, chunk: int = 2048) -> TopK:
    """Top-``k`` next tokens and their log-probabilities from hidden states
    ``h`` [n, H] and the LM head ``W`` [V, H], ``chunk`` rows of logits at a
    time (no [n, V] tensor), in fp32 after the GEMM."""
    n = h.shape[0]
    lp = torch.empty(n, k, device=h.device, dtype=torch.float32)
    tok = torch.empty(n, k, device=h.device, dtype=torch.long)
    with torch.no_grad():
        for s in range(0, n, chunk):
            logits = (h[s : s + chunk] @ W.t()).float()
            v, i = logits.topk(k, dim=-1)
            lp[s : s + chunk] = v - torch.logsumexp(logits, dim=-1, keepdim=True)
            tok[s : s + chunk] = i
    return TopK(logprobs=lp, tokens=tok)


def activation_bytes_per_token(cfg, dtype_bytes: int = 2) -> int:
    """Activations the backward keeps per token and layer of this trainer's
    decoder (inputs of every projection, attention output and statistics,
    the gate/up product), summed over layers: the planner's estimate."""
    H = cfg.hidden_size
    F = cfg.moe_intermediate_size * cfg.num_experts_per_tok if cfg.is_moe else cfg.intermediate_size
    per_layer = (4 * H + (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * cfg.head_dim
                 + cfg.num_attention_heads * cfg.head_dim + 3 * F) * dtype_bytes + 8 * cfg.num_attention_heads
    return per_layer * cfg.num_hidden_layers


def plan_micro_batches(token_counts: Sequence[int], budget_bytes: int, bytes_per_token: int) -> list[list[int]]:
    """Group inputs (in order) into micro batches whose summed activation
    estimate stays under ``budget_bytes``; an input larger than the budget
    gets a micro batch of its own (reference ``trainer_rank`` memory-checked
    micro batching, ``__init__.py:895-977``)."""
    groups: list[list[int]] = []
    cur: list[int] = []
    used = 0
    for i, n in enumerate(token_counts):
        need = int(n) * bytes_per_token
        if cur and used + need > budget_bytes:
            groups.append(cur)
            cur, used = [], 0
        cur.append(i)
        used += need
    if cur:
        groups.append(cur)
    return groups


class TrainerRank:
    def __init__(self, trainer) -> None:
        self.tr = trainer
        self.slots: dict[str, torch.Tensor] = {}
        self._active: str | None = None
        self._stack: list[str | None] = []
        self.checkpoints: dict[str, dict] = {}  # trainable slots with their optimizer state
        self._live_checkpoint: str | None = None

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
            if inp.group_ids is not None:
                # the target at t is the row token t + 1, which must be t's own continuation
                cut = sel[(sel + 1) >= kend.index_select(0, sel).long()]
                if cut.numel():
                    raise ValueError(f"scored positions {cut.tolist()[:8]} end a branch of the prefix tree: the "
                                     f"next row token is not their continuation")
            targets = toks[sel + 1].to(dev)
            ctx = {"group_ids": None if inp.group_ids is None else torch.tensor(list(inp.group_ids)),
                   "parent_ids": None if inp.parent_ids is None else torch.tensor(list(inp.parent_ids))}
            grad = self._active is None and torch.is_grad_enabled()
            model = self.tr.model
            W = model.lm_head
            # families with their own logits (Gemma-4 soft-caps them) provide them
            own_lp = getattr(model, "token_logprobs_hidden", None)
            own_logits = getattr(model, "logits", None)
            with self._adapter(), torch.set_grad_enabled(grad):
                h = model.forward(toks.to(dev), meta, ctx)
                hs = h.index_select(0, sel.to(dev))
                if own_lp is not None:
                    lp, ent = own_lp(hs, targets, self.tr.logprob_chunk, inp.entropy)
                else:
                    lp, ent = fused.lm_head_logprobs(hs, W, targets, self.tr.logprob_chunk, inp.entropy)
                logits = None
                if inp.logits:
                    logits = own_logits(hs) if own_logits is not None else hs @ W.t()
            topk = None
            if inp.top_k:
                if own_logits is not None:
                    with torch.no_grad():
                        v, i = torch.log_softmax(own_logits(hs.detach()).float(), -1).topk(inp.top_k, dim=-1)
                    topk = TopK(logprobs=v, tokens=i)
                else:
                    topk = top_k_logprobs(hs.detach(), W, inp.top_k)
            outs.append(ForwardOutput(logprobs=lp, entropy=ent, targets=targets, top_k=topk, logits=logits,
                                      hidden_states=hs if inp.hidden_states else None))
        return outs

    def forward_micro_batches(self, inputs: Sequence[ForwardInput], memory_budget_bytes: int | None = None):
        """Yield ``(indices, outputs)`` per micro batch, sized so the kept
        activations of one micro batch stay under ``memory_budget_bytes``
        (default: half of the device's free memory); the caller runs its
        loss and ``backward()`` per micro batch before the next forward."""
        counts = [len(inp.tokens) for inp in inputs]
        if memory_budget_bytes is None:
            if self.tr.device.type == "cuda":
                free, _ = torch.cuda.mem_get_info(self.tr.device)
                memory_budget_bytes = free // 2
            else:
                memory_budget_bytes = 1 << 34
        bpt = activation_bytes_per_token(self.tr.model.cfg, torch.empty(0, dtype=self.tr.model.dtype).element_size())
        for group in plan_micro_batches(counts, memory_budget_bytes, bpt):
            yield group, self.forward([inputs[i] for i in group])

    # ------------------------------------------------------------------ checkpoint slots
    def save_checkpoint_slot(self, name: str) -> None:
        """Keep the live adapter and its optimizer state as a named slot
        (reference checkpoint slots: several adapters trained in turn, each
        with its own AdamW moments)."""
        tr = self.tr
        tr.prepare_checkpoint()
        st = tr.store
        self.checkpoints[name] = {"master": st.master.clone(), "exp_avg": st.exp_avg.clone(),
                                  "exp_avg_sq": st.exp_avg_sq.clone(), "step": st.step}

    def set_checkpoint(self, name: str) -> None:
        """Make slot ``name`` the live, trainable adapter (the live one is
        kept under the slot name it was last loaded from, if any)."""
        if name not in self.checkpoints:
            raise KeyError(f"no checkpoint slot named {name!r}")
        if self._live_checkpoint is not None and self._live_checkpoint != name:
            self.save_checkpoint_slot(self._live_checkpoint)
        st, c = self.tr.store, self.checkpoints[name]
        st.master.copy_(c["master"])
        st.exp_avg.copy_(c["exp_avg"])
        st.exp_avg_sq.copy_(c["exp_avg_sq"])
        st.step = int(c["step"])
        st.sync_compute()
        st.grad.zero_()
        self._live_checkpoint = name

    def load_checkpoint_slot(self, name: str, path: str) -> None:
        """A PEFT checkpoint directory (adapter + optimizer state, if present)
        as checkpoint slot ``name``."""
        from .checkpoint import load_adapter

        st = self.tr.store
        saved = {k: getattr(st, k).clone() for k in ("master", "exp_avg", "exp_avg_sq")}
        step = st.step
        try:
            st.exp_avg.zero_()
            st.exp_avg_sq.zero_()
            st.step = 0
            opt = load_adapter(path, st, strict=False)
            if opt is not None:
                self.tr.optim.load_state_dict(opt)
            self.checkpoints[name] = {"master": st.master.clone(), "exp_avg": st.exp_avg.clone(),
                                      "exp_avg_sq": st.exp_avg_sq.clone(), "step": st.step}
        finally:
            for k, v in saved.items():
                getattr(st, k).copy_(v)
            st.step = step

    def checkpoint_slot_optimizer_state(self, name: str) -> dict | None:
        c = self.checkpoints.get(name)
        if c is None:
            return None
        return {"exp_avg": c["exp_avg"], "exp_avg_sq": c["exp_avg_sq"], "step": c["step"]}

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
