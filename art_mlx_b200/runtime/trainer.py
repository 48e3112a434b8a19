"""GRPO training step over packed prefix-tree rows.

Semantics follow the reference's multi-GPU trainer
(``src/art/megatron/train.py:1407-1605``, ``training/microbatches.py:145-170``):

* one packed row per micro step; rows are interleaved across data-parallel
  ranks (rank ``r`` takes rows ``r, r+N, ...``);
* new logprobs are the model's log-softmax at the next packed token; the loss
  is summed over tokens and normalised by the number of trainable tokens of
  the whole step (all micro steps, all ranks);
* gradients are reduced over the data-parallel group, then one clipped AdamW
  update is applied;
* with ``kl_penalty_coef > 0`` the reference logprobs come from the same
  model with the adapter disabled (the frozen base).

B200 specifics: the LM head runs only on trainable positions (all other
positions have zero loss weight), in vocab chunks whose logits are reused
in place for the gradient; the loss, its gradient and the optimizer are
fused kernels; there is no host synchronisation inside a step except the
final metric read.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Mapping

import numpy as np
import torch
import torch.distributed as dist

from ..loss import AlignedLossInputs, loss_fn, resolve_clip
from ..models.config import LoRASpec, ModelConfig
from ..models.transformer import DecoderLM
from ..ops import fused
from ..ops.fused import AttnMeta
from ..parallel import mutation
from ..preprocessing.prefix_tree import visibility_ends
from .optimizer import AdamWConfig, FlatAdamW


@dataclass
class MicroBatch:
    """One packed row staged on the device."""

    tokens: torch.Tensor  # [L] int64
    meta: AttnMeta
    sel: torch.Tensor  # [n] int64 positions with a trainable next token
    targets: torch.Tensor  # [n] int64
    old: torch.Tensor  # [n] fp32 (NaN = missing)
    adv: torch.Tensor  # [n]
    w: torch.Tensor  # [n]
    group: torch.Tensor  # [n] group id of the scored token
    original: torch.Tensor | None = None
    routes: torch.Tensor | None = None  # [L, layers, k] replayed MoE routes
    # per MoE layer, tokens routed to each expert (host lists, from the replayed
    # routes): the single-GPU MoE path sizes its expert groups without a sync
    route_counts: list | None = None
    n_tokens: int = 0  # valid (non-padding) tokens in the row
    n_train: int = 0
    h2d_bytes: int = 0  # bytes copied host -> device to stage this row
    group_ids: torch.Tensor | None = None  # [L] host copies (tree-structured layers)
    parent_ids: torch.Tensor | None = None
    cp_plan: Any = None  # context-parallel plan (parallel/cp.py) when the row is split across ranks
    # per MoE layer, [EP world, experts] slots every EP rank routes to each
    # expert in this micro step (host; from every rank's replayed routes)
    ep_counts: Any = None

    @property
    def L(self) -> int:
        return int(self.tokens.numel())


def _route_counts(routes: torch.Tensor) -> list[list[int]]:
    """Tokens per expert for every MoE layer of a row's replayed routes
    ``[T, layers, k]`` (host tensor); each list is a bincount over the expert
    ids seen (the MoE layer pads it to its expert count)."""
    r = routes.to(torch.int64).numpy()
    return [np.bincount(r[:, layer, :].reshape(-1)).tolist() for layer in range(r.shape[1])]


def _valid_length(group_ids: torch.Tensor) -> int:
    nz = (group_ids >= 0).nonzero()
    return int(nz[-1].item()) + 1 if nz.numel() else 0


_PAD_VALUES = {"tokens": -100, "group_ids": -1, "parent_ids": -1, "input_pos": 0, "assistant_mask": False,
               "logprobs": float("nan"), "advantages": 0.0, "weights": 0.0, "original_logprobs": float("nan")}


def pad_packed_length(packed: Mapping[str, Any], multiple: int) -> dict[str, Any]:
    """A copy of ``packed`` whose row length is padded up to a multiple of
    ``multiple`` with padding tokens (group -1: never attended, never
    trained); replayed routes are padded with expert 0 and no coverage."""
    S = int(packed["tokens"].shape[1])
    extra = (-S) % multiple
    if not extra:
        return dict(packed)
    out = dict(packed)
    for k, v in _PAD_VALUES.items():
        t = packed.get(k)
        if isinstance(t, torch.Tensor) and t.dim() == 2 and t.shape[1] == S:
            out[k] = torch.nn.functional.pad(t, (0, extra), value=v) if t.dtype != torch.bool else torch.cat(
                [t, t.new_zeros(t.shape[0], extra)], dim=1)
    rr = packed.get("moe_routing_replay")
    if rr is not None:
        import dataclasses

        ei = rr.expert_indices
        pad_e = ei.new_zeros((ei.shape[0], extra) + tuple(ei.shape[2:]))
        tm = rr.token_mask
        out["moe_routing_replay"] = dataclasses.replace(
            rr, expert_indices=torch.cat([ei, pad_e], dim=1),
            token_mask=torch.cat([tm, tm.new_zeros((tm.shape[0], extra) + tuple(tm.shape[2:]))], dim=1))
    return out


def stage_row(
    packed: Mapping[str, Any],
    row: int,
    device: torch.device,
    pad_to: int = 64,
    pin: bool = True,
    cp: Any = None,
    conv_width: int = 4,
    linear_layers: bool = False,
) -> MicroBatch:
    """Slice one row of CPU packed tensors, trim trailing padding (rounded up
    to ``pad_to``), build the attention metadata and copy it to ``device``.

    With a context-parallel group ``cp`` every rank of the group stages the
    same row but keeps only its contiguous token slice (plus the plan that
    the attention and gated DeltaNet layers use to exchange the rest)."""
    gids = packed["group_ids"][row]
    n_valid = max(_valid_length(gids), 1)
    L = min(int(gids.numel()), (n_valid + pad_to - 1) // pad_to * pad_to)
    tokens = packed["tokens"][row, :L].clone()
    tokens[tokens < 0] = 0
    mask = packed["assistant_mask"][row, :L]
    # aligned (shifted) views: position t scores token t+1
    m_al = torch.zeros(L, dtype=torch.bool)
    m_al[:-1] = mask[1:]
    sel = m_al.nonzero().squeeze(1)
    nxt = sel + 1
    kend = visibility_ends(packed["group_ids"][row : row + 1, :L], packed["parent_ids"][row : row + 1, :L])[0]
    pos = packed["input_pos"][row, :L]
    if cp is not None and cp.world > 1:
        return _stage_row_cp(packed, row, device, L, kend, pos, sel, n_valid, cp, pin, conv_width, linear_layers)

    moved = [0]

    def dev(t: torch.Tensor) -> torch.Tensor:
        t = t.contiguous()
        moved[0] += t.numel() * t.element_size()
        if pin and device.type == "cuda":
            t = t.pin_memory()
        return t.to(device, non_blocking=True)

    routes = None
    route_counts = None
    rr = packed.get("moe_routing_replay")
    if rr is not None:
        host_routes = rr.expert_indices[row, :L]
        routes = dev(host_routes)
        route_counts = _route_counts(host_routes)
    orig = packed.get("original_logprobs")
    meta = AttnMeta.build(pos, kend, device)
    moved[0] += sum(t.numel() * t.element_size()
                    for t in (meta.positions, meta.kend, meta.tile_kmax, meta.tile_kmin, meta.bwd_units))
    return MicroBatch(
        tokens=dev(tokens),
        meta=meta,
        sel=dev(sel),
        targets=dev(packed["tokens"][row, nxt]),
        old=dev(packed["logprobs"][row, nxt].float()),
        adv=dev(packed["advantages"][row, nxt].float()),
        w=dev(packed["weights"][row, nxt].float()),
        group=dev(packed["group_ids"][row, nxt]),
        original=dev(orig[row, nxt].float()) if orig is not None else None,
        routes=routes,
        route_counts=route_counts,
        n_tokens=n_valid,
        n_train=int(sel.numel()),
        h2d_bytes=moved[0],
        group_ids=packed["group_ids"][row, :L].clone(),
        parent_ids=packed["parent_ids"][row, :L].clone(),
    )


def _stage_row_cp(packed, row, device, L, kend, pos, sel, n_valid, cp, pin, conv_width, linear_layers) -> MicroBatch:
    from ..parallel.cp import CPPlan

    assert L % (cp.world * 64) == 0, "context-parallel rows must split into 64-token multiples"
    gids = packed["group_ids"][row, :L]
    pids = packed["parent_ids"][row, :L]
    plan = CPPlan(cp, kend, pos, gids, pids, conv_width, linear_layers)
    a, b = plan.a, plan.b
    moved = [sum(t.numel() * t.element_size() for t in (plan.meta.positions, plan.meta.kend,
                                                         plan.meta.tile_kmax, plan.meta.tile_kmin,
                                                         plan.meta.bwd_units))]

    def dev(t: torch.Tensor) -> torch.Tensor:
        t = t.contiguous()
        moved[0] += t.numel() * t.element_size()
        if pin and device.type == "cuda":
            t = t.pin_memory()
        return t.to(device, non_blocking=True)

    tokens = packed["tokens"][row, a:b].clone()
    tokens[tokens < 0] = 0
    sel = sel[(sel >= a) & (sel < b)]
    nxt = sel + 1
    routes = None
    rr = packed.get("moe_routing_replay")
    if rr is not None:
        routes = dev(rr.expert_indices[row, a:b])
    orig = packed.get("original_logprobs")
    return MicroBatch(
        tokens=dev(tokens),
        meta=plan.meta,
        sel=dev(sel - a),
        targets=dev(packed["tokens"][row, nxt]),
        old=dev(packed["logprobs"][row, nxt].float()),
        adv=dev(packed["advantages"][row, nxt].float()),
        w=dev(packed["weights"][row, nxt].float()),
        group=dev(packed["group_ids"][row, nxt]),
        original=dev(orig[row, nxt].float()) if orig is not None else None,
        routes=routes,
        n_tokens=max(0, min(n_valid, b) - a),
        n_train=int(sel.numel()),
        h2d_bytes=moved[0],
        group_ids=gids.clone(),
        parent_ids=pids.clone(),
        cp_plan=plan,
    )


def zero_weight(mb: MicroBatch) -> MicroBatch:
    """A micro batch that contributes nothing to the loss or the gradients."""
    mb.w = torch.zeros_like(mb.w)
    mb.adv = torch.zeros_like(mb.adv)
    mb.n_tokens = 0
    return mb


@dataclass
class StepMetrics:
    loss: torch.Tensor
    entropy: torch.Tensor
    probs_corr: torch.Tensor
    kl: torch.Tensor
    grad_norm: torch.Tensor
    n_train: int
    n_tokens: int | torch.Tensor
    # status words of the step's bounded device waits (0 = every wait
    # completed); read with the metrics in the same device->host copy
    health: torch.Tensor | None = None
    health_names: tuple[str, ...] = ()

    def to_host(self) -> dict[str, float]:
        """Metrics as host floats (one device->host copy).  Raises
        :class:`DeviceWaitTimeout` when a bounded device wait of the step gave
        up: the step's gradients or parameters are then partial, so no
        checkpoint may be written from it."""
        parts = [self.loss, self.entropy, self.probs_corr, self.kl, self.grad_norm.reshape(())]
        tok = self.n_tokens
        parts.append(tok.reshape(()) if torch.is_tensor(tok) else self.loss.new_tensor(float(tok)))
        nh = 0
        if self.health is not None:
            nh = int(self.health.numel())
            parts.extend(self.health.float().unbind(0))
        vals = torch.stack([p.float().reshape(()) for p in parts]).cpu().tolist()
        loss, ent, pc, kl, gn, ntok = vals[:6]
        bad = [f"{name}={int(v)}" for name, v in zip(self.health_names, vals[6 : 6 + nh]) if v != 0]
        if bad:
            raise DeviceWaitTimeout("a bounded device wait gave up during the step (" + ", ".join(bad) +
                                    "); its gradients or parameters are incomplete")
        return {
            "loss/train": loss,
            "loss/entropy": ent,
            "loss/probs_corr": pc,
            "loss/kl_policy_ref": kl,
            "loss/grad_norm": gn,
            "data/step_trainer_tokens": float(self.n_train),
            "data/step_packed_tokens": float(ntok),
        }


class DeviceWaitTimeout(RuntimeError):
    """A kernel's bounded wait (peer barrier, tensor-core pipeline barrier)
    ran out and recorded a status instead of hanging."""


def _probs_corr_device(old: torch.Tensor, new: torch.Tensor) -> torch.Tensor:
    """Pearson correlation of exp(old) and exp(new) over non-NaN ``old``
    without host synchronisation (0 when undefined)."""
    have = ~torch.isnan(old)
    n = have.sum().float()
    po = torch.where(have, old, torch.zeros_like(old)).exp() * have
    pn = new.detach().exp() * have
    mo = po.sum() / n.clamp_min(1)
    mn = pn.sum() / n.clamp_min(1)
    do = (po - mo) * have
    dn = (pn - mn) * have
    cov = (do * dn).sum()
    so = (do * do).sum().sqrt()
    sn = (dn * dn).sum().sqrt()
    den = so * sn
    ok = (n >= 2) & (den > 0)
    return torch.where(ok, cov / torch.where(den > 0, den, torch.ones_like(den)), torch.zeros_like(den))


class GRPOTrainer:
    """Owns the model, the LoRA store and the optimizer on one device/rank."""

    def __init__(
        self,
        cfg: ModelConfig,
        lora: LoRASpec,
        device: torch.device | str = "cpu",
        seed: int = 0,
        adamw: AdamWConfig | None = None,
        group: dist.ProcessGroup | None = None,
        logprob_chunk: int = 4096,
        fused_dp: bool = True,
        max_tokens_per_rank: int = 16384,
        tp_size: int = 1,
        cp_size: int = 1,
        etp_size: int = 1,
        allow_unvalidated_arch: bool = False,
        recompute: bool | None = None,
        stream_weights: bool = False,
    ) -> None:
        """``recompute``: full activation recompute per layer (``None``: the
        ``ART_B200_RECOMPUTE`` environment switch).  ``stream_weights``: the
        layers' base weights stay in pinned host memory and are streamed to
        the GPU one layer at a time (implies recompute)."""
        from ..models.registry import check_parallelism, get_model_support

        self.support = get_model_support(cfg, allow_unvalidated_arch)
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.grad_sync = None  # fused data-parallel reducer (parallel/dp.py) on GPUs
        store = None
        if self.world > 1 and self.device.type == "cuda" and fused_dp:
            from ..models.lora import LoRAStore
            from ..models.transformer import lora_specs_for
            from ..parallel.dp import FusedDataParallel

            specs = lora_specs_for(cfg, lora)
            dtype = torch.bfloat16
            self.grad_sync = FusedDataParallel(LoRAStore.numel_for(specs), dtype, group, self.device)
            store = LoRAStore(specs, self.device, dtype, compute_buf=self.grad_sync.compute,
                              grad_buf=self.grad_sync.grad)
            store.init_(seed + 1)
        self.ep = None
        self.tp = None
        self.tp_size = tp_size if self.world > 1 else 1
        self.cp_size = cp_size if self.world > 1 else 1
        if self.tp_size > 1 and self.cp_size > 1:
            raise ValueError("tensor and context parallelism are not combined")
        if self.world % (self.tp_size * self.cp_size) != 0:
            raise ValueError(f"tp={self.tp_size} x cp={self.cp_size} does not divide world={self.world}")
        if self.tp_size > 1:
            from ..parallel.topology import shard_subgroup
            from ..parallel.tp import TPContext

            self.tp = TPContext(shard_subgroup(group, self.tp_size), self.device, max_tokens_per_rank,
                                cfg.hidden_size)
        self.cp = None
        if self.cp_size > 1:
            # context parallelism: every rank of a CP group takes a contiguous
            # slice of the group's packed rows
            from ..parallel.cp import CPContext
            from ..parallel.topology import shard_subgroup

            self.cp = CPContext(shard_subgroup(group, self.cp_size), self.device)
        check_parallelism(self.support, tp=self.tp_size, cp=self.cp_size, etp=etp_size if self.world > 1 else 1)
        self.etp = None
        self.etp_size = etp_size if self.world > 1 else 1
        if self.etp_size > 1 and not cfg.is_moe:
            raise ValueError("expert tensor parallelism applies to MoE models")
        if cfg.is_moe and self.world > 1:
            from ..parallel.ep import EPContext

            ep_group = group
            if self.etp_size > 1:
                # ETP groups of consecutive ranks; the EP group of a rank holds
                # the ranks with the same position in their ETP group
                from ..parallel.etp import ETPContext
                from ..parallel.topology import strided_subgroup

                if self.world % self.etp_size != 0:
                    raise ValueError(f"etp={self.etp_size} does not divide world={self.world}")
                self.etp = ETPContext(group, self.etp_size, self.device)
                ep_group = strided_subgroup(group, self.etp_size)
            if self.world // self.etp_size > 1:
                cap = 2 * max_tokens_per_rank * cfg.num_experts_per_tok * self.etp_size
                self.ep = EPContext(ep_group, cfg.num_experts, cfg.hidden_size, self.device, cap)
        if self.tp is not None:
            from ..models.tp_decoder import TPDecoderLM

            self.model = TPDecoderLM(cfg, lora, self.device, self.tp, seed=seed, store=store)
        elif cfg.family == "gemma4":
            from ..models.gemma4 import Gemma4LM

            self.model = Gemma4LM(cfg, lora, self.device, seed=seed, store=store, ep=self.ep, etp=self.etp)
        else:
            self.model = DecoderLM(cfg, lora, self.device, seed=seed, store=store, ep=self.ep, etp=self.etp)
        if recompute is not None:
            if recompute and not hasattr(self.model, "recompute"):
                raise ValueError(f"activation recompute is not available for {type(self.model).__name__}")
            if hasattr(self.model, "recompute"):
                self.model.recompute = bool(recompute)
        if stream_weights:
            if not hasattr(self.model, "enable_weight_streaming"):
                raise ValueError(f"weight streaming is not available for {type(self.model).__name__}")
            self.model.enable_weight_streaming()
        self.store = self.model.store
        self.optim = FlatAdamW(self.store, adamw)
        self.logprob_chunk = logprob_chunk
        self.ref_flat: torch.Tensor | None = None  # KL reference adapter (compute dtype)

    def prepare_checkpoint(self, moments: bool = True) -> None:
        """Collective: make the full master weights (and, with ``moments``,
        the AdamW moments) current on every rank (with the fused data-parallel
        optimizer each rank updates only its shard).  Every rank must call it
        before rank 0 writes a checkpoint.  With ``moments=False`` the moments
        stay sharded: each rank then writes its own shard
        (:meth:`optimizer_shard`)."""
        if self.grad_sync is not None:
            self.grad_sync.gather_full_state(self.store, moments)

    def optimizer_shard(self) -> tuple[int, int, int, int] | None:
        """``(offset, numel, rank, world)`` of the optimizer-state shard this
        rank owns under the fused data-parallel optimizer (else ``None``)."""
        if self.grad_sync is None:
            return None
        off, n = self.grad_sync.shards[self.grad_sync.rank]
        return off, n, self.grad_sync.rank, self.grad_sync.world

    def offload(self) -> int:
        """Move the model, LoRA store and optimizer state to pinned host
        memory (the GPU is free for other work until :meth:`reload`)."""
        if self.grad_sync is not None or self.tp is not None or self.ep is not None or self.etp is not None:
            raise RuntimeError("offload applies to a single-GPU trainer (peer-mapped buffers stay resident)")
        from .offload import OffloadState

        self._offload = OffloadState(self.model, self.store, self.optim)
        return self._offload.offload()

    def reload(self) -> None:
        st = getattr(self, "_offload", None)
        if st is not None:
            st.reload()
            self._offload = None

    def health_words(self) -> tuple[list[str], list[torch.Tensor]]:
        """The device status words of every bounded wait this trainer's
        kernels use: the peer barriers of the data-, context-, tensor- and
        expert-parallel exchanges and the error word of the tensor-core
        kernels (attention, GEMMs).  Non-zero = a wait gave up."""
        names: list[str] = []
        words: list[torch.Tensor] = []

        def add(name: str, t: Any) -> None:
            if torch.is_tensor(t):
                names.append(name)
                words.append(t)

        if self.grad_sync is not None:
            add("dp_barrier", self.grad_sync.status)
        if self.cp is not None:
            add("cp_barrier", getattr(self.cp, "status", None))
        if self.tp is not None:
            add("tp_barrier", getattr(self.tp, "status", None))
        if self.ep is not None:
            add("ep_barrier", getattr(self.ep.transport, "status", None))
            if getattr(self.ep, "fused", None) is not None:
                add("ep_fused_barrier", self.ep.fused.status)
        if self.etp is not None:
            add("etp_barrier", getattr(self.etp, "status", None))
        if self.device.type == "cuda":
            from ..ops import native

            add("tensor_core_wait", native.lib().tc_error_word())
        return names, words

    def _health(self) -> tuple[torch.Tensor | None, tuple[str, ...]]:
        names, words = self.health_words()
        if not words:
            return None, ()
        return torch.stack([w.reshape(-1)[0].to(torch.int32) for w in words]), tuple(names)

    def check_health(self) -> None:
        """Raise :class:`DeviceWaitTimeout` if any bounded wait gave up (one
        device->host read)."""
        health, names = self._health()
        if health is None:
            return
        vals = health.cpu().tolist()
        bad = [f"{n}={v}" for n, v in zip(names, vals) if v != 0]
        if bad:
            raise DeviceWaitTimeout("a bounded device wait gave up (" + ", ".join(bad) + ")")

    def set_reference_adapter(self, state: Mapping[str, torch.Tensor] | None) -> None:
        """Use a saved adapter (PEFT state dict) as the KL reference; ``None``
        means the frozen base model (adapter disabled)."""
        if state is None:
            self.ref_flat = None
            return
        st = self.store
        flat = torch.zeros_like(st.compute)
        for name, e in st.entries.items():
            if name in state:
                flat[e.offset : e.offset + e.numel].copy_(state[name].reshape(-1).to(flat.dtype))
        self.ref_flat = flat

    def _reference_logprobs(self, mb: "MicroBatch", ctx: dict[str, Any]) -> torch.Tensor:
        st = self.store
        with torch.no_grad():
            if self.ref_flat is None:
                self.model.lora_enabled = False
                try:
                    ref, _ = self._logprobs(mb, dict(ctx), entropy=False)
                finally:
                    self.model.lora_enabled = True
                return ref
            saved = st.compute.clone()
            st.compute.copy_(self.ref_flat)
            st.version += 1
            try:
                ref, _ = self._logprobs(mb, dict(ctx), entropy=False)
            finally:
                st.compute.copy_(saved)
                st.version += 1
            return ref

    # ------------------------------------------------------------------
    def _logprobs(self, mb: MicroBatch, ctx: dict[str, Any], entropy: bool) -> tuple[torch.Tensor, torch.Tensor | None]:
        if self.tp is not None:
            return self.model.token_logprobs(mb.tokens, mb.meta, mb.sel, mb.targets, ctx, entropy)
        h = self.model.forward(mb.tokens, mb.meta, ctx)
        hs = h.index_select(0, mb.sel)
        own = getattr(self.model, "token_logprobs_hidden", None)  # families with their own logits (soft-capping)
        if own is not None:
            return own(hs, mb.targets, self.logprob_chunk, entropy)
        return fused.lm_head_logprobs(hs, self.model.lm_head, mb.targets, self.logprob_chunk, entropy)

    def micro_step(
        self, mb: MicroBatch, cfg: Mapping[str, Any], total_tokens: float
    ) -> dict[str, torch.Tensor]:
        """Forward + backward of one packed row; gradients accumulate into the
        store.  Returns device scalars (loss contribution, entropy sum, ...)."""
        ctx: dict[str, Any] = {"group_ids": mb.group_ids, "parent_ids": mb.parent_ids}
        if mb.cp_plan is not None:
            ctx["cp_plan"], ctx["cp"] = mb.cp_plan, self.cp
        if mb.routes is not None:
            ctx["replay_routes"] = mb.routes
            if mb.route_counts is not None:
                ctx["replay_counts"] = mb.route_counts
            if mb.ep_counts is not None:
                ctx["ep_counts"] = mb.ep_counts
        ref = None
        kl_coef = float(cfg.get("kl_penalty_coef", 0.0) or 0.0)
        if kl_coef > 0:
            ref = self._reference_logprobs(mb, ctx)
        lp, ent = self._logprobs(mb, ctx, entropy=True)
        n = lp.numel()
        level = cfg.get("importance_sampling_level", "token")
        if self.device.type == "cuda" and level == "token":
            cfg_t = torch.tensor(fused.grpo_loss_config(dict(cfg), n, total_tokens), dtype=torch.float32)
            cfg_t = cfg_t.to(self.device, non_blocking=True)
            ones = torch.ones(n, device=self.device, dtype=torch.float32)
            loss, stats = fused.grpo_token_loss(lp, mb.old, mb.adv, mb.w, ones, ref, mb.original, cfg_t)
            kl = stats[2]
        else:
            inputs = AlignedLossInputs(
                assistant_mask=torch.ones(1, n, dtype=torch.bool, device=self.device),
                old_logprobs=mb.old.view(1, n),
                advantages=mb.adv.view(1, n),
                weights=mb.w.view(1, n),
                group_ids=mb.group.view(1, n),
                original_logprobs=None if mb.original is None else mb.original.view(1, n),
                entropies_are_aligned=True,
            )
            out = loss_fn(inputs, lp.view(1, n), None if ref is None else ref.view(1, n), None, cfg, reduction="sum")
            loss = out.policy_loss / total_tokens
            kl = out.kl_policy_ref if out.kl_policy_ref is not None else lp.new_zeros(())
        loss.backward()
        ent_sum = (ent * mb.w).sum() / total_tokens if ent is not None else lp.new_zeros(())
        return {
            "loss": loss.detach(),
            "entropy": ent_sum.detach(),
            "probs_corr": _probs_corr_device(mb.old, lp),
            "kl": kl.detach() if torch.is_tensor(kl) else lp.new_tensor(float(kl)),
        }

    def rows_needed(self, n_rows: int) -> set[int]:
        """Rows of a step of ``n_rows`` packed rows that this rank stages
        (:meth:`stage`): a packer may materialize only these."""
        shard = self.tp_size * self.cp_size
        dp_world = self.world // shard
        dp_rank = self.rank // shard
        rows = set(range(n_rows)[dp_rank::dp_world])
        if (self.ep is not None or self.etp is not None) and n_rows:
            rows.add(dp_rank % n_rows)  # the zero-weight copy of a short rank
        return rows

    def stage(self, packed: Mapping[str, Any]) -> list[MicroBatch]:
        """Stage this rank's rows of ``packed`` on the device.

        Rows are interleaved over the data-parallel groups; the ranks of one
        tensor- or context-parallel group stage the same rows (TP: whole
        rows, CP: each its slice).  With expert parallelism every rank runs
        the same number of micro steps (the expert exchange is collective),
        so short ranks get zero-weight copies.
        """
        n_rows = int(packed["tokens"].shape[0])
        shard = self.tp_size * self.cp_size  # ranks that split one row
        dp_world = self.world // shard
        dp_rank = self.rank // shard
        pad_to = 128 * shard if shard > 1 else 64
        if self.etp is not None:
            # the ETP all-gather wants equal token counts on every member: rows
            # keep their full packed length
            pad_to = max(int(packed["tokens"].shape[1]), 1)
        if shard > 1 and int(packed["tokens"].shape[1]) % pad_to:
            # rows split over ranks need a length the split divides evenly
            packed = pad_packed_length(packed, pad_to)
        cfgm = self.model.cfg
        linear = any(cfgm.layer_kind(i) != "attention" for i in range(cfgm.num_hidden_layers))

        def one(r: int) -> MicroBatch:
            return stage_row(packed, r, self.device, pad_to=pad_to, cp=self.cp,
                             conv_width=cfgm.linear_conv_kernel_dim, linear_layers=linear)

        mbs = [one(r) for r in list(range(n_rows))[dp_rank::dp_world]]
        if self.ep is not None or self.etp is not None:
            per_rank = (n_rows + dp_world - 1) // dp_world
            while len(mbs) < per_rank:
                mbs.append(zero_weight(one(dp_rank % n_rows)))
        return mbs

    def train_step(
        self,
        packed: Mapping[str, Any],
        learning_rate: float,
        cfg: Mapping[str, Any] | None = None,
        micro_batches: list[MicroBatch] | None = None,
    ) -> StepMetrics:
        """One optimizer step over every row of ``packed`` (CPU tensors).

        ``micro_batches`` may carry rows already staged on the device (this
        rank's rows, in order); the step then performs no host→device copy.
        """
        cfg = dict(cfg or {})
        mask = packed["assistant_mask"]
        # trainable (scored) tokens of the whole step (a packer that filled
        # only this rank's rows states the step's count itself)
        total = float(packed["trainable_tokens"]) if "trainable_tokens" in packed else float(mask[:, 1:].sum().item())
        if micro_batches is None:
            micro_batches = self.stage(packed)
        if mutation.active("dp_local_token_normalization"):
            total = float(sum(int(mb.sel.numel()) for mb in micro_batches))
        self._attach_ep_counts(micro_batches)
        acc = {k: torch.zeros((), device=self.device) for k in ("loss", "entropy", "probs_corr", "kl")}
        n_tokens = 0
        for mb in micro_batches:
            out = self.micro_step(mb, cfg, max(total, 1.0))
            for k in acc:
                acc[k] += out[k]
            n_tokens += mb.n_tokens
        nmb = max(len(micro_batches), 1)
        acc["probs_corr"] /= nmb
        acc["kl"] /= nmb
        packed_tokens: int | torch.Tensor = n_tokens
        if self.world > 1:
            # tensor-parallel ranks hold identical copies of the loss statistics
            # (and of the packed tokens of their row)
            rep = float(self.tp_size)
            stats = torch.stack([acc["loss"] / rep, acc["entropy"] / rep, acc["probs_corr"] / self.world,
                                 acc["kl"] / self.world, acc["loss"].new_tensor(n_tokens / rep)])
            if self.grad_sync is not None:
                self.grad_sync.reduce_and_step(self.optim, learning_rate, stats)
            else:
                if not mutation.active("dp_skip_grad_reduce"):
                    dist.all_reduce(self.store.grad, group=self.group)
                dist.all_reduce(stats, group=self.group)
                self.optim.step(learning_rate)
            acc["loss"], acc["entropy"], acc["probs_corr"], acc["kl"], packed_tokens = stats.unbind(0)
        else:
            self.optim.step(learning_rate)
        health, names = self._health()
        # step_trainer_tokens and step_packed_tokens both count the whole step
        # (every rank's rows)
        return StepMetrics(
            loss=acc["loss"], entropy=acc["entropy"], probs_corr=acc["probs_corr"], kl=acc["kl"],
            grad_norm=self.optim.grad_norm, n_train=int(total), n_tokens=packed_tokens,
            health=health, health_names=names,
        )

    def _attach_ep_counts(self, micro_batches: list[MicroBatch]) -> None:
        """With replayed routes, give every micro batch the per-layer slot
        counts of every expert-parallel rank (one host all-gather per step;
        the fused exchange then plans each MoE layer without a device sync)."""
        ep = self.ep
        if ep is None or getattr(ep, "fused", None) is None or self.etp is not None:
            return
        if not micro_batches or any(mb.route_counts is None for mb in micro_batches):
            return
        if all(mb.ep_counts is not None for mb in micro_batches):
            return
        E = self.model.cfg.num_experts
        mine = []
        for mb in micro_batches:
            per_layer = np.zeros((len(mb.route_counts), E), dtype=np.int64)
            for j, c in enumerate(mb.route_counts):
                per_layer[j, : len(c)] = c
            mine.append(per_layer)
        gathered: list = [None] * ep.world
        dist.all_gather_object(gathered, mine, group=ep.group)
        for m, mb in enumerate(micro_batches):
            mb.ep_counts = [np.stack([gathered[q][m][j] for q in range(ep.world)])
                            for j in range(len(mb.route_counts))]

    def train_steps(
        self,
        packed: Mapping[str, Any],
        learning_rate: float,
        cfg: Mapping[str, Any] | None = None,
        grad_accumulation_sequences: int | None = None,
    ) -> list[StepMetrics]:
        """Optimizer steps over ``packed``: one over every row when
        ``grad_accumulation_sequences`` is ``None``, else one per consecutive
        block of that many rows (reference ``megatron/training/microbatches.py:
        115-170``: ``ceil(rows / sequences)`` gradient steps, each normalised by
        its own trainable tokens; its blocks are spread over the data-parallel
        ranks like a whole call)."""
        from ..preprocessing.pack import select_rows

        n = int(packed["tokens"].shape[0])
        g = grad_accumulation_sequences
        if g is None or g >= n:
            return [self.train_step(packed, learning_rate, cfg)]
        return [self.train_step(select_rows(packed, list(range(a, min(n, a + g)))), learning_rate, cfg)
                for a in range(0, n, g)]

    # ------------------------------------------------------------------
    def sft_step(self, batch: list[tuple[list[int], list[int]]], learning_rate: float) -> dict[str, float]:
        """One supervised step: mean negative log-likelihood of the label
        tokens (``-100`` = ignored) over the whole batch, then AdamW."""
        rows = batch[self.rank :: self.world]
        total = sum(sum(1 for v in labels[1:] if v != -100) for _, labels in batch)
        total = max(total, 1)
        acc = torch.zeros((), device=self.device)
        for ids, labels in rows:
            L = len(ids)
            lab = torch.tensor(labels, dtype=torch.long)
            sel = (lab[1:] != -100).nonzero().squeeze(1)
            kend = torch.full((L,), L, dtype=torch.int32)
            meta = AttnMeta.build(torch.arange(L), kend, self.device)
            toks = torch.tensor(ids, dtype=torch.long).to(self.device)
            h = self.model.forward(toks, meta, {})
            hs = h.index_select(0, sel.to(self.device))
            lp, _ = fused.lm_head_logprobs(hs, self.model.lm_head, lab[1:][sel].to(self.device), self.logprob_chunk, False)
            loss = -lp.sum() / total
            loss.backward()
            acc += loss.detach()
        if self.grad_sync is not None:
            # the fused data-parallel step: every rank updates its own shard
            # of the master weights and moments (a full local step would start
            # from the other shards' stale copies)
            stats = acc.reshape(1)
            self.grad_sync.reduce_and_step(self.optim, learning_rate, stats)
            acc = stats[0]
        elif self.world > 1:
            dist.all_reduce(self.store.grad, group=self.group)
            dist.all_reduce(acc, group=self.group)
            self.optim.step(learning_rate)
        else:
            self.optim.step(learning_rate)
        health, names = self._health()
        parts = [acc.reshape(()), self.optim.grad_norm.reshape(())]
        if health is not None:
            parts.extend(health.float().unbind(0))
        vals = torch.stack([p.float() for p in parts]).cpu().tolist()
        bad = [f"{n}={int(v)}" for n, v in zip(names, vals[2:]) if v != 0]
        if bad:
            raise DeviceWaitTimeout("a bounded device wait gave up during the SFT step (" + ", ".join(bad) + ")")
        return {"loss/train": vals[0], "loss/grad_norm": vals[1], "data/step_trainer_tokens": float(total)}
