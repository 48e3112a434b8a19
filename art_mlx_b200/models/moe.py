"""Mixture-of-experts FFN (Qwen3-MoE style) with per-expert LoRA and
routing replay.

Routing: ``softmax(h W_router^T)`` over experts, top-k, renormalised when
``norm_topk_prob``.  With routing replay (reference
``src/art/megatron/routing_replay.py:696-1084``) the top-k expert ids come
from the rollout engine's record for each token and layer; the weights are
still the current router's probabilities at those ids, so the router's
computation graph matches the sampled policy.

Expert compute is a grouped GEMM over tokens sorted by expert.  The LoRA
factors of all experts of a layer are stacked views ``[E, ...]`` into the
flat store, so the adapter update is itself two grouped GEMMs.
"""

from __future__ import annotations

from typing import Any, Callable

import torch

from .config import LoRASpec, ModelConfig
from ..ops.fused import grad_anchor
from .lora import LoRAStore, peft_key


def moe_lora_specs(cfg: ModelConfig, i: int, spec: LoRASpec) -> list[tuple[str, tuple[int, ...], str]]:
    r, H, F, E = spec.r, cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts
    t = set(spec.expert_targets) & set(spec.target_modules)
    out: list[tuple[str, tuple[int, ...], str]] = []
    if {"gate_proj", "up_proj"} <= t:
        for e in range(E):
            for p in ("gate_proj", "up_proj"):
                out.append((peft_key(i, "mlp", p, "A", e), (r, H), "A"))
        for e in range(E):
            for p in ("gate_proj", "up_proj"):
                out.append((peft_key(i, "mlp", p, "B", e), (F, r), "B"))
    if "down_proj" in t:
        for e in range(E):
            out.append((peft_key(i, "mlp", "down_proj", "A", e), (r, F), "A"))
        for e in range(E):
            out.append((peft_key(i, "mlp", "down_proj", "B", e), (H, r), "B"))
    return out


def grouped_mm(x: torch.Tensor, w: torch.Tensor, counts: list[int]) -> torch.Tensor:
    """Rows of ``x`` [N, K] are grouped by expert (``counts``); returns
    ``[N, M]`` with group ``e`` multiplied by ``w[e]`` ([E, K, M])."""
    outs = []
    s = 0
    for e, c in enumerate(counts):
        if c:
            outs.append(x[s : s + c] @ w[e])
        s += c
    if not outs:
        return x.new_zeros(0, w.shape[-1])
    return torch.cat(outs)


def grouped_wgrad(a: torch.Tensor, b: torch.Tensor, counts: list[int], out: torch.Tensor, alpha: float) -> None:
    """``out[e] += alpha * a_e^T b_e`` (fp32 accumulate) for row groups ``e``."""
    s = 0
    for e, c in enumerate(counts):
        if c:
            ae, be = a[s : s + c], b[s : s + c]
            if out.device.type == "cuda" and ae.dtype != torch.float32:
                torch.addmm(out[e], ae.t(), be, beta=1.0, alpha=alpha, out_dtype=torch.float32, out=out[e])
            else:
                out[e].addmm_(ae.t().float(), be.float(), alpha=alpha)
        s += c


class _ExpertsFn(torch.autograd.Function):
    """Grouped SwiGLU experts with LoRA on gate/up and down."""

    @staticmethod
    def forward(ctx, xs, counts, gu_w_t, down_w_t, A_gu, B_gu, A_d, B_d, g_A_gu, g_B_gu, g_A_d, g_B_d, scale, enabled, anchor):
        # xs [N, H] sorted by expert; gu_w_t [E, H, 2F]; down_w_t [E, F, H]
        gu = grouped_mm(xs, gu_w_t, counts)
        u_gu = None
        if enabled and A_gu is not None:
            u_gu = grouped_mm(xs, A_gu.transpose(1, 2), counts)  # [N, 2r]
            E, _, F, r = B_gu.shape
            r2 = 2 * r
            # block-diagonal per expert: gate rows use u[:, :r], up rows u[:, r:]
            lo = grouped_mm(u_gu[:, :r].contiguous(), B_gu[:, 0].transpose(1, 2), counts)
            hi = grouped_mm(u_gu[:, r:r2].contiguous(), B_gu[:, 1].transpose(1, 2), counts)
            gu = gu + scale * torch.cat([lo, hi], dim=1)
        Fh = gu.shape[1] // 2
        g, up = gu[:, :Fh], gu[:, Fh:]
        sg = torch.sigmoid(g.float())
        act = (g.float() * sg).to(gu.dtype) * up
        out = grouped_mm(act, down_w_t, counts)
        u_d = None
        if enabled and A_d is not None:
            u_d = grouped_mm(act, A_d.transpose(1, 2), counts)  # [N, r]
            out = out + scale * grouped_mm(u_d, B_d.transpose(1, 2), counts)
        ctx.save_for_backward(xs, gu, act, u_gu if u_gu is not None else xs.new_empty(0), u_d if u_d is not None else xs.new_empty(0))
        ctx.counts = counts
        ctx.w = (gu_w_t, down_w_t, A_gu, B_gu, A_d, B_d)
        ctx.g = (g_A_gu, g_B_gu, g_A_d, g_B_d)
        ctx.scale = scale
        ctx.enabled = enabled
        return out

    @staticmethod
    def backward(ctx, dout):
        xs, gu, act, u_gu, u_d = ctx.saved_tensors
        counts, s = ctx.counts, ctx.scale
        gu_w_t, down_w_t, A_gu, B_gu, A_d, B_d = ctx.w
        g_A_gu, g_B_gu, g_A_d, g_B_d = ctx.g
        dout = dout.contiguous()
        dact = grouped_mm(dout, down_w_t.transpose(1, 2), counts)
        if ctx.enabled and A_d is not None:
            dyB = grouped_mm(dout, B_d, counts)  # [N, r]
            grouped_wgrad(dout, u_d, counts, g_B_d, s)  # [E, H, r]
            grouped_wgrad(dyB, act, counts, g_A_d, s)  # [E, r, F]
            dact = dact + s * grouped_mm(dyB, A_d, counts)
        Fh = gu.shape[1] // 2
        g, up = gu[:, :Fh].float(), gu[:, Fh:].float()
        sg = torch.sigmoid(g)
        da = dact.float()
        dup = da * g * sg
        dg = da * up * sg * (1 + g * (1 - sg))
        dgu = torch.cat([dg, dup], dim=1).to(gu.dtype)
        dxs = grouped_mm(dgu, gu_w_t.transpose(1, 2), counts)
        if ctx.enabled and A_gu is not None:
            r = B_gu.shape[-1]
            dyB_lo = grouped_mm(dgu[:, :Fh].contiguous(), B_gu[:, 0], counts)
            dyB_hi = grouped_mm(dgu[:, Fh:].contiguous(), B_gu[:, 1], counts)
            grouped_wgrad(dgu[:, :Fh], u_gu[:, :r], counts, g_B_gu[:, 0], s)
            grouped_wgrad(dgu[:, Fh:], u_gu[:, r:], counts, g_B_gu[:, 1], s)
            dyB = torch.cat([dyB_lo, dyB_hi], dim=1)
            grouped_wgrad(dyB, xs, counts, g_A_gu, s)
            dxs = dxs + s * grouped_mm(dyB, A_gu, counts)
        return (dxs,) + (None,) * 14


class MoEBlock:
    def __init__(self, cfg: ModelConfig, i: int, gen, dev, dt, store: LoRAStore, spec: LoRASpec) -> None:
        from .transformer import _randn

        self.cfg, self.index = cfg, i
        E, H, F = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
        self.router_w = _randn((E, H), gen, dev, dt)
        # stored transposed for row-major grouped GEMMs: x [N,H] @ [H, 2F]
        self.gu_w_t = _randn((E, H, 2 * F), gen, dev, dt)
        self.down_w_t = _randn((E, F, H), gen, dev, dt)
        self.shared = None
        if cfg.shared_expert_intermediate_size:
            Fs = cfg.shared_expert_intermediate_size
            self.shared = (
                _randn((2 * Fs, H), gen, dev, dt),
                _randn((H, Fs), gen, dev, dt),
                _randn((1, H), gen, dev, dt),
            )
        self.scale = spec.scale
        r = spec.r

        def stacked(names: list[str], shape: tuple[int, ...]):
            if not names or names[0] not in store.entries:
                return None, None
            off, n = store.contiguous_span(names)
            return (
                store.compute[off : off + n].view(shape),
                store.grad[off : off + n].view(shape),
            )

        self.A_gu, self.g_A_gu = stacked(
            [peft_key(i, "mlp", p, "A", e) for e in range(E) for p in ("gate_proj", "up_proj")], (E, 2 * r, H)
        )
        self.B_gu, self.g_B_gu = stacked(
            [peft_key(i, "mlp", p, "B", e) for e in range(E) for p in ("gate_proj", "up_proj")], (E, 2, F, r)
        )
        self.A_d, self.g_A_d = stacked([peft_key(i, "mlp", "down_proj", "A", e) for e in range(E)], (E, r, F))
        self.B_d, self.g_B_d = stacked([peft_key(i, "mlp", "down_proj", "B", e) for e in range(E)], (E, H, r))

    def num_parameters(self) -> int:
        n = self.router_w.numel() + self.gu_w_t.numel() + self.down_w_t.numel()
        if self.shared is not None:
            n += sum(t.numel() for t in self.shared)
        return n

    def route(self, h: torch.Tensor, ctx: dict[str, Any]) -> tuple[torch.Tensor, torch.Tensor]:
        cfg = self.cfg
        logits = (h @ self.router_w.t()).float()
        probs = torch.softmax(logits, dim=-1)
        replay = ctx.get("replay_routes")  # [T, L, k] int
        if replay is not None:
            idx = replay[:, self.index].long()
            wts = probs.gather(1, idx)
        else:
            wts, idx = probs.topk(cfg.num_experts_per_tok, dim=-1)
        if cfg.norm_topk_prob:
            wts = wts / wts.sum(-1, keepdim=True)
        rec = ctx.get("record_routes")
        if rec is not None:
            rec[self.index] = idx.detach().to(torch.int32)
        return idx, wts

    def __call__(self, h: torch.Tensor, version: int, enabled: bool, ctx: dict[str, Any]) -> torch.Tensor:
        T, H = h.shape
        E, k = self.cfg.num_experts, self.cfg.num_experts_per_tok
        idx, wts = self.route(h, ctx)
        flat = idx.reshape(-1)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=E).tolist()
        tok = order // k
        xs = h[tok]
        ys = _ExpertsFn.apply(
            xs, counts, self.gu_w_t, self.down_w_t, self.A_gu, self.B_gu, self.A_d, self.B_d,
            self.g_A_gu, self.g_B_gu, self.g_A_d, self.g_B_d, self.scale, enabled,
            grad_anchor(h.device) if enabled else None,
        )
        w_sorted = wts.reshape(-1)[order].to(ys.dtype).unsqueeze(1)
        out = torch.zeros(T, H, device=h.device, dtype=ys.dtype).index_add(0, tok, ys * w_sorted)
        if self.shared is not None:
            gu_w, down_w, gate_w = self.shared
            gu = h @ gu_w.t()
            Fs = gu.shape[1] // 2
            sh = (torch.nn.functional.silu(gu[:, :Fs]) * gu[:, Fs:]) @ down_w.t()
            out = out + torch.sigmoid(h @ gate_w.t()) * sh
        return out

    def load_hf(self, sd: dict[str, torch.Tensor], prefix: str, g: Callable[[str], torch.Tensor]) -> None:
        self.router_w.copy_(g(prefix + "gate.weight"))
        for e in range(self.cfg.num_experts):
            p = f"{prefix}experts.{e}."
            self.gu_w_t[e].copy_(torch.cat([g(p + "gate_proj.weight"), g(p + "up_proj.weight")]).t())
            self.down_w_t[e].copy_(g(p + "down_proj.weight").t())
