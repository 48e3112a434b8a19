"""Mixture-of-experts FFN (Qwen3-MoE style) with per-expert LoRA, routing
replay and expert parallelism.

Routing: ``softmax(h W_router^T)`` over experts, top-k, renormalised when
``norm_topk_prob``.  With routing replay (reference
``src/art/megatron/routing_replay.py:696-1084``) the top-k expert ids come
from the rollout engine's record for each token and layer; the weights are
still the current router's probabilities at those ids, so gradients reach the
router exactly as for the sampled policy.

Experts run as grouped GEMMs over tokens laid out expert-contiguous.  The
LoRA factors of all experts of a layer are stacked ``[E, ...]`` views into the
flat store, so the adapter is itself grouped GEMMs (rank-r).  Under expert
parallelism (:mod:`art_mlx_b200.parallel.ep`) a rank holds the base weights
of its ``E / world`` experts; the LoRA store keeps every expert (non-local
experts simply receive zero gradient on this rank), which lets the
data-parallel optimizer reduce expert and shared parameters alike.
"""

from __future__ import annotations

from typing import Any, Callable

import torch

from ..ops.fused import grad_anchor
from .config import LoRASpec, ModelConfig
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


# ---------------------------------------------------------------------------
# grouped GEMM helpers
# ---------------------------------------------------------------------------


def _h2d(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    """Host -> device without a stream sync: a copy from pageable memory waits
    for the stream to drain first, one from pinned memory is queued like a
    kernel (the grouped GEMMs call this for every expert layout)."""
    if device.type == "cuda":
        return t.pin_memory().to(device, non_blocking=True)
    return t.to(device)


def _offsets(counts: list[int], device: torch.device) -> torch.Tensor:
    return _h2d(torch.tensor(counts, dtype=torch.int64).cumsum(0).to(torch.int32), device)


def _use_library_grouped(x: torch.Tensor, k: int, m: int) -> bool:
    return (
        x.device.type == "cuda" and x.dtype == torch.bfloat16 and hasattr(torch, "_grouped_mm")
        and k % 8 == 0 and m % 8 == 0
    )


def grouped_mm(x: torch.Tensor, w: torch.Tensor, counts: list[int]) -> torch.Tensor:
    """Rows of ``x`` [N, K] grouped by expert (``counts``) times ``w[e]``
    ([E, K, M]) -> [N, M].  On GPUs this is one grouped GEMM launch."""
    if _use_library_grouped(x, x.shape[1], w.shape[-1]):
        if x.shape[0] == 0:
            return x.new_zeros(0, w.shape[-1])
        return torch._grouped_mm(x.contiguous(), w, offs=_offsets(counts, x.device))
    outs = []
    s = 0
    for e, c in enumerate(counts):
        if c:
            outs.append(x[s : s + c] @ w[e])
        s += c
    if not outs:
        return x.new_zeros(0, w.shape[-1])
    return torch.cat(outs)


def pad_groups(x: torch.Tensor, counts: list[int], multiple: int = 8) -> tuple[torch.Tensor, list[int]]:
    """Copy row groups into a buffer where every group starts at a multiple of
    ``multiple`` rows (zero rows in between); returns (padded, padded counts)."""
    padded_counts = [(c + multiple - 1) // multiple * multiple for c in counts]
    if padded_counts == list(counts):
        return x, list(counts)
    dst = torch.empty(x.shape[0], dtype=torch.int64)
    s = d = 0
    for c, pc in zip(counts, padded_counts):
        dst[s : s + c] = torch.arange(d, d + c)
        s += c
        d += pc
    out = x.new_zeros(d, *x.shape[1:])
    out.index_copy_(0, _h2d(dst, x.device), x)
    return out, padded_counts


def grouped_wgrad(a: torch.Tensor, b: torch.Tensor, counts: list[int], out: torch.Tensor, alpha: float) -> None:
    """``out[e] += alpha * a_e^T b_e`` (fp32 accumulate) for row groups ``e``."""
    if _use_library_grouped(a, a.shape[1], b.shape[1]) and a.shape[0] > 0:
        # the reduced (token) dimension of each group must span a multiple of
        # 16 bytes: align every group to 8 rows with zero padding
        ap, pc = pad_groups(a, counts)
        bp, _ = pad_groups(b, counts)
        # one launch for all experts; the per-expert product is rounded to
        # bf16 once (fp32 accumulation inside the GEMM) before the fp32 add
        g = torch._grouped_mm(ap.t().contiguous(), bp.contiguous(), offs=_offsets(pc, a.device))
        out.add_(g.view(out.shape).float(), alpha=alpha)
        return
    s = 0
    for e, c in enumerate(counts):
        if c:
            ae, be = a[s : s + c], b[s : s + c]
            if out.device.type == "cuda" and ae.dtype != torch.float32:
                torch.addmm(out[e], ae.t(), be, beta=1.0, alpha=alpha, out_dtype=torch.float32, out=out[e])
            else:
                out[e].addmm_(ae.t().to(out.dtype), be.to(out.dtype), alpha=alpha)
        s += c


class ExpertParams:
    """Base weights of the experts held by this rank plus their LoRA views."""

    def __init__(self, gu_w_t, down_w_t, A_gu, B_gu, A_d, B_d, g_A_gu, g_B_gu, g_A_d, g_B_d, scale):
        self.gu_w_t, self.down_w_t = gu_w_t, down_w_t  # [E_l, H, 2F], [E_l, F, H]
        self.A_gu, self.B_gu, self.A_d, self.B_d = A_gu, B_gu, A_d, B_d
        self.g_A_gu, self.g_B_gu, self.g_A_d, self.g_B_d = g_A_gu, g_B_gu, g_A_d, g_B_d
        self.scale = scale
        # every expert's A of gate/up and B of down (origin-side rank rows of
        # the fused expert-parallel exchange; None without expert parallelism)
        self.A_all_gu = None
        self.B_all_d = None
        # GPT-OSS experts: frozen biases ([E_l, 2F] of [gate | up], [E_l, H])
        # and the clamped GLU instead of SwiGLU
        self.gu_b = None
        self.down_b = None
        self.act = "swiglu"
        self.alpha, self.limit = 1.702, 7.0

    def for_compute(self) -> "ExpertParams":
        """Contiguous copies of the factors the products read (slices under
        expert tensor parallelism are strided views of the flat store); the
        gradient views stay the store's."""
        facs = (self.A_gu, self.B_gu, self.A_d, self.B_d)
        if all(t is None or t.is_contiguous() for t in facs):
            return self
        c = lambda t: None if t is None else t.contiguous()  # noqa: E731
        out = ExpertParams(self.gu_w_t, self.down_w_t, c(self.A_gu), c(self.B_gu), c(self.A_d), c(self.B_d),
                           self.g_A_gu, self.g_B_gu, self.g_A_d, self.g_B_d, self.scale)
        out.A_all_gu, out.B_all_d = self.A_all_gu, self.B_all_d
        out.gu_b, out.down_b, out.act, out.alpha, out.limit = self.gu_b, self.down_b, self.act, self.alpha, self.limit
        return out

    @property
    def plain(self) -> bool:
        """SwiGLU experts without biases (what the expert-parallel paths run)."""
        return self.act == "swiglu" and self.gu_b is None and self.down_b is None


def _row_bias(b: torch.Tensor | None, counts: list[int], like: torch.Tensor) -> torch.Tensor | None:
    """Per-row bias of expert-sorted rows: ``b[e]`` for the rows of expert e."""
    if b is None:
        return None
    idx = torch.repeat_interleave(torch.arange(len(counts), device=like.device),
                                  torch.tensor(counts, device=like.device))
    return b[idx].to(like.dtype)


def _act_fwd(gu: torch.Tensor, p: "ExpertParams") -> torch.Tensor:
    """Expert activation over the [gate | up] halves of ``gu``."""
    Fh = gu.shape[1] // 2
    if gu.device.type == "cuda" and gu.dtype == torch.bfloat16:
        from ..ops import native

        C = native.lib()
        if p.act == "clamped_glu":
            return C.glu_clamp_fwd(gu.contiguous(), p.alpha, p.limit)
        return C.swiglu_fwd(gu.contiguous())
    g, up = gu[:, :Fh].float(), gu[:, Fh:].float()
    if p.act == "clamped_glu":
        g = g.clamp(max=p.limit)
        up = up.clamp(-p.limit, p.limit)
        return ((up + 1) * g * torch.sigmoid(g * p.alpha)).to(gu.dtype)
    return (g * torch.sigmoid(g)).to(gu.dtype) * gu[:, Fh:]


def _act_bwd(dact: torch.Tensor, gu: torch.Tensor, p: "ExpertParams") -> torch.Tensor:
    Fh = gu.shape[1] // 2
    if gu.device.type == "cuda" and gu.dtype == torch.bfloat16:
        from ..ops import native

        C = native.lib()
        if p.act == "clamped_glu":
            return C.glu_clamp_bwd(dact.contiguous(), gu.contiguous(), p.alpha, p.limit)
        return C.swiglu_bwd(dact.contiguous(), gu)
    g, up = gu[:, :Fh].float(), gu[:, Fh:].float()
    da = dact.float()
    if p.act == "clamped_glu":
        gc = g.clamp(max=p.limit)
        uc = up.clamp(-p.limit, p.limit)
        sg = torch.sigmoid(gc * p.alpha)
        du = torch.where((up >= -p.limit) & (up <= p.limit), da * gc * sg, torch.zeros_like(da))
        dg = torch.where(g <= p.limit, da * (uc + 1) * (sg + p.alpha * gc * sg * (1 - sg)), torch.zeros_like(da))
        return torch.cat([dg, du], dim=1).to(gu.dtype)
    sg = torch.sigmoid(g)
    return torch.cat([da * up * sg * (1 + g * (1 - sg)), da * g * sg], dim=1).to(gu.dtype)


def _tc_grouped(x: torch.Tensor, p: ExpertParams) -> bool:
    """Whether the experts run on the tcgen05 grouped GEMM (base product and
    LoRA in one kernel, ops/csrc/gemm_tc.cu ``gemm_tc_grouped``)."""
    if x.device.type != "cuda" or x.dtype != torch.bfloat16 or x.shape[0] == 0:
        return False
    H, F2 = p.gu_w_t.shape[1], p.gu_w_t.shape[2]
    return H % 64 == 0 and F2 % 128 == 0 and p.gu_w_t.is_contiguous() and p.down_w_t.is_contiguous()


def _offs(counts: list[int]) -> list[int]:
    out = [0]
    for c in counts:
        out.append(out[-1] + int(c))
    return out


def _lr_rows(x: torch.Tensor, W: torch.Tensor, counts: list[int], transposed: bool = False,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-expert rank-side product ``x_e @ W_e^T`` with ``W`` [E, R, K]
    (``transposed``: ``x_e @ W_e`` with ``W`` [E, K, R]) on the low-rank
    kernels (no library grouped GEMM)."""
    from ..ops import lowrank

    if transposed:
        E, K, R = W.shape
        st = (W.stride(0), W.stride(2), W.stride(1))
    else:
        E, R, K = W.shape
        st = (W.stride(0), W.stride(1), W.stride(2))
    return lowrank.rows(x, W, st, R, K, counts=counts, out=out)


def _lr_wgrad(P: torch.Tensor, Q: torch.Tensor, G: torch.Tensor, counts: list[int], alpha: float,
              transposed: bool = False) -> None:
    """Per-expert ``G_e += alpha P_e^T Q_e`` with ``G`` [E, R, C] fp32
    (``transposed``: ``G`` [E, C, R] receives ``alpha Q_e^T P_e``)."""
    from ..ops import lowrank

    if transposed:
        E, C, R = G.shape
        st = (G.stride(0), G.stride(2), G.stride(1))
    else:
        E, R, C = G.shape
        st = (G.stride(0), G.stride(1), G.stride(2))
    lowrank.wgrad(P, Q, G, st, R, C, alpha, counts=counts)


def _experts_forward_tc(xs, counts, p: ExpertParams, lora: bool):
    """Gate/up and down as grouped tcgen05 GEMMs with the LoRA products as a
    K-extension of each (x A^T is the small library grouped GEMM)."""
    from ..ops import native

    C = native.lib()
    s = p.scale
    E, H, F2 = p.gu_w_t.shape
    Fh = F2 // 2
    offs = _offs(counts)
    a2 = b2 = u_gu = u_d = None
    if lora and p.A_gu is not None:
        r = p.B_gu.shape[-1]
        u_gu = _lr_rows(xs, p.A_gu, counts)  # [N, 2r]
        bd = xs.new_zeros(E, F2, 2 * r)  # per expert: block-diagonal s*[B_gate, B_up]
        bd[:, :Fh, :r] = s * p.B_gu[:, 0]
        bd[:, Fh:, r:] = s * p.B_gu[:, 1]
        a2, b2 = u_gu.contiguous(), bd.view(E * F2, 2 * r)
    gu = C.gemm_tc_grouped(xs.contiguous(), p.gu_w_t.view(E * H, F2), offs, F2, a2, b2, True)
    if p.gu_b is not None:
        gu.add_(_row_bias(p.gu_b, counts, gu))
    act = _act_fwd(gu, p)  # fused activation over the [gate | up] halves
    a2 = b2 = None
    if lora and p.A_d is not None:
        u_d = _lr_rows(act, p.A_d, counts)  # [N, r]
        a2, b2 = u_d, (s * p.B_d).reshape(E * H, -1).contiguous()
    out = C.gemm_tc_grouped(act, p.down_w_t.view(E * Fh, H), offs, H, a2, b2, True)
    if p.down_b is not None:
        out.add_(_row_bias(p.down_b, counts, out))
    return out, (xs, gu, act, u_gu, u_d, counts, lora)


def experts_forward(xs: torch.Tensor, counts: list[int], p: ExpertParams, lora: bool):
    """Grouped SwiGLU experts with LoRA on gate/up and down.  Returns
    ``(out, saved)`` where ``saved`` feeds :func:`experts_backward`."""
    if _tc_grouped(xs, p):
        return _experts_forward_tc(xs, counts, p, lora)
    s = p.scale
    gu = grouped_mm(xs, p.gu_w_t, counts)
    u_gu = u_d = None
    if lora and p.A_gu is not None:
        r = p.B_gu.shape[-1]
        u_gu = grouped_mm(xs, p.A_gu.transpose(1, 2), counts)  # [N, 2r]
        lo = grouped_mm(u_gu[:, :r].contiguous(), p.B_gu[:, 0].transpose(1, 2), counts)
        hi = grouped_mm(u_gu[:, r:].contiguous(), p.B_gu[:, 1].transpose(1, 2), counts)
        gu = gu + s * torch.cat([lo, hi], dim=1)
    if p.gu_b is not None:
        gu = gu + _row_bias(p.gu_b, counts, gu)
    act = _act_fwd(gu, p)
    out = grouped_mm(act, p.down_w_t, counts)
    if lora and p.A_d is not None:
        u_d = grouped_mm(act, p.A_d.transpose(1, 2), counts)  # [N, r]
        out = out + s * grouped_mm(u_d, p.B_d.transpose(1, 2), counts)
    if p.down_b is not None:
        out = out + _row_bias(p.down_b, counts, out)
    return out, (xs, gu, act, u_gu, u_d, counts, lora)


def experts_backward(dout: torch.Tensor, saved, p: ExpertParams) -> torch.Tensor:
    xs, gu, act, u_gu, u_d, counts, lora = saved
    s = p.scale
    dout = dout.contiguous()
    tc = _tc_grouped(xs, p)
    E, H, F2 = p.gu_w_t.shape
    if tc:
        from ..ops import native

        C = native.lib()
        offs = _offs(counts)
    if tc:
        a2 = b2 = None
        if lora and p.A_d is not None:
            dyB = _lr_rows(dout, p.B_d, counts, transposed=True)  # [N, r] = dout_e B_d[e]
            _lr_wgrad(u_d, dout, p.g_B_d, counts, s, transposed=True)  # dB_d[e] += s dout_e^T u_d
            _lr_wgrad(dyB, act, p.g_A_d, counts, s)  # dA_d[e] += s dyB^T act
            a2, b2 = dyB, (s * p.A_d.transpose(1, 2)).reshape(E * (F2 // 2), -1).contiguous()
        dact = C.gemm_tc_grouped(dout, p.down_w_t.view(E * (F2 // 2), H), offs, F2 // 2, a2, b2, False)
    else:
        dact = grouped_mm(dout, p.down_w_t.transpose(1, 2), counts)
    if not tc and lora and p.A_d is not None:
        dyB = grouped_mm(dout, p.B_d, counts)  # [N, r]
        grouped_wgrad(dout, u_d, counts, p.g_B_d, s)
        grouped_wgrad(dyB, act, counts, p.g_A_d, s)
        dact = dact + s * grouped_mm(dyB, p.A_d, counts)
    Fh = gu.shape[1] // 2
    dgu = _act_bwd(dact, gu, p)  # [dgate | dup] (fused kernel on the GPU)
    if tc:
        a2 = b2 = None
        if lora and p.A_gu is not None:
            r = p.B_gu.shape[-1]
            dyB = dgu.new_empty(dgu.shape[0], 2 * r)
            _lr_rows(dgu[:, :Fh], p.B_gu[:, 0], counts, transposed=True, out=dyB[:, :r])
            _lr_rows(dgu[:, Fh:], p.B_gu[:, 1], counts, transposed=True, out=dyB[:, r:])
            _lr_wgrad(u_gu[:, :r], dgu[:, :Fh], p.g_B_gu[:, 0], counts, s, transposed=True)
            _lr_wgrad(u_gu[:, r:], dgu[:, Fh:], p.g_B_gu[:, 1], counts, s, transposed=True)
            _lr_wgrad(dyB, xs, p.g_A_gu, counts, s)
            a2, b2 = dyB, (s * p.A_gu.transpose(1, 2)).reshape(E * H, -1).contiguous()
        return C.gemm_tc_grouped(dgu, p.gu_w_t.view(E * H, F2), offs, H, a2, b2, False)
    dxs = grouped_mm(dgu, p.gu_w_t.transpose(1, 2), counts)
    if lora and p.A_gu is not None:
        r = p.B_gu.shape[-1]
        dyB = torch.cat(
            [grouped_mm(dgu[:, :Fh].contiguous(), p.B_gu[:, 0], counts),
             grouped_mm(dgu[:, Fh:].contiguous(), p.B_gu[:, 1], counts)], dim=1)
        grouped_wgrad(dgu[:, :Fh], u_gu[:, :r], counts, p.g_B_gu[:, 0], s)
        grouped_wgrad(dgu[:, Fh:], u_gu[:, r:], counts, p.g_B_gu[:, 1], s)
        grouped_wgrad(dyB, xs, counts, p.g_A_gu, s)
        dxs = dxs + s * grouped_mm(dyB, p.A_gu, counts)
    return dxs


class _LocalExperts(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xs, counts, params, lora, anchor):
        out, saved = experts_forward(xs, counts, params, lora)
        _save_expert_state(ctx, saved)
        ctx.params = params
        return out

    @staticmethod
    def backward(ctx, dout):
        dxs = experts_backward(dout, _expert_state(ctx, ctx.saved_tensors), ctx.params)
        return dxs, None, None, None, None


def _save_expert_state(ctx, saved, *extra: torch.Tensor | None) -> None:
    """Keep the expert activations through ``save_for_backward`` (so that
    activation recompute can drop and regenerate them); the group sizes and
    the LoRA flag stay on ``ctx``."""
    xs, gu, act, u_gu, u_d, counts, lora = saved
    ctx.save_for_backward(xs, gu, act, u_gu, u_d, *extra)
    ctx.expert_meta = (counts, lora)


def _expert_state(ctx, saved_tensors):
    """The ``experts_backward`` state from ``ctx.saved_tensors`` (read once
    per backward: under recompute each read regenerates the tensors)."""
    xs, gu, act, u_gu, u_d = saved_tensors[:5]
    return (xs, gu, act, u_gu, u_d, *ctx.expert_meta)


def native_combine(slots: torch.Tensor, w: torch.Tensor | None, k: int) -> torch.Tensor:
    """``y[t] = sum_j w[t, j] * slots[t*k + j]`` (fused kernel on CUDA)."""
    if slots.device.type == "cuda":
        from ..ops import native

        ww = None if w is None else w.reshape(-1).float().contiguous()
        return native.lib().combine_rows(slots.contiguous(), ww, k)
    T = slots.shape[0] // k
    sl = slots.view(T, k, -1).to(torch.float64 if slots.dtype == torch.float64 else torch.float32)
    if w is not None:
        sl = sl * w.view(T, k, 1).to(sl.dtype)
    return sl.sum(1).to(slots.dtype)


class _EPExperts(torch.autograd.Function):
    """Dispatch -> local experts -> combine across the expert-parallel group."""

    @staticmethod
    def forward(ctx, h, w, idx, ep, params, lora, anchor):
        plan = ep.plan(idx)
        tr = ep.transport
        recv = tr.push(plan, h, None, 0)
        xs = recv.clone()
        out, saved = experts_forward(xs, plan.local_counts, params, lora)
        tr.publish(out, 1)
        slots = tr.pull(plan, 1)
        from ..parallel import mutation

        y = native_combine(slots, None if mutation.active("ep_skip_combine_weights") else w, plan.k)
        ctx.plan, ctx.ep, ctx.params = plan, ep, params
        _save_expert_state(ctx, saved, slots, w)
        return y

    @staticmethod
    def backward(ctx, dy):
        saved = ctx.saved_tensors
        slots, w = saved[5:]
        plan, ep, params = ctx.plan, ctx.ep, ctx.params
        tr = ep.transport
        dy = dy.contiguous()
        T, k = plan.T, plan.k
        dw = (slots.view(T, k, -1).float() * dy.view(T, 1, -1).float()).sum(-1)
        d_recv = tr.push(plan, dy, w.reshape(-1).float().contiguous(), 2)
        dxs = experts_backward(d_recv.clone(), _expert_state(ctx, saved), params)
        tr.publish(dxs, 3)
        dslots = tr.pull(plan, 3)
        dh = native_combine(dslots, None, k)
        return dh, dw.to(w.dtype), None, None, None, None, None


class MoEBlock:
    def __init__(self, cfg: ModelConfig, i: int, gen, dev, dt, store: LoRAStore, spec: LoRASpec,
                 ep: Any = None, etp: Any = None) -> None:
        from .transformer import _randn

        self.cfg, self.index, self.ep, self.etp = cfg, i, ep, etp
        E, H, F = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
        self.router_w = _randn((E, H), gen, dev, dt)
        self.router_b = _randn((E,), gen, dev, dt) if cfg.router_bias else None
        e0 = ep.first_expert if ep is not None else 0
        El = ep.E_local if ep is not None else E
        f0, Fl = etp.slice(F) if etp is not None else (0, F)
        self.f0, self.F_local = f0, Fl
        # the expert weights are drawn in one piece so the random init does not
        # depend on the expert- or expert-tensor-parallel degree; each rank
        # keeps its experts and, under ETP, its intermediate slice
        gu = _randn((E, H, 2 * F), gen, dev, dt)
        dn = _randn((E, F, H), gen, dev, dt)
        if El != E or Fl != F:
            gu = torch.cat([gu[e0 : e0 + El, :, f0 : f0 + Fl], gu[e0 : e0 + El, :, F + f0 : F + f0 + Fl]], dim=2)
            dn = dn[e0 : e0 + El, f0 : f0 + Fl].contiguous()
        self.gu_w_t = gu.contiguous()  # [E_local, H, 2F_local]
        self.down_w_t = dn  # [E_local, F_local, H]
        self.shared = None
        if cfg.shared_expert_intermediate_size:
            Fs = cfg.shared_expert_intermediate_size
            self.shared = (
                _randn((2 * Fs, H), gen, dev, dt),
                _randn((H, Fs), gen, dev, dt),
                _randn((1, H), gen, dev, dt),
            )
        r = spec.r

        def stacked(names: list[str], shape: tuple[int, ...]):
            if not names or names[0] not in store.entries:
                return None, None
            off, n = store.contiguous_span(names)
            return store.compute[off : off + n].view(shape), store.grad[off : off + n].view(shape)

        A_gu, g_A_gu = stacked([peft_key(i, "mlp", p, "A", e) for e in range(E) for p in ("gate_proj", "up_proj")], (E, 2 * r, H))
        B_gu, g_B_gu = stacked([peft_key(i, "mlp", p, "B", e) for e in range(E) for p in ("gate_proj", "up_proj")], (E, 2, F, r))
        A_d, g_A_d = stacked([peft_key(i, "mlp", "down_proj", "A", e) for e in range(E)], (E, r, F))
        B_d, g_B_d = stacked([peft_key(i, "mlp", "down_proj", "B", e) for e in range(E)], (E, H, r))
        sl = slice(e0, e0 + El)
        fs = slice(f0, f0 + Fl)
        pick = lambda t: None if t is None else t[sl]  # noqa: E731
        pick_bgu = lambda t: None if t is None else t[sl, :, fs]  # noqa: E731  gate/up B: rows of the F slice
        pick_ad = lambda t: None if t is None else t[sl, :, fs]  # noqa: E731  down A: columns of the F slice
        self.params = ExpertParams(
            self.gu_w_t, self.down_w_t, pick(A_gu), pick_bgu(B_gu), pick_ad(A_d), pick(B_d),
            pick(g_A_gu), pick_bgu(g_B_gu), pick_ad(g_A_d), pick(g_B_d), spec.scale,
        )
        self.params.A_all_gu, self.params.B_all_d = A_gu, B_d
        if cfg.expert_bias:
            self.params.gu_b = _randn((El, 2 * Fl), gen, dev, dt)
            self.params.down_b = _randn((El, H), gen, dev, dt)
        self.params.act, self.params.alpha, self.params.limit = cfg.expert_act, cfg.glu_alpha, cfg.glu_limit

    def num_parameters(self) -> int:
        n = self.router_w.numel() + self.gu_w_t.numel() + self.down_w_t.numel()
        if self.shared is not None:
            n += sum(t.numel() for t in self.shared)
        return n

    def route(self, h: torch.Tensor, ctx: dict[str, Any]) -> tuple[torch.Tensor, torch.Tensor]:
        cfg = self.cfg
        logits = (h @ self.router_w.t()).float()
        if self.router_b is not None:
            logits = logits + self.router_b.float()
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
        E, k = self.cfg.num_experts, self.cfg.num_experts_per_tok
        idx, wts = self.route(h, ctx)
        anchor = grad_anchor(h.device) if enabled else None
        hx, wx, ix = h, wts, idx
        if self.etp is not None:  # the ETP group's whole token set, every member its F slice
            hx, wx, ix = self.etp.gather(h), self.etp.gather(wts), self.etp.gather_nograd(idx)
        T, H = hx.shape
        params = self.params.for_compute()
        if self.ep is not None and self.ep.world > 1:
            if not params.plain:
                raise NotImplementedError("expert parallelism runs SwiGLU experts without biases (not GPT-OSS)")
            fused = getattr(self.ep, "fused", None)
            counts = ctx.get("ep_counts")
            if fused is not None and counts is not None and self.etp is None:
                # routes replayed and every rank's counts known on the host:
                # the exchanges fused into the expert GEMMs
                from ..parallel.ep_fused import FusedEPExperts

                out = FusedEPExperts.apply(hx, wx, ix, fused, params, enabled, counts[self.index], anchor)
            else:
                out = _EPExperts.apply(hx, wx, ix, self.ep, params, enabled, anchor)
        else:
            flat = ix.reshape(-1)
            order = torch.argsort(flat, stable=True)
            host = ctx.get("replay_counts") if self.etp is None else None
            if host is not None:  # replayed routes: group sizes known on the host, no device sync
                counts = list(host[self.index]) + [0] * (E - len(host[self.index]))
            else:
                counts = torch.bincount(flat, minlength=E).tolist()
            tok = order // k
            xs = hx[tok]
            ys = _LocalExperts.apply(xs, counts, params, enabled, anchor)
            w_sorted = wx.reshape(-1)[order].to(ys.dtype).unsqueeze(1)
            out = torch.zeros(T, H, device=hx.device, dtype=ys.dtype).index_add(0, tok, ys * w_sorted)
        if self.etp is not None:  # sum the F slices, back to this rank's tokens
            out = self.etp.reduce_scatter(out)
        if self.shared is not None:
            gu_w, down_w, gate_w = self.shared
            gu = h @ gu_w.t()
            Fs = gu.shape[1] // 2
            sh = (torch.nn.functional.silu(gu[:, :Fs]) * gu[:, Fs:]) @ down_w.t()
            out = out + torch.sigmoid(h @ gate_w.t()) * sh
        return out

    def load_hf(self, sd: dict[str, torch.Tensor], prefix: str, g: Callable[[str], torch.Tensor]) -> None:
        e0 = self.ep.first_expert if self.ep is not None else 0
        fs = slice(self.f0, self.f0 + self.F_local)
        if prefix + "router.weight" in sd:  # GPT-OSS: stacked experts, gate/up interleaved by column
            El = self.gu_w_t.shape[0]
            es = slice(e0, e0 + El)
            self.router_w.copy_(g(prefix + "router.weight"))
            if self.router_b is not None:
                self.router_b.copy_(g(prefix + "router.bias"))
            gu = g(prefix + "experts.gate_up_proj")[es]  # [E, H, 2F]
            self.gu_w_t.copy_(torch.cat([gu[..., 0::2][..., fs], gu[..., 1::2][..., fs]], dim=2))
            self.down_w_t.copy_(g(prefix + "experts.down_proj")[es][:, fs])
            if self.params.gu_b is not None:
                b = g(prefix + "experts.gate_up_proj_bias")[es]
                self.params.gu_b.copy_(torch.cat([b[:, 0::2][:, fs], b[:, 1::2][:, fs]], dim=1))
                self.params.down_b.copy_(g(prefix + "experts.down_proj_bias")[es])
            return
        self.router_w.copy_(g(prefix + "gate.weight"))
        if self.shared is not None and prefix + "shared_expert.gate_proj.weight" in sd:
            gu_w, down_w, gate_w = self.shared
            gu_w.copy_(torch.cat([g(prefix + "shared_expert.gate_proj.weight"), g(prefix + "shared_expert.up_proj.weight")]))
            down_w.copy_(g(prefix + "shared_expert.down_proj.weight"))
            gate_w.copy_(g(prefix + "shared_expert_gate.weight"))
        for le in range(self.gu_w_t.shape[0]):
            p = f"{prefix}experts.{e0 + le}."
            self.gu_w_t[le].copy_(torch.cat([g(p + "gate_proj.weight")[fs], g(p + "up_proj.weight")[fs]]).t())
            self.down_w_t[le].copy_(g(p + "down_proj.weight")[:, fs].t())
