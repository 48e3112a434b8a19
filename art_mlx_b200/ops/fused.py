"""Autograd wrappers of the fused kernels.

Every op has one implementation per device: CUDA tensors run the sm_100a
kernels of ``ops/csrc`` (and raise if the extension is missing), CPU tensors
run the same math in plain PyTorch (the fp32 plumbing configuration and the
numerics oracle of the GPU tests).

Ops:
* :func:`add_rmsnorm` - residual add fused with RMSNorm (frozen weight).
* :func:`rope_attention` - qk-RMSNorm + RoPE on packed positions + prefix-tree
  attention, returning the attention output; its backward produces the
  gradient of the whole raw QKV projection in one buffer.
* :func:`swiglu` - ``silu(gate) * up`` on a fused ``[gate | up]`` projection.
* :func:`lora_linear` - frozen base GEMM plus LoRA, accumulating the LoRA
  gradients straight into the flat fp32 gradient buffer.
* :func:`lm_head_logprobs` - chunked LM head + log-softmax gather + entropy.
* :func:`grpo_token_loss` - the token-level GRPO/CISPO/PPO loss with its
  closed-form gradient.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import Any, Sequence

import numpy as np
import torch

from . import lowrank, native


def _cuda(t: torch.Tensor) -> bool:
    return t.device.type == "cuda"


def _acc(t: torch.Tensor) -> torch.Tensor:
    """Accumulation precision of the CPU reference path: fp32, or fp64 when
    the inputs already are fp64."""
    return t if t.dtype == torch.float64 else t.float()


# ---------------------------------------------------------------------------
# Attention metadata (per packed row)
# ---------------------------------------------------------------------------


BWD_KEYS = 128  # key block of the warp-level attention backward kernel
BWD_Q = 32  # query tile of the warp-level attention backward kernel
BWD_MAX_QTILES = 8  # query tiles per warp-level backward work unit


def attention_bwd_units(kend: torch.Tensor, max_qtiles: int = BWD_MAX_QTILES) -> torch.Tensor:
    """Work units ``[n, 3]`` = (key block, q tile lo, q tile hi) of the
    warp-level backward (``attn_bwd`` and its allocation-free C entry point;
    training runs the tensor-core backward, :func:`attention_bwd_units_tc`).

    Key block ``kb`` (128 keys) is seen by queries ``[128 kb, max kend)``;
    that range (in 32-query tiles) is split into units of at most
    ``max_qtiles`` tiles so a shared prompt attended by every completion is
    spread over many CTAs instead of serialising on a few.
    """
    T = int(kend.numel())
    if T == 0:
        return torch.zeros(0, 3, dtype=torch.int32)
    nkb = (T + BWD_KEYS - 1) // BWD_KEYS
    kp = torch.nn.functional.pad(kend.to(torch.int64), (0, nkb * BWD_KEYS - T), value=0)
    kmax = kp.view(nkb, BWD_KEYS).amax(1).clamp(max=T).tolist()
    units = []
    for kb in range(nkb):
        lo = kb * BWD_KEYS // BWD_Q
        hi = (kmax[kb] + BWD_Q - 1) // BWD_Q
        for a in range(lo, hi, max_qtiles):
            units.append((kb, a, min(hi, a + max_qtiles)))
    return torch.tensor(units, dtype=torch.int32).view(-1, 3)


TC_TILE = 128  # key block and query tile of the tensor-core backward
TC_MAX_QTILES = 4  # query tiles per tensor-core backward work unit


def attention_bwd_units_tc(kend: torch.Tensor, q_off: int = 0, Tq: int | None = None,
                           max_qtiles: int = TC_MAX_QTILES, kv_heads: int = 4, min_ctas: int = 2 * 148) -> torch.Tensor:
    """Work units ``[n, 3]`` = (128-key block, first, end local 128-query
    tile) of the tensor-core backward for local queries ``[q_off, q_off+Tq)``
    (global positions) against every key.  A key block is seen by the
    queries ``[128 kb, max kend)``; that range is cut into units of at most
    ``max_qtiles`` tiles so shared-prompt blocks spread over many CTAs, and
    the cut is made finer (down to one tile) while the launch
    (units x ``kv_heads``) would not fill ``min_ctas`` CTAs."""
    T = int(kend.numel())
    Tq = T - q_off if Tq is None else Tq
    if T == 0 or Tq <= 0:
        return torch.zeros(0, 3, dtype=torch.int32)
    nkb = (T + TC_TILE - 1) // TC_TILE
    kp = torch.nn.functional.pad(kend.to(torch.int64), (0, nkb * TC_TILE - T), value=0)
    kmax = kp.view(nkb, TC_TILE).amax(1).clamp(max=T).tolist()
    spans = []
    for kb in range(nkb):
        lo = max(kb * TC_TILE, q_off) - q_off
        hi = min(kmax[kb], q_off + Tq) - q_off
        if hi > lo:
            spans.append((kb, lo // TC_TILE, (hi + TC_TILE - 1) // TC_TILE))
    m = max_qtiles
    while m > 1 and sum((b - a + m - 1) // m for _, a, b in spans) * kv_heads < min_ctas:
        m //= 2
    units = [(kb, a, min(b, a + m)) for kb, lo, b in spans for a in range(lo, b, m)]
    return torch.tensor(units, dtype=torch.int32).view(-1, 3)


@dataclass
class AttnMeta:
    """Per-row attention metadata shared by every layer of one micro step.

    ``kend[j]``: query ``i`` may attend key ``j`` iff ``j <= i < kend[j]``.
    ``tile_kmax[t]`` / ``tile_kmin[t]``: max / min of ``kend`` over keys
    ``[64t, 64t+64)`` (tile skipping, and tiles that need no mask).
    ``bwd_units``: load-balanced work list of the tensor-core attention
    backward (128-key blocks x 128-query tiles).
    """

    positions: torch.Tensor  # int32 [T]
    kend: torch.Tensor  # int32 [T]
    tile_kmax: torch.Tensor  # int32 [ceil(T/64)]
    T: int
    bwd_units: torch.Tensor | None = None  # int32 [n, 3]
    tile_kmin: torch.Tensor | None = None  # int32 [ceil(T/64)]
    # sliding window (0: none): the variant of this row for windowed layers
    window: int = 0
    tile_pmax: torch.Tensor | None = None  # int32 [ceil(T/128)]: max position per 128-key tile
    _windowed: dict = field(default_factory=dict, repr=False)
    _host: tuple | None = field(default=None, repr=False)  # (positions, kend) on the CPU

    def windowed(self, window: int | None) -> "AttnMeta":
        """The metadata of this row for a layer with a sliding window of
        ``window`` tokens (``None``/0: this one).  Key ``j`` then reaches the
        queries ``i`` with ``j <= i < kend_w[j]`` and ``pos[i] - pos[j] <
        window``; ``kend_w`` (:func:`window_visibility_ends`) tightens the
        interval so tile skipping and the backward work list see only the
        window.  Built once per row and window, shared by the layers."""
        if not window:
            return self
        w = self._windowed.get(window)
        if w is None:
            if self._host is None:
                raise ValueError("this AttnMeta was built without host positions; rebuild it with AttnMeta.build")
            pos, kend = self._host
            if pos is None:  # built from device positions: fetch them once
                pos = self.positions.to("cpu", torch.int32)
                self._host = (pos, kend)
            kw = window_visibility_ends(pos, kend, window)
            w = AttnMeta.build(pos, kw, self.kend.device, window=window)
            self._windowed[window] = w
        return w

    @staticmethod
    def build(positions: torch.Tensor, kend: torch.Tensor, device: torch.device, window: int = 0) -> "AttnMeta":
        """``kend`` may live on any device; the work list is planned on the CPU."""
        T = int(kend.numel())
        pad = (-T) % 64
        k_cpu = kend.detach().to("cpu", torch.int32)
        kp = torch.nn.functional.pad(k_cpu, (0, pad), value=0)
        tile = kp.view(-1, 64).amax(dim=1).to(torch.int32)
        kq = torch.nn.functional.pad(k_cpu, (0, pad), value=torch.iinfo(torch.int32).max)
        tile_min = kq.view(-1, 64).amin(dim=1).to(torch.int32)
        units = attention_bwd_units_tc(k_cpu)
        pin = device.type == "cuda"
        mv = lambda t: (t.pin_memory() if pin else t).to(device, non_blocking=True)  # noqa: E731
        if positions.device.type == "cpu":  # host positions: no device round trip for windowed variants
            p_cpu = positions.detach().to(torch.int32).contiguous()
            pos_dev = mv(p_cpu)
        else:
            p_cpu = None
            pos_dev = positions.to(device=device, dtype=torch.int32, non_blocking=True)
        tile_pmax = None
        if window:
            if p_cpu is None:
                p_cpu = positions.detach().to("cpu", torch.int32)
            pp = torch.nn.functional.pad(p_cpu, (0, (-T) % 128), value=torch.iinfo(torch.int32).min)
            tile_pmax = mv(pp.view(-1, 128).amax(dim=1).to(torch.int32))
        return AttnMeta(
            positions=pos_dev,
            kend=mv(k_cpu),
            tile_kmax=mv(tile),
            T=T,
            bwd_units=mv(units),
            tile_kmin=mv(tile_min),
            window=int(window or 0),
            tile_pmax=tile_pmax,
            _host=(p_cpu, k_cpu),
        )


def window_visibility_ends(positions: torch.Tensor, kend: torch.Tensor, window: int) -> torch.Tensor:
    """Visibility ends under a sliding window of ``window`` positions.

    The packed row is cut into runs where ``kend`` is constant and positions
    rise by one (a prefix-tree segment, merged with an only child).  Queries
    of key ``j``'s own run are ``j..run_end`` at positions ``pos[j] + (i -
    j)``; every later query of its subtree sits at a position of at least
    ``pos[run_end - 1] + 1``.  So if the run's end is ``window`` or more
    positions past ``j``, no later query is in the window and the interval
    shrinks to ``[j, min(run_end, j + window))``; otherwise it stays
    ``[j, kend[j])``.  The result bounds the visible queries from above; the
    kernels still check ``pos[i] - pos[j] < window`` per pair (the
    reference's sliding-window block masks, ``src/art/megatron/
    prefix_tree_state.py:67,94-102``)."""
    k = kend.detach().to("cpu", torch.int64).numpy()
    p = positions.detach().to("cpu", torch.int64).numpy()
    T = k.shape[0]
    if T == 0:
        return kend.to("cpu", torch.int32)
    brk = np.ones(T, dtype=bool)
    brk[1:] = (k[1:] != k[:-1]) | (p[1:] != p[:-1] + 1)
    starts = np.flatnonzero(brk)
    ends = np.append(starts[1:], T)
    e = ends[np.cumsum(brk) - 1]
    j = np.arange(T)
    kw = np.where((k > e) & (e - j < window), k, np.minimum(e, j + window))
    return torch.from_numpy(kw.astype(np.int32))


def rope_inv_freq(head_dim: int, theta: float, device: torch.device, scaling: dict | None = None) -> torch.Tensor:
    """RoPE inverse frequencies ``theta^(-2i/d)``, with the checkpoint's
    frequency scaling: ``linear`` (positions divided by ``factor``) or
    ``llama3`` (long wavelengths divided by ``factor``, short ones kept, a
    linear blend in between, as published with Llama 3.1).  Other scaling
    types are refused rather than silently ignored."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64, device="cpu") / head_dim))
    kind = (scaling or {}).get("rope_type") or (scaling or {}).get("type") or "default"
    if kind == "linear":
        inv = inv / float(scaling["factor"])
    elif kind == "llama3":
        factor = float(scaling["factor"])
        lo, hi = float(scaling["low_freq_factor"]), float(scaling["high_freq_factor"])
        ctx = float(scaling["original_max_position_embeddings"])
        wavelen = 2 * math.pi / inv
        smooth = ((ctx / wavelen - lo) / (hi - lo)).clamp(0.0, 1.0)
        blended = (1 - smooth) * inv / factor + smooth * inv
        inv = torch.where(wavelen < ctx / hi, inv, torch.where(wavelen > ctx / lo, inv / factor, blended))
    elif kind == "yarn":
        inv = _yarn_inv_freq(inv, head_dim, theta, scaling)
    elif kind != "default":
        raise NotImplementedError(f"RoPE scaling {kind!r} is not supported")
    return inv.to(device=device, dtype=torch.float32)


def _yarn_mscale(scale: float, m: float = 1.0) -> float:
    return 0.1 * m * math.log(scale) + 1.0 if scale > 1 else 1.0


def _yarn_inv_freq(inv: torch.Tensor, head_dim: int, theta: float, sc: dict) -> torch.Tensor:
    """YaRN (Peng et al., 2023, "YaRN: Efficient Context Window Extension of
    Large Language Models"): frequencies that complete fewer than
    ``beta_slow`` turns over the original context are interpolated (divided
    by ``factor``), those with more than ``beta_fast`` turns kept, with a
    linear ramp in between over the dimension index."""
    factor = float(sc["factor"])
    ctx = float(sc.get("original_max_position_embeddings") or 4096)
    b_fast, b_slow = float(sc.get("beta_fast", 32.0)), float(sc.get("beta_slow", 1.0))

    def dim_of(turns: float) -> float:  # dimension index whose wavelength gives `turns` over ctx
        return head_dim * math.log(ctx / (turns * 2 * math.pi)) / (2 * math.log(theta))

    lo, hi = dim_of(b_fast), dim_of(b_slow)
    if sc.get("truncate", True):
        lo, hi = math.floor(lo), math.ceil(hi)
    lo, hi = max(lo, 0), min(hi, head_dim - 1)
    if lo == hi:
        hi += 0.001
    ramp = ((torch.arange(head_dim // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0.0, 1.0)
    keep = 1.0 - ramp  # 1: extrapolate (keep), 0: interpolate
    return inv / factor * (1 - keep) + inv * keep


def partial_rotary(head_dim: int, rotary_dim: int, theta: float, device: torch.device,
                   scaling: dict | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE on the first ``rotary_dim`` dims of each head only (rotate-half
    within them; Qwen3-Next / Qwen3.5).  Returns the frequencies of the
    kernels' pair layout (pair ``i`` = dims ``(i, i + head_dim/2)`` of an
    internal order) and ``perm``: internal dim -> head column.  The rotated
    dims and their partners take the first pairs; the untouched dims fill the
    rest with zero frequency.  Attention reads q and k in the internal order
    (dot products do not change when both are permuted alike); weights,
    LoRA factors and v stay in the checkpoint's order."""
    D, rd = head_dim, rotary_dim
    assert rd % 2 == 0 and 0 < rd <= D
    inv = torch.zeros(D // 2, dtype=torch.float32)
    inv[: rd // 2] = rope_inv_freq(rd, theta, torch.device("cpu"), scaling)
    perm = torch.empty(D, dtype=torch.int64)
    half, rest = rd // 2, (D - rd) // 2
    for i in range(D // 2):
        if i < half:
            perm[i], perm[i + D // 2] = i, i + half
        else:
            j = i - half
            perm[i], perm[i + D // 2] = rd + j, rd + rest + j
    return inv.to(device), perm.to(device)


def rope_attention_factor(scaling: dict | None) -> float:
    """Factor by which the checkpoint's RoPE scales cos / sin (YaRN's
    ``0.1 ln(factor) + 1``, or the configured ``attention_factor``); q and k
    both carry it, so attention scores carry its square."""
    sc = scaling or {}
    kind = sc.get("rope_type") or sc.get("type") or "default"
    if kind != "yarn":
        return 1.0
    if sc.get("attention_factor") is not None:
        return float(sc["attention_factor"])
    factor = float(sc["factor"])
    m, m_all = sc.get("mscale"), sc.get("mscale_all_dim")
    if m and m_all:
        return _yarn_mscale(factor, float(m)) / _yarn_mscale(factor, float(m_all))
    return _yarn_mscale(factor)


# ---------------------------------------------------------------------------
# RMSNorm with fused residual add
# ---------------------------------------------------------------------------


def _rmsnorm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = _acc(x)
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * r).to(x.dtype) * w


class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, res, w, eps):
        y, xs, rstd = native.lib().rmsnorm_fwd(x, res, w, eps)
        ctx.save_for_backward(xs, w, rstd)
        ctx.has_res = res is not None
        return y, xs

    @staticmethod
    def backward(ctx, dy, dxs):
        xs, w, rstd = ctx.saved_tensors
        dres = dxs.contiguous() if dxs is not None else None
        dx = native.lib().rmsnorm_bwd(dy.contiguous(), xs, w, rstd, dres)
        return dx, (dx if ctx.has_res else None), None, None


def add_rmsnorm(
    x: torch.Tensor, res: torch.Tensor | None, w: torch.Tensor, eps: float
) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns ``(rmsnorm(x + res) * w, x + res)``; ``res=None`` skips the add."""
    if _cuda(x):
        return _AddRMSNorm.apply(x, res, w, eps)
    s = x if res is None else x + res
    return _rmsnorm_ref(s, w, eps), s


# ---------------------------------------------------------------------------
# RoPE + prefix-tree attention
# ---------------------------------------------------------------------------


def _rope_ref(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    # x [T, H, D]; rotate-half convention
    ang = _acc(pos.to(x.dtype) if x.dtype == torch.float64 else pos.float()).unsqueeze(-1) * inv_freq.to(
        torch.float64 if x.dtype == torch.float64 else torch.float32
    ).unsqueeze(0)  # [T, D/2]
    cos = torch.cat([ang.cos(), ang.cos()], -1).unsqueeze(1).to(x.dtype)
    sin = torch.cat([ang.sin(), ang.sin()], -1).unsqueeze(1).to(x.dtype)
    d = x.shape[-1] // 2
    rot = torch.cat([-x[..., d:], x[..., :d]], -1)
    return x * cos + rot * sin


def attention_ref(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kend: torch.Tensor, scale: float,
    positions: torch.Tensor | None = None, window: int = 0, sinks: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Dense-mask prefix-tree attention in fp32 math (oracle). q [T,Hq,D].

    ``window`` > 0 also requires ``pos[i] - pos[j] < window``; ``sinks``
    ([Hq], natural log) adds ``exp(sink)`` to every row's denominator."""
    T, Hq, D = q.shape
    G = Hq // k.shape[1]
    kx = _acc(k).repeat_interleave(G, dim=1)
    vx = _acc(v).repeat_interleave(G, dim=1)
    s = torch.einsum("ihd,jhd->hij", _acc(q), kx) * scale
    i = torch.arange(T, device=q.device).view(T, 1)
    j = torch.arange(T, device=q.device).view(1, T)
    mask = (j <= i) & (i < kend.to(q.device).long().view(1, T))
    if window:
        pos = positions.to(q.device).long()
        mask &= (pos.view(T, 1) - pos.view(1, T)) < window
    s = s.masked_fill(~mask.unsqueeze(0), float("-inf"))
    if sinks is not None:
        sk = _acc(sinks).view(Hq, 1, 1).expand(Hq, T, 1)
        lse = torch.logsumexp(torch.cat([s, sk], -1), dim=-1)  # [Hq, T]
        p = torch.exp(s - lse.unsqueeze(-1))
    else:
        lse = torch.logsumexp(s, dim=-1)  # [Hq, T]
        p = torch.softmax(s, dim=-1).nan_to_num(0.0)
    o = torch.einsum("hij,jhd->ihd", p, vx)
    return o.to(q.dtype), lse


ATTN_HEAD_DIM = 128  # head size of the tcgen05 attention kernels


def _pad_head(x: torch.Tensor) -> torch.Tensor:
    """Heads narrower than the kernels' 128 columns, zero-padded (zero
    columns change no score and give zero output columns)."""
    D = x.shape[-1]
    if D == ATTN_HEAD_DIM:
        return x
    if D > ATTN_HEAD_DIM:
        raise NotImplementedError(f"attention head_dim {D} > {ATTN_HEAD_DIM} on the GPU")
    return torch.nn.functional.pad(x, (0, ATTN_HEAD_DIM - D)).contiguous()


class _RopeAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, meta, inv_freq, nq, nkv, D, qn_w, kn_w, eps, scale, sinks, perm):
        C = native.lib()
        T = qkv.shape[0]
        qk, rstd = C.rope_fwd(qkv, meta.positions, inv_freq, nq, nkv, D, qn_w, kn_w, eps, perm)
        q = qk[:, : nq * D].view(T, nq, D)
        k = qk[:, nq * D :].view(T, nkv, D)
        v = qkv[:, (nq + nkv) * D : (nq + 2 * nkv) * D].unflatten(1, (nkv, D))
        win = meta.window
        q, k, v = _pad_head(q), _pad_head(k), _pad_head(v)
        o, lse = C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, scale, 0,
                               meta.positions if win else None, meta.tile_pmax if win else None, win, sinks)
        ctx.save_for_backward(qkv, qk, o, lse, inv_freq, qn_w if qn_w is not None else qkv.new_empty(0),
                              kn_w if kn_w is not None else qkv.new_empty(0),
                              rstd if rstd is not None and rstd.numel() else qkv.new_empty(0, dtype=torch.float32))
        ctx.meta = meta
        ctx.perm = perm
        ctx.dims = (nq, nkv, D, scale, qn_w is not None)
        return o[..., :D].reshape(T, nq * D)

    @staticmethod
    def backward(ctx, do):
        C = native.lib()
        qkv, qk, o, lse, inv_freq, qn_w, kn_w, rstd = ctx.saved_tensors
        nq, nkv, D, scale, has_norm = ctx.dims
        meta = ctx.meta
        T = qkv.shape[0]
        do = _pad_head(do.contiguous().view(T, nq, D))
        q = _pad_head(qk[:, : nq * D].view(T, nq, D))
        k = _pad_head(qk[:, nq * D :].view(T, nkv, D))
        v = _pad_head(qkv[:, (nq + nkv) * D : (nq + 2 * nkv) * D].unflatten(1, (nkv, D)))
        dqkv = torch.empty_like(qkv)
        win = meta.window
        dq_acc, dk_acc, dv_acc, _ = C.attn_bwd_tc(do, q, k, v, o, lse, meta.kend, meta.bwd_units, scale, 0,
                                                 meta.positions if win else None, win)
        # the fp32 accumulators straight into dqkv (RoPE / norm backward for
        # q and k, v converted) in one launch
        C.rope_bwd_f32(dq_acc, dk_acc, dv_acc, qkv, meta.positions, inv_freq, nq, nkv, D,
                       qn_w if has_norm else None, kn_w if has_norm else None,
                       rstd if has_norm else None, dqkv, ctx.perm)
        return dqkv, None, None, None, None, None, None, None, None, None, None, None


def rope_attention(
    qkv: torch.Tensor,
    meta: AttnMeta,
    inv_freq: torch.Tensor,
    nq: int,
    nkv: int,
    D: int,
    qn_w: torch.Tensor | None,
    kn_w: torch.Tensor | None,
    eps: float,
    sinks: torch.Tensor | None = None,
    scale: float | None = None,
    perm: torch.Tensor | None = None,
) -> torch.Tensor:
    """Raw QKV projection ``[T, (nq+2nkv)*D]`` -> attention output ``[T, nq*D]``.

    ``meta`` carries the row's mask (``meta.windowed(w)`` for a sliding-window
    layer); ``sinks`` are frozen per-head sink logits (fp32 [nq])."""
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if _cuda(qkv):
        if sinks is not None:
            sinks = sinks.float().contiguous()
        if perm is not None:
            perm = perm.to(device=qkv.device, dtype=torch.int16).contiguous()
        return _RopeAttention.apply(qkv, meta, inv_freq, nq, nkv, D, qn_w, kn_w, eps, scale, sinks, perm)
    T = qkv.shape[0]
    q = qkv[:, : nq * D].view(T, nq, D)
    k = qkv[:, nq * D : (nq + nkv) * D].view(T, nkv, D)
    v = qkv[:, (nq + nkv) * D :].reshape(T, nkv, D)
    if qn_w is not None:
        q = _rmsnorm_ref(q, qn_w, eps)
        k = _rmsnorm_ref(k, kn_w, eps)
    pos = meta.positions
    if perm is not None:  # partial rotary: the kernels' internal dim order
        q, k = q[..., perm.long()], k[..., perm.long()]
    q = _rope_ref(q, pos, inv_freq)
    k = _rope_ref(k, pos, inv_freq)
    o, _ = attention_ref(q, k, v, meta.kend, scale, pos, meta.window, sinks)
    return o.reshape(T, nq * D)


# ---------------------------------------------------------------------------
# SwiGLU
# ---------------------------------------------------------------------------


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        ctx.save_for_backward(gu)
        return native.lib().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, da):
        (gu,) = ctx.saved_tensors
        return native.lib().swiglu_bwd(da.contiguous(), gu)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    if _cuda(gu):
        return _SwiGLU.apply(gu)
    F = gu.shape[-1] // 2
    g, u = gu[..., :F], gu[..., F:]
    return torch.nn.functional.silu(g) * u


# ---------------------------------------------------------------------------
# LoRA linear
# ---------------------------------------------------------------------------


@dataclass
class LoRABinding:
    """The LoRA factors of one (possibly fused) projection.

    ``A`` is the row-concatenation of the per-slice ``A`` matrices
    ``[n*r, in]``; ``B_blocks[k]`` is slice ``k``'s ``B`` ``[out_k, r]``,
    placed at output rows ``slices[k]`` and LoRA columns ``[k*r, (k+1)*r)``.
    ``gA``/``gB_blocks`` are the matching fp32 gradient slots.
    """

    A: torch.Tensor
    B_blocks: Sequence[torch.Tensor | None]
    gA: torch.Tensor
    gB_blocks: Sequence[torch.Tensor | None]
    slices: Sequence[tuple[int, int]]
    r: int
    scale: float
    out_features: int
    _bd: torch.Tensor | None = None
    _bd_version: int = -1

    _bd_s: torch.Tensor | None = None
    _at_s: torch.Tensor | None = None
    _fused_version: int = -1

    def fused_factors(self, version: int) -> tuple[torch.Tensor, torch.Tensor]:
        """``(scale * B_blockdiag [out, n*r], scale * A^T [in, n*r])``: the
        K-extension operands of the forward and input-gradient GEMMs (cached
        until the parameters change)."""
        if self._fused_version != version or self._bd_s is None:
            self._bd_s = (self.block_diag(version) * self.scale).contiguous()
            self._at_s = (self.A.t() * self.scale).contiguous()
            self._fused_version = version
        return self._bd_s, self._at_s

    def block_diag_t(self, version: int) -> torch.Tensor:
        """``block_diag(version)^T`` as a contiguous ``[n*r, out]`` matrix (the
        W operand of the rank-side input gradient ``dy B``; cached)."""
        if getattr(self, "_bdt_version", -1) != version or getattr(self, "_bdt", None) is None:
            self._bdt = self.block_diag(version).t().contiguous()
            self._bdt_version = version
        return self._bdt

    def block_diag(self, version: int) -> torch.Tensor:
        """Dense ``[out, n*r]`` B with the slice blocks on its diagonal (cached
        until the parameters change)."""
        if len(self.B_blocks) == 1 and self.B_blocks[0] is not None:
            return self.B_blocks[0]
        if self._bd is None or self._bd_version != version:
            n = len(self.B_blocks)
            bd = self.A.new_zeros(self.out_features, n * self.r)
            for k, (blk, (s, e)) in enumerate(zip(self.B_blocks, self.slices)):
                if blk is not None:
                    bd[s:e, k * self.r : (k + 1) * self.r] = blk
            self._bd = bd
            self._bd_version = version
        return self._bd


def _lowrank_ok(t: torch.Tensor, R: int, wgrad: bool = False) -> bool:
    """Whether a rank-side product with ``R`` low-rank columns runs on the
    low-rank kernels (CUDA bf16, 16-byte rows)."""
    return (LOWRANK and t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 2
            and R in (lowrank.WGRAD_WIDTHS if wgrad else lowrank.ROWS_WIDTHS)
            and R in lowrank.WGRAD_WIDTHS and t.stride(1) == 1 and t.stride(0) % 8 == 0
            and t.data_ptr() % 16 == 0 and t.shape[1] % 8 == 0)


def _accum_mm(slot: torch.Tensor, a: torch.Tensor, b: torch.Tensor, alpha: float) -> None:
    """``slot += alpha * a @ b`` with fp32 accumulation into the fp32 slot."""
    if _cuda(slot) and a.dtype != torch.float32:
        torch.addmm(slot, a, b, beta=1.0, alpha=alpha, out_dtype=torch.float32, out=slot)
    else:
        slot.addmm_(a.to(slot.dtype), b.to(slot.dtype), alpha=alpha)


_ANCHORS: dict[torch.device, torch.Tensor] = {}


def grad_anchor(device: torch.device) -> torch.Tensor:
    """A scalar that requires grad.  Ops whose trainable state lives outside
    autograd (the flat LoRA store) take it as an input so their outputs join
    the graph and their backward runs even when no other input needs a grad."""
    a = _ANCHORS.get(device)
    if a is None:
        a = torch.zeros((), device=device, requires_grad=True)
        _ANCHORS[device] = a
    return a


PAIR_GEMM = os.environ.get("ART_B200_PAIR_GEMM", "1") != "0"
PAIR_MIN_ROWS = 1024
PAIR_MAX_CONTRACTION = int(os.environ.get("ART_B200_PAIR_MAX_K", str(1 << 30)))
# the dense LoRA rank-side products on ops/csrc/lowrank.cu (1) or cuBLAS (0);
# the MoE experts' grouped rank-side products always use the low-rank kernels
LOWRANK = os.environ.get("ART_B200_LOWRANK", "0") != "0"


def _pair_ok(x: torch.Tensor, W: torch.Tensor, bias: torch.Tensor | None, contraction: int) -> bool:
    """Calls the CTA-pair tcgen05 GEMM takes: bf16, 16-byte rows, out and in
    features multiples of 128 and enough rows to fill the GPU (decode-sized
    calls stay on cuBLAS).  Every contraction length runs on it: under the
    1 kW power cap the step time ties cuBLAS on the long ones (down
    projection, gate/up input gradient; ``ART_B200_PAIR_MAX_K`` caps it)."""
    return (PAIR_GEMM and _cuda(x) and x.dim() == 2 and x.dtype == torch.bfloat16 and W.dtype == torch.bfloat16
            and x.shape[0] >= PAIR_MIN_ROWS and W.shape[0] % 128 == 0 and W.shape[1] % 128 == 0
            and contraction <= PAIR_MAX_CONTRACTION
            and x.is_contiguous() and W.is_contiguous() and (bias is None or bias.dtype == torch.bfloat16))


class _LoRALinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, W, bias, lora, version, enabled, anchor):
        u = None
        on = enabled and lora is not None
        pair = _pair_ok(x, W, bias, W.shape[1])
        if on:
            R, K = lora.A.shape
            if _lowrank_ok(x, R):
                u = lowrank.rows(x, lora.A, (0, lora.A.stride(0), 1), R, K)  # [T, n*r]
            else:
                u = x @ lora.A.t()  # [T, n*r]
        if pair:
            # base GEMM + LoRA as one more k-block of the same accumulator
            bd_s = lora.fused_factors(version)[0] if on else None
            y = native.lib().gemm_pair(x, W, u, bd_s, bias)
        else:
            y = torch.nn.functional.linear(x, W, bias)
            if on:
                y.addmm_(u, lora.block_diag(version).t(), alpha=lora.scale)
        ctx.save_for_backward(x, W, u if u is not None else x.new_empty(0))
        ctx.lora = lora if on else None
        ctx.version = version
        ctx.pair_dgrad = _pair_ok(x, W, None, W.shape[0])
        return y

    @staticmethod
    def backward(ctx, dy):
        x, W, u = ctx.saved_tensors
        lora = ctx.lora
        dy = dy.contiguous()
        dyB = None
        if lora is not None:
            s = lora.scale
            R = lora.A.shape[0]
            if _lowrank_ok(dy, R) and _lowrank_ok(x, R):
                # the rank-side products on the low-rank kernels (ops/csrc/lowrank.cu)
                bdt = lora.block_diag_t(ctx.version)
                dyB = lowrank.rows(dy, bdt, (0, bdt.stride(0), 1), R, bdt.shape[1])  # [T, n*r]
                lowrank.wgrad(dyB, x, lora.gA, (0, lora.gA.stride(0), 1), R, x.shape[1], s)  # dA = s dyB^T x
                for k, (gB, (a, b)) in enumerate(zip(lora.gB_blocks, lora.slices)):
                    if gB is None:
                        continue
                    uk = u[:, k * lora.r : (k + 1) * lora.r]
                    dyk = dy[:, a:b]
                    if _lowrank_ok(uk, lora.r, wgrad=True) and dyk.data_ptr() % 16 == 0 and (b - a) % 8 == 0:
                        # dB_k^T (r x out_k) = s u_k^T dy_k, stored into dB_k [out_k, r]
                        lowrank.wgrad(uk, dyk, gB, (0, gB.stride(1), gB.stride(0)), lora.r, b - a, s)
                    else:
                        _accum_mm(gB, dyk.t(), uk, s)
            else:
                bd = lora.block_diag(ctx.version)
                dyB = dy @ bd  # [T, n*r]
                # dA = s * dyB^T x
                _accum_mm(lora.gA, dyB.t(), x, s)
                # dB_k = s * dy[:, slice_k]^T u[:, k-block]
                for k, (gB, (a, b)) in enumerate(zip(lora.gB_blocks, lora.slices)):
                    if gB is None:
                        continue
                    _accum_mm(gB, dy[:, a:b].t(), u[:, k * lora.r : (k + 1) * lora.r], s)
        if not ctx.needs_input_grad[0]:
            # the input needs no gradient (e.g. the first layer over the frozen
            # embedding): the LoRA gradients above are all this pass owes
            return None, None, None, None, None, None, None
        if ctx.pair_dgrad:
            # dx = dy W + (dy B) (s A): W read in its stored [out, in] layout
            at_s = lora.fused_factors(ctx.version)[1] if lora is not None else None
            dx = native.lib().gemm_pair(dy, W, dyB, at_s, None, None, False, None, True)
        else:
            dx = dy @ W
            if lora is not None:
                dx.addmm_(dyB, lora.A, alpha=lora.scale)
        return dx, None, None, None, None, None, None


def lora_linear(
    x: torch.Tensor,
    W: torch.Tensor,
    bias: torch.Tensor | None,
    lora: LoRABinding | None,
    version: int = 0,
    enabled: bool = True,
) -> torch.Tensor:
    """``y = x W^T + b + scale * (x A^T) B^T`` with frozen ``W``/``b``; the LoRA
    gradients are accumulated into ``lora.gA`` / ``lora.gB_blocks``."""
    anchor = grad_anchor(x.device) if (enabled and lora is not None) else None
    return _LoRALinear.apply(x, W, bias, lora, version, enabled, anchor)


# ---------------------------------------------------------------------------
# LM head log-probabilities
# ---------------------------------------------------------------------------


class _LMHeadLogprobs(torch.autograd.Function):
    """``log softmax(h W^T)[target]`` without the logits in memory.

    Forward: the CTA-pair tcgen05 GEMM keeps each 256x256 logits tile in TMEM
    (fp32) and its epilogue folds it into per-row online-softmax partials and
    the target logit (``lm_head_fwd``); a merge kernel gives lse, logprob and
    entropy.  Two backward modes, chosen by size (``LMHEAD_KEEP_BYTES``):
    * kept logits: the forward epilogue also stores the bf16 logits; the
      backward turns them into ``dlogits`` in place (one elementwise pass)
      and runs ``dh = dlogits W`` -- no second logits GEMM;
    * recompute: nothing of size [T, V] survives the forward; per row chunk
      the same GEMM recomputes the tiles and writes ``dlogits = g (onehot -
      softmax)`` (bf16) from its epilogue, then ``dh = dlogits W``.
    ``dh = dlogits W`` runs on the pair GEMM with ``W`` in its stored layout.
    (``dh`` cannot stay in TMEM across the vocabulary: one 128-row block of it
    is 128 x hidden fp32, several times the 512 TMEM columns.)
    Reference: the chunked logprob / entropy of
    ``src/art/trainer_rank/__init__.py:2162-2290``."""

    @staticmethod
    def forward(ctx, h, W, targets, chunk, want_entropy):
        C = native.lib()
        h = h.contiguous()
        T, V = h.shape[0], W.shape[0]
        # keep the bf16 logits for the backward when they fit the budget
        # (saves the recomputing GEMM); else recompute them tile by tile
        logits = None
        if ctx.needs_input_grad[0] and T * V * 2 <= LMHEAD_KEEP_BYTES:
            logits = torch.empty(T, V, device=h.device, dtype=h.dtype)
        lp, ent, lse = C.lm_head_fwd(h, W, targets, want_entropy, logits)
        ctx.save_for_backward(h, W, targets, lse)
        ctx.logits = logits
        ctx.chunk = chunk
        if want_entropy:
            ctx.mark_non_differentiable(ent)
            return lp, ent
        return lp, None

    @staticmethod
    def backward(ctx, glp, gent):
        C = native.lib()
        h, W, targets, lse = ctx.saved_tensors
        T, V = h.shape[0], W.shape[0]
        glp = glp.float().contiguous()
        pair_dgrad = W.shape[1] % 128 == 0
        if ctx.logits is not None:  # kept logits: gradient in place, then dh = dlogits W
            logits, ctx.logits = ctx.logits, None
            C.logits_grad_(logits, targets, lse, glp)
            return (C.gemm_pair(logits, W, b_transposed=True) if pair_dgrad else logits @ W), None, None, None, None
        dh = torch.empty_like(h)
        chunk = max(128, min(ctx.chunk, T))
        dl = torch.empty(chunk, V, device=h.device, dtype=h.dtype)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            if e - s < 128:  # a short tail: recompute over the last 128 rows, keep the new ones
                s0 = e - 128
                d = dl[:128]
                C.lm_head_grad_logits(h[s0:e], W, targets[s0:e], lse[s0:e], glp[s0:e], d)
                part = C.gemm_pair(d, W, b_transposed=True) if pair_dgrad else d @ W
                dh[s:e] = part[s - s0 :]
                continue
            d = dl[: e - s]
            C.lm_head_grad_logits(h[s:e], W, targets[s:e], lse[s:e], glp[s:e], d)
            if pair_dgrad:
                C.gemm_pair(d, W, out=dh[s:e], b_transposed=True)
            else:
                torch.mm(d, W, out=dh[s:e])
        return dh, None, None, None, None


# bf16 logits kept from the LM-head forward to its backward up to this many
# bytes per call (8192 tokens x 152k vocabulary = 2.5 GB); larger calls
# recompute the logits tiles in the backward instead
LMHEAD_KEEP_BYTES = int(float(os.environ.get("ART_B200_LMHEAD_KEEP_GB", "8")) * (1 << 30))


# the library baseline of the LM head (cuBLAS logits GEMM kept for the
# backward, separate statistics and gradient kernels): the unfused
# comparison point of the benchmark, not the default
LMHEAD_LIBRARY = os.environ.get("ART_B200_LMHEAD_LIBRARY", "0") != "0"


class _LMHeadLogprobsLibrary(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, W, targets, chunk, want_entropy):
        C = native.lib()
        T = h.shape[0]
        lp = torch.empty(T, device=h.device, dtype=torch.float32)
        ent = torch.empty(T, device=h.device, dtype=torch.float32) if want_entropy else None
        saved, lses = [], []
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            logits = h[s:e] @ W.t()
            lse, tgt, en = C.logits_stats(logits, targets[s:e], want_entropy)
            lp[s:e] = tgt - lse
            if want_entropy:
                ent[s:e] = en
            saved.append(logits)
            lses.append(lse)
        ctx.saved_logits = saved
        ctx.save_for_backward(W, targets, torch.cat(lses) if lses else lp.new_empty(0))
        ctx.chunk = chunk
        if want_entropy:
            ctx.mark_non_differentiable(ent)
        return lp, ent

    @staticmethod
    def backward(ctx, glp, gent):
        C = native.lib()
        W, targets, lse = ctx.saved_tensors
        T = targets.shape[0]
        dh = torch.empty(T, W.shape[1], device=W.device, dtype=W.dtype)
        glp = glp.float().contiguous()
        for idx, s in enumerate(range(0, T, ctx.chunk)):
            e = min(T, s + ctx.chunk)
            logits = ctx.saved_logits[idx]
            C.logits_grad_(logits, targets[s:e], lse[s:e], glp[s:e])
            torch.mm(logits, W, out=dh[s:e])
        ctx.saved_logits = None
        return dh, None, None, None, None


def _lm_head_native_ok(h: torch.Tensor, W: torch.Tensor) -> bool:
    return (_cuda(h) and h.dtype == torch.bfloat16 and W.dtype == torch.bfloat16 and W.is_contiguous()
            and W.shape[0] % 32 == 0 and W.shape[0] >= 128 and h.shape[1] % 8 == 0)


def lm_head_logprobs(
    h: torch.Tensor, W: torch.Tensor, targets: torch.Tensor, chunk: int = 4096, entropy: bool = True
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Per-row ``log softmax(h W^T)[target]`` (fp32) and entropy (no grad)."""
    if _cuda(h):
        if LMHEAD_LIBRARY:
            return _LMHeadLogprobsLibrary.apply(h, W, targets.contiguous(), chunk, entropy)
        if not _lm_head_native_ok(h, W):
            raise ValueError(f"LM head on the GPU needs bf16 operands and a vocabulary that is a multiple of 32 "
                             f"(got {h.dtype}/{W.dtype}, V={W.shape[0]})")
        T = h.shape[0]
        if T < 128:  # the tile loads want 128 rows: pad with zero rows that have no target
            hp = torch.cat([h, h.new_zeros(128 - T, h.shape[1])])
            tp = torch.cat([targets, targets.new_full((128 - T,), -1)])
            lp, ent = _LMHeadLogprobs.apply(hp, W, tp, chunk, entropy)
            return lp[:T], (ent[:T] if ent is not None else None)
        return _LMHeadLogprobs.apply(h, W, targets.contiguous(), chunk, entropy)
    logits = _acc(h @ W.t())
    lse = torch.logsumexp(logits, dim=-1)
    lp = logits.gather(-1, targets.clamp_min(0).unsqueeze(-1)).squeeze(-1) - lse
    ent = None
    if entropy:
        with torch.no_grad():
            logp = logits - lse.unsqueeze(-1)
            ent = -(logp.exp() * logp).sum(-1)
    return lp, ent


# ---------------------------------------------------------------------------
# GRPO token loss (token-level importance ratio)
# ---------------------------------------------------------------------------


def grpo_loss_config(cfg: dict[str, Any], T: int, denominator: float) -> list[float]:
    from ..loss import resolve_clip

    ppo, eps, eps_hi = resolve_clip(cfg)
    return [
        float(ppo),
        eps,
        eps_hi,
        float(cfg.get("kl_penalty_coef", 0.0) or 0.0),
        1.0 if cfg.get("kl_penalty_source", "current_learner") == "sample" else 0.0,
        float(cfg.get("truncated_importance_sampling") or 0.0),
        1.0 if cfg.get("mask_prob_ratio", False) else 0.0,
        float(cfg.get("kimi_k2_tau") or 0.0),
        float(cfg.get("max_negative_advantage_importance_sampling_weight") or 0.0),
        float(denominator),
        float(T),
    ]


class _GRPOTokenLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, newlp, oldlp, adv, w, mask, reflp, origlp, cfg):
        grad, out = native.lib().grpo_token_loss(
            newlp.contiguous(), oldlp.contiguous(), adv.contiguous(), w.contiguous(),
            mask.contiguous(), reflp, origlp, cfg
        )
        ctx.save_for_backward(grad)
        ctx.mark_non_differentiable(out)
        return out[0] / out[1], out

    @staticmethod
    def backward(ctx, gloss, gout):
        (grad,) = ctx.saved_tensors
        return grad * gloss, None, None, None, None, None, None, None


def grpo_token_loss(
    newlp: torch.Tensor,
    oldlp: torch.Tensor,
    adv: torch.Tensor,
    w: torch.Tensor,
    mask: torch.Tensor,
    reflp: torch.Tensor | None,
    origlp: torch.Tensor | None,
    cfg: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused token-level loss on 1-D aligned vectors (CUDA).  Returns
    ``(reduced_loss, stats[3] = {loss_sum, denominator, mean_kl})``."""
    return _GRPOTokenLoss.apply(newlp, oldlp, adv, w, mask, reflp, origlp, cfg)
