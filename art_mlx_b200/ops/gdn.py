"""Autograd wrappers of the gated DeltaNet kernels (``csrc/gdn.cu``).

* :func:`scan` - the sequential chunk scan of the gated delta rule
  (``U = U0 - W S``, ``O = gq S + QKM U``, ``S <- gC S + Kd^T U``).  On CUDA
  the recurrences run in ``gdn_scan_fwd`` / ``gdn_scan_bwd``; the gradient
  products that contract over the value width (``dgq = dO S^T``,
  ``dW = -dU S^T``, ``dQKM = dO U^T``, ``dKd = U dS^T``, ``dgC``) are batched
  GEMMs over all chunks.  With ``peer_out`` the kernel also stores the final
  state into every listed address (the fused context-parallel summary
  exchange).  CPU tensors run the same recurrence as a Python loop.
* :func:`conv_silu` - depthwise causal conv over a packed prefix-tree row
  (each token's predecessors from a table, crossing into the parent segment)
  followed by SiLU, fp32 output; the backward gathers over a successor table
  (:func:`successors`).

Role of the reference's FLA chunked delta rule and packed varlen conv
(``src/art/megatron/gdn/fla_cp.py:143-227``, ``gdn/conv_gelu.py:72-430``).
"""

from __future__ import annotations

import numpy as np
import torch

from . import native

CHUNK = 64


def _rows(t: torch.Tensor, lead: int) -> torch.Tensor:
    """Flatten the first ``lead`` dims into one and make it contiguous fp32."""
    return t.reshape(-1, *t.shape[lead:]).float().contiguous()


class _Scan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gq, W, U0, QKM, Kd, gC, S0, want_out, peer_out):
        N, H, nc, C, dk = W.shape
        dv = U0.shape[-1]
        need = any(ctx.needs_input_grad[:7])
        args = [_rows(t, 2) for t in (gq, W, U0, QKM, Kd)] + [gC.reshape(-1, nc).float().contiguous()]
        s0 = None if S0 is None else S0.reshape(-1, dk, dv).float().contiguous()
        O, S_end, states, U = native.lib().gdn_scan_fwd(*args, s0, want_out, need, peer_out)
        ctx.shape = (N, H, nc, C, dk, dv)
        ctx.has_s0 = S0 is not None
        ctx.want_out = want_out
        if need:
            gq_, W_, _, QKM_, Kd_, gC_ = args
            ctx.save_for_backward(gq_, W_, QKM_, Kd_, gC_, states, U)
        O = O.view(N, H, nc, C, dv) if want_out else O
        if not want_out:
            ctx.mark_non_differentiable(O)
        return O, S_end.view(N, H, dk, dv)

    @staticmethod
    def backward(ctx, dO, dS_end):
        N, H, nc, C, dk, dv = ctx.shape
        gq, W, QKM, Kd, gC, states, U = ctx.saved_tensors
        R = N * H
        dO_ = dO.reshape(R, nc, C, dv).float().contiguous() if (ctx.want_out and dO is not None) else None
        dSe = dS_end.reshape(R, dk, dv).float().contiguous() if dS_end is not None else None
        dU, dSa, dS0 = native.lib().gdn_scan_bwd(dO_, dSe, gq, W, QKM, Kd, gC, dv)
        St = states.transpose(-1, -2)  # [R, nc, dv, dk]
        if dO_ is not None:
            dgq = torch.matmul(dO_, St)
            dQKM = torch.matmul(dO_, U.transpose(-1, -2))
        else:
            dgq = torch.zeros_like(gq)
            dQKM = torch.zeros_like(QKM)
        dW = torch.matmul(dU, St).neg_()
        dKd = torch.matmul(U, dSa.transpose(-1, -2))
        dgC = (states * dSa).sum((-1, -2))
        shp = lambda t, *tail: t.view(N, H, nc, *tail)  # noqa: E731
        return (shp(dgq, C, dk), shp(dW, C, dk), shp(dU, C, dv), shp(dQKM, C, C), shp(dKd, C, dk),
                dgC.view(N, H, nc), dS0.view(N, H, dk, dv) if ctx.has_s0 else None, None, None)


def _scan_ref(gq, W, U0, QKM, Kd, gC, S0, want_out):
    N, H, nc, C, dk = W.shape
    dv = U0.shape[-1]
    S = S0 if S0 is not None else W.new_zeros(N, H, dk, dv)
    outs = []
    for c in range(nc):
        U = U0[:, :, c] - W[:, :, c] @ S
        if want_out:
            outs.append(gq[:, :, c] @ S + QKM[:, :, c] @ U)
        S = gC[:, :, c, None, None] * S + Kd[:, :, c].transpose(-1, -2) @ U
    O = torch.stack(outs, dim=2) if want_out and outs else W.new_zeros(N, H, nc, C, dv)
    return (O if want_out else W.new_zeros(0)), S


def scan(gq, W, U0, QKM, Kd, gC, S0=None, want_out: bool = True, peer_out: torch.Tensor | None = None):
    """Chunk scan over ``[N, H, nc, C, *]`` operands; returns ``(O [N, H, nc,
    C, dv] (empty unless want_out), S_end [N, H, dk, dv])``."""
    if W.device.type == "cuda" and W.shape[3] == CHUNK:
        return _Scan.apply(gq, W, U0, QKM, Kd, gC, S0, want_out, peer_out)
    if peer_out is not None:
        raise ValueError("peer_out needs the CUDA scan")
    return _scan_ref(gq, W, U0, QKM, Kd, gC, S0, want_out)


def summary_scan(W, U0, Kd, gC, peer_out: torch.Tensor | None = None) -> torch.Tensor:
    """Affine summary ``[A | B]`` (``S_out = A S_in + B``) of every row's
    chunk span: the scan of the augmented state ``[I | 0]`` with ``U0``
    extended by zero columns.  Returns ``[N, H, dk, dk + dv]``."""
    N, H, nc, C, dk = W.shape
    U0a = torch.cat([U0.new_zeros(N, H, nc, C, dk), U0], dim=-1)
    eye = torch.eye(dk, device=W.device, dtype=W.dtype)
    S0a = torch.cat([eye.expand(N, H, dk, dk), W.new_zeros(N, H, dk, U0.shape[-1])], dim=-1)
    if W.device.type == "cuda" and C == CHUNK:
        dummy = W.new_zeros(N, H, nc, C, dk)
        dqkm = W.new_zeros(N, H, nc, C, C)
        return _Scan.apply(dummy, W, U0a, dqkm, Kd, gC, S0a, False, peer_out)[1]
    if peer_out is not None:
        raise ValueError("peer_out needs the CUDA scan")
    return _scan_ref(None, W, U0a, None, Kd, gC, S0a, False)[1]


# ---------------------------------------------------------------------------
# tree causal conv + SiLU
# ---------------------------------------------------------------------------


def successors(prev: torch.Tensor, device: torch.device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Inverse of a predecessor table ``prev [T, W-1]``: CSR ``(ptr [T+1],
    idx, tap)`` listing, for every token j, the tokens i that read it and at
    which tap (``tap`` = positions back, 0 = the token itself)."""
    p = prev.detach().cpu().numpy()
    T, K = p.shape
    js, is_, ts = [np.arange(T)], [np.arange(T)], [np.zeros(T, np.int8)]
    for m in range(K):
        sel = p[:, m] >= 0
        js.append(p[sel, m])
        is_.append(np.nonzero(sel)[0])
        ts.append(np.full(int(sel.sum()), m + 1, np.int8))
    j = np.concatenate(js)
    order = np.argsort(j, kind="stable")
    ptr = np.zeros(T + 1, np.int64)
    ptr[1:] = np.cumsum(np.bincount(j, minlength=T))
    idx = np.concatenate(is_)[order].astype(np.int64)
    tap = np.concatenate(ts)[order]
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device, non_blocking=True)  # noqa: E731
    return to(ptr), to(idx), to(tap)


def _conv_ref(x: torch.Tensor, w: torch.Tensor, prev: torch.Tensor) -> torch.Tensor:
    y = x * w[:, -1]
    for m in range(prev.shape[1]):
        idx = prev[:, m]
        valid = (idx >= 0).unsqueeze(1).to(x.dtype)
        y = y + x.index_select(0, idx.clamp_min(0)) * valid * w[:, -2 - m]
    return y


class _ConvSiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, prev, succ):
        xc, wc = x.contiguous(), w.to(x.dtype).contiguous()
        y = native.lib().gdn_conv_fwd(xc, wc, prev)
        ctx.save_for_backward(xc, wc, prev, *succ)
        ctx.w_dtype = w.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, prev, ptr, idx, tap = ctx.saved_tensors
        dx, dw = native.lib().gdn_conv_bwd(dy.float().contiguous(), x, w, prev, ptr, idx, tap)
        return dx, dw.to(ctx.w_dtype), None, None


def conv_silu(x: torch.Tensor, w: torch.Tensor, prev: torch.Tensor,
              succ: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    """``silu(causal_conv(x))`` in fp32; ``x [T, C]``, ``w [C, width]``,
    ``prev [T, width-1]`` (int64, -1 before a sequence start)."""
    if x.device.type == "cuda":
        if succ is None:
            succ = successors(prev, x.device)
        return _ConvSiLU.apply(x, w, prev.contiguous(), succ)
    return torch.nn.functional.silu(_conv_ref(x, w, prev).float())
