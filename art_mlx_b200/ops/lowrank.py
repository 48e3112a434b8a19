"""Low-rank (LoRA) side products over row segments.

``rows``  : ``Y[n] = scale[n] * X[src[n]] @ W_g^T`` for the rows ``n`` of
            segment ``s`` (group ``g = groups[s]``), ``W_g`` an ``R x K``
            matrix read through strides (so a stored ``B`` can be used as
            ``B^T`` without a copy);
``wgrad`` : ``G_g(r, c) += alpha * sum_{n in s} P[n, r] * Q[n, c]`` into an
            fp32 gradient addressed through strides.

One segment covers a dense linear layer; one segment per expert covers the
grouped expert adapters of a MoE layer (rows expert-contiguous).  On CUDA
both are the kernels of ``ops/csrc/lowrank.cu``; elsewhere (CPU tests, fp32)
the same math in PyTorch.  Reference counterpart: the grouped LoRA GEMMs of
``src/art/megatron/kernels/cute_grouped_lora_quack.py:257-680``.
"""

from __future__ import annotations

from typing import Sequence

import torch

ROWS_WIDTHS = (8, 16, 24, 32, 48, 64, 96)
WGRAD_WIDTHS = (8, 16, 24, 32, 48, 64, 96, 128)


def _aligned(t: torch.Tensor) -> bool:
    return t.stride(-1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0


def _segs(n: int, counts: Sequence[int] | None, groups: Sequence[int] | None) -> tuple[list[int], list[int]]:
    if counts is None:
        return [0, n], [0]
    off = [0]
    for c in counts:
        off.append(off[-1] + int(c))
    grp = list(range(len(counts))) if groups is None else [int(g) for g in groups]
    return off, grp


def native_ok(x: torch.Tensor, R: int, widths: Sequence[int]) -> bool:
    return x.is_cuda and x.dtype == torch.bfloat16 and R in widths and _aligned(x)


def rows(
    x: torch.Tensor,
    w: torch.Tensor,
    w_strides: tuple[int, int, int],
    R: int,
    K: int,
    counts: Sequence[int] | None = None,
    groups: Sequence[int] | None = None,
    src: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``[N, R]`` rows of ``scale * x[src] @ W_g^T``; ``w_strides = (group,
    row r, column k)`` element strides of ``w``."""
    n = int(sum(counts)) if counts is not None else (int(src.numel()) if src is not None else int(x.shape[0]))
    off, grp = _segs(n, counts, groups)
    if native_ok(x, R, ROWS_WIDTHS) and K % 8 == 0 and w.dtype == torch.bfloat16 and (
            out is None or (out.stride(-1) == 1 and out.stride(0) % 2 == 0)):
        from . import native

        return native.lib().lowrank_rows(x, src, None if scale is None else scale.float().contiguous(), off, grp, w,
                                         R, w_strides[0], w_strides[1], w_strides[2], K, out)
    y = x.new_zeros(n, R) if out is None else out
    gs, rs, ks = w_strides
    for s in range(len(grp)):
        a, b = off[s], off[s + 1]
        if a == b:
            continue
        Wg = torch.as_strided(w, (R, K), (rs, ks), w.storage_offset() + grp[s] * gs)
        xs = x[src[a:b]] if src is not None else x[a:b]
        v = xs[:, :K].float() @ Wg.float().t()
        if scale is not None:
            v = v * scale[a:b].float().unsqueeze(1)
        y[a:b] = v.to(y.dtype)
    return y


def wgrad(
    p: torch.Tensor,
    q: torch.Tensor,
    g: torch.Tensor,
    g_strides: tuple[int, int, int],
    R: int,
    C: int,
    alpha: float,
    counts: Sequence[int] | None = None,
    groups: Sequence[int] | None = None,
) -> None:
    """``G_g(r, c) += alpha * sum_n p[n, r] q[n, c]`` per segment, ``G``
    fp32 with element strides ``g_strides = (group, r, c)``."""
    n = int(sum(counts)) if counts is not None else int(p.shape[0])
    off, grp = _segs(n, counts, groups)
    if (native_ok(p, R, WGRAD_WIDTHS) and q.is_cuda and q.dtype == torch.bfloat16 and _aligned(q) and C % 8 == 0
            and g.dtype == torch.float32):
        from . import native

        native.lib().lowrank_wgrad(p, q, off, grp, g, R, C, g_strides[0], g_strides[1], g_strides[2], float(alpha))
        return
    gs, rs, cs = g_strides
    for s in range(len(grp)):
        a, b = off[s], off[s + 1]
        if a == b:
            continue
        G = torch.as_strided(g, (R, C), (rs, cs), g.storage_offset() + grp[s] * gs)
        G.add_((p[a:b, :R].to(G.dtype).t() @ q[a:b, :C].to(G.dtype)), alpha=alpha)
