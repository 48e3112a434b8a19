"""Low-rank (LoRA) side-product kernels against fp32 PyTorch references.

``lowrank_rows``: per-segment ``scale * X[src] @ W_g^T`` with W read through
strides (as stored, or transposed); ``lowrank_wgrad``: per-segment
``G_g += alpha P^T Q`` into fp32, also into a transposed layout.  Segments
include empty ones and lengths that are not multiples of the 64-row tile.
"""

import pytest
import torch

from art_mlx_b200.ops import lowrank, native

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize("R", [8, 16, 24, 48, 96])
@pytest.mark.parametrize("transposed_w", [False, True])
def test_rows_matches_fp32(cuda, R, transposed_w):
    torch.manual_seed(R)
    C = native.lib()
    K = 1536 + 64
    counts = [37, 0, 128, 5, 200]
    E = len(counts)
    N = sum(counts)
    T = 300
    x = torch.randn(T, K, device=cuda, dtype=torch.bfloat16)
    src = torch.randint(0, T, (N,), device=cuda)
    scale = torch.rand(N, device=cuda) + 0.5
    if transposed_w:
        Wst = torch.randn(E, K, R, device=cuda, dtype=torch.bfloat16)  # stored [E, K, R]: use as W_g = Wst[g]^T
        W = Wst.transpose(1, 2)
        strides = (Wst.stride(0), Wst.stride(2), Wst.stride(1))
        base = Wst
    else:
        W = torch.randn(E, R, K, device=cuda, dtype=torch.bfloat16)
        strides = (W.stride(0), W.stride(1), W.stride(2))
        base = W
    y = lowrank.rows(x, base, strides, R, K, counts=counts, src=src, scale=scale)
    off = 0
    ref = torch.empty(N, R, device=cuda)
    for e, c in enumerate(counts):
        ref[off : off + c] = (x[src[off : off + c]].float() @ W[e].float().t()) * scale[off : off + c, None]
        off += c
    assert _rel(y, ref) < 1e-2
    # identity rows, one segment, written into a column slice of a wider output
    out = torch.zeros(T, 2 * R, device=cuda, dtype=torch.bfloat16)
    lowrank.rows(x, base, strides, R, K, out=out[:, R:])
    ref2 = x.float() @ W[0].float().t()
    assert _rel(out[:, R:], ref2) < 1e-2
    assert float(out[:, :R].abs().max()) == 0.0
    del C


@pytest.mark.parametrize("R", [8, 16, 32, 48, 128])
@pytest.mark.parametrize("transposed_g", [False, True])
def test_wgrad_matches_fp32(cuda, R, transposed_g):
    torch.manual_seed(100 + R)
    Cc = 768 + 40
    counts = [513, 0, 77, 2048, 9]
    E = len(counts)
    N = sum(counts)
    p = torch.randn(N, R, device=cuda, dtype=torch.bfloat16)
    q = torch.randn(N, Cc, device=cuda, dtype=torch.bfloat16)
    if transposed_g:
        G = torch.randn(E, Cc, R, device=cuda)
        G0 = G.clone()
        strides = (G.stride(0), G.stride(2), G.stride(1))
    else:
        G = torch.randn(E, R, Cc, device=cuda)
        G0 = G.clone()
        strides = (G.stride(0), G.stride(1), G.stride(2))
    lowrank.wgrad(p, q, G, strides, R, Cc, 0.5, counts=counts)
    off = 0
    for e, c in enumerate(counts):
        upd = 0.5 * (p[off : off + c].float().t() @ q[off : off + c].float())  # [R, Cc]
        exp = G0[e] + (upd.t() if transposed_g else upd)
        assert _rel(G[e], exp) < 1e-4 + (0 if c else 0), f"expert {e}"
        off += c


def test_dense_lora_linear_uses_lowrank_and_matches_fp32(cuda):
    """A LoRA projection's gradients through the low-rank kernels equal an
    fp32 autograd reference."""
    from art_mlx_b200.ops import fused

    fused.LOWRANK = True  # the dense path on the low-rank kernels for this test
    torch.manual_seed(3)
    T, Kin, out, r = 1100, 512, 768, 16
    x = torch.randn(T, Kin, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    W = (torch.randn(out, Kin, device=cuda) * 0.05).to(torch.bfloat16)
    A = (torch.randn(2 * r, Kin, device=cuda) * 0.05).to(torch.bfloat16)
    B0 = (torch.randn(512, r, device=cuda) * 0.05).to(torch.bfloat16)
    B1 = (torch.randn(256, r, device=cuda) * 0.05).to(torch.bfloat16)
    gA = torch.zeros(2 * r, Kin, device=cuda)
    gB0 = torch.zeros(512, r, device=cuda)
    gB1 = torch.zeros(256, r, device=cuda)
    lora = fused.LoRABinding(A=A, B_blocks=[B0, B1], gA=gA, gB_blocks=[gB0, gB1], slices=[(0, 512), (512, 768)],
                             r=r, scale=2.0, out_features=out)
    y = fused.lora_linear(x, W, None, lora, 0, True)
    dy = torch.randn_like(y)
    y.backward(dy)
    # fp32 reference
    xf = x.detach().float().requires_grad_(True)
    Af = A.float().requires_grad_(True)
    B0f = B0.float().requires_grad_(True)
    B1f = B1.float().requires_grad_(True)
    u = xf @ Af.t()
    yf = xf @ W.float().t() + 2.0 * torch.cat([u[:, :r] @ B0f.t(), u[:, r:] @ B1f.t()], 1)
    yf.backward(dy.float())
    assert _rel(y, yf) < 2e-2
    assert _rel(x.grad, xf.grad) < 2e-2
    assert _rel(gA, Af.grad) < 2e-2
    assert _rel(gB0, B0f.grad) < 2e-2
    assert _rel(gB1, B1f.grad) < 2e-2
