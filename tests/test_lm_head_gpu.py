"""Fused LM head (tcgen05 pair GEMM with softmax epilogues) against fp32 PyTorch.

The forward keeps the logits in TMEM and reduces them to per-row lse, target
logit and entropy; the backward recomputes each tile and writes only the
logits gradient.  Both are compared with the same op on fp32 tensors."""

import pytest
import torch

from art_mlx_b200.ops import fused

pytestmark = pytest.mark.gpu


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _ref(h, W, tgt):
    hf = h.detach().float().requires_grad_()
    logits = hf @ W.float().t()
    lse = torch.logsumexp(logits, -1)
    lp = logits.gather(1, tgt.clamp_min(0)[:, None])[:, 0] - lse
    lp = torch.where(tgt >= 0, lp, -lse)
    logp = logits - lse[:, None]
    ent = -(logp.exp() * logp).sum(-1)
    return hf, lp, ent


@pytest.mark.parametrize("wide", ["0", "1"])
@pytest.mark.parametrize("keep", [True, False])
@pytest.mark.parametrize("T,H,V", [(300, 256, 4096), (77, 128, 2080), (1000, 512, 32000 + 32), (4100, 3584, 152064)])
def test_lm_head_fwd_bwd_matches_fp32(cuda, T, H, V, keep, wide, monkeypatch):
    """Both backward modes (logits kept from the forward, or recomputed) and
    both tile widths of the pair GEMM."""
    monkeypatch.setattr(fused, "LMHEAD_KEEP_BYTES", 1 << 40 if keep else 0)
    monkeypatch.setenv("ART_B200_PAIR_WIDE", wide)
    torch.manual_seed(T + V)
    h = (torch.randn(T, H, device=cuda) * 0.5).to(torch.bfloat16).requires_grad_()
    W = (torch.randn(V, H, device=cuda) / H**0.5 * 2).to(torch.bfloat16)
    tgt = torch.randint(0, V, (T,), device=cuda)
    tgt[::13] = -1  # rows without a target
    lp, ent = fused.lm_head_logprobs(h, W, tgt, chunk=1024, entropy=True)
    hf, lp_r, ent_r = _ref(h, W, tgt)
    assert torch.allclose(lp, lp_r.detach(), atol=2e-3, rtol=1e-3), float((lp - lp_r).abs().max())
    assert torch.allclose(ent, ent_r.detach(), atol=5e-3, rtol=1e-3)
    g = torch.randn(T, device=cuda)
    g[::7] = 0.0
    lp.backward(g)
    lp_r.backward(g)
    assert rel_err(h.grad, hf.grad) < 2e-2


def test_lm_head_two_calls_and_no_entropy(cuda):
    torch.manual_seed(3)
    T, H, V = 513, 256, 8192
    h = torch.randn(T, H, device=cuda).to(torch.bfloat16)
    W = (torch.randn(V, H, device=cuda) / 8).to(torch.bfloat16)
    tgt = torch.randint(0, V, (T,), device=cuda)
    a, e = fused.lm_head_logprobs(h, W, tgt, entropy=False)
    b, _ = fused.lm_head_logprobs(h, W, tgt, entropy=False)
    assert e is None
    assert torch.equal(a, b)  # the partials are rewritten, nothing carries over between calls
    _, lp_r, _ = _ref(h, W, tgt)
    assert torch.allclose(a, lp_r.detach(), atol=2e-3, rtol=1e-3)
