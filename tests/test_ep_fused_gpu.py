"""The fused expert-parallel exchange on one GPU (the group of one rank pushes
to itself) against an fp32 PyTorch reference of the MoE experts with LoRA.

Exercises every piece of ``ops/csrc/ep_gemm.cu`` that does not need a second
GPU: the push warps, the per-expert arrival counters and bounded waits, the
grouped GEMM with the rank-side LoRA rows pushed alongside the token rows,
the scatter epilogue into the slot buffer with its counter, and the waiting
combine; plus the backward (dispatch of the weighted gradients, owner-side
LoRA gradients on the low-rank kernels, scatter of the input gradients).
Three exchanges in a row with different routes check the cumulative
counter targets.  The 2-GPU test in ``test_distributed.py`` covers the peer
path.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _reference(h, w, idx, P, s):
    """fp32 autograd reference; returns y and the leaf tensors."""
    leaves = {k: v.detach().float().requires_grad_(True) for k, v in P.items()}
    x = h.detach().float().requires_grad_(True)
    wf = w.detach().float().requires_grad_(True)
    T, k = idx.shape
    F = leaves["B_gu"].shape[2]
    r = leaves["B_gu"].shape[3]
    y = torch.zeros(T, x.shape[1], device=x.device)
    for e in range(leaves["gu"].shape[0]):
        tt, jj = (idx == e).nonzero(as_tuple=True)
        if tt.numel() == 0:
            continue
        xe = x[tt]
        u = xe @ leaves["A_gu"][e].t()
        gu = xe @ leaves["gu"][e] + s * torch.cat([u[:, :r] @ leaves["B_gu"][e, 0].t(),
                                                   u[:, r:] @ leaves["B_gu"][e, 1].t()], 1)
        act = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
        out = act @ leaves["dn"][e] + s * (act @ leaves["A_d"][e].t()) @ leaves["B_d"][e].t()
        y = y.index_add(0, tt, out * wf[tt, jj].unsqueeze(1))
    return y, x, wf, leaves


def test_fused_ep_single_rank_matches_fp32(cuda):
    from art_mlx_b200.models.moe import ExpertParams
    from art_mlx_b200.ops.fused import grad_anchor
    from art_mlx_b200.parallel.ep_fused import FusedEP, FusedEPExperts

    torch.manual_seed(11)
    E, H, F, r, k, T = 8, 256, 128, 8, 2, 300
    s = 2.0
    bf = torch.bfloat16
    P = {
        "gu": torch.randn(E, H, 2 * F, device=cuda) * 0.06,
        "dn": torch.randn(E, F, H, device=cuda) * 0.08,
        "A_gu": torch.randn(E, 2 * r, H, device=cuda) * 0.06,
        "B_gu": torch.randn(E, 2, F, r, device=cuda) * 0.1,
        "A_d": torch.randn(E, r, F, device=cuda) * 0.08,
        "B_d": torch.randn(E, H, r, device=cuda) * 0.1,
    }
    Pb = {kk: v.to(bf).contiguous() for kk, v in P.items()}
    g = {kk: torch.zeros(v.shape, device=cuda) for kk, v in P.items() if kk not in ("gu", "dn")}
    params = ExpertParams(Pb["gu"], Pb["dn"], Pb["A_gu"], Pb["B_gu"], Pb["A_d"], Pb["B_d"],
                          g["A_gu"], g["B_gu"], g["A_d"], g["B_d"], s)
    params.A_all_gu, params.B_all_d = Pb["A_gu"], Pb["B_d"]
    fep = FusedEP(None, E, H, cuda, capacity_rows=4096, max_slots=2048)
    for call in range(3):
        for t in g.values():
            t.zero_()
        idx = torch.stack([torch.randperm(E, device=cuda)[:k] for _ in range(T)])
        w = torch.softmax(torch.randn(T, k, device=cuda), -1)
        h = (torch.randn(T, H, device=cuda) * 0.5).to(bf).requires_grad_(True)
        wr = w.clone().requires_grad_(True)
        counts = np.bincount(idx.reshape(-1).cpu().numpy(), minlength=E).reshape(1, E)
        y = FusedEPExperts.apply(h, wr, idx, fep, params, True, counts, grad_anchor(cuda))
        dy = torch.randn_like(y)
        y.backward(dy)
        torch.cuda.synchronize()
        from art_mlx_b200.ops import native

        assert int(native.lib().tc_error_code()) == 0, "a bounded wait gave up"
        ref, x, wf, leaves = _reference(h, w, idx, Pb, s)
        ref.backward(dy.float())
        assert _rel(y, ref) < 3e-2, f"call {call}: y"
        assert _rel(h.grad, x.grad) < 3e-2, f"call {call}: dh"
        assert _rel(wr.grad, wf.grad) < 3e-2, f"call {call}: dw"
        for name in ("A_gu", "B_gu", "A_d", "B_d"):
            assert _rel(g[name], leaves[name].grad) < 3e-2, f"call {call}: d{name}"
