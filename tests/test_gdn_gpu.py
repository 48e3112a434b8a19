"""Gated DeltaNet kernels on the GPU (``ops/csrc/gdn.cu``) against fp32/fp64
PyTorch references: the chunk scan (forward, backward, affine summary), the
tree causal conv + SiLU, and the whole prefix-tree delta rule."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a GPU", allow_module_level=True)

from art_mlx_b200.models.gdn import (  # noqa: E402
    TreePlan,
    chunk_parts,
    delta_rule,
    delta_rule_reference,
    sequence_predecessors,
    tree_delta_rule,
)
from art_mlx_b200.ops import gdn as gdn_ops  # noqa: E402
from art_mlx_b200.ops import native  # noqa: E402
from art_mlx_b200.ops.fused import AttnMeta  # noqa: E402
from art_mlx_b200.preprocessing.prefix_tree import prefix_tree_pack, visibility_ends  # noqa: E402

DEV = torch.device("cuda")


def _operands(N, H, nc, dk, dv, seed):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s, sc=1.0: (torch.randn(*s, generator=g, dtype=torch.float64) * sc)  # noqa: E731
    gq = r(N, H, nc, 64, dk, sc=0.1)
    W = r(N, H, nc, 64, dk, sc=0.02)
    U0 = r(N, H, nc, 64, dv)
    QKM = r(N, H, nc, 64, 64, sc=0.1)
    Kd = r(N, H, nc, 64, dk, sc=0.05)
    gC = 0.5 + 0.5 * torch.rand(N, H, nc, generator=g, dtype=torch.float64)
    S0 = r(N, H, dk, dv, sc=0.3)
    return [gq, W, U0, QKM, Kd, gC, S0]


@pytest.mark.parametrize("dk,dv", [(128, 128), (64, 96)])
def test_scan_forward_backward_matches_reference(dk, dv):
    ops = _operands(2, 3, 5, dk, dv, seed=dk + dv)
    ref_in = [t.clone().requires_grad_(True) for t in ops]
    O_r, S_r = gdn_ops._scan_ref(*ref_in, True)
    g = torch.Generator().manual_seed(7)
    dO = torch.randn(O_r.shape, generator=g, dtype=torch.float64)
    dS = torch.randn(S_r.shape, generator=g, dtype=torch.float64)
    ((O_r * dO).sum() + (S_r * dS).sum()).backward()

    gpu_in = [t.float().to(DEV).requires_grad_(True) for t in ops]
    O, S = gdn_ops.scan(*gpu_in)
    assert "gdn_scan_fwd" in dir(native.lib())
    ((O * dO.float().to(DEV)).sum() + (S * dS.float().to(DEV)).sum()).backward()
    torch.cuda.synchronize()
    rel = lambda a, b: float((a.detach().double().cpu() - b).norm() / b.norm().clamp_min(1e-30))  # noqa: E731
    assert rel(O, O_r.detach()) < 1e-5
    assert rel(S, S_r.detach()) < 1e-5
    for name, a, b in zip(["gq", "W", "U0", "QKM", "Kd", "gC", "S0"], gpu_in, ref_in):
        assert rel(a.grad, b.grad) < 1e-4, name


def test_summary_scan_matches_reference_and_composes():
    ops = _operands(1, 4, 6, 128, 64, seed=3)
    _, W, U0, _, Kd, gC, _ = ops
    ref_in = [t.clone().requires_grad_(True) for t in (W, U0, Kd, gC)]
    AB_r = gdn_ops.summary_scan(*ref_in)
    up = torch.randn(AB_r.shape, dtype=torch.float64)
    (AB_r * up).sum().backward()
    gpu_in = [t.float().to(DEV).requires_grad_(True) for t in (W, U0, Kd, gC)]
    AB = gdn_ops.summary_scan(*gpu_in)
    (AB * up.float().to(DEV)).sum().backward()
    rel = lambda a, b: float((a.detach().double().cpu() - b).norm() / b.norm().clamp_min(1e-30))  # noqa: E731
    assert rel(AB, AB_r.detach()) < 1e-5
    for a, b in zip(gpu_in, ref_in):
        assert rel(a.grad, b.grad) < 1e-4


def test_delta_rule_on_gpu_matches_token_recurrence():
    g = torch.Generator().manual_seed(0)
    N, L, H, dk, dv = 2, 200, 4, 128, 128
    q = torch.nn.functional.normalize(torch.randn(N, L, H, dk, generator=g), dim=-1) / dk**0.5
    k = torch.nn.functional.normalize(torch.randn(N, L, H, dk, generator=g), dim=-1)
    v = torch.randn(N, L, H, dv, generator=g)
    gg = -torch.rand(N, L, H, generator=g) * 0.2
    beta = torch.rand(N, L, H, generator=g)
    o_r, S_r = delta_rule_reference(q.double(), k.double(), v.double(), gg.double(), beta.double())
    o, S = delta_rule(*(t.to(DEV) for t in (q, k, v, gg, beta)))
    assert float((o.double().cpu() - o_r).abs().max()) < 2e-4
    assert float((S.double().cpu() - S_r).abs().max()) < 2e-4


def _tree():
    torch.manual_seed(0)
    prompt = torch.randint(0, 50, (150,))
    seqs = [torch.cat([prompt, torch.randint(50, 99, (n,))]) for n in (70, 9, 130)]
    pack = prefix_tree_pack(seqs, max_depth=8, shareable_lengths=[149] * 3)
    T = pack.tokens.shape[1]
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    return pack, T, kend


def test_conv_silu_matches_reference_on_a_tree():
    pack, T, kend = _tree()
    segs_plan = TreePlan(AttnMeta.build(pack.position_ids[0], kend, torch.device("cpu")), pack.group_ids[0],
                         pack.parent_ids[0], T)
    prev = segs_plan.prev
    C = 200
    g = torch.Generator().manual_seed(1)
    x = torch.randn(T, C, generator=g).bfloat16()
    w = (torch.randn(C, 4, generator=g) * 0.3).bfloat16()
    dy = torch.randn(T, C, generator=g)
    xr = x.float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    y_r = torch.nn.functional.silu(gdn_ops._conv_ref(xr, wr, prev))
    (y_r * dy).sum().backward()
    xg = x.to(DEV).requires_grad_(True)
    wg = w.to(DEV).requires_grad_(True)
    y = gdn_ops.conv_silu(xg, wg, prev.to(DEV))
    (y * dy.to(DEV)).sum().backward()
    assert float((y.cpu() - y_r.detach()).abs().max()) < 1e-4
    assert float((xg.grad.float().cpu() - xr.grad).abs().max()) < 3e-2  # dx rounded to bf16
    assert float((wg.grad.float().cpu() - wr.grad).abs().max() / wr.grad.abs().max()) < 1e-2


def test_tree_delta_rule_gradients_match_cpu():
    pack, T, kend = _tree()
    H, dk, dv = 2, 64, 64
    g = torch.Generator().manual_seed(2)
    q = torch.nn.functional.normalize(torch.randn(T, H, dk, generator=g), dim=-1) / dk**0.5
    k = torch.nn.functional.normalize(torch.randn(T, H, dk, generator=g), dim=-1)
    v = torch.randn(T, H, dv, generator=g)
    gg = -torch.rand(T, H, generator=g) * 0.3
    beta = torch.rand(T, H, generator=g)
    up = torch.randn(T, H, dv, generator=g)
    outs = {}
    for dev in ("cpu", "cuda"):
        d = torch.device(dev)
        meta = AttnMeta.build(pack.position_ids[0], kend, d)
        plan = TreePlan(meta, pack.group_ids[0], pack.parent_ids[0], T)
        ins = [t.double().to(d) if dev == "cpu" else t.to(d) for t in (q, k, v, gg, beta)]
        ins = [t.requires_grad_(True) for t in ins]
        o = tree_delta_rule(*ins, plan)
        (o * up.to(o.dtype).to(d)).sum().backward()
        outs[dev] = (o.detach().double().cpu(), [t.grad.double().cpu() for t in ins])
    o_c, g_c = outs["cpu"]
    o_g, g_g = outs["cuda"]
    assert float((o_g - o_c).abs().max()) < 2e-4
    for a, b in zip(g_g, g_c):
        assert float((a - b).norm() / b.norm()) < 1e-3
