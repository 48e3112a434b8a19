"""tcgen05 / TMEM attention forward (ops/csrc/attention_tc.cu) against the
fp32 PyTorch reference of the prefix-tree mask."""

import math

import pytest
import torch

from art_mlx_b200.ops import fused, native
from art_mlx_b200.preprocessing.prefix_tree import prefix_tree_pack, visibility_ends

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _tree_kend(n_completions, prompt, comp):
    p = torch.randint(0, 1000, (prompt,))
    seqs = [torch.cat([p, torch.randint(0, 1000, (comp,))]) for _ in range(n_completions)]
    pack = prefix_tree_pack(seqs, max_depth=4096, shareable_lengths=[prompt - 1] * n_completions)
    return visibility_ends(pack.group_ids, pack.parent_ids)[0]


def _ref_rows(q, k, v, kend, scale, q_off):
    Tq, Hq, D = q.shape
    Tk = k.shape[0]
    G = Hq // k.shape[1]
    kx = k.float().repeat_interleave(G, 1)
    vx = v.float().repeat_interleave(G, 1)
    s = torch.einsum("ihd,jhd->hij", q.float(), kx) * scale
    i = (torch.arange(Tq, device=q.device) + q_off).view(Tq, 1)
    j = torch.arange(Tk, device=q.device).view(1, Tk)
    mask = (j <= i) & (i < kend.long().view(1, Tk))
    s = s.masked_fill(~mask.unsqueeze(0), float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.einsum("hij,jhd->ihd", torch.softmax(s, -1).nan_to_num(0.0), vx)
    return o, lse


@pytest.mark.parametrize("shape", [(3, 200, 90, 4, 2), (5, 130, 64, 8, 1), (1, 333, 0, 4, 4), (4, 256, 128, 2, 2)])
def test_attention_tc_fwd_matches_reference(cuda, shape):
    n, prompt, comp, Hq, Hkv = shape
    torch.manual_seed(5)
    kend = _tree_kend(n, prompt, comp)
    T, D = kend.numel(), 128
    # q/k/v as strided views of one fused projection, like the model's
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=cuda, dtype=torch.bfloat16) * 2
    q = qkv[:, : Hq * D].view(T, Hq, D)
    k = qkv[:, Hq * D : (Hq + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D :].view(T, Hkv, D)
    meta = fused.AttnMeta.build(torch.arange(T), kend, cuda)
    scale = 1 / math.sqrt(D)
    C = native.lib()
    o, lse = C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, scale)
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    orf, lser = _ref_rows(q, k, v, meta.kend, scale, 0)
    assert rel_err(o, orf) < 1e-2
    fin = torch.isfinite(lser)
    assert torch.allclose(lse[fin], lser[fin], atol=2e-2, rtol=1e-3)
    assert bool(torch.isinf(lse[~fin]).all())
    # same numbers as the warp-level kernel
    o2, lse2 = C.attn_fwd(q, k, v, meta.kend, meta.tile_kmax, scale)
    assert rel_err(o, o2) < 1e-2


def test_attention_tc_fwd_query_offset(cuda):
    """Local queries at a global offset (context-parallel slice) against all keys."""
    torch.manual_seed(6)
    kend = _tree_kend(4, 300, 100)
    T, D, Hq, Hkv = kend.numel(), 128, 4, 2
    T = T // 128 * 128
    kend = kend[:T].clamp(max=T).contiguous()
    k = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    q_all = torch.randn(T, Hq, D, device=cuda, dtype=torch.bfloat16)
    meta = fused.AttnMeta.build(torch.arange(T), kend, cuda)
    C = native.lib()
    a = T // 2
    q = q_all[a:]
    o, lse = C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, 1 / math.sqrt(D), a)
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    orf, _ = _ref_rows(q, k, v, meta.kend, 1 / math.sqrt(D), a)
    assert rel_err(o, orf) < 1e-2


def test_attention_tc_fwd_large_tree(cuda):
    """The benchmark's row shape: 1024-token prompt shared by 16 completions of 512."""
    torch.manual_seed(7)
    kend = _tree_kend(16, 1024, 512)
    T, D, Hq, Hkv = kend.numel(), 128, 28, 4
    q = torch.randn(T, Hq, D, device=cuda, dtype=torch.bfloat16)
    k = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    meta = fused.AttnMeta.build(torch.arange(T), kend, cuda)
    C = native.lib()
    o, lse = C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, 1 / math.sqrt(D))
    o2, lse2 = C.attn_fwd(q, k, v, meta.kend, meta.tile_kmax, 1 / math.sqrt(D))
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    assert rel_err(o, o2) < 1e-2
    assert torch.allclose(lse, lse2, atol=2e-2, rtol=1e-3)


@pytest.mark.parametrize("shape", [(3, 200, 90, 4, 2), (5, 130, 64, 8, 1), (4, 256, 128, 2, 2)])
def test_attention_tc_bwd_matches_reference(cuda, shape):
    n, prompt, comp, Hq, Hkv = shape
    torch.manual_seed(8)
    kend = _tree_kend(n, prompt, comp)
    T, D = kend.numel(), 128
    q = torch.randn(T, Hq, D, device=cuda, dtype=torch.bfloat16)
    k = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    meta = fused.AttnMeta.build(torch.arange(T), kend, cuda)
    scale = 1 / math.sqrt(D)
    C = native.lib()
    o, lse = C.attn_fwd(q, k, v, meta.kend, meta.tile_kmax, scale)
    do = torch.randn_like(o)
    units = fused.attention_bwd_units_tc(kend).to(cuda)
    dq, dk, dv, _ = C.attn_bwd_tc(do, q, k, v, o, lse, meta.kend, units, scale)
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    orf, _ = fused.attention_ref(qr, kr, vr, kend.to(cuda), scale)
    orf.backward(do.float())
    assert rel_err(dv, vr.grad) < 2e-2
    assert rel_err(dk, kr.grad) < 2e-2
    assert rel_err(dq, qr.grad) < 2e-2


def _tree(n_completions, prompt, comp):
    p = torch.randint(0, 1000, (prompt,))
    seqs = [torch.cat([p, torch.randint(0, 1000, (comp + 7 * i,))]) for i in range(n_completions)]
    pack = prefix_tree_pack(seqs, max_depth=4096, shareable_lengths=[prompt - 1] * n_completions)
    return visibility_ends(pack.group_ids, pack.parent_ids)[0], pack.position_ids[0].to(torch.int32)


@pytest.mark.parametrize("window,sink", [(128, False), (200, True), (0, True), (1000, True)])
def test_attention_tc_window_and_sinks(cuda, window, sink):
    """Sliding window (positions of the packed prefix tree) and attention
    sinks, forward and backward, against the fp32 dense-mask reference."""
    torch.manual_seed(11 + window)
    kend, pos = _tree(4, 300, 170)
    T, D, Hq, Hkv = kend.numel(), 128, 4, 2
    q = torch.randn(T, Hq, D, device=cuda, dtype=torch.bfloat16)
    k = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(T, Hkv, D, device=cuda, dtype=torch.bfloat16)
    sinks = (torch.randn(Hq, device=cuda) * 2).float() if sink else None
    meta = fused.AttnMeta.build(pos, kend, cuda).windowed(window)
    scale = 1 / math.sqrt(D)
    C = native.lib()
    w = meta.window
    o, lse = C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, scale, 0,
                           meta.positions if w else None, meta.tile_pmax if w else None, w, sinks)
    do = torch.randn_like(o)
    dq, dk, dv, _ = C.attn_bwd_tc(do, q, k, v, o, lse, meta.kend, meta.bwd_units, scale, 0,
                                  meta.positions if w else None, w)
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    orf, lser = fused.attention_ref(qr, kr, vr, kend.to(cuda), scale, pos.to(cuda), window, sinks)
    assert rel_err(o, orf) < 1e-2
    assert torch.allclose(lse, lser, atol=2e-2, rtol=1e-3)
    orf.backward(do.float())
    assert rel_err(dv, vr.grad) < 2e-2
    assert rel_err(dk, kr.grad) < 2e-2
    assert rel_err(dq, qr.grad) < 2e-2
