"""tcgen05 GEMM (with the fused low-rank extension) vs an fp32 PyTorch reference."""

import pytest
import torch

from art_mlx_b200.ops import native

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.parametrize(
    "M,K,N,K2,bias,acc",
    [
        (128, 64, 256, 0, False, False),
        (300, 512, 512, 0, True, False),
        (1000, 3584, 4608, 48, True, False),
        (777, 1024, 3584, 16, False, True),
        (64, 192, 96, 8, False, False),
    ],
)
def test_gemm_tc_matches_fp32(cuda, M, K, N, K2, bias, acc):
    C = native.lib()
    torch.manual_seed(M + K + N)
    a = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=cuda, dtype=torch.bfloat16) * 0.05
    a2 = torch.randn(M, K2, device=cuda, dtype=torch.bfloat16) if K2 else None
    b2 = torch.randn(N, K2, device=cuda, dtype=torch.bfloat16) * 0.05 if K2 else None
    bb = torch.randn(N, device=cuda, dtype=torch.bfloat16) if bias else None
    out = torch.randn(M, N, device=cuda, dtype=torch.bfloat16) if acc else None
    ref = a.float() @ b.float().t()
    if K2:
        ref += a2.float() @ b2.float().t()
    if bias:
        ref += bb.float()
    if acc:
        ref += out.float()
    got = C.gemm_tc(a, b, a2, b2, bb, out, acc)
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    assert rel_err(got, ref) < 1e-2


def test_gemm_tc_repeated_calls_stable(cuda):
    C = native.lib()
    a = torch.randn(2048, 1024, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(2048, 1024, device=cuda, dtype=torch.bfloat16) * 0.05
    r0 = C.gemm_tc(a, b, None, None, None, None, False)
    for _ in range(5):
        r = C.gemm_tc(a, b, None, None, None, None, False)
        assert torch.equal(r, r0)
    assert C.tc_error_code() == 0


@pytest.mark.parametrize("E,K,N,K2,wt", [(8, 256, 512, 0, False), (16, 2048, 1536, 16, False), (4, 512, 96, 8, False),
                                         (8, 256, 512, 0, True), (16, 2048, 1536, 32, True), (4, 200, 64, 8, True)])
def test_gemm_tc_grouped_matches_fp32(cuda, E, K, N, K2, wt):
    """Per-expert rows (some experts empty, counts not multiples of 128)."""
    C = native.lib()
    g = torch.Generator().manual_seed(E * K)
    counts = [int(c) for c in torch.randint(0, 300, (E,), generator=g)]
    counts[1] = 0
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + c)
    M = offs[-1]
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    w = torch.randn(E * N, K, device=cuda, dtype=torch.bfloat16) * 0.05
    a2 = torch.randn(M, K2, device=cuda, dtype=torch.bfloat16) if K2 else None
    b2 = torch.randn(E * N, K2, device=cuda, dtype=torch.bfloat16) * 0.05 if K2 else None
    if wt:  # the same matrices handed over transposed, stacked as [E*K, N]
        wt_ = w.view(E, N, K).transpose(1, 2).contiguous().view(E * K, N)
        out = C.gemm_tc_grouped(x, wt_, offs, N, a2, b2, True)
    else:
        out = C.gemm_tc_grouped(x, w, offs, N, a2, b2)
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    ref = torch.empty(M, N, device=cuda)
    for e in range(E):
        r = slice(offs[e], offs[e + 1])
        ref[r] = x[r].float() @ w[e * N : (e + 1) * N].float().t()
        if K2:
            ref[r] += a2[r].float() @ b2[e * N : (e + 1) * N].float().t()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize(
    "M,K,N,K2,bias,acc",
    [
        (256, 64, 256, 0, False, False),
        (300, 512, 512, 0, True, False),
        (1000, 3584, 4608, 48, True, False),
        (777, 1024, 3584, 16, False, True),
        (64, 192, 96, 8, False, False),
        (2048, 2048, 800, 16, False, False),
    ],
)
@pytest.mark.parametrize("wide", ["0", "1"])
def test_gemm_pair_matches_fp32(cuda, M, K, N, K2, bias, acc, wide, monkeypatch):
    """The CTA-pair (cta_group::2) tcgen05 GEMM against an fp32 reference,
    with 256- and 512-wide tiles (ART_B200_PAIR_WIDE forces the width)."""
    monkeypatch.setenv("ART_B200_PAIR_WIDE", wide)
    C = native.lib()
    torch.manual_seed(M + K + N + 1)
    a = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=cuda, dtype=torch.bfloat16) * 0.05
    a2 = torch.randn(M, K2, device=cuda, dtype=torch.bfloat16) if K2 else None
    b2 = torch.randn(N, K2, device=cuda, dtype=torch.bfloat16) * 0.05 if K2 else None
    bb = torch.randn(N, device=cuda, dtype=torch.bfloat16) if bias else None
    out = torch.randn(M, N, device=cuda, dtype=torch.bfloat16) if acc else None
    ref = a.float() @ b.float().t()
    if K2:
        ref += a2.float() @ b2.float().t()
    if bias:
        ref += bb.float()
    if acc:
        ref += out.float()
    got = C.gemm_pair(a, b, a2, b2, bb, out, acc)
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    assert rel_err(got, ref) < 1e-2


@pytest.mark.parametrize("M,K,N,K2", [(300, 512, 256, 0), (1000, 3584, 3584, 48), (2048, 4608, 3584, 16)])
@pytest.mark.parametrize("wide", ["0", "1"])
def test_gemm_pair_transposed_b_matches_fp32(cuda, M, K, N, K2, wide, monkeypatch):
    """Input-gradient form: out = a @ bt (+ a2 @ b2^T) with bt = [K, N] row-major."""
    monkeypatch.setenv("ART_B200_PAIR_WIDE", wide)
    C = native.lib()
    torch.manual_seed(M + K + N + 2)
    a = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    bt = torch.randn(K, N, device=cuda, dtype=torch.bfloat16) * 0.05
    a2 = torch.randn(M, K2, device=cuda, dtype=torch.bfloat16) if K2 else None
    b2 = torch.randn(N, K2, device=cuda, dtype=torch.bfloat16) * 0.05 if K2 else None
    ref = a.float() @ bt.float()
    if K2:
        ref += a2.float() @ b2.float().t()
    got = C.gemm_pair(a, bt, a2, b2, None, None, False, None, True)
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    assert rel_err(got, ref) < 1e-2


@pytest.mark.parametrize("wide", ["0", "1"])
def test_gemm_pair_reduce_scatter_epilogue(cuda, wide, monkeypatch):
    """The pair GEMM's reduce-scatter epilogue: row block r of the product
    lands in destination r's slot (here local buffers stand in for the
    peers' staging arenas)."""
    monkeypatch.setenv("ART_B200_PAIR_WIDE", wide)
    C = native.lib()
    torch.manual_seed(9)
    world, rows, K, N, K2 = 3, 320, 1024, 1536, 16
    a = torch.randn(world * rows, K, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=cuda, dtype=torch.bfloat16) * 0.05
    a2 = torch.randn(world * rows, K2, device=cuda, dtype=torch.bfloat16)
    b2 = torch.randn(N, K2, device=cuda, dtype=torch.bfloat16) * 0.05
    slot = 1
    stages = [torch.zeros(2 * rows, N, device=cuda, dtype=torch.bfloat16) for _ in range(world)]
    C.gemm_pair_rs(a, b, a2, b2, [t.data_ptr() for t in stages], rows, N, slot)
    torch.cuda.synchronize()
    assert C.tc_error_code() == 0
    ref = a.float() @ b.float().t() + a2.float() @ b2.float().t()
    for r in range(world):
        assert rel_err(stages[r][slot * rows :], ref[r * rows : (r + 1) * rows]) < 1e-2
        assert not bool(stages[r][:rows].any())  # the other slot is untouched
