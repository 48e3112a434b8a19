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
