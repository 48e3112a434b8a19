"""Kernel microbenchmarks (CUDA-event timing) behind the performance notes.

    python -m art_mlx_b200.ops.microbench attn [--small]   # tcgen05 vs warp-level prefix-tree attention
    python -m art_mlx_b200.ops.microbench gemm             # tcgen05 GEMM (+ fused LoRA) vs cuBLAS
    python -m art_mlx_b200.ops.microbench gemm_one         # 3 pair-GEMM calls, gate_up shape (ncu target)
    python -m art_mlx_b200.ops.microbench gdn              # gated DeltaNet scan / conv kernels vs PyTorch
    python -m art_mlx_b200.ops.microbench norm             # residual-add RMSNorm: warp-per-row vs block-per-row
    python -m torch.distributed.run --nnodes 1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29533 -m art_mlx_b200.ops.microbench comm   # fused comm paths vs NCCL

Single-GPU cases: 3 warm-up calls, then the median of 5 repetitions of 5
back-to-back calls, with a 256 MiB write between repetitions to flush L2.
Multi-rank cases: 3 warm-up + 10 timed calls bracketed by barrier +
synchronize, the MAX over ranks.  Every line printed is one JSON object.
"""

from __future__ import annotations

import json
import math
import os
import sys
from typing import Callable

import torch

LINK_BPS = 770e9  # measured peer-copy bandwidth per direction per GPU
GEMM_PEAK = 1.6486e15  # measured cuBLAS bf16 burst peak (8192^3, best of 10)


def _timed(fn: Callable[[], object], reps: int = 5, inner: int = 5) -> float:
    dev = torch.device("cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(3):
        fn()
    ts = []
    for _ in range(reps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(inner):
            fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b) / inner)
    ts.sort()
    return ts[len(ts) // 2]


def _emit(**kw) -> None:
    print(json.dumps(kw), flush=True)


# ---------------------------------------------------------------------------
def bench_attn(small: bool = False) -> None:
    from . import fused, native
    from ..preprocessing.prefix_tree import prefix_tree_pack, visibility_ends

    torch.manual_seed(0)
    n, P, Cl = (4, 512, 256) if small else (16, 1024, 512)
    p = torch.randint(0, 1000, (P,))
    seqs = [torch.cat([p, torch.randint(0, 1000, (Cl,))]) for _ in range(n)]
    pack = prefix_tree_pack(seqs, max_depth=4096, shareable_lengths=[P - 1] * n)
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    T, D, Hq, Hkv = kend.numel(), 128, 28, 4
    dev = torch.device("cuda")
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev, dtype=torch.bfloat16)
    q = qkv[:, : Hq * D].view(T, Hq, D)
    k = qkv[:, Hq * D : (Hq + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D :].view(T, Hkv, D)
    meta = fused.AttnMeta.build(torch.arange(T), kend, dev)
    C = native.lib()
    ke = kend.long()
    i = torch.arange(T).view(T, 1)
    j = torch.arange(T).view(1, T)
    pairs = int(((j <= i) & (i < ke.view(1, T))).sum())
    flops = 4 * D * Hq * pairs
    sc = 1 / math.sqrt(D)
    units_tc = fused.attention_bwd_units_tc(kend).to(dev)
    units_w = fused.attention_bwd_units(kend).to(dev)
    o, lse = C.attn_fwd(q, k, v, meta.kend, meta.tile_kmax, sc)
    do = torch.randn_like(o)
    cases = [
        ("attn_fwd_warp_mma_sync", lambda: C.attn_fwd(q, k, v, meta.kend, meta.tile_kmax, sc), flops),
        ("attn_fwd_tcgen05", lambda: C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, sc), flops),
        ("attn_bwd_warp_mma_sync", lambda: C.attn_bwd(do, q, k, v, o, lse, meta.kend, units_w, sc), 2.5 * flops),
        ("attn_bwd_tcgen05", lambda: C.attn_bwd_tc(do, q, k, v, o, lse, meta.kend, units_tc, sc), 2.5 * flops),
    ]
    for name, fn, fl in cases:
        t = _timed(fn, reps=2 if small else 5)
        _emit(case=name, T=T, visible_pairs=pairs, ms=round(t, 4), tflops=round(fl / t / 1e9, 1),
              frac_of_measured_peak=round(fl / t / 1e-3 / GEMM_PEAK, 3))
    o2, _ = C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, sc)
    g1 = C.attn_bwd(do, q, k, v, o, lse, meta.kend, units_w, sc)
    g2 = C.attn_bwd_tc(do, q, k, v, o, lse, meta.kend, units_tc, sc)
    rel = lambda a, b: float((a.float() - b.float()).norm() / b.float().norm())  # noqa: E731
    _emit(case="attn_tc_vs_warp_rel_diff", fwd=rel(o2, o), dq=rel(g2[0], g1[0]), dk=rel(g2[1], g1[1]),
          dv=rel(g2[2], g1[2]), tc_error=int(C.tc_error_code()))


def attn_diag(small: bool = False) -> None:
    """Where a forward attention CTA's cycles go on the benchmark row: the
    kernel's phase clocks (per CTA, SM cycles), as medians over CTAs."""
    from . import fused, native
    from ..preprocessing.prefix_tree import prefix_tree_pack, visibility_ends

    torch.manual_seed(0)
    n, P, Cl = (4, 512, 256) if small else (16, 1024, 512)
    p = torch.randint(0, 1000, (P,))
    seqs = [torch.cat([p, torch.randint(0, 1000, (Cl,))]) for _ in range(n)]
    pack = prefix_tree_pack(seqs, max_depth=4096, shareable_lengths=[P - 1] * n)
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    T, D, Hq, Hkv = kend.numel(), 128, 28, 4
    dev = torch.device("cuda")
    q = torch.randn(T, Hq, D, device=dev, dtype=torch.bfloat16)
    k = torch.randn(T, Hkv, D, device=dev, dtype=torch.bfloat16)
    v = torch.randn(T, Hkv, D, device=dev, dtype=torch.bfloat16)
    meta = fused.AttnMeta.build(torch.arange(T), kend, dev)
    C = native.lib()
    sc = 1 / math.sqrt(D)
    ctas = (T + 127) // 128 * Hq
    dg = torch.zeros(ctas, 96, dtype=torch.int64, device=dev)
    t_plain = _timed(lambda: C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, sc))
    t_diag = _timed(lambda: C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, sc, diag=dg))
    dg.zero_()
    C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, sc, diag=dg)
    torch.cuda.synchronize()
    d = dg.cpu().double()
    t0 = d[:, 0:1]
    ntl = d[:, 36].clamp(min=1)
    med = lambda x: round(float(x.median()), 1)  # noqa: E731
    tiles = [n for n in range(16)]
    soft = torch.stack([d[:, 3 + 2 * n] - d[:, 2 + 2 * n] for n in tiles], 1)
    gap = torch.stack([d[:, 2 + 2 * (n + 1)] - d[:, 3 + 2 * n] for n in tiles[:-1]], 1)
    valid = torch.arange(16).view(1, 16) < d[:, 36:37]
    vgap = torch.arange(15).view(1, 15) < (d[:, 36:37] - 1)
    _emit(case="attn_fwd_diag", T=T, ctas=ctas, ms_plain=round(t_plain, 4), ms_diag=round(t_diag, 4),
          tiles_per_cta=med(ntl), cycles_total=med(d[:, 46] - t0), setup=med(d[:, 1] - t0),
          first_s_issue=med(d[:, 42] - t0), first_s_ready=med(d[:, 2] - t0),
          loop=med(d[:, 34] - d[:, 2]), loop_per_tile=med((d[:, 34] - d[:, 2]) / ntl),
          softmax_per_tile=round(float(soft[valid].median()), 1),
          wait_s_per_tile=round(float(gap[vgap].median()), 1) if vgap.any() else None,
          epilogue=med(d[:, 35] - d[:, 34]), tail=med(d[:, 46] - d[:, 35]),
          mma_wait_k=med(d[:, 37] / ntl), mma_wait_s_empty=med(d[:, 38] / ntl), mma_wait_p=med(d[:, 39] / ntl),
          mma_wait_v=med(d[:, 40] / ntl), mma_wait_q=med(d[:, 41]), prod_wait_k_empty=med(d[:, 44] / ntl),
          prod_wait_v_empty=med(d[:, 45] / ntl), mma_issue_s=med(d[:, 80] / ntl), mma_issue_pv=med(d[:, 81] / ntl),
          tc_error=int(C.tc_error_code()))
    # one CTA's timeline (SM cycles from its start): MMA-thread issue ends and softmax spans per tile
    i = int(torch.argmax((d[:, 36] >= 10).double() * (d[:, 0] > 0).double()))
    row = d[i]
    rel = lambda x: int(x - row[0]) if x > 0 else None  # noqa: E731
    m = int(min(row[36].item(), 16))
    _emit(case="attn_fwd_diag_timeline", cta=i, tiles=int(row[36]), setup=rel(row[1]),
          s_issued=[rel(row[48 + n]) for n in range(m)], pv_issued=[rel(row[64 + n]) for n in range(m)],
          softmax_start=[rel(row[2 + 2 * n]) for n in range(m)], softmax_end=[rel(row[3 + 2 * n]) for n in range(m)],
          epilogue_end=rel(row[35]), end=rel(row[46]))


def attn_bwd_diag(small: bool = False) -> None:
    """Where a backward attention CTA's cycles go on the benchmark row
    (phase clocks of the diag build, medians over CTAs, SM cycles)."""
    from . import fused, native
    from ..preprocessing.prefix_tree import prefix_tree_pack, visibility_ends

    torch.manual_seed(0)
    n, P, Cl = (4, 512, 256) if small else (16, 1024, 512)
    p = torch.randint(0, 1000, (P,))
    seqs = [torch.cat([p, torch.randint(0, 1000, (Cl,))]) for _ in range(n)]
    pack = prefix_tree_pack(seqs, max_depth=4096, shareable_lengths=[P - 1] * n)
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    T, D, Hq, Hkv = kend.numel(), 128, 28, 4
    dev = torch.device("cuda")
    q = torch.randn(T, Hq, D, device=dev, dtype=torch.bfloat16)
    k = torch.randn(T, Hkv, D, device=dev, dtype=torch.bfloat16)
    v = torch.randn(T, Hkv, D, device=dev, dtype=torch.bfloat16)
    meta = fused.AttnMeta.build(torch.arange(T), kend, dev)
    C = native.lib()
    sc = 1 / math.sqrt(D)
    units = fused.attention_bwd_units_tc(kend).to(dev)
    o, lse = C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, sc)
    do = torch.randn_like(o)
    ctas = units.shape[0] * Hkv
    dg = torch.zeros(ctas, 128, dtype=torch.int64, device=dev)
    t_plain = _timed(lambda: C.attn_bwd_tc(do, q, k, v, o, lse, meta.kend, units, sc))
    t_diag = _timed(lambda: C.attn_bwd_tc(do, q, k, v, o, lse, meta.kend, units, sc, diag=dg))
    dg.zero_()
    C.attn_bwd_tc(do, q, k, v, o, lse, meta.kend, units, sc, diag=dg)
    torch.cuda.synchronize()
    d = dg.cpu().double()
    it = d[:, 2].clamp(min=1)
    med = lambda x: round(float(x.median()), 1)  # noqa: E731
    m = 16
    valid = torch.arange(m).view(1, m) < d[:, 2:3]
    soft = torch.stack([d[:, 5 + 4 * i] - d[:, 4 + 4 * i] for i in range(m)], 1)
    wdq = torch.stack([d[:, 6 + 4 * i] - d[:, 5 + 4 * i] for i in range(m)], 1)
    rdq = torch.stack([d[:, 7 + 4 * i] - d[:, 6 + 4 * i] for i in range(m)], 1)
    vn = torch.arange(m - 1).view(1, m - 1) < (d[:, 2:3] - 1)
    wsd = torch.stack([d[:, 4 + 4 * (i + 1)] - d[:, 7 + 4 * i] for i in range(m - 1)], 1)
    _emit(case="attn_bwd_diag", T=T, ctas=ctas, ms_plain=round(t_plain, 4), ms_diag=round(t_diag, 4),
          iters_per_cta=med(it), setup=med(d[:, 1] - d[:, 0]), loop_per_iter=med((d[:, 68] - d[:, 4]) / it),
          softmax=round(float(soft[valid].median()), 1), wait_dq=round(float(wdq[valid].median()), 1),
          dq_readout=round(float(rdq[valid].median()), 1),
          wait_next_s=round(float(wsd[vn].median()), 1) if vn.any() else None,
          epilogue=med(d[:, 69] - d[:, 68]), mma_wait_qdo=med(d[:, 70] / it), mma_wait_dv_done=med(d[:, 71] / it),
          mma_issue_dp=med(d[:, 72] / it), mma_wait_dq_free=med(d[:, 73] / it), mma_issue_s=med(d[:, 74] / it),
          mma_wait_ds=med(d[:, 75] / it), mma_issue_dvdk=med(d[:, 76] / it), mma_issue_dq=med(d[:, 77] / it),
          prod_wait_qdo_empty=med(d[:, 78] / it),
          softmax_to_first_ld=med(torch.stack([d[:, 80 + 2 * i] - d[:, 4 + 4 * i] for i in range(8)], 1)[:, 1:].flatten()),
          softmax_compute=med(torch.stack([d[:, 81 + 2 * i] - d[:, 80 + 2 * i] for i in range(8)], 1)[:, 1:].flatten()),
          softmax_tail=med(torch.stack([d[:, 5 + 4 * i] - d[:, 81 + 2 * i] for i in range(8)], 1)[:, 1:].flatten()),
          chunk0_math=med(torch.stack([d[:, 96 + 4 * i] - d[:, 80 + 2 * i] for i in range(8)], 1)[:, 1:].flatten()),
          chunk0_stage_wait=med(torch.stack([d[:, 97 + 4 * i] - d[:, 96 + 4 * i] for i in range(8)], 1)[:, 1:].flatten()),
          chunk0_stores=med(torch.stack([d[:, 98 + 4 * i] - d[:, 97 + 4 * i] for i in range(8)], 1)[:, 1:].flatten()),
          chunk1_all=med(torch.stack([d[:, 81 + 2 * i] - d[:, 98 + 4 * i] for i in range(8)], 1)[:, 1:].flatten()),
          tc_error=int(C.tc_error_code()))


# ---------------------------------------------------------------------------
def bench_gemm() -> None:
    from . import native

    C = native.lib()
    dev = torch.device("cuda")
    M = 9280
    shapes = [("qkv", 3584, 4608, 48), ("o", 3584, 3584, 16), ("gate_up", 3584, 37888, 32),
              ("down", 18944, 3584, 16), ("lm_head", 3584, 152064, 0)]
    for name, K, N, r in shapes:
        rows = 8192 if name == "lm_head" else M
        a = torch.randn(rows, K, device=dev, dtype=torch.bfloat16)
        b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
        fl = 2 * rows * K * N
        t_ours = _timed(lambda: C.gemm_tc(a, b, None, None, None, None, False))
        os.environ["ART_B200_PAIR_WIDE"] = "1"
        t_wide = _timed(lambda: C.gemm_pair(a, b, None, None, None, None, False))
        os.environ["ART_B200_PAIR_WIDE"] = "0"
        t_pair = _timed(lambda: C.gemm_pair(a, b, None, None, None, None, False))
        os.environ.pop("ART_B200_PAIR_WIDE")
        t_cublas = _timed(lambda: torch.matmul(a, b.t()))
        row = dict(case=f"gemm_{name}", M=rows, K=K, N=N, ours_1cta_ms=round(t_ours, 4),
                   ours_pair_ms=round(t_pair, 4), ours_wide_ms=round(t_wide, 4), cublas_ms=round(t_cublas, 4),
                   ours_wide_tflops=round(fl / t_wide / 1e9, 1),
                   ours_1cta_tflops=round(fl / t_ours / 1e9, 1), ours_pair_tflops=round(fl / t_pair / 1e9, 1),
                   cublas_tflops=round(fl / t_cublas / 1e9, 1))
        if r:
            a2 = torch.randn(rows, r, device=dev, dtype=torch.bfloat16)
            b2 = torch.randn(N, r, device=dev, dtype=torch.bfloat16)
            row["ours_1cta_lora_ms"] = round(_timed(lambda: C.gemm_tc(a, b, a2, b2, None, None, False)), 4)
            row["ours_pair_lora_ms"] = round(_timed(lambda: C.gemm_pair(a, b, a2, b2, None, None, False)), 4)
            row["cublas_lora_ms"] = round(_timed(lambda: torch.addmm(torch.matmul(a, b.t()), a2, b2.t())), 4)
        if r:
            # input-gradient form: dx = dy W (+ (dy B) (s A)), W in its stored [N, K] layout
            dy = torch.randn(rows, N, device=dev, dtype=torch.bfloat16)
            dyb = torch.randn(rows, r, device=dev, dtype=torch.bfloat16)
            at = torch.randn(K, r, device=dev, dtype=torch.bfloat16)
            A = at.t().contiguous()
            row["dgrad_pair_ms"] = round(_timed(lambda: C.gemm_pair(dy, b, None, None, None, None, False, None, True)), 4)
            row["dgrad_cublas_ms"] = round(_timed(lambda: torch.matmul(dy, b)), 4)
            row["dgrad_pair_lora_ms"] = round(_timed(lambda: C.gemm_pair(dy, b, dyb, at, None, None, False, None, True)), 4)
            row["dgrad_cublas_lora_ms"] = round(_timed(lambda: torch.matmul(dy, b).addmm_(dyb, A)), 4)
        diff = (C.gemm_pair(a, b, None, None, None, None, False).float() - torch.matmul(a, b.t()).float())
        row["pair_vs_cublas_rel"] = float(diff.norm() / torch.matmul(a, b.t()).float().norm())
        row["tc_error"] = int(C.tc_error_code())
        _emit(**row)


def bench_lmhead() -> None:
    """LM head of the benchmark (8192 rows x 3584 -> 152,064 vocab): the fused
    statistics epilogue (with and without the kept bf16 logits) against the
    plain CTA-pair GEMM of the same shape, and the gradient-logits pass."""
    from . import native

    C = native.lib()
    dev = torch.device("cuda")
    T, H, V = 8192, 3584, 152064
    h = torch.randn(T, H, device=dev, dtype=torch.bfloat16)
    w = torch.randn(V, H, device=dev, dtype=torch.bfloat16) * 0.02
    tg = torch.randint(0, V, (T,), device=dev)
    logits = torch.empty(T, V, device=dev, dtype=torch.bfloat16)
    fl = 2 * T * H * V
    t_gemm = _timed(lambda: C.gemm_pair(h, w, None, None, None, None, False))
    t_stats = _timed(lambda: C.lm_head_fwd(h, w, tg, True, None))
    t_keep = _timed(lambda: C.lm_head_fwd(h, w, tg, True, logits))
    _, _, lse = C.lm_head_fwd(h, w, tg, False, None)
    g = torch.randn(T, device=dev)
    d = torch.empty(T, V, device=dev, dtype=torch.bfloat16)
    t_grad = _timed(lambda: C.lm_head_grad_logits(h, w, tg, lse, g, d))
    _emit(case="lm_head", gemm_ms=round(t_gemm, 4), stats_ms=round(t_stats, 4), stats_keep_ms=round(t_keep, 4),
          grad_logits_ms=round(t_grad, 4), stats_tflops=round(fl / t_stats / 1e9, 1), tc_error=int(C.tc_error_code()))


def gemm_one() -> None:
    """Three CTA-pair GEMM calls on the gate_up shape: a small, self-ending
    target for a one-launch profiler capture."""
    from . import native

    C = native.lib()
    dev = torch.device("cuda")
    a = torch.randn(9280, 3584, device=dev, dtype=torch.bfloat16)
    b = torch.randn(37888, 3584, device=dev, dtype=torch.bfloat16) * 0.02
    for _ in range(3):
        C.gemm_pair(a, b)
    torch.cuda.synchronize()
    _emit(case="gemm_one", tc_error=int(C.tc_error_code()))


def gemm_diag() -> None:
    """Where the pair GEMM's time goes on the gate_up shape: full kernel vs
    the mainloop alone (epilogue skipped), and the MMA thread's counters."""
    from . import native

    C = native.lib()
    dev = torch.device("cuda")
    a = torch.randn(9280, 3584, device=dev, dtype=torch.bfloat16)
    b = torch.randn(37888, 3584, device=dev, dtype=torch.bfloat16) * 0.02
    fl = 2 * 9280 * 3584 * 37888
    diag = torch.zeros(5, dtype=torch.int64, device=dev)
    t_full = _timed(lambda: C.gemm_pair(a, b))
    t_main = _timed(lambda: C.gemm_pair_mainloop(a, b, diag))
    diag.zero_()
    C.gemm_pair_mainloop(a, b, diag)
    torch.cuda.synchronize()
    d_main = [int(x) for x in diag.tolist()]
    diag.zero_()
    C.gemm_pair(a, b, None, None, None, None, False, diag)
    torch.cuda.synchronize()
    d_full = [int(x) for x in diag.tolist()]

    def frac(d):
        tot = max(d[2], 1)
        return dict(wait_operands=round(d[0] / tot, 4), wait_accumulator=round(d[1] / tot, 4),
                    blocks_not_ready=round(d[3] / max(d[4], 1), 4))

    _emit(case="gemm_diag_gate_up", full_ms=round(t_full, 4), mainloop_ms=round(t_main, 4),
          full_tflops=round(fl / t_full / 1e9, 1), mainloop_tflops=round(fl / t_main / 1e9, 1),
          full=frac(d_full), mainloop=frac(d_main), tc_error=int(C.tc_error_code()))


def gemm_pair_vs_cublas_one() -> None:
    """Two CTA-pair GEMM calls, then two cuBLAS calls, on the gate_up shape
    (a small, self-ending target for a profiler capture of both kernels)."""
    from . import native

    C = native.lib()
    dev = torch.device("cuda")
    a = torch.randn(9280, 3584, device=dev, dtype=torch.bfloat16)
    b = torch.randn(37888, 3584, device=dev, dtype=torch.bfloat16) * 0.02
    for _ in range(2):
        C.gemm_pair(a, b)
    for _ in range(2):
        torch.matmul(a, b.t())
    torch.cuda.synchronize()
    _emit(case="gemm_pair_vs_cublas_one", tc_error=int(C.tc_error_code()))


def bench_norm() -> None:
    """Residual add + RMSNorm forward and backward on one packed row of the
    benchmark (9231 tokens x 3584): warp-per-row kernels vs the block-per-row
    ones, as achieved HBM bandwidth."""
    from . import native

    C = native.lib()
    dev = torch.device("cuda")
    T, H = 9231, 3584
    x = torch.randn(T, H, device=dev).bfloat16()
    res = torch.randn(T, H, device=dev).bfloat16()
    w = torch.ones(H, device=dev).bfloat16()
    dy = torch.randn(T, H, device=dev).bfloat16()
    dres = torch.randn(T, H, device=dev).bfloat16()
    _, xs, rstd = C.rmsnorm_fwd(x, res, w, 1e-6)
    row = T * H * 2
    for legacy in (False, True):
        tf = _timed(lambda: C.rmsnorm_fwd(x, res, w, 1e-6, legacy))
        tb = _timed(lambda: C.rmsnorm_bwd(dy, xs, w, rstd, dres, legacy))
        _emit(case="rmsnorm_block_per_row" if legacy else "rmsnorm_warp_per_row", T=T, H=H,
              fwd_ms=round(tf, 4), fwd_tbps=round(4 * row / tf / 1e9, 2),  # x, res in; y, sum out
              bwd_ms=round(tb, 4), bwd_tbps=round(4 * row / tb / 1e9, 2))  # dy, x, dres in; dx out


# ---------------------------------------------------------------------------
def bench_gdn() -> None:
    from ..models import gdn as G
    from . import gdn as gops

    dev = torch.device("cuda")
    T, H, dk, dv = 8192, 16, 128, 128  # one CP=8 slice of the hybrid config's 65536-token row
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.nn.functional.normalize(torch.randn(1, T, H, dk, device=dev, generator=g), dim=-1) / dk**0.5
    k = torch.nn.functional.normalize(torch.randn(1, T, H, dk, device=dev, generator=g), dim=-1)
    v = torch.randn(1, T, H, dv, device=dev, generator=g)
    gg = -torch.rand(1, T, H, device=dev, generator=g) * 0.2
    beta = torch.rand(1, T, H, device=dev, generator=g)
    ins = [t.requires_grad_(True) for t in (q, k, v, gg, beta)]
    up = torch.randn(1, T, H, dv, device=dev, generator=g)
    parts = G.chunk_parts(*(t.detach() for t in ins))
    nc = parts[0].shape[2]
    scan_mac = nc * H * (3 * 64 * dk * dv + 64 * 64 * dv)

    def layer_step():
        o, _ = G.delta_rule(*ins)
        (o * up).sum().backward()

    def scan_only():
        gops.scan(*parts)

    def summary_only():
        gops.summary_scan(parts[1], parts[2], parts[4], parts[5])

    t_layer = _timed(layer_step, reps=3, inner=2)
    t_scan = _timed(scan_only)
    t_summ = _timed(summary_only)
    orig = gops.scan
    gops.scan = lambda *a: gops._scan_ref(*a, None, True) if len(a) == 6 else gops._scan_ref(*a, True)
    try:
        t_layer_ref = _timed(layer_step, reps=2, inner=1)
        t_scan_ref = _timed(scan_only, reps=2, inner=1)
    finally:
        gops.scan = orig
    _emit(case="gdn_delta_rule_fwd_bwd", T=T, heads=H, dk=dk, dv=dv, kernel_ms=round(t_layer, 3),
          pytorch_loop_ms=round(t_layer_ref, 3), speedup=round(t_layer_ref / t_layer, 2))
    _emit(case="gdn_scan_fwd", kernel_ms=round(t_scan, 3), pytorch_loop_ms=round(t_scan_ref, 3),
          fp32_tflops=round(2 * scan_mac / t_scan / 1e9, 2))
    _emit(case="gdn_summary_scan", kernel_ms=round(t_summ, 3), width=dk + dv)
    # tree causal conv + SiLU, fwd + bwd, qkv channels of the hybrid layer
    Cc = 2 * H * dk + H * dv
    segs = [(0, T // 2, -1)] + [(T // 2 + i * (T // 16), T // 2 + (i + 1) * (T // 16), 0) for i in range(8)]
    prev_cpu = G.sequence_predecessors(segs, T, 4)
    succ = gops.successors(prev_cpu, dev)
    prev = prev_cpu.to(dev)
    x = torch.randn(T, Cc, device=dev).bfloat16().requires_grad_(True)
    w = (torch.randn(Cc, 4, device=dev) * 0.3).bfloat16().requires_grad_(True)
    dy = torch.randn(T, Cc, device=dev)
    t_conv = _timed(lambda: (gops.conv_silu(x, w, prev, succ) * dy).sum().backward())
    t_conv_ref = _timed(lambda: (torch.nn.functional.silu(gops._conv_ref(x, w, prev).float()) * dy).sum().backward())
    _emit(case="gdn_conv_silu_fwd_bwd", T=T, channels=Cc, kernel_ms=round(t_conv, 3),
          pytorch_ms=round(t_conv_ref, 3))


# ---------------------------------------------------------------------------
def bench_comm() -> None:
    from datetime import timedelta

    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    def timed(fn, iters=10, warm=3):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    out = []
    # DP: LoRA-grad reduce-scatter + AdamW + all-gather, Qwen2.5-7B r16
    from ..models.config import LoRASpec, get_config
    from ..models.lora import LoRAStore
    from ..models.transformer import lora_specs_for
    from ..parallel.dp import FusedDataParallel
    from ..runtime.optimizer import FlatAdamW

    specs = lora_specs_for(get_config("qwen2.5-7b"), LoRASpec(r=16, alpha=32))
    numel = LoRAStore.numel_for(specs)
    fdp = FusedDataParallel(numel, torch.bfloat16, dist.group.WORLD, dev)
    store = LoRAStore(specs, dev, torch.bfloat16, compute_buf=fdp.compute, grad_buf=fdp.grad)
    store.init_(1)
    opt = FlatAdamW(store)
    store2 = LoRAStore(specs, dev, torch.bfloat16)
    store2.init_(1)
    opt2 = FlatAdamW(store2)

    def fused_dp():
        store.grad.normal_()
        fdp.reduce_and_step(opt, 1e-5)

    def nccl_dp():
        store2.grad.normal_()
        dist.all_reduce(store2.grad)
        opt2.step(1e-5)

    gen = timed(lambda: store.grad.normal_())
    t_f, t_n = timed(fused_dp) - gen, timed(nccl_dp) - gen
    byts = (world - 1) / world * numel * (4 + 2)
    out.append(dict(path="dp_reduce_adamw_allgather", world=world, numel=numel, fused_ms=t_f, nccl_ms=t_n,
                    roofline_ms=byts / LINK_BPS * 1e3))
    # TP: AG->GEMM and GEMM->RS, Qwen3-32B shapes
    from ..parallel.tp import TPContext

    T, H = 8192, 5120
    tp = TPContext(dist.group.WORLD, dev, T, max(H, 25600 // world))
    N_col = (64 * 128 + 2 * 8 * 128) // world
    x_sh = torch.randn(T // world, H, device=dev, dtype=torch.bfloat16)
    Wc = torch.randn(N_col, H, device=dev, dtype=torch.bfloat16) * 0.02
    t_ag = timed(lambda: tp.ag_gemm(x_sh, Wc))
    t_ag_n = timed(lambda: torch.matmul(tp.all_gather(x_sh), Wc.t()))
    fl, byts = 2 * T * H * N_col, (world - 1) / world * T * H * 2
    out.append(dict(path="tp_allgather_gemm", world=world, T=T, K=H, N=N_col, fused_ms=t_ag, nccl_ms=t_ag_n,
                    roofline_ms=max(fl / GEMM_PEAK, byts / LINK_BPS) * 1e3))
    K_row = 25600 // world
    tp2 = TPContext(dist.group.WORLD, dev, T, H)
    xr = torch.randn(T, K_row, device=dev, dtype=torch.bfloat16)
    Wr = torch.randn(H, K_row, device=dev, dtype=torch.bfloat16) * 0.02
    t_rs = timed(lambda: tp2.gemm_rs(xr, Wr))
    t_rs_n = timed(lambda: tp2.reduce_scatter(torch.matmul(xr, Wr.t())))
    fl = 2 * T * K_row * H
    out.append(dict(path="tp_gemm_reducescatter", world=world, T=T, K=K_row, N=H, fused_ms=t_rs, nccl_ms=t_rs_n,
                    roofline_ms=max(fl / GEMM_PEAK, byts / LINK_BPS) * 1e3))
    # EP: dispatch / combine, Qwen3-30B-A3B shapes
    from ..parallel.ep import EPContext

    Tt, k, E, He = 8192, 8, 128, 2048
    idx = torch.randint(0, E, (Tt, k), device=dev)
    ep = EPContext(dist.group.WORLD, E, He, dev, 2 * Tt * k)
    ep_n = EPContext(dist.group.WORLD, E, He, dev, 2 * Tt * k, transport="a2a")
    h = torch.randn(Tt, He, device=dev, dtype=torch.bfloat16)
    plan, plan_n = ep.plan(idx), ep_n.plan(idx)

    def ep_roundtrip(e, pl):
        rx = e.transport.push(pl, h, None, 0)
        e.transport.publish(rx, 1)
        return e.transport.pull(pl, 1)

    t_ep = timed(lambda: ep_roundtrip(ep, plan))
    t_ep_n = timed(lambda: ep_roundtrip(ep_n, plan_n))
    byts = 2 * (world - 1) / world * Tt * k * He * 2
    out.append(dict(path="ep_dispatch_combine", world=world, tokens=Tt, topk=k, hidden=He, fused_ms=t_ep,
                    nccl_ms=t_ep_n, roofline_ms=byts / LINK_BPS * 1e3))
    # CP: gated DeltaNet summary scan + exchange (hybrid config: 16 heads, dk = dv = 128, 8192 local tokens)
    from ..models import gdn as G
    from ..ops import gdn as gops
    from ..parallel.cp import CPContext, _ArenaGather

    Hh, dk, dv, Tl = 16, 128, 128, 8192
    gen_ = torch.Generator(device=dev).manual_seed(rank)
    qq = torch.nn.functional.normalize(torch.randn(1, Tl, Hh, dk, device=dev, generator=gen_), dim=-1)
    kk = torch.nn.functional.normalize(torch.randn(1, Tl, Hh, dk, device=dev, generator=gen_), dim=-1)
    vv = torch.randn(1, Tl, Hh, dv, device=dev, generator=gen_)
    g_ = -torch.rand(1, Tl, Hh, device=dev, generator=gen_) * 0.2
    b_ = torch.rand(1, Tl, Hh, device=dev, generator=gen_)
    _, Wm, U0, _, Kd, gC = G.chunk_parts(qq, kk, vv, g_, b_)
    cpf = CPContext(dist.group.WORLD, dev)
    cpn = CPContext(dist.group.WORLD, dev, transport="nccl")
    slot = Hh * dk * (dk + dv)

    def cp_fused():
        off = cpf.exchange_region(world * slot * 4)
        s = gops.summary_scan(Wm, U0, Kd, gC, cpf.arena.table(off + rank * slot * 4))
        return _ArenaGather.apply(s, cpf, off)

    def cp_nccl():
        s = gops.summary_scan(Wm, U0, Kd, gC)
        return cpn.all_gather(s.contiguous())

    ref = cp_nccl()
    got = cp_fused()
    err = float((got - ref).abs().max())
    t_cf, t_cn = timed(cp_fused), timed(cp_nccl)
    t_scan = timed(lambda: gops.summary_scan(Wm, U0, Kd, gC))
    out.append(dict(path="cp_gdn_summary_scan_exchange", world=world, tokens=Tl, heads=Hh, fused_ms=t_cf,
                    nccl_ms=t_cn, scan_only_ms=t_scan, max_abs_diff_vs_nccl=err,
                    bytes_per_rank=slot * 4 * world))
    cpf.check()
    if rank == 0:
        for o in out:
            _emit(**o)
    if cpf.arena is not None:
        cpf.arena.close()
    dist.barrier()
    dist.destroy_process_group()


def main(argv: list[str]) -> None:
    which = argv[0] if argv else "attn"
    if which == "attn":
        bench_attn(small="--small" in argv)
    elif which == "gemm":
        bench_gemm()
    elif which == "lmhead":
        bench_lmhead()
    elif which == "gemm_one":
        gemm_one()
    elif which == "gemm_diag":
        gemm_diag()
    elif which == "attn_diag":
        attn_diag(small="--small" in argv)
    elif which == "attn_bwd_diag":
        attn_bwd_diag(small="--small" in argv)
    elif which == "gemm_pair_vs_cublas_one":
        gemm_pair_vs_cublas_one()
    elif which == "gdn":
        bench_gdn()
    elif which == "norm":
        bench_norm()
    elif which == "comm":
        bench_comm()
    else:
        raise SystemExit(f"unknown case {which!r}: attn | attn_diag | attn_bwd_diag | gemm | lmhead | gemm_one | gemm_diag | gemm_pair_vs_cublas_one | gdn | norm | comm")


if __name__ == "__main__":
    main(sys.argv[1:])
