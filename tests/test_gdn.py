"""Gated DeltaNet: chunked affine form vs the token recurrence, prefix trees,
and packed-vs-independent parity of the hybrid (GDN + attention + MoE) model."""

import torch

from art_mlx_b200.models.config import LoRASpec, ModelConfig
from art_mlx_b200.models.gdn import TreePlan, causal_conv, delta_rule, delta_rule_reference, tree_delta_rule
from art_mlx_b200.models.transformer import DecoderLM
from art_mlx_b200.ops import fused
from art_mlx_b200.ops.fused import AttnMeta
from art_mlx_b200.preprocessing.prefix_tree import prefix_tree_pack, visibility_ends


def _inputs(N, L, H, dk, dv, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(N, L, H, dk, generator=g, dtype=torch.float64), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(N, L, H, dk, generator=g, dtype=torch.float64), dim=-1)
    v = torch.randn(N, L, H, dv, generator=g, dtype=torch.float64)
    gg = -torch.rand(N, L, H, generator=g, dtype=torch.float64) * 0.3
    beta = torch.rand(N, L, H, generator=g, dtype=torch.float64)
    return q, k, v, gg, beta


def test_chunked_matches_recurrence():
    q, k, v, g, b = _inputs(2, 150, 3, 16, 8)
    S0 = torch.randn(2, 3, 16, 8, dtype=torch.float64)
    o, S = delta_rule(q, k, v, g, b, S0, C=32)
    o_r, S_r = delta_rule_reference(q, k, v, g, b, S0)
    assert torch.allclose(o, o_r, atol=1e-10)
    assert torch.allclose(S, S_r, atol=1e-10)


def test_tree_delta_rule_matches_independent_sequences():
    torch.manual_seed(0)
    prompt = torch.randint(0, 50, (37,))
    seqs = [torch.cat([prompt, torch.randint(50, 99, (n,))]) for n in (21, 9, 40)]
    pack = prefix_tree_pack(seqs, max_depth=8, shareable_lengths=[36] * 3)
    T = pack.tokens.shape[1]
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    meta = AttnMeta.build(pack.position_ids[0], kend, torch.device("cpu"))
    plan = TreePlan(meta, pack.group_ids[0], pack.parent_ids[0], T)
    # per-token features derived from the token id and position so that shared
    # prefix tokens have identical inputs in every sequence
    def feats(tok, pos):
        g = torch.Generator().manual_seed(1)
        table = torch.randn(100, 2, 4 * 6 + 2, generator=g, dtype=torch.float64)
        f = table[tok, 0] + 0.01 * pos.unsqueeze(-1).double()
        q = torch.nn.functional.normalize(f[..., :12].view(-1, 2, 6), dim=-1)
        k = torch.nn.functional.normalize(f[..., 12:24].view(-1, 2, 6), dim=-1)
        v = f[..., :10].view(-1, 2, 5)
        gg = -torch.sigmoid(f[..., 24:26])
        b = torch.sigmoid(f[..., 24:26] * 0.5)
        return q, k, v, gg, b
    q, k, v, gg, b = feats(pack.tokens[0], pack.position_ids[0])
    out = tree_delta_rule(q, k, v, gg, b, plan)
    for n, s in enumerate(seqs):
        qs, ks, vs, gs, bs = feats(s, torch.arange(s.numel()))
        ref, _ = delta_rule_reference(qs[None], ks[None], vs[None], gs[None], bs[None])
        pos = pack.positions_by_sequence[n]
        assert torch.allclose(out[pos], ref[0], atol=1e-10)
    # causal conv follows the sequence into the parent segment
    x = torch.randn(T, 3, dtype=torch.float64)
    w = torch.randn(3, 4, dtype=torch.float64)
    y = causal_conv(x, w, plan.prev)
    for n, s in enumerate(seqs):
        pos = pack.positions_by_sequence[n]
        xs = x[pos]
        ref = torch.nn.functional.conv1d(xs.t()[None], w.flip(-1).flip(-1)[:, None, :], padding=3, groups=3)[0, :, : xs.shape[0]].t()
        assert torch.allclose(y[pos], ref, atol=1e-12)


HYBRID = ModelConfig(
    name="hybrid-tiny", family="qwen3_next", vocab_size=97, hidden_size=64, num_hidden_layers=4,
    num_attention_heads=4, num_key_value_heads=2, head_dim=16, intermediate_size=0, qk_norm=True,
    num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32, shared_expert_intermediate_size=32,
    full_attention_interval=4, linear_num_key_heads=2, linear_num_value_heads=2, linear_key_head_dim=16,
    linear_value_head_dim=16, attn_output_gate=True,
)


def test_hybrid_model_packed_matches_independent():
    torch.manual_seed(0)
    m = DecoderLM(HYBRID, LoRASpec(r=4, alpha=8), "cpu", dtype=torch.float64, seed=0)
    m.store.master.normal_(0, 0.05)
    m.store.sync_compute()
    prompt = torch.randint(0, 97, (23,))
    seqs = [torch.cat([prompt, torch.randint(0, 97, (n,))]) for n in (7, 12)]
    pack = prefix_tree_pack(seqs, max_depth=8, shareable_lengths=[22, 22])
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    meta = AttnMeta.build(pack.position_ids[0], kend, torch.device("cpu"))
    h = m.forward(pack.tokens[0], meta, {"group_ids": pack.group_ids[0], "parent_ids": pack.parent_ids[0]})
    logp = torch.log_softmax(h @ m.lm_head.t(), -1)
    for n, s in enumerate(seqs):
        L = s.numel()
        mi = AttnMeta.build(torch.arange(L), torch.full((L,), L, dtype=torch.int32), torch.device("cpu"))
        hi = m.forward(s, mi, {})
        ref = torch.log_softmax(hi @ m.lm_head.t(), -1)
        pos = pack.positions_by_sequence[n]
        assert torch.allclose(logp[pos[:-1], s[1:]], ref[torch.arange(L - 1), s[1:]], atol=1e-9)


def test_summary_scan_matches_composed_chunk_maps():
    from art_mlx_b200.models.gdn import chunk_parts, chunk_summaries
    from art_mlx_b200.ops.gdn import summary_scan
    from art_mlx_b200.parallel.cp import compose

    q, k, v, g, b = _inputs(2, 96, 3, 16, 8)
    _, W, U0, _, Kd, gC = chunk_parts(q, k, v, g, b, C=32)
    AB = summary_scan(W, U0, Kd, gC)
    parts = chunk_summaries(q, k, v, g, b, C=32)
    A, B = compose(parts[4], parts[5])
    assert torch.allclose(AB[..., :16], A, atol=1e-10)
    assert torch.allclose(AB[..., 16:], B, atol=1e-10)


def test_conv_successor_table_inverts_predecessors():
    from art_mlx_b200.models.gdn import sequence_predecessors
    from art_mlx_b200.ops.gdn import successors

    segs = [(0, 10, -1), (10, 12, 0), (12, 20, 0), (20, 23, 1)]
    prev = sequence_predecessors(segs, 23, 4)
    ptr, idx, tap = successors(prev, torch.device("cpu"))
    seen = set()
    for j in range(23):
        for e in range(int(ptr[j]), int(ptr[j + 1])):
            i, t = int(idx[e]), int(tap[e])
            if t == 0:
                assert i == j
            else:
                assert int(prev[i, t - 1]) == j
            seen.add((i, t))
    want = {(i, 0) for i in range(23)} | {(i, m + 1) for i in range(23) for m in range(3) if prev[i, m] >= 0}
    assert seen == want
