"""Packed prefix-tree rows compute exactly what independent sequences compute
(the invariant behind shared-prompt packing; reference
``tests/unit/test_prefix_tree_grad_parity.py``)."""

import torch

from art_mlx_b200.models.config import LoRASpec, ModelConfig
from art_mlx_b200.models.transformer import DecoderLM
from art_mlx_b200.ops import fused
from art_mlx_b200.ops.fused import AttnMeta
from art_mlx_b200.preprocessing.prefix_tree import prefix_tree_pack, visibility_ends

CFG = ModelConfig(
    name="parity", family="qwen3", vocab_size=97, hidden_size=64, num_hidden_layers=2,
    num_attention_heads=4, num_key_value_heads=2, head_dim=16, intermediate_size=96, qk_norm=True,
)


def _logprobs(model, tokens, positions, kend):
    meta = AttnMeta.build(positions, kend, torch.device("cpu"))
    h = model.forward(tokens, meta)
    sel = torch.arange(tokens.numel() - 1)
    lp, _ = fused.lm_head_logprobs(h[sel], model.lm_head, tokens[1:], entropy=False)
    return lp


def test_packed_tree_matches_independent_sequences():
    torch.manual_seed(0)
    model = DecoderLM(CFG, LoRASpec(r=4, alpha=8), "cpu", dtype=torch.float64, seed=0)
    # give B non-zero values so the adapter participates
    model.store.master.normal_(0, 0.05)
    model.store.sync_compute()
    prompt = torch.randint(0, 97, (11,))
    seqs = [torch.cat([prompt, torch.randint(0, 97, (n,))]) for n in (5, 8, 3)]
    pack = prefix_tree_pack(seqs, max_depth=16, shareable_lengths=[10, 10, 10])
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    toks = pack.tokens[0]
    meta = AttnMeta.build(pack.position_ids[0], kend, torch.device("cpu"))
    h = model.forward(toks, meta)
    logits = h @ model.lm_head.t()
    logp = torch.log_softmax(logits, -1)
    for k, s in enumerate(seqs):
        pos = pack.positions_by_sequence[k]
        ind = _logprobs(model, s, torch.arange(s.numel()), torch.full((s.numel(),), s.numel(), dtype=torch.int32))
        # packed: position pos[t] predicts the sequence's token t+1
        packed_lp = logp[pos[:-1], s[1:]]
        assert torch.allclose(packed_lp, ind, atol=1e-10, rtol=0)


def test_lora_grads_match_between_packed_and_independent():
    torch.manual_seed(1)
    spec = LoRASpec(r=4, alpha=8)
    m1 = DecoderLM(CFG, spec, "cpu", dtype=torch.float64, seed=0)
    m2 = DecoderLM(CFG, spec, "cpu", dtype=torch.float64, seed=0)
    vals = torch.randn(m1.store.numel, dtype=torch.float32) * 0.05
    for m in (m1, m2):
        m.store.master.copy_(vals)
        m.store.sync_compute()
    prompt = torch.randint(0, 97, (9,))
    seqs = [torch.cat([prompt, torch.randint(0, 97, (n,))]) for n in (4, 6)]
    # packed
    pack = prefix_tree_pack(seqs, max_depth=16, shareable_lengths=[8, 8])
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    meta = AttnMeta.build(pack.position_ids[0], kend, torch.device("cpu"))
    h = m1.forward(pack.tokens[0], meta)
    logp = torch.log_softmax(h @ m1.lm_head.t(), -1)
    total = 0
    for k, s in enumerate(seqs):
        pos = pack.positions_by_sequence[k]
        total = total + logp[pos[8:-1], s[9:]].sum()  # completion tokens only
    total.backward()
    # independent
    tot2 = 0
    for s in seqs:
        L = s.numel()
        meta = AttnMeta.build(torch.arange(L), torch.full((L,), L, dtype=torch.int32), torch.device("cpu"))
        h = m2.forward(s, meta)
        lp = torch.log_softmax(h @ m2.lm_head.t(), -1)
        tot2 = tot2 + lp[torch.arange(8, L - 1), s[9:]].sum()
    tot2.backward()
    # the fp32 gradient buffer accumulates fp64 products: agreement to fp32 rounding
    err = (m1.store.grad - m2.store.grad).norm() / m2.store.grad.norm()
    assert err < 1e-6, err
    assert m1.store.grad.abs().sum() > 0
