"""Sliding-window visibility on packed prefix-tree rows: the tightened
interval ``kend_w`` with the per-pair position check gives exactly the
windowed prefix-tree mask (reference ``src/art/megatron/prefix_tree_state.py:
67,94-102``), and the fp32 attention oracle honours windows and sinks."""

import random

import torch

from art_mlx_b200.ops import fused
from art_mlx_b200.preprocessing.prefix_tree import prefix_tree_pack, visibility_ends


def _random_pack(rng: random.Random):
    prompt = [rng.randrange(50) for _ in range(rng.randint(3, 40))]
    seqs = []
    for _ in range(rng.randint(1, 5)):
        mid = prompt[: rng.randint(1, len(prompt))] + [rng.randrange(50) for _ in range(rng.randint(0, 8))]
        seqs.append(torch.tensor(mid + [rng.randrange(50) for _ in range(rng.randint(1, 30))]))
    pack = prefix_tree_pack(seqs, max_depth=64, shareable_lengths=[len(s) - 1 for s in seqs])
    return visibility_ends(pack.group_ids, pack.parent_ids)[0], pack.position_ids[0]


def test_window_ends_give_exact_windowed_mask():
    rng = random.Random(0)
    for trial in range(200):
        kend, pos = _random_pack(rng)
        T = kend.numel()
        window = rng.choice([1, 2, 3, 5, 8, 17, 64])
        kw = fused.window_visibility_ends(pos, kend, window)
        assert bool((kw <= kend).all()) and bool((kw >= torch.arange(1, T + 1)).all())
        i = torch.arange(T).view(T, 1)
        j = torch.arange(T).view(1, T)
        near = (pos.view(T, 1).long() - pos.view(1, T).long()) < window
        exact = (j <= i) & (i < kend.long().view(1, T)) & near
        tight = (j <= i) & (i < kw.long().view(1, T)) & near
        assert torch.equal(exact, tight), trial


def test_attention_ref_window_and_sinks():
    torch.manual_seed(0)
    kend, pos = _random_pack(random.Random(3))
    T, H, D = kend.numel(), 2, 8
    q, k, v = (torch.randn(T, H, D, dtype=torch.float64) for _ in range(3))
    window = 4
    sinks = torch.randn(H, dtype=torch.float64)
    o, lse = fused.attention_ref(q, k, v, kend, 0.5, pos, window, sinks)
    for h in range(H):
        for t in range(T):
            vis = [jj for jj in range(T) if jj <= t < int(kend[jj]) and int(pos[t]) - int(pos[jj]) < window]
            s = torch.stack([(q[t, h] * k[jj, h]).sum() * 0.5 for jj in vis])
            z = torch.logsumexp(torch.cat([s, sinks[h].view(1)]), 0)
            assert torch.allclose(lse[h, t], z)
            ref = sum(torch.exp(s[n] - z) * v[jj, h] for n, jj in enumerate(vis))
            assert torch.allclose(o[t, h], ref)


def test_windowed_meta_is_cached_and_tight():
    kend, pos = _random_pack(random.Random(5))
    meta = fused.AttnMeta.build(pos, kend, torch.device("cpu"))
    w = meta.windowed(4)
    assert w is meta.windowed(4) and meta.windowed(0) is meta
    assert w.window == 4 and w.tile_pmax is not None
    assert bool((w.kend <= meta.kend).all())
