"""Tokenize / advantages / prefix-tree packing / packed tensor format (CPU)."""

import math
import random

import pytest
import torch

from art_mlx_b200.preprocessing.pack import (
    packed_tensors_from_dir,
    packed_tensors_from_tokenized_results,
    packed_tensors_to_dir,
)
from art_mlx_b200.preprocessing.prefix_tree import (
    dense_prefix_tree_mask,
    estimate_prefix_tree_packed_tokens,
    parse_prefix_tree_row,
    prefix_tree_pack,
    visibility_ends,
)
from art_mlx_b200.preprocessing.synthetic import synthetic_groups
from art_mlx_b200.preprocessing.tokenize import group_advantages, tokenize_trajectory_groups
from art_mlx_b200.trajectories import Trajectory, TrajectoryGroup
from art_mlx_b200.utils.group_aggregate import group_aggregate


def T(*v):
    return torch.tensor(v, dtype=torch.long)


def test_prefix_tree_pack_shares_common_prefix():
    a = T(1, 2, 3, 4, 5)
    b = T(1, 2, 3, 9, 9, 9)
    c = T(7, 8)
    p = prefix_tree_pack([a, b, c], max_depth=8)
    assert p.tokens.tolist() == [[1, 2, 3, 4, 5, 9, 9, 9, 7, 8]]
    g = p.group_ids[0].tolist()
    par = p.parent_ids[0].tolist()
    # shared root, two children pointing at it, separate root for c
    assert g[:3] == [1, 1, 1] and par[:3] == [1, 1, 1]
    assert g[3] != g[5] and par[3] == 1 and par[5] == 1
    assert g[8] == par[8]
    assert p.position_ids[0].tolist() == [0, 1, 2, 3, 4, 3, 4, 5, 0, 1]
    assert p.positions_by_sequence[1].tolist() == [0, 1, 2, 5, 6, 7]
    assert estimate_prefix_tree_packed_tokens([a, b, c], max_depth=8) == 10


def test_prefix_tree_pack_respects_shareable_lengths_and_depth0():
    a = T(1, 2, 3, 4)
    b = T(1, 2, 3, 5)
    p = prefix_tree_pack([a, b], max_depth=8, shareable_lengths=[2, 2])
    assert p.tokens.tolist() == [[1, 2, 3, 4, 3, 5]]
    p0 = prefix_tree_pack([a, b], max_depth=0)
    assert p0.tokens.tolist() == [[1, 2, 3, 4, 1, 2, 3, 5]]


def _reference_depth1_mask(group_ids, parent_ids):
    S = group_ids.shape[-1]
    causal = torch.tril(torch.ones(S, S, dtype=torch.bool))
    gm = group_ids.unsqueeze(2) == group_ids.unsqueeze(1)
    pm = parent_ids.unsqueeze(2) == group_ids.unsqueeze(1)
    return causal & (gm | pm)


def test_visibility_interval_matches_group_parent_mask_for_depth1():
    random.seed(0)
    prompt = [random.randrange(100) for _ in range(20)]
    seqs = [torch.tensor(prompt + [random.randrange(100) for _ in range(7)]) for _ in range(5)]
    p = prefix_tree_pack(seqs, max_depth=64, shareable_lengths=[19] * 5)
    kend = visibility_ends(p.group_ids, p.parent_ids)
    ours = dense_prefix_tree_mask(kend)
    ref = _reference_depth1_mask(p.group_ids, p.parent_ids)
    assert torch.equal(ours, ref)


def test_visibility_handles_nested_trees():
    # two-level tree: root -> mid -> {leaf1, leaf2}; keys of root visible to leaves
    seqs = [T(1, 2, 3, 4, 5, 6), T(1, 2, 3, 4, 7, 8), T(1, 2, 9, 9)]
    p = prefix_tree_pack(seqs, max_depth=8)
    segs = parse_prefix_tree_row(p.group_ids[0], p.parent_ids[0])
    assert [len(s.ancestors) for s in segs] == [0, 1, 2, 2, 1]
    m = dense_prefix_tree_mask(visibility_ends(p.group_ids, p.parent_ids))[0]
    # every query of a packed sequence sees exactly its own prefix
    for k, pos in enumerate(p.positions_by_sequence):
        pos = pos.tolist()
        for qi, q in enumerate(pos):
            visible = set(m[q].nonzero().flatten().tolist())
            assert visible == set(pos[: qi + 1])


def _choice_groups():
    return synthetic_groups(num_groups=3, rollouts_per_group=4, prompt_len=10, completion_len=5, vocab_size=50, seed=1)


def test_group_advantages_match_reference_formula():
    r = [1.0, 0.0, 0.5, 0.5]
    mean = sum(r) / 4
    std = math.sqrt(sum((x - mean) ** 2 for x in r) / 4)
    assert group_advantages(r, True) == [(x - mean) / (std + 1e-6) for x in r]
    assert group_advantages(r, False) == [x - mean for x in r]


def test_tokenize_prompt_length_weights_and_dropping():
    groups = _choice_groups()
    groups[0].trajectories[0].reward = groups[0].trajectories[1].reward  # keep variety
    flat = [TrajectoryGroup([Trajectory(messages_and_choices=t.messages_and_choices, reward=1.0) for t in groups[2]])]
    res = list(tokenize_trajectory_groups(None, groups[:2] + flat, False, True, rng=random.Random(0)))
    # the all-equal-reward group produces no results (zero advantages dropped)
    assert len(res) == 8
    for r in res:
        assert r.prompt_length == 9  # common prefix 10 capped before first sampled token, minus one
        assert abs(r.weight - 1 / 5) < 1e-5
        assert len(r.token_ids) == 15 and sum(r.assistant_mask) == 5


def test_pack_normalisations_and_disk_roundtrip(tmp_path):
    groups = _choice_groups()
    res = list(tokenize_trajectory_groups(None, groups, False, True, rng=random.Random(0)))
    p = packed_tensors_from_tokenized_results(res, 128, rng=random.Random(0))
    m = p["assistant_mask"]
    assert torch.allclose(p["weights"][m].mean(), torch.tensor(1.0))
    assert torch.allclose((p["advantages"][m].abs() * p["weights"][m]).mean(), torch.tensor(1.0), atol=1e-5)
    assert (p["weights"][~m] == 0).all() and (p["advantages"][~m] == 0).all()
    assert torch.isnan(p["logprobs"][~m]).all()
    # each group's 4 completions share one 9-token prompt segment
    assert int((p["group_ids"] >= 0).sum()) == 3 * (9 + 4 * 6)
    disk = packed_tensors_to_dir(p, str(tmp_path / "t"))
    q = packed_tensors_from_dir(**disk)
    for k in ("tokens", "group_ids", "parent_ids", "input_pos", "assistant_mask", "advantages", "weights"):
        assert torch.equal(q[k], p[k])
    assert torch.equal(torch.isnan(q["logprobs"]), torch.isnan(p["logprobs"]))


def test_pack_refuses_to_share_trainable_tokens():
    from art_mlx_b200.preprocessing.tokenize import TokenizedResult

    a = TokenizedResult(advantage=1.0, token_ids=[1, 2, 3], input_pos=[0, 1, 2], assistant_mask=[0, 1, 1],
                        logprobs=[float("nan"), -1.0, -1.0], weight=0.5, prompt_length=1)
    b = TokenizedResult(advantage=-1.0, token_ids=[1, 2, 4], input_pos=[0, 1, 2], assistant_mask=[0, 1, 1],
                        logprobs=[float("nan"), -1.0, -1.0], weight=0.5, prompt_length=1)
    p = packed_tensors_from_tokenized_results([a, b], 16)
    # shareable length is min(prompt_length, first_trainable - 1) = 0: nothing shared
    assert int((p["group_ids"] >= 0).sum()) == 6


@pytest.mark.parametrize("reduce", ["sum", "mean", "var", "std", "count", "min", "max"])
def test_group_aggregate_matches_naive(reduce):
    torch.manual_seed(0)
    v = torch.randn(3, 20)
    by = torch.randint(0, 4, (3, 20))
    out = group_aggregate(v, by=by, reduce=reduce)
    for b in range(3):
        for g in by[b].unique():
            sel = v[b][by[b] == g]
            n = sel.numel()
            if reduce == "sum":
                e = sel.sum()
            elif reduce == "mean":
                e = sel.sum() / (n + 1e-8)
            elif reduce == "count":
                e = torch.tensor(float(n))
            elif reduce == "min":
                e = sel.min()
            elif reduce == "max":
                e = sel.max()
            else:
                mean = sel.sum() / (n + 1e-8)
                var = torch.clamp((sel * sel).sum() / (n + 1e-8) - mean * mean, min=0)
                e = var if reduce == "var" else torch.sqrt(var + 1e-8)
            assert torch.allclose(out[b][by[b] == g], e.expand(n), atol=1e-5)


def test_pad_groups_aligns_each_group():
    from art_mlx_b200.models.moe import pad_groups

    x = torch.arange(11, dtype=torch.float32).view(11, 1)
    out, pc = pad_groups(x, [3, 0, 8])
    assert pc == [8, 0, 8]
    assert out.shape[0] == 16
    assert out[:3, 0].tolist() == [0, 1, 2] and out[3:8].abs().sum() == 0
    assert out[8:, 0].tolist() == list(range(3, 11))
    # weight-gradient of padded groups equals the unpadded per-group products
    a = torch.randn(11, 4)
    b = torch.randn(11, 5)
    ap, pcs = pad_groups(a, [3, 0, 8])
    bp, _ = pad_groups(b, [3, 0, 8])
    s0 = 0
    for e, (c, p) in enumerate(zip([3, 0, 8], pcs)):
        ref = a[sum([3, 0, 8][:e]) : sum([3, 0, 8][:e]) + c].t() @ b[sum([3, 0, 8][:e]) : sum([3, 0, 8][:e]) + c]
        got = ap[s0 : s0 + p].t() @ bp[s0 : s0 + p]
        assert torch.allclose(ref, got)
        s0 += p


def test_row_assignment_matches_planning_every_candidate_row():
    """The packer's length-bound shortcut takes the same row decisions as
    re-planning the prefix tree of every candidate row."""
    import math
    import random as _random

    from art_mlx_b200.preprocessing import pack as P
    from art_mlx_b200.preprocessing.tokenize import TokenizedResult

    rng = _random.Random(0)
    for trial in range(30):
        seq_len = rng.choice([48, 64, 96])
        results = []
        for g in range(rng.randint(1, 6)):
            prompt = [rng.randrange(2, 50) for _ in range(rng.randint(1, 30))]
            for _ in range(rng.randint(1, 6)):
                comp = [rng.randrange(2, 50) for _ in range(rng.randint(1, 40))]
                n = len(prompt)
                results.append(TokenizedResult(
                    advantage=rng.uniform(-1, 1), token_ids=prompt + comp, input_pos=list(range(n + len(comp))),
                    assistant_mask=[0] * n + [1] * len(comp), logprobs=[math.nan] * n + [-1.0] * len(comp),
                    weight=1.0, prompt_id=g, prompt_length=n))
        got = P.packed_tensors_from_tokenized_results(results, seq_len, rng=_random.Random(trial))
        rows = [[]]
        for r in results:
            it = P._item(r, seq_len)
            if rows[-1] and P._row_len([*rows[-1], it], seq_len) > seq_len:
                rows.append([])
            rows[-1].append(it)
        _random.Random(trial).shuffle(rows)
        ref = P._padded([P._pack_row(row, seq_len, True)["tokens"] for row in rows], seq_len, -100, torch.long)
        assert torch.equal(got["tokens"], ref), trial


def test_pad_packed_length_keeps_rows_inert():
    import random as _r

    from art_mlx_b200.preprocessing.pack import packed_tensors_from_tokenized_results
    from art_mlx_b200.preprocessing.synthetic import synthetic_groups
    from art_mlx_b200.preprocessing.tokenize import tokenize_trajectory_groups
    from art_mlx_b200.runtime.trainer import pad_packed_length

    groups = synthetic_groups(num_groups=2, rollouts_per_group=3, prompt_len=30, completion_len=9, vocab_size=99, seed=1)
    res = list(tokenize_trajectory_groups(None, groups, False, True, rng=_r.Random(0)))
    p = packed_tensors_from_tokenized_results(res, 100, rng=_r.Random(0))
    q = pad_packed_length(p, 128)
    assert q["tokens"].shape[1] == 128 and torch.equal(q["tokens"][:, :100], p["tokens"])
    assert bool((q["group_ids"][:, 100:] == -1).all()) and not bool(q["assistant_mask"][:, 100:].any())
    assert float(q["assistant_mask"].sum()) == float(p["assistant_mask"].sum())
