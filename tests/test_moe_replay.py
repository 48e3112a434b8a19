"""Routing replay: expert ids recorded in a forward pass and replayed by the
training pass give the same update as routing on the fly (same weights, so
the same experts), and the replayed rows carry per-layer expert counts
computed on the host (the single-GPU MoE path then needs no device sync)."""

import random

import numpy as np
import torch

from art_mlx_b200.models.config import LoRASpec
from art_mlx_b200.preprocessing.pack import PackedMoeRoutingReplay, packed_tensors_from_tokenized_results
from art_mlx_b200.preprocessing.synthetic import synthetic_groups
from art_mlx_b200.preprocessing.tokenize import tokenize_trajectory_groups
from art_mlx_b200.runtime.trainer import GRPOTrainer

from test_distributed import MOE_CPU


def _packed():
    groups = synthetic_groups(num_groups=3, rollouts_per_group=4, prompt_len=24, completion_len=12,
                              vocab_size=MOE_CPU.vocab_size, seed=5)
    res = list(tokenize_trajectory_groups(None, groups, False, True, rng=random.Random(0)))
    return packed_tensors_from_tokenized_results(res, 128, rng=random.Random(0))


def test_replayed_routes_match_live_routing_and_carry_host_counts():
    packed = _packed()
    dev = torch.device("cpu")
    rec_tr = GRPOTrainer(MOE_CPU, LoRASpec(r=8, alpha=16), dev, seed=0)
    rows, S = packed["tokens"].shape
    L, k = MOE_CPU.num_hidden_layers, MOE_CPU.num_experts_per_tok
    idx = torch.zeros(rows, S, L, k, dtype=torch.int64)
    mask = torch.zeros(rows, S, dtype=torch.bool)
    for r, mb in enumerate(rec_tr.stage(packed)):
        rec: dict = {}
        with torch.no_grad():
            rec_tr.model.forward(mb.tokens, mb.meta, {"record_routes": rec, "group_ids": mb.group_ids,
                                                      "parent_ids": mb.parent_ids})
        routes = torch.stack([rec[i] for i in sorted(rec)], dim=1).long()
        idx[r, : routes.shape[0]] = routes
        mask[r, : routes.shape[0]] = True
    replay = dict(packed)
    replay["moe_routing_replay"] = PackedMoeRoutingReplay(idx, mask, L, k, MOE_CPU.num_experts)

    live = GRPOTrainer(MOE_CPU, LoRASpec(r=8, alpha=16), dev, seed=0)
    m_live = live.train_step(packed, 1e-3, {}).to_host()
    rep = GRPOTrainer(MOE_CPU, LoRASpec(r=8, alpha=16), dev, seed=0)
    mbs = rep.stage(replay)
    for mb in mbs:
        assert mb.route_counts is not None and len(mb.route_counts) == L
        want = np.bincount(mb.routes[:, 0, :].reshape(-1).numpy())
        assert mb.route_counts[0] == want.tolist()
    m_rep = rep.train_step(replay, 1e-3, {}, micro_batches=mbs).to_host()
    assert torch.allclose(rep.store.master, live.store.master, atol=1e-6)
    assert abs(m_rep["loss/train"] - m_live["loss/train"]) < 1e-6


def test_shared_prefix_route_conflicts_are_counted_and_first_routes_kept():
    from art_mlx_b200.preprocessing.tokenize import TokenizedResult

    nan = float("nan")

    def res(completion, adv, routes):
        return TokenizedResult(advantage=adv, token_ids=[1, 2, 3, 4, *completion], input_pos=list(range(6)),
                               assistant_mask=[0, 0, 0, 0, 1, 1], logprobs=[nan] * 4 + [-1.0, -1.0],
                               weight=1.0, prompt_id=0, prompt_length=4, moe_routed_experts=routes)

    a = [[[0, 1], [2, 3]], [[4, 5], [6, 7]], [[0, 2], [1, 3]], [[5, 6], [7, 0]], [[1, 1], [1, 1]], [[2, 2], [2, 2]]]
    b = [r for r in a]
    b[1] = [[4, 6], [6, 7]]  # a different expert set in layer 0: a conflict
    b[2] = [[2, 0], [3, 1]]  # same sets in another order: no conflict
    b[4], b[5] = [[3, 3], [3, 3]], [[4, 4], [4, 4]]
    packed = packed_tensors_from_tokenized_results([res([5, 6], 1.0, a), res([7, 8], -1.0, b)], 16,
                                                   include_moe_routing=True, rng=random.Random(0))
    rr = packed["moe_routing_replay"]
    # the prompt is packed once except its last token, which each branch re-emits (it predicts
    # the branch's first completion token): [1 2 3 4 5 6 | 4 7 8]
    assert packed["tokens"][0, :9].tolist() == [1, 2, 3, 4, 5, 6, 4, 7, 8]
    assert rr.shared_route_tokens == 3 and rr.route_conflict_tokens == 1
    assert rr.expert_indices[0, 1].tolist() == a[1]  # the first sequence's routes are kept
    assert rr.expert_indices[0, 6].tolist() == b[3] and rr.expert_indices[0, 7].tolist() == b[4]
    assert bool(rr.token_mask[0, :9].all())
