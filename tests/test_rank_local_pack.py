"""A data-parallel rank may fill only the rows it trains: the filled rows,
the normalised weights / advantages and the step's scored-token count are the
same as those of the full pack."""

import random

import torch

from art_mlx_b200.preprocessing.pack import packed_tensors_from_tokenized_results
from art_mlx_b200.preprocessing.synthetic import synthetic_groups
from art_mlx_b200.preprocessing.tokenize import tokenize_trajectory_groups


def _results():
    groups = synthetic_groups(num_groups=6, rollouts_per_group=4, prompt_len=40, completion_len=17,
                              vocab_size=500, seed=3, reward="bernoulli")
    return list(tokenize_trajectory_groups(None, groups, False, True, rng=random.Random(1)))


def test_rank_rows_match_full_pack():
    res = _results()
    for balance in (0.0, 0.3, -0.2):
        full = packed_tensors_from_tokenized_results(res, 128, rng=random.Random(2), advantage_balance=balance)
        n = full["tokens"].shape[0]
        total = float(full["assistant_mask"][:, 1:].sum())
        for rank, world in ((0, 2), (1, 2), (2, 4)):
            part = packed_tensors_from_tokenized_results(
                res, 128, rng=random.Random(2), advantage_balance=balance,
                rows_needed=lambda n_rows, r=rank, w=world: set(range(n_rows)[r::w]))
            assert part["tokens"].shape == full["tokens"].shape
            assert part["trainable_tokens"] == total
            for row in range(n):
                if row % world != rank:
                    assert not bool(part["assistant_mask"][row].any())
                    continue
                for key in ("tokens", "group_ids", "parent_ids", "input_pos", "assistant_mask"):
                    assert torch.equal(part[key][row], full[key][row]), key
                for key in ("advantages", "weights"):
                    assert torch.allclose(part[key][row], full[key][row], rtol=1e-5, atol=1e-6), key
