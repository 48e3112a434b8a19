"""Trainability on CPU (role of the reference's yes/no trainability suite,
``tests/integration/megatron/trainability/``, without a rollout engine): GRPO
steps on a group whose completions differ in one token must raise the
log-probability of the rewarded completion and lower the other's, through the
same packer, loss and optimizer as the benchmark step."""

import math
import random

import torch

from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.preprocessing.pack import packed_tensors_from_tokenized_results
from art_mlx_b200.preprocessing.tokenize import TokenizedResult
from art_mlx_b200.runtime.trainer import GRPOTrainer
from art_mlx_b200.runtime.trainer_rank import ForwardInput, TrainerRank

PROMPT = [5, 6, 7, 8, 9]
GOOD, BAD = 100, 200


def _result(tok: int, adv: float) -> TokenizedResult:
    n = len(PROMPT)
    return TokenizedResult(advantage=adv, token_ids=[*PROMPT, tok, 3], input_pos=list(range(n + 2)),
                           assistant_mask=[0] * n + [1, 1], logprobs=[math.nan] * (n + 2),
                           weight=1.0, prompt_id=0, prompt_length=n)


def _logprob(rank: TrainerRank, tok: int) -> float:
    with torch.no_grad():
        out = rank.forward([ForwardInput(tokens=[*PROMPT, tok], score_positions=[len(PROMPT) - 1])])
    return float(out[0].logprobs[0])


def _run(loss_fn: str) -> tuple[list[float], list[float]]:
    trainer = GRPOTrainer(get_config("tiny-qwen3"), LoRASpec(r=8, alpha=16), torch.device("cpu"), seed=0)
    rank = TrainerRank(trainer)
    group = [_result(GOOD, 1.0) for _ in range(4)] + [_result(BAD, -1.0) for _ in range(4)]
    good, bad = [_logprob(rank, GOOD)], [_logprob(rank, BAD)]
    for step in range(4):
        packed = packed_tensors_from_tokenized_results(group, 64, rng=random.Random(step))
        trainer.train_step(packed, 3e-3, {"loss_fn": loss_fn})
        good.append(_logprob(rank, GOOD))
        bad.append(_logprob(rank, BAD))
    return good, bad


def test_grpo_steps_move_probability_toward_the_rewarded_completion():
    # old logprobs are NaN (replaced by the current ones), so every step is on-policy: the ratio
    # is 1 and CISPO and PPO have the same gradient; the default (CISPO) is checked
    good, bad = _run("cispo")
    assert good[-1] > good[0] + 2.0, good
    assert bad[-1] < bad[0] - 2.0, bad
    # monotone over the steps, not only at the end
    assert all(b > a for a, b in zip(good, good[1:])), good
    assert all(b < a for a, b in zip(bad, bad[1:])), bad
