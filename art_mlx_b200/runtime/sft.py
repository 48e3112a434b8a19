"""SFT batches from trajectories whose assistant turns carry token ids.

Each trajectory becomes ``(input_ids, labels)``: the prompt tokens of its
first trainable choice followed by every assistant completion (merged
append-only, like the RL tokenizer); labels keep only assistant tokens.
Chat-template tokenisation for plain-text trajectories is
:func:`art_mlx_b200.preprocessing.tokenize.tokenize_sft_batch`.
"""

from __future__ import annotations

from ..preprocessing.tokenize import tokenize_histories
from ..trajectories import History, Trajectory


def trajectory_to_sft_example(t: Trajectory) -> tuple[list[int], list[int]] | None:
    results = tokenize_histories(
        [History(messages_and_choices=t.messages_and_choices, tools=t.tools)],
        advantage=0.0, allow_training_without_logprobs=True, trajectory=t,
    )
    if not results:
        return None
    r = results[0]
    labels = [tok if m else -100 for tok, m in zip(r.token_ids, r.assistant_mask)]
    return r.token_ids, labels


def sft_batches_from_trajectories(trajs: list[Trajectory], batch_size: int) -> list[list[tuple[list[int], list[int]]]]:
    examples = [e for e in (trajectory_to_sft_example(t) for t in trajs) if e is not None]
    return [examples[i : i + batch_size] for i in range(0, len(examples), batch_size)]
