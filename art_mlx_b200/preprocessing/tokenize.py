"""Trajectory → token sequences, with GRPO group advantages.

Follows the reference ``src/art/preprocessing/tokenize.py:388-606``:

* tokens are never re-templated: each trainable ``Choice`` carries the
  rollout server's ``prompt_token_ids`` and completion ``token_ids`` in its
  ``model_extra`` (see :func:`choice_token_ids`), and its sampled logprobs;
* consecutive turns are merged append-only: a turn whose prompt extends the
  running sequence appends only the new suffix, otherwise a new sequence is
  started;
* group advantage ``(r - mean) / (std + 1e-6)`` (population std), with
  zero-advantage trajectories dropped;
* per-trajectory weight ``1 / assistant_tokens``;
* the group's shareable prompt length is the longest common prefix capped
  just before the first sampled token, minus one;
* results inside a group are shuffled (``random.shuffle``).
"""

from __future__ import annotations

import math
import random
from dataclasses import dataclass, field
from typing import Any, Generator, Iterable, Literal

import numpy as np
import torch

from ..trajectories import History, Trajectory, TrajectoryGroup, get_messages


def _int_list(raw: Any, name: str) -> list[int]:
    if raw is None:
        raise RuntimeError(f"Missing {name}")
    if not isinstance(raw, list):
        raise RuntimeError(f"Expected {name} list, got {type(raw)}")
    return list(map(int, raw))


def choice_token_ids(choice: Any) -> tuple[list[int], list[int]] | None:
    """(prompt_token_ids, completion token_ids) attached to a ``Choice``."""
    extra = getattr(choice, "model_extra", None) or {}
    if "prompt_token_ids" not in extra or "token_ids" not in extra:
        return None
    return (
        _int_list(extra.get("prompt_token_ids"), "prompt_token_ids"),
        _int_list(extra.get("token_ids"), "token_ids"),
    )


def attach_token_ids_to_choice(
    choice: Any, response_payload: dict[str, Any], choice_index: int = 0
) -> None:
    """Copy token ids from a raw server response onto the parsed ``Choice``."""
    prompt = response_payload.get("prompt_token_ids")
    raw_choices = response_payload.get("choices")
    if not isinstance(raw_choices, list) or choice_index >= len(raw_choices):
        return
    raw = raw_choices[choice_index]
    if not isinstance(raw, dict) or prompt is None or raw.get("token_ids") is None:
        return
    extra = choice.model_extra
    extra["prompt_token_ids"] = _int_list(prompt, "prompt_token_ids")
    extra["token_ids"] = _int_list(raw.get("token_ids"), "token_ids")
    if raw.get("routed_experts") is not None:
        extra["routed_experts"] = raw.get("routed_experts")


@dataclass
class TokenizedResult:
    advantage: float
    token_ids: list[int]
    input_pos: list[int]
    assistant_mask: list[int]
    logprobs: list[float]
    trajectory: Trajectory | None = None
    choice_offsets: list[int] = field(default_factory=list)
    chat: str = ""
    weight: float = 0.0
    prompt_id: int = 0
    prompt_length: int = 0
    moe_routed_experts: list[Any] | None = None
    extra_logprobs: dict[str, list[float]] = field(default_factory=dict)
    pixel_values: torch.Tensor | None = None
    image_grid_thw: torch.Tensor | None = None

    def without_prompt(self) -> "TokenizedResult":
        k = self.prompt_length
        return TokenizedResult(
            advantage=self.advantage,
            token_ids=self.token_ids[k:],
            input_pos=self.input_pos[k:],
            assistant_mask=self.assistant_mask[k:],
            logprobs=self.logprobs[k:],
            trajectory=self.trajectory,
            choice_offsets=self.choice_offsets,
            chat=self.chat,
            weight=self.weight,
            prompt_id=self.prompt_id,
            prompt_length=0,
            moe_routed_experts=(
                self.moe_routed_experts[k:] if self.moe_routed_experts is not None else None
            ),
            extra_logprobs={n: v[k:] for n, v in self.extra_logprobs.items()},
        )


def _choice_logprobs(choice: Any, n: int, allow_missing: bool) -> list[float]:
    lp = getattr(choice, "logprobs", None)
    if lp is None:
        if allow_missing:
            return [float("nan")] * n
        raise RuntimeError("Trainable Choice is missing logprobs")
    entries = lp.content or getattr(lp, "refusal", None) or []
    if len(entries) != n:
        raise RuntimeError(
            f"Choice logprob length does not match completion token ids: {len(entries)} != {n}"
        )
    return [float(e.logprob) for e in entries]


def _routes_for(choice: Any, prompt_len: int, completion_len: int) -> list[Any] | None:
    extra = getattr(choice, "model_extra", None) or {}
    routes = extra.get("routed_experts")
    if routes is None:
        return None
    return list(routes)


def tokenize_histories(
    histories: list[History],
    *,
    advantage: float,
    allow_training_without_logprobs: bool,
    trajectory: Trajectory | None,
) -> list[TokenizedResult]:
    """Merge the trainable turns of ``histories`` into append-only sequences."""
    results: list[TokenizedResult] = []
    ids: list[int] = []
    mask: list[int] = []
    lps: list[float] = []
    offsets: list[int] = []
    routes: list[Any] = []
    have_routes = True
    open_turns = 0

    def flush() -> None:
        nonlocal ids, mask, lps, offsets, routes, have_routes, open_turns
        if open_turns:
            results.append(
                TokenizedResult(
                    advantage=advantage,
                    token_ids=ids,
                    input_pos=list(range(len(ids))),
                    assistant_mask=mask,
                    logprobs=lps,
                    trajectory=trajectory,
                    choice_offsets=offsets,
                    moe_routed_experts=routes if have_routes and routes else None,
                )
            )
        ids, mask, lps, offsets, routes = [], [], [], [], []
        have_routes = True
        open_turns = 0

    for history in histories:
        for item in history.messages_and_choices:
            if isinstance(item, dict) or not hasattr(item, "message"):
                continue
            if item.logprobs is None and not allow_training_without_logprobs:
                continue
            meta = choice_token_ids(item)
            if meta is None:
                raise RuntimeError(
                    "Trainable Choice is missing prompt_token_ids/token_ids; "
                    "the rollout server must return token ids"
                )
            prompt, completion = meta
            comp_lps = _choice_logprobs(item, len(completion), allow_training_without_logprobs)
            if ids and len(prompt) >= len(ids) and prompt[: len(ids)] == ids:
                suffix = prompt[len(ids) :]
            else:
                flush()
                suffix = prompt
            ids.extend(suffix)
            mask.extend([0] * len(suffix))
            lps.extend([float("nan")] * len(suffix))
            offsets.append(len(ids))
            ids.extend(completion)
            mask.extend([1] * len(completion))
            lps.extend(comp_lps)
            r = _routes_for(item, len(prompt), len(completion))
            if r is None:
                have_routes = False
            else:
                # the route list covers prompt + completion of this turn;
                # keep the entries of the tokens appended now
                total = len(prompt) + len(completion)
                start = total - len(suffix) - len(completion)
                routes.extend(r[start:total] if len(r) >= total else [None] * (len(suffix) + len(completion)))
            open_turns += 1
    flush()
    return results


def group_advantages(rewards: list[float], scale_rewards: bool) -> list[float]:
    n = len(rewards)
    mean = sum(rewards) / n
    std = math.sqrt(sum((r - mean) ** 2 for r in rewards) / n)
    out = []
    for r in rewards:
        a = r - mean
        if scale_rewards:
            a /= std + 1e-6
        out.append(a)
    return out


def _common_prefix_len(rows: list) -> int:
    """Length of the prefix shared by every token sequence."""
    n = min(len(r) for r in rows)
    first = np.asarray(rows[0][:n], dtype=np.int64)
    common = n
    for r in rows[1:]:
        diff = np.flatnonzero(np.asarray(r[:common], dtype=np.int64) != first[:common])
        if diff.size:
            common = int(diff[0])
    return common


def _first_sampled(logprobs) -> int:
    """Index of the first token with a logprob (the first sampled token)."""
    hit = np.flatnonzero(~np.isnan(np.asarray(logprobs, dtype=np.float64)))
    return int(hit[0]) if hit.size else len(logprobs)


def tokenize_trajectory_groups(
    tokenizer: Any,
    trajectory_groups: Iterable[TrajectoryGroup],
    allow_training_without_logprobs: bool,
    scale_rewards: bool,
    shuffle_group_trajectories: bool = True,
    drop_zero_advantage_trajectories: bool = True,
    rng: random.Random | None = None,
) -> Generator[TokenizedResult, None, None]:
    """Yield tokenized results group by group (the tokenizer is unused: token
    ids come from the rollout server; it is accepted for API parity)."""
    del tokenizer
    shuffle = (rng or random).shuffle
    randint = (rng or random).randint
    for group in trajectory_groups:
        if not len(group):
            continue
        trajs = list(group)
        advs = group_advantages([t.reward for t in trajs], scale_rewards)
        results: list[TokenizedResult] = []
        for traj, adv in zip(trajs, advs):
            if adv == 0 and drop_zero_advantage_trajectories:
                continue
            rs = tokenize_histories(
                [
                    History(messages_and_choices=traj.messages_and_choices, tools=traj.tools),
                    *traj.additional_histories,
                ],
                advantage=adv,
                allow_training_without_logprobs=allow_training_without_logprobs,
                trajectory=traj,
            )
            w = 1 / (sum(sum(r.assistant_mask) for r in rs) + 1e-6)
            for r in rs:
                r.weight = w
            results.extend(rs)
        if not results:
            continue
        prompt_id = randint(-(2**63), 2**63 - 1)
        common = _common_prefix_len([r.token_ids for r in results])
        first_sampled = min(_first_sampled(r.logprobs) for r in results)
        prompt_length = max(min(common, first_sampled) - 1, 0)
        for r in results:
            r.prompt_id = prompt_id
            r.prompt_length = prompt_length
        if shuffle_group_trajectories:
            shuffle(results)
        yield from results


# ---------------------------------------------------------------------------
# SFT tokenization (chat template, response-only labels)
# ---------------------------------------------------------------------------


@dataclass
class SFTBatch:
    trajectory_tensors: list[dict[str, torch.Tensor]]
    learning_rate: float
    num_trajectories: int
    num_tokens: int
    num_trainable_tokens: int
    num_dropped_trajectories: int = 0


def _find(seq: list[int], pattern: list[int], start: int) -> int:
    n = len(pattern)
    for i in range(start, len(seq) - n + 1):
        if seq[i : i + n] == pattern:
            return i
    return -1


def response_only_labels(
    input_ids: list[int], *, instruction_ids: list[int], response_ids: list[int]
) -> list[int]:
    """Labels that keep only assistant responses: every span after a
    response marker up to the next instruction marker (reference
    ``preprocessing/response_masking.py:26-50``)."""
    labels = [-100] * len(input_ids)
    pos = 0
    while True:
        r = _find(input_ids, response_ids, pos)
        if r < 0:
            break
        begin = r + len(response_ids)
        nxt = _find(input_ids, instruction_ids, begin)
        end = len(input_ids) if nxt < 0 else nxt
        labels[begin:end] = input_ids[begin:end]
        pos = end
    return labels


def tokenize_sft_batch(
    trajectory_batch: list[Trajectory],
    learning_rate: float,
    tokenizer: Any,
    instruction_part: str,
    response_part: str,
    max_seq_length: int | None = None,
    assistant_turns: Literal["all", "last"] = "all",
) -> SFTBatch:
    if max_seq_length is not None and max_seq_length < 1:
        raise ValueError(f"max_seq_length must be positive, got {max_seq_length}")
    enc = lambda text: list(tokenizer(text, add_special_tokens=False)["input_ids"])  # noqa: E731
    instruction_ids = enc(instruction_part)
    response_ids = enc(response_part)
    tensors: list[dict[str, torch.Tensor]] = []
    n_tok = n_train = dropped = 0
    for traj in trajectory_batch:
        messages = get_messages(traj.messages_and_choices)
        if assistant_turns == "last":
            if not messages or messages[-1].get("role") != "assistant":
                raise ValueError("assistant_turns='last' requires a final assistant message")
            prompt_text = tokenizer.apply_chat_template(
                messages[:-1], tools=traj.tools, tokenize=False, add_generation_prompt=True
            )
            full_text = tokenizer.apply_chat_template(
                messages, tools=traj.tools, tokenize=False, add_generation_prompt=False
            )
            if not full_text.startswith(prompt_text):
                raise ValueError("completed chat does not extend its generation prompt")
            p_ids = enc(prompt_text)
            t_ids = enc(full_text[len(prompt_text) :])
            input_ids = p_ids + t_ids
            labels = [-100] * len(p_ids) + t_ids
        else:
            out = tokenizer.apply_chat_template(
                messages, tools=traj.tools, tokenize=True, add_generation_prompt=False
            )
            if isinstance(out, dict) or hasattr(out, "keys"):
                out = out["input_ids"]
            input_ids = list(out[0] if out and isinstance(out[0], list) else out)
            labels = response_only_labels(
                input_ids, instruction_ids=instruction_ids, response_ids=response_ids
            )
        if max_seq_length is not None and len(input_ids) > max_seq_length:
            dropped += 1
            continue
        tensors.append(
            {
                "input_ids": torch.tensor([input_ids], dtype=torch.long),
                "attention_mask": torch.ones(1, len(input_ids), dtype=torch.long),
                "labels": torch.tensor([labels], dtype=torch.long),
            }
        )
        n_tok += len(input_ids)
        n_train += sum(1 for v in labels if v != -100)
    return SFTBatch(tensors, learning_rate, len(tensors), n_tok, n_train, dropped)
