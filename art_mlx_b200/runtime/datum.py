"""Datum-level training client: the hosted-service training API run locally.

Role of the reference's Tinker-native backend
(``src/art/tinker_native/data.py:22-281``, ``backend.py:306-460``): each
trajectory history with a sampled ``Choice`` becomes one *datum* (the model
input, the next token at every position, the sampler's log-probabilities,
the advantage and a mask of the trained positions); a training client runs
``forward_backward(datums, loss_fn)`` and then ``optim_step(adam_params)``.
The reference sends those calls to the hosted Tinker service; here the same
calls run on this machine's :class:`TrainerRank` (the prefix-tree attention
and LM-head kernels, the flat LoRA store and its fused AdamW), so code
written against the datum API trains without the service.

Loss functions, all summed over the masked positions (``r`` is the ratio of
the learner's to the sampler's token probability, ``A`` the advantage):

* ``cross_entropy``: ``-w * logp`` (supervised; ``weights`` per position);
* ``importance_sampling``: ``-r * A``;
* ``ppo``: ``-min(r * A, clip(r, 1 - eps, 1 + eps_high) * A)``;
* ``cispo``: ``-stopgrad(clip(r, 1 - eps, 1 + eps_high)) * A * logp``;
* ``dro``: ``-(A * logp - beta / 2 * (logp - logp_sampler)^2)``.

A KL penalty against the base model (LoRA off, the ``"base"`` slot) shifts
each datum's advantages by ``coef * (mean KL - token KL)`` with the KL
estimated from the sampler's log-probabilities, as the reference's
``_apply_kl_penalty`` (``backend.py:85-150``) does.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Iterable, Literal, Sequence

import torch

from ..trajectories import History, Trajectory, TrajectoryGroup, get_messages
from ..types import Choice
from .trainer_rank import ForwardInput, TrainerRank

LossName = Literal["cross_entropy", "importance_sampling", "ppo", "cispo", "dro"]


@dataclass
class Datum:
    """One training sequence: ``tokens[t]`` predicts ``target_tokens[t]``."""

    tokens: list[int]
    target_tokens: list[int]
    logprobs: list[float] = field(default_factory=list)  # sampler log-probabilities (0 where untrained)
    advantages: list[float] = field(default_factory=list)
    mask: list[float] = field(default_factory=list)  # 1 on trained positions
    weights: list[float] | None = None  # cross-entropy weights (default: the mask)

    def __post_init__(self) -> None:
        n = len(self.tokens)
        if len(self.target_tokens) != n:
            raise ValueError("tokens and target_tokens differ in length")
        for name in ("logprobs", "advantages", "mask"):
            v = getattr(self, name)
            if not v:
                setattr(self, name, [0.0 if name != "mask" else 1.0] * n)
            elif len(v) != n:
                raise ValueError(f"{name} has {len(v)} entries for {n} positions")


@dataclass
class AdamParams:
    learning_rate: float = 1e-5
    beta1: float = 0.9
    beta2: float = 0.95
    eps: float = 1e-8
    weight_decay: float | None = None  # None: keep the trainer's
    max_grad_norm: float | None = None


def compute_advantages(rewards: Sequence[float], normalize: bool = True) -> list[float]:
    """Group-relative advantages: rewards minus the group mean, divided by
    the group's (sample) standard deviation when ``normalize`` (all zero
    when the rewards do not differ)."""
    if not rewards:
        return []
    r = torch.tensor(list(rewards), dtype=torch.float64)
    c = r - r.mean()
    if not normalize:
        return c.tolist()
    s = r.std() if r.numel() > 1 else torch.tensor(0.0, dtype=torch.float64)
    return (c / s).tolist() if s > 1e-8 else [0.0] * len(rewards)


def build_datum(prompt_tokens: Sequence[int], completion_tokens: Sequence[int], logprobs: Sequence[float],
                advantage: float) -> Datum | None:
    """The datum of a prompt and its sampled completion: positions before the
    completion carry no loss."""
    if not prompt_tokens or not completion_tokens or len(completion_tokens) != len(logprobs):
        return None
    seq = list(prompt_tokens) + list(completion_tokens)
    ob = len(prompt_tokens) - 1
    C = len(completion_tokens)
    return Datum(tokens=seq[:-1], target_tokens=seq[1:], logprobs=[0.0] * ob + [float(x) for x in logprobs],
                 advantages=[0.0] * ob + [float(advantage)] * C, mask=[0.0] * ob + [1.0] * C)


def choice_tokens(choice: Any, tokenizer: Any) -> tuple[list[int], list[float]]:
    """Sampled token ids and log-probabilities of a ``Choice`` (entries of
    the form ``token_id:<n>`` are read directly; others through the
    tokenizer's vocabulary)."""
    lp = getattr(choice, "logprobs", None)
    entries = (getattr(lp, "content", None) or getattr(lp, "refusal", None) or []) if lp is not None else []
    toks, lps = [], []
    for e in entries:
        s = e.token or ""
        if s.startswith("token_id:"):
            try:
                tid = int(s.split(":", 1)[1])
            except ValueError:
                continue
        else:
            tid = tokenizer.convert_tokens_to_ids(s) if tokenizer is not None else None
            if tid is None:
                continue
        toks.append(int(tid))
        lps.append(float(e.logprob))
    return toks, lps


def history_to_datum(history: History, advantage: float, tokenizer: Any) -> Datum | None:
    """The datum of a history's last sampled ``Choice``: the prompt is the
    chat template applied to the messages before it (with the history's
    tools and a generation prompt)."""
    mc = history.messages_and_choices
    idx = next((i for i in range(len(mc) - 1, -1, -1) if isinstance(mc[i], Choice)), None)
    if idx is None:
        return None
    comp, lps = choice_tokens(mc[idx], tokenizer)
    if not comp:
        return None
    out = tokenizer.apply_chat_template(get_messages(mc[:idx]), tools=history.tools, tokenize=True,
                                        add_generation_prompt=True)
    if isinstance(out, dict) or hasattr(out, "keys"):
        out = out["input_ids"]
    prompt = list(out[0] if out and isinstance(out[0], list) else out)
    return build_datum(prompt, comp, lps, advantage)


def _histories(t: Trajectory) -> Iterable[History]:
    yield History(messages_and_choices=t.messages_and_choices, tools=t.tools)
    yield from t.additional_histories


def trajectory_groups_to_datums(groups: Iterable[TrajectoryGroup], tokenizer: Any,
                                normalize_advantages: bool = True) -> list[Datum]:
    """One datum per history that ends in a sampled choice; groups whose
    advantages are all zero contribute nothing."""
    out: list[Datum] = []
    for g in groups:
        if not g.trajectories:
            continue
        for t in g.trajectories:
            if not any(isinstance(m, Choice) for m in t.messages_and_choices):
                raise ValueError("a trajectory has no sampled Choice: nothing in it can be trained")
        adv = compute_advantages([t.reward for t in g.trajectories], normalize_advantages)
        if all(a == 0.0 for a in adv):
            continue
        for t, a in zip(g.trajectories, adv):
            for h in _histories(t):
                d = history_to_datum(h, a, tokenizer)
                if d is not None:
                    out.append(d)
    return out


def datum_loss(name: LossName, logp: torch.Tensor, d: Datum, config: dict[str, Any]) -> torch.Tensor:
    """The summed loss of one datum from the learner's log-probabilities."""
    dev = logp.device
    mask = torch.tensor(d.mask, dtype=torch.float32, device=dev)
    if name == "cross_entropy":
        w = torch.tensor(d.weights if d.weights is not None else d.mask, dtype=torch.float32, device=dev)
        return -(w * logp).sum()
    old = torch.tensor(d.logprobs, dtype=torch.float32, device=dev)
    adv = torch.tensor(d.advantages, dtype=torch.float32, device=dev)
    ratio = torch.exp(logp - old)
    eps = float(config.get("epsilon", 0.2))
    eps_hi = float(config.get("epsilon_high", eps))
    if name == "importance_sampling":
        per = -ratio * adv
    elif name == "ppo":
        per = -torch.minimum(ratio * adv, ratio.clamp(1 - eps, 1 + eps_hi) * adv)
    elif name == "cispo":
        per = -ratio.detach().clamp(1 - eps, 1 + eps_hi) * adv * logp
    elif name == "dro":
        beta = float(config.get("beta", 0.05))
        per = -(adv * logp - 0.5 * beta * (logp - old) ** 2)
    else:
        raise ValueError(f"unknown loss function {name!r}")
    return (per * mask).sum()


class DatumTrainingClient:
    """``forward`` / ``forward_backward`` / ``optim_step`` over datums on a
    local :class:`TrainerRank` (gradients accumulate across
    ``forward_backward`` calls until ``optim_step``)."""

    def __init__(self, rank: TrainerRank) -> None:
        self.rank = rank

    def _inputs(self, datums: Sequence[Datum]) -> list[ForwardInput]:
        # ForwardInput scores position t against tokens[t + 1]: append the last target
        return [ForwardInput(tokens=list(d.tokens) + [d.target_tokens[-1]],
                             score_positions=list(range(len(d.tokens)))) for d in datums]

    def _check(self, datums: Sequence[Datum], outs) -> None:
        for d, o in zip(datums, outs):
            if o.targets.tolist() != list(d.target_tokens):
                raise ValueError("a datum's target tokens are not its next tokens: only shifted sequences are "
                                 "supported")

    def forward(self, datums: Sequence[Datum], lora: str | None = None) -> list[torch.Tensor]:
        """Per-position log-probabilities of the targets (no gradient);
        ``lora`` selects an adapter slot (``"base"``: LoRA off)."""
        with torch.no_grad(), self.rank.push_lora(lora):
            outs = self.rank.forward(self._inputs(datums))
        self._check(datums, outs)
        return [o.logprobs.detach().float() for o in outs]

    def apply_kl_penalty(self, datums: Sequence[Datum], coef: float) -> dict[str, float]:
        """Shift the advantages by ``coef * (mean KL - token KL)`` against the
        base model, the KL estimated as sampler minus base log-probability
        on the trained positions."""
        base = self.forward(datums, lora="base")
        toks = [(torch.tensor(d.logprobs) - b.cpu()) * torch.tensor(d.mask) for d, b in zip(datums, base)]
        n = sum(float(sum(d.mask)) for d in datums)
        mean = sum(float(k.sum()) for k in toks) / max(n, 1.0)
        for d, k in zip(datums, toks):
            m = torch.tensor(d.mask)
            d.advantages = (torch.tensor(d.advantages) + coef * (mean - k) * m).tolist()
        return {"loss/kl_policy_ref": mean}

    def forward_backward(self, datums: Sequence[Datum], loss_fn: LossName = "cispo",
                         loss_fn_config: dict[str, Any] | None = None) -> dict[str, Any]:
        """Run the loss on every datum and accumulate its gradient; returns
        the learner's log-probabilities and the summed loss."""
        cfg = dict(loss_fn_config or {})
        logps, total, n_tok = [], 0.0, 0.0
        for d in datums:  # one datum at a time: activations of one sequence are alive at once
            out = self.rank.forward(self._inputs([d]))[0]
            self._check([d], [out])
            lp = out.logprobs.float()
            loss = datum_loss(loss_fn, lp, d, cfg)
            if loss.requires_grad:
                loss.backward()
            total += float(loss.detach())
            n_tok += float(sum(d.mask))
            logps.append(lp.detach())
        return {"logprobs": logps, "loss": total,
                "metrics": {"loss/train": total / max(n_tok, 1.0), "data/step_trainer_tokens": float(n_tok)}}

    def optim_step(self, adam: AdamParams | float) -> dict[str, float]:
        """One AdamW step with these hyperparameters; clears the gradient."""
        if not isinstance(adam, AdamParams):
            adam = AdamParams(learning_rate=float(adam))
        c = self.rank.tr.optim.cfg
        c.beta1, c.beta2, c.eps = adam.beta1, adam.beta2, adam.eps
        if adam.weight_decay is not None:
            c.weight_decay = adam.weight_decay
        if adam.max_grad_norm is not None:
            c.max_grad_norm = adam.max_grad_norm
        gn = self.rank.optim_step(adam.learning_rate)
        self.rank.zero_grad()
        if not math.isfinite(gn):
            raise FloatingPointError(f"non-finite gradient norm {gn}")
        return {"loss/grad_norm": gn}

    def save_state(self, name: str) -> None:
        """Keep the adapter and its optimizer moments as slot ``name``."""
        self.rank.save_checkpoint_slot(name)

    def load_state(self, name: str) -> None:
        self.rank.set_checkpoint(name)

    def save_weights(self, output_dir: str) -> None:
        """Write the live adapter as a PEFT directory (what a sampler loads)."""
        self.rank.save_lora_slot(None, output_dir)


def train_on_groups(client: DatumTrainingClient, groups: Iterable[TrajectoryGroup], tokenizer: Any, *,
                    learning_rate: float = 1e-5, loss_fn: LossName = "cispo", normalize_advantages: bool = True,
                    loss_fn_config: dict[str, Any] | None = None, adam_params: AdamParams | None = None,
                    kl_penalty_coef: float = 0.0) -> dict[str, float]:
    """The reference backend's ``train``: datums, optional KL shaping, one
    ``forward_backward`` and one ``optim_step``."""
    datums = trajectory_groups_to_datums(list(groups), tokenizer, normalize_advantages)
    metrics: dict[str, float] = {"data/step_num_datums": float(len(datums))}
    if not datums:
        return metrics
    if kl_penalty_coef > 0:
        metrics.update(client.apply_kl_penalty(datums, kl_penalty_coef))
    fb = client.forward_backward(datums, loss_fn, loss_fn_config)
    metrics.update(fb["metrics"])
    metrics.update(client.optim_step(adam_params or AdamParams(learning_rate=learning_rate)))
    return metrics
