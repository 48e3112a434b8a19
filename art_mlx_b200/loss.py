"""GRPO / CISPO / PPO token loss (PyTorch oracle).

This is the fp32 reference of the loss math in the reference's
``src/art/loss.py:104-225``; the fused CUDA kernels in
``art_mlx_b200/ops/csrc/loss.cu`` (called through ``ops/fused.py``:
``grpo_token_loss``, ``lm_head_logprobs``) compute the same per-token
quantities and are tested against this module.

Per token ``t`` (inputs are shifted by one so position ``t`` scores the
token at ``t+1``):

* missing rollout logprobs (NaN) are replaced by the current ones;
* ``ratio = exp(new - old)`` at token level, or the group mean of the
  log-ratio over a sequence (``sequence``), or their arithmetic or
  geometric average;
* CISPO (default): ``-clip(ratio.detach(), 1-eps, 1+eps_hi) * A * new``
  with ``eps=1, eps_hi=4``; PPO: ``-min(r*A, clip(r)*A)`` with ``eps=0.2``;
* optional KL penalty folded into the advantage as
  ``coef * (mean_kl - kl_t)``, truncated importance sampling, Kimi-K2 tau;
* reduction ``sum(loss * weight * mask) / denom`` (``denom = 1`` for
  ``reduction="sum"``, the masked token count for ``"mean"``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Literal, Mapping

import torch

from . import dev
from .utils.group_aggregate import group_aggregate


def shift_tensor(tensor: torch.Tensor, pad: int | float | bool) -> torch.Tensor:
    """``out[:, t] = tensor[:, t + 1]``; the last column is ``pad``."""
    return torch.nn.functional.pad(tensor[:, 1:], (0, 1), value=pad)


@dataclass
class Loss:
    reduction: Literal["mean", "sum"]
    policy_loss: torch.Tensor
    entropy: torch.Tensor | None
    policy_loss_sum: torch.Tensor
    probs_corr: torch.Tensor
    kl_policy_ref: torch.Tensor | None = None


@dataclass
class AlignedLossInputs:
    """Loss inputs already shifted so that column ``t`` scores token ``t+1``."""

    assistant_mask: torch.Tensor
    old_logprobs: torch.Tensor
    advantages: torch.Tensor
    weights: torch.Tensor
    group_ids: torch.Tensor
    original_logprobs: torch.Tensor | None = None
    entropies_are_aligned: bool = False

    def align_inputs(self) -> "AlignedLossInputs":
        return self

    def group_mean(self, values: torch.Tensor, by: torch.Tensor) -> torch.Tensor:
        return group_aggregate(values, by=by, reduce="mean")

    def masked_mean(self, values: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        return values.sum() / (mask.sum() + 1e-18)

    def denominator(self, mask: torch.Tensor, reduction: str) -> torch.Tensor | float:
        return 1.0 if reduction == "sum" else mask.sum() + 1e-18

    def aligned_entropies(self, entropies: torch.Tensor | None) -> torch.Tensor | None:
        if entropies is None or self.entropies_are_aligned:
            return entropies
        return shift_tensor(entropies, 0.0)


@dataclass
class LossInputs:
    """Packed (unshifted) tensors: tokens' own logprobs/advantages/weights."""

    inputs: Mapping[str, Any]

    def align_inputs(self) -> AlignedLossInputs:
        x = self.inputs
        return AlignedLossInputs(
            assistant_mask=shift_tensor(x["assistant_mask"], False),
            old_logprobs=shift_tensor(x["logprobs"], float("nan")),
            advantages=shift_tensor(x["advantages"], 0.0),
            weights=shift_tensor(x["weights"], 0.0),
            group_ids=shift_tensor(x["group_ids"], 0),
            original_logprobs=(
                shift_tensor(x["original_logprobs"], 0.0)
                if "original_logprobs" in x
                else None
            ),
        )


def compute_probs_corr(old_logprobs: torch.Tensor, new_logprobs: torch.Tensor) -> torch.Tensor:
    """Pearson correlation of sampler vs learner token probabilities over the
    tokens that have a sampler logprob (0 when undefined)."""
    have = ~torch.isnan(old_logprobs)
    p_old = torch.exp(old_logprobs[have])
    p_new = torch.exp(new_logprobs[have].detach())
    if p_old.numel() < 2:
        return new_logprobs.new_zeros(())
    s_old = p_old.std(unbiased=False)
    s_new = p_new.std(unbiased=False)
    if not (torch.isfinite(s_old) and torch.isfinite(s_new)) or s_old == 0 or s_new == 0:
        return new_logprobs.new_zeros(())
    return torch.corrcoef(torch.stack([p_old, p_new]))[0, 1]


def resolve_clip(config: Mapping[str, Any]) -> tuple[bool, float, float]:
    """(ppo, epsilon, epsilon_high) with the reference defaults."""
    ppo = bool(config.get("ppo", False))
    eps = config.get("epsilon", 0.2 if ppo else 1.0)
    eps_hi = config.get("epsilon_high", None if ppo else 4.0)
    if eps_hi is None:
        eps_hi = eps
    return ppo, float(eps), float(eps_hi)


def loss_fn(
    inputs: LossInputs | AlignedLossInputs,
    new_logprobs: torch.Tensor,
    ref_logprobs: torch.Tensor | None,
    entropies: torch.Tensor | None,
    experimental_config: dev.TrainConfig | Mapping[str, Any],
    reduction: Literal["mean", "sum"] = "mean",
) -> Loss:
    cfg = experimental_config
    a = inputs.align_inputs()
    mask = a.assistant_mask.to(new_logprobs.dtype)
    weights = a.weights
    advantages = a.advantages
    probs_corr = compute_probs_corr(a.old_logprobs, new_logprobs)

    old = torch.where(torch.isnan(a.old_logprobs), new_logprobs.detach(), a.old_logprobs)
    log_ratio = new_logprobs - old
    ratio = torch.exp(log_ratio)
    level = cfg.get("importance_sampling_level", "token")
    if level != "token":
        seq_ratio = torch.exp(a.group_mean(log_ratio, by=a.group_ids * mask))
        if level == "sequence":
            ratio = seq_ratio
        elif level == "average":
            ratio = (ratio + seq_ratio) / 2
        elif level == "geometric_average":
            ratio = (ratio**0.5) * (seq_ratio**0.5)

    ppo, eps, eps_hi = resolve_clip(cfg)
    if cap := cfg.get("max_negative_advantage_importance_sampling_weight", None):
        ratio = torch.clamp(ratio, max=cap)
    if cfg.get("mask_prob_ratio", False):
        ratio = torch.where((ratio > 1 - eps) & (ratio < 1 + eps_hi), ratio, 0.0)
    if tau := cfg.get("kimi_k2_tau", None):
        advantages = advantages - tau * log_ratio.detach()

    kl_policy_ref = None
    kl_coef = cfg.get("kl_penalty_coef", 0.0)
    if kl_coef > 0 and ref_logprobs is not None:
        source = cfg.get("kl_penalty_source", "current_learner")
        if source == "sample":
            src = old.detach()
        elif source == "current_learner":
            src = new_logprobs.detach()
        else:
            raise AssertionError(source)
        kl_tok = (src - ref_logprobs).detach() * mask
        avg_kl = a.masked_mean(kl_tok, mask)
        advantages = advantages + kl_coef * (avg_kl - kl_tok) * mask
        kl_policy_ref = avg_kl

    if ppo:
        policy_loss = -torch.min(
            ratio * advantages, torch.clip(ratio, 1 - eps, 1 + eps_hi) * advantages
        )
    else:
        policy_loss = -(
            torch.clip(ratio.detach(), 1 - eps, 1 + eps_hi) * advantages * new_logprobs
        )

    if upper := cfg.get("truncated_importance_sampling", None):
        tis_ratio = ratio
        if a.original_logprobs is not None:
            orig = torch.where(
                torch.isnan(a.original_logprobs), new_logprobs.detach(), a.original_logprobs
            )
            tis_ratio = torch.exp(old - orig)
        policy_loss = policy_loss * torch.clamp(tis_ratio, max=upper).detach()

    policy_loss = policy_loss * weights * mask
    denom = a.denominator(mask, reduction)
    ent = a.aligned_entropies(entropies)
    return Loss(
        reduction=reduction,
        policy_loss=policy_loss.sum() / denom,
        entropy=None if ent is None else (ent * weights * mask).sum() / denom,
        policy_loss_sum=policy_loss.sum(),
        probs_corr=probs_corr,
        kl_policy_ref=kl_policy_ref,
    )
