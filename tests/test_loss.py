"""GRPO/CISPO/PPO loss math (CPU, fp64)."""

import math

import torch

from art_mlx_b200.loss import AlignedLossInputs, LossInputs, loss_fn, shift_tensor


def _inputs(n=12, seed=0):
    g = torch.Generator().manual_seed(seed)
    old = -torch.rand(1, n, generator=g, dtype=torch.float64) * 3
    old[0, 3] = float("nan")
    return AlignedLossInputs(
        assistant_mask=torch.ones(1, n, dtype=torch.bool),
        old_logprobs=old,
        advantages=torch.randn(1, n, generator=g, dtype=torch.float64),
        weights=torch.rand(1, n, generator=g, dtype=torch.float64),
        group_ids=torch.ones(1, n, dtype=torch.long),
    )


def test_shift_tensor():
    t = torch.tensor([[1, 2, 3]])
    assert shift_tensor(t, 0).tolist() == [[2, 3, 0]]


def test_cispo_default_matches_closed_form():
    inp = _inputs()
    new = (-torch.rand(1, 12, dtype=torch.float64) * 3).requires_grad_()
    out = loss_fn(inp, new, None, None, {}, reduction="sum")
    old = torch.where(torch.isnan(inp.old_logprobs), new.detach(), inp.old_logprobs)
    r = torch.exp(new.detach() - old).clamp(0.0, 5.0)  # eps=1, eps_hi=4
    expect = -(r * inp.advantages * new * inp.weights).sum()
    assert torch.allclose(out.policy_loss, expect)
    out.policy_loss.backward()
    assert torch.allclose(new.grad, -(r * inp.advantages * inp.weights))


def test_ppo_clip_and_mean_reduction():
    inp = _inputs(seed=1)
    new = (-torch.rand(1, 12, dtype=torch.float64) * 3)
    out = loss_fn(inp, new, None, None, {"ppo": True}, reduction="mean")
    old = torch.where(torch.isnan(inp.old_logprobs), new, inp.old_logprobs)
    r = torch.exp(new - old)
    a = inp.advantages
    per = -torch.min(r * a, r.clamp(0.8, 1.2) * a) * inp.weights
    assert torch.allclose(out.policy_loss, per.sum() / (12 + 1e-18))


def test_kl_penalty_folds_into_advantage():
    inp = _inputs(seed=2)
    new = -torch.rand(1, 12, dtype=torch.float64)
    ref = -torch.rand(1, 12, dtype=torch.float64)
    coef = 0.3
    out = loss_fn(inp, new, ref, None, {"kl_penalty_coef": coef}, reduction="sum")
    kl = new - ref
    avg = kl.sum() / 12
    adv = inp.advantages + coef * (avg - kl)
    old = torch.where(torch.isnan(inp.old_logprobs), new, inp.old_logprobs)
    r = torch.exp(new - old).clamp(0.0, 5.0)
    assert torch.allclose(out.policy_loss, -(r * adv * new * inp.weights).sum())
    assert torch.allclose(out.kl_policy_ref, avg)


def test_sequence_level_ratio_uses_group_mean():
    inp = _inputs(seed=3)
    inp.group_ids = torch.tensor([[1] * 6 + [2] * 6])
    new = -torch.rand(1, 12, dtype=torch.float64)
    out = loss_fn(inp, new, None, None, {"importance_sampling_level": "sequence", "ppo": True}, reduction="sum")
    old = torch.where(torch.isnan(inp.old_logprobs), new, inp.old_logprobs)
    d = new - old
    seq = torch.cat([d[:, :6].mean().expand(6), d[:, 6:].mean().expand(6)]).view(1, 12).exp()
    a = inp.advantages
    per = -torch.min(seq * a, seq.clamp(0.8, 1.2) * a) * inp.weights
    assert torch.allclose(out.policy_loss, per.sum(), atol=1e-6)


def test_loss_inputs_align_shift():
    packed = {
        "assistant_mask": torch.tensor([[0, 1, 1]], dtype=torch.bool),
        "logprobs": torch.tensor([[math.nan, -1.0, -2.0]]),
        "advantages": torch.tensor([[0.0, 1.0, 1.0]]),
        "weights": torch.tensor([[0.0, 0.5, 0.5]]),
        "group_ids": torch.tensor([[1, 1, 1]]),
    }
    a = LossInputs(inputs=packed).align_inputs()
    assert a.assistant_mask.tolist() == [[True, True, False]]
    assert a.old_logprobs[0, :2].tolist() == [-1.0, -2.0]
