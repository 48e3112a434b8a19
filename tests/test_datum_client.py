"""Datum-level training client (the hosted-service training API run on a
local TrainerRank; reference counterpart ``src/art/tinker_native/``):
trajectory groups become datums, each loss function has the gradient its
definition gives, and a train call steps the adapter."""

import math

import pytest
import torch
from openai.types.chat.chat_completion import Choice, ChoiceLogprobs
from openai.types.chat.chat_completion_message import ChatCompletionMessage
from openai.types.chat.chat_completion_token_logprob import ChatCompletionTokenLogprob

from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.runtime import datum as D
from art_mlx_b200.runtime.trainer import GRPOTrainer
from art_mlx_b200.runtime.trainer_rank import TrainerRank
from art_mlx_b200.trajectories import History, Trajectory, TrajectoryGroup


class Tok:
    """Chat template: each message is its role id then its characters."""

    def apply_chat_template(self, messages, tools=None, tokenize=True, add_generation_prompt=False):
        ids = []
        for m in messages:
            ids += [1 if m["role"] == "system" else 2] + [3 + ord(c) % 50 for c in m["content"]]
        return ids + ([9] if add_generation_prompt else [])

    def convert_tokens_to_ids(self, s):
        return None


def _choice(tokens, lps=None):
    lps = lps or [-1.0] * len(tokens)
    content = [ChatCompletionTokenLogprob(token=f"token_id:{t}", logprob=lp, bytes=None, top_logprobs=[])
               for t, lp in zip(tokens, lps)]
    return Choice(index=0, finish_reason="stop", logprobs=ChoiceLogprobs(content=content),
                  message=ChatCompletionMessage(role="assistant", content="x"))


def _client():
    tr = GRPOTrainer(get_config("tiny-qwen3"), LoRASpec(r=4, alpha=8), "cpu", seed=0)
    g = torch.Generator().manual_seed(3)
    tr.store.master.copy_(torch.randn(tr.store.numel, generator=g) * 0.05)
    tr.store.sync_compute()
    return tr, D.DatumTrainingClient(TrainerRank(tr))


def test_advantages_and_datum_layout():
    assert D.compute_advantages([1.0, 1.0]) == [0.0, 0.0]
    a = D.compute_advantages([0.0, 1.0, 2.0])
    assert a == pytest.approx([-1.0, 0.0, 1.0])
    assert D.compute_advantages([0.0, 2.0], normalize=False) == pytest.approx([-1.0, 1.0])
    d = D.build_datum([5, 6, 7], [8, 9], [-0.5, -0.25], 2.0)
    assert d.tokens == [5, 6, 7, 8] and d.target_tokens == [6, 7, 8, 9]
    assert d.mask == [0, 0, 1, 1] and d.advantages == [0, 0, 2.0, 2.0] and d.logprobs == [0, 0, -0.5, -0.25]
    assert D.build_datum([], [1], [0.0], 1.0) is None


def test_groups_to_datums():
    sys_ = {"role": "system", "content": "s"}
    t0 = Trajectory(messages_and_choices=[sys_, {"role": "user", "content": "ab"}, _choice([11, 12])], reward=0.0)
    t1 = Trajectory(messages_and_choices=[sys_, {"role": "user", "content": "cd"}, _choice([13])], reward=1.0,
                    additional_histories=[History(messages_and_choices=[{"role": "user", "content": "e"},
                                                                        _choice([14, 15, 16])])])
    flat = TrajectoryGroup([t0, t0.model_copy()])  # equal rewards: nothing to learn
    ds = D.trajectory_groups_to_datums([TrajectoryGroup([t0, t1]), flat], Tok())
    assert len(ds) == 3
    prompt = Tok().apply_chat_template([sys_, {"role": "user", "content": "ab"}], add_generation_prompt=True)
    assert ds[0].tokens == prompt + [11] and ds[0].target_tokens == prompt[1:] + [11, 12]
    assert ds[0].advantages[-1] < 0 < ds[1].advantages[-1] == ds[2].advantages[-1]
    with pytest.raises(ValueError):
        D.trajectory_groups_to_datums([TrajectoryGroup([Trajectory(messages_and_choices=[sys_]), t1])], Tok())


def _datums(vocab, n=2, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for k in range(n):
        seq = torch.randint(0, vocab, (14 + 3 * k,), generator=g).tolist()
        out.append(D.build_datum(seq[:8], seq[8:], [-1.0] * (len(seq) - 8), 1.5 - k))
    return out


def test_policy_losses_share_their_gradient_on_policy():
    """With the sampler's log-probabilities equal to the learner's (ratio
    1, nothing clipped), importance sampling, PPO and CISPO all have the
    gradient ``-A * dlogp``; cross-entropy on the mask with weight A too."""
    tr, c = _client()
    ds = _datums(tr.model.cfg.vocab_size)
    for d, lp in zip(ds, c.forward(ds)):
        d.logprobs = [float(x) if m else 0.0 for x, m in zip(lp, d.mask)]
    grads = {}
    for name in ("importance_sampling", "ppo", "cispo", "cross_entropy"):
        if name == "cross_entropy":
            for d in ds:
                d.weights = [a * m for a, m in zip(d.advantages, d.mask)]
        tr.store.grad.zero_()
        out = c.forward_backward(ds, name)
        grads[name] = tr.store.grad.clone()
        if name == "importance_sampling":
            assert out["loss"] == pytest.approx(-sum(a * m for d in ds for a, m in zip(d.advantages, d.mask)),
                                                rel=1e-4)
    g0 = grads["importance_sampling"]
    assert g0.norm() > 0
    for name, g in grads.items():
        assert torch.allclose(g, g0, atol=1e-6, rtol=1e-4), name


def test_clipping_and_dro():
    tr, c = _client()
    d = _datums(tr.model.cfg.vocab_size, n=1)[0]
    lp = c.forward([d])[0]
    d.logprobs = [float(x) - 1.0 if m else 0.0 for x, m in zip(lp, d.mask)]  # ratio e > 1 + eps: clipped
    ppo = D.datum_loss("ppo", lp, d, {"epsilon": 0.2})
    m = torch.tensor(d.mask)
    assert float(ppo) == pytest.approx(float(-(1.2 * 1.5 * m).sum()), rel=1e-5)  # A > 0: min picks the clip
    dro = D.datum_loss("dro", lp, d, {"beta": 0.1})
    want = -((1.5 * lp - 0.05 * torch.ones_like(lp)) * m).sum()
    assert float(dro) == pytest.approx(float(want), rel=1e-5)
    with pytest.raises(ValueError):
        D.datum_loss("nope", lp, d, {})  # type: ignore[arg-type]


def test_kl_penalty_against_the_base_model():
    tr, c = _client()
    ds = _datums(tr.model.cfg.vocab_size)
    base = c.forward(ds, lora="base")
    for d, b in zip(ds, base):
        d.logprobs = [float(x) + (0.3 if i % 2 else 0.0) if m else 0.0
                      for i, (x, m) in enumerate(zip(b, d.mask))]
    before = [list(d.advantages) for d in ds]
    out = c.apply_kl_penalty(ds, 0.5)
    kl = [(torch.tensor(d.logprobs) - b) * torch.tensor(d.mask) for d, b in zip(ds, base)]
    mean = sum(float(k.sum()) for k in kl) / sum(sum(d.mask) for d in ds)
    assert out["loss/kl_policy_ref"] == pytest.approx(mean, abs=1e-6)
    for d, b0, k in zip(ds, before, kl):
        want = torch.tensor(b0) + 0.5 * (mean - k) * torch.tensor(d.mask)
        assert torch.allclose(torch.tensor(d.advantages), want, atol=1e-6)


def test_train_on_groups_steps_the_adapter(tmp_path):
    tr, c = _client()
    V = tr.model.cfg.vocab_size
    mk = lambda toks, r: Trajectory(messages_and_choices=[{"role": "user", "content": "hi"}, _choice(toks)],  # noqa
                                    reward=r)
    groups = [TrajectoryGroup([mk([5, 6, 7], 0.0), mk([8 % V, 9], 1.0), mk([10, 11, 12, 13], 0.5)])]
    before = tr.store.master.clone()
    m = D.train_on_groups(c, groups, Tok(), learning_rate=1e-3, loss_fn="importance_sampling",
                          adam_params=D.AdamParams(learning_rate=1e-3, beta2=0.999), kl_penalty_coef=0.1)
    assert m["data/step_num_datums"] == 3 and math.isfinite(m["loss/train"]) and m["loss/grad_norm"] > 0
    assert "loss/kl_policy_ref" in m
    assert tr.optim.cfg.beta2 == 0.999
    assert not torch.equal(before, tr.store.master)
    assert float(tr.store.grad.abs().sum()) == 0.0  # cleared for the next step
    c.save_weights(str(tmp_path / "w"))
    assert any((tmp_path / "w").iterdir())
    c.save_state("a")
    saved = tr.store.master.clone()
    D.train_on_groups(c, groups, Tok(), learning_rate=1e-3)
    c.load_state("a")
    assert torch.equal(tr.store.master, saved)


def test_a_langgraph_rollout_trains_through_the_datum_client():
    """Choices built from LangChain response metadata carry token ids the
    datum path reads, so an agent rollout trains without conversion code."""
    import asyncio

    from art_mlx_b200 import langgraph as lg
    from test_langgraph import FakeChat, FakeModel, Msg

    def ai(ids):
        lp = {"content": [{"token": f"token_id:{t}", "logprob": -0.7, "bytes": None, "top_logprobs": []}
                          for t in ids]}
        return Msg("ai", "ok", response_metadata={"logprobs": lp, "finish_reason": "stop"})

    async def rollout(ids, reward):
        await lg.init_chat_model(FakeChat([ai(ids)])).ainvoke([Msg("human", "hi")])
        return Trajectory(reward=reward)

    w = lg.wrap_rollout(FakeModel(), rollout, log_dir=None)
    trajs = [asyncio.run(w([5, 6, 7], 0.0)), asyncio.run(w([8, 9], 1.0))]
    ds = D.trajectory_groups_to_datums([TrajectoryGroup(trajs)], Tok())
    assert [d.target_tokens[-3:] for d in ds] == [[5, 6, 7], [9, 8, 9]]
    assert ds[0].logprobs[-1] == pytest.approx(-0.7)
    tr, c = _client()
    before = tr.store.master.clone()
    m = D.train_on_groups(c, [TrajectoryGroup(trajs)], Tok(), learning_rate=1e-3, loss_fn="ppo")
    assert m["data/step_num_datums"] == 2 and not torch.equal(before, tr.store.master)
