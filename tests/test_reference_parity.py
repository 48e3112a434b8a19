"""Parity with the reference's own Python: its GRPO/CISPO/PPO loss, its
prefix-tree packer and its packed-tensor builder, loaded read-only from the
reference source tree by file path (parent packages are stubbed so that their
``__init__`` files, which need packages this image does not have, never run).

The reference tree is found through ``ART_B200_REFERENCE_SRC`` (the directory
holding its ``art`` package) or as the ``reference/src`` sibling of this
repository; the tests are skipped where it is absent (GPU boxes).
"""

from __future__ import annotations

import importlib
import math
import os
import random
import sys
import types

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.environ.get("ART_B200_REFERENCE_SRC") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference",
                                                                "src")
ART = os.path.join(SRC, "art")
pytestmark = pytest.mark.skipif(not os.path.isdir(ART), reason="reference source tree not available")


@pytest.fixture(scope="module")
def ref():
    """The reference modules, imported under their own names with stub parents;
    the stubs are removed again afterwards."""
    saved = {k: v for k, v in sys.modules.items() if k == "art" or k.startswith("art.")}
    for k in saved:
        del sys.modules[k]
    for name, sub in (("art", ""), ("art.utils", "utils"), ("art.preprocessing", "preprocessing"),
                      ("art.megatron", "megatron")):
        pkg = types.ModuleType(name)
        pkg.__path__ = [os.path.join(ART, sub)]
        sys.modules[name] = pkg
    mods = types.SimpleNamespace(
        loss=importlib.import_module("art.loss"),
        tree=importlib.import_module("art.megatron.prefix_tree_packing"),
        tokenize=importlib.import_module("art.preprocessing.tokenize"),
        pack=importlib.import_module("art.preprocessing.pack"),
    )
    yield mods
    for k in [k for k in sys.modules if k == "art" or k.startswith("art.")]:
        del sys.modules[k]
    sys.modules.update(saved)


def _packed_inputs(seed: int, S: int = 96):
    g = torch.Generator().manual_seed(seed)
    mask = torch.rand(1, S, generator=g) < 0.6
    mask[0, :5] = False
    logprobs = -torch.rand(1, S, generator=g) * 3
    logprobs[~mask] = float("nan")
    logprobs[0, 7::11] = float("nan")  # some sampled logprobs missing
    adv = torch.randn(1, S, generator=g)
    w = torch.rand(1, S, generator=g)
    gids = torch.zeros(1, S, dtype=torch.long)
    gids[0, S // 2 :] = 1
    new = (-torch.rand(1, S, generator=g) * 3).requires_grad_()
    refl = -torch.rand(1, S, generator=g) * 3
    orig = -torch.rand(1, S, generator=g) * 3
    return {"assistant_mask": mask, "logprobs": logprobs, "advantages": adv, "weights": w, "group_ids": gids,
            "original_logprobs": orig}, new, refl


CONFIGS = [
    {},
    {"ppo": True},
    {"ppo": True, "epsilon": 0.1, "epsilon_high": 0.3},
    {"kl_penalty_coef": 0.05},
    {"kl_penalty_coef": 0.05, "kl_penalty_source": "sample"},
    {"importance_sampling_level": "sequence"},
    {"importance_sampling_level": "average", "ppo": True},
    {"importance_sampling_level": "geometric_average"},
    {"mask_prob_ratio": True},
    {"kimi_k2_tau": 0.5},
    {"max_negative_advantage_importance_sampling_weight": 2.0},
    {"truncated_importance_sampling": 2.0},
]


@pytest.mark.parametrize("cfg", CONFIGS, ids=[",".join(f"{k}={v}" for k, v in c.items()) or "default" for c in CONFIGS])
@pytest.mark.parametrize("reduction", ["mean", "sum"])
def test_loss_matches_reference(ref, cfg, reduction):
    from art_mlx_b200 import loss as ours

    inputs, new, refl = _packed_inputs(len(str(cfg)) + (reduction == "sum"))
    ent = torch.rand(1, new.shape[1])
    new2 = new.detach().clone().requires_grad_()
    a = ref.loss.loss_fn(ref.loss.LossInputs(inputs=inputs), new, refl, ent, dict(cfg), reduction)
    b = ours.loss_fn(ours.LossInputs(inputs=inputs), new2, refl, ent, dict(cfg), reduction)
    for name in ("policy_loss", "policy_loss_sum", "probs_corr"):
        x, y = getattr(a, name), getattr(b, name)
        assert torch.allclose(x.float(), y.float(), rtol=1e-5, atol=1e-6, equal_nan=True), name
    for name in ("entropy", "kl_policy_ref"):
        x, y = getattr(a, name), getattr(b, name)
        assert (x is None) == (y is None), name
        if x is not None:
            assert torch.allclose(torch.as_tensor(x).float(), torch.as_tensor(y).float(), rtol=1e-5, atol=1e-6), name
    a.policy_loss.backward()
    b.policy_loss.backward()
    assert torch.allclose(new.grad, new2.grad, rtol=1e-5, atol=1e-7)


def test_prefix_tree_pack_matches_reference(ref):
    from art_mlx_b200.preprocessing.prefix_tree import prefix_tree_pack

    rng = random.Random(0)
    for trial in range(60):
        prompt = [rng.randrange(30) for _ in range(rng.randint(1, 25))]
        seqs = []
        for _ in range(rng.randint(1, 6)):
            cut = rng.randint(0, len(prompt))
            seqs.append(torch.tensor(prompt[:cut] + [rng.randrange(30) for _ in range(rng.randint(1, 12))]))
        depth = rng.choice([0, 4, 64])
        share = [max(0, len(s) - rng.randint(1, 5)) for s in seqs] if rng.random() < 0.5 else None
        a = ref.tree.prefix_tree_pack(seqs, max_depth=depth, shareable_lengths=share)
        b = prefix_tree_pack(seqs, max_depth=depth, shareable_lengths=share)
        for name in ("tokens", "group_ids", "parent_ids", "position_ids"):
            assert torch.equal(getattr(a, name), getattr(b, name)), (trial, name)
        assert len(a.positions_by_sequence) == len(b.positions_by_sequence)
        for x, y in zip(a.positions_by_sequence, b.positions_by_sequence):
            assert torch.equal(x, y), trial


def _tokenized(ref_tokenize, ours_tokenize, rng: random.Random):
    """The same sequences as the reference's and this package's result types."""
    out_ref, out_ours = [], []
    prompt_id = 0
    for g in range(rng.randint(2, 5)):
        prompt_id += 1
        prompt = [rng.randrange(100) for _ in range(rng.randint(4, 30))]
        for _ in range(rng.randint(1, 4)):
            comp = [rng.randrange(100) for _ in range(rng.randint(1, 20))]
            ids = prompt + comp
            mask = [0] * len(prompt) + [1] * len(comp)
            lps = [math.nan] * len(prompt) + [-rng.random() for _ in comp]
            fields = dict(advantage=rng.uniform(-1, 1), token_ids=ids, input_pos=list(range(len(ids))),
                          assistant_mask=mask, logprobs=lps, prompt_id=prompt_id, prompt_length=len(prompt) - 1,
                          weight=1.0 / len(comp))
            out_ref.append(_make(ref_tokenize.TokenizedResult, fields))
            out_ours.append(_make(ours_tokenize.TokenizedResult, fields))
    return out_ref, out_ours


def _make(cls, fields):
    import dataclasses

    names = {f.name for f in dataclasses.fields(cls)}
    kw = {k: v for k, v in fields.items() if k in names}
    for f in dataclasses.fields(cls):
        if f.name in kw or f.default is not dataclasses.MISSING or f.default_factory is not dataclasses.MISSING:
            continue
        kw[f.name] = None
    obj = cls(**kw)
    for k in ("weight", "prompt_id", "prompt_length"):
        if k in fields:
            setattr(obj, k, fields[k])
    return obj


def test_packed_tensors_match_reference(ref):
    from art_mlx_b200.preprocessing import pack as ours_pack
    from art_mlx_b200.preprocessing import tokenize as ours_tokenize

    for seed in range(6):
        rng = random.Random(seed)
        r_ref, r_ours = _tokenized(ref.tokenize, ours_tokenize, rng)
        a = ref.pack.packed_tensors_from_tokenized_results(r_ref, 128, verbosity=0)
        b = ours_pack.packed_tensors_from_tokenized_results(r_ours, 128, verbosity=0)
        assert a["tokens"].shape == b["tokens"].shape
        # rows are shuffled by each implementation's own generator: compare as sets of rows
        key = lambda p, r: tuple(p["tokens"][r].tolist())  # noqa: E731
        ia = sorted(range(a["tokens"].shape[0]), key=lambda r: key(a, r))
        ib = sorted(range(b["tokens"].shape[0]), key=lambda r: key(b, r))
        for ra, rb in zip(ia, ib):
            for name in ("tokens", "group_ids", "parent_ids", "input_pos", "assistant_mask"):
                assert torch.equal(a[name][ra], b[name][rb]), (seed, name)
            for name in ("advantages", "weights", "logprobs"):
                assert torch.allclose(a[name][ra].float(), b[name][rb].float(), rtol=1e-5, atol=1e-6,
                                      equal_nan=True), (seed, name)
