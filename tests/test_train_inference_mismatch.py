"""Train-vs-inference mismatch: the logprobs the rollout engine reports for
the tokens it sampled equal the logprobs the trainer computes for the same
tokens in a prefix-tree packed row (shared prompt stored once), on the same
model and adapter.  A mismatch here is what the importance ratio of the
GRPO loss would absorb as spurious off-policyness (reference counterpart:
``tests/integration/megatron/train_inf_mismatch/``)."""

import math

import pytest
import torch

from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.preprocessing.pack import packed_tensors_from_tokenized_results
from art_mlx_b200.preprocessing.tokenize import TokenizedResult
from art_mlx_b200.runtime.generate import GenerationEngine, SamplingParams
from art_mlx_b200.runtime.trainer import GRPOTrainer
from test_distributed import CONFIGS


@pytest.mark.parametrize("name", ["tiny-qwen3", "hybrid-tiny"])
def test_rollout_logprobs_match_training_logprobs(name):
    cfg = CONFIGS.get(name) or get_config(name)
    tr = GRPOTrainer(cfg, LoRASpec(r=4, alpha=8), "cpu", seed=0)
    g = torch.Generator().manual_seed(1)
    tr.store.master.copy_(torch.randn(tr.store.numel, generator=g) * 0.05)  # a non-trivial adapter
    tr.store.sync_compute()
    eng = GenerationEngine(tr.model, max_len=256)
    prompt = [int(x) for x in torch.randint(0, cfg.vocab_size, (24,), generator=g)]
    outs = eng.generate([prompt] * 4, SamplingParams(max_tokens=10, temperature=1.0, seed=5))
    results = []
    for k, o in enumerate(outs):
        ids = o.prompt_token_ids + o.token_ids
        P, C = len(o.prompt_token_ids), len(o.token_ids)
        results.append(TokenizedResult(
            advantage=float(k) - 1.5, token_ids=ids, input_pos=list(range(len(ids))),
            assistant_mask=[0] * P + [1] * C, logprobs=[math.nan] * P + list(o.logprobs),
            weight=1.0 / C, prompt_length=P))
    packed = packed_tensors_from_tokenized_results(results, 128)
    assert packed["tokens"].shape[0] == 1  # one row: the prompt is stored once
    n = 0
    for mb in tr.stage(packed):
        ctx = {"group_ids": mb.group_ids, "parent_ids": mb.parent_ids}
        with torch.no_grad():
            lp, _ = tr._logprobs(mb, ctx, entropy=False)
        ok = ~torch.isnan(mb.old)
        assert ok.any()
        diff = (lp[ok] - mb.old[ok]).abs().max().item()
        assert diff < 1e-4, f"{name}: train-vs-inference logprob mismatch {diff}"
        n += int(ok.sum())
    assert n == sum(len(o.token_ids) for o in outs)
