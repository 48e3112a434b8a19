"""Gemma-4 in the trainer: a prefix-tree packed row gives every sequence the
hidden states it has on its own (sliding windows, kv-shared layers and the
per-layer inputs included), GRPO steps train its adapter, and the GPU step
matches the CPU fp32 one.  (Logit parity with transformers is in
``test_hf_parity.py``.)"""

import random

import pytest
import torch

pytest.importorskip("transformers")

from art_mlx_b200.models.config import LoRASpec, ModelConfig  # noqa: E402
from art_mlx_b200.models.gemma4 import Gemma4LM  # noqa: E402
from art_mlx_b200.ops import fused  # noqa: E402
from art_mlx_b200.preprocessing.pack import packed_tensors_from_tokenized_results  # noqa: E402
from art_mlx_b200.preprocessing.prefix_tree import prefix_tree_pack, visibility_ends  # noqa: E402
from art_mlx_b200.preprocessing.synthetic import synthetic_groups  # noqa: E402
from art_mlx_b200.preprocessing.tokenize import tokenize_trajectory_groups  # noqa: E402
from art_mlx_b200.runtime.trainer import GRPOTrainer  # noqa: E402
from test_hf_parity import _tiny_gemma4  # noqa: E402


def _cfg(moe: bool = True) -> ModelConfig:
    d = _tiny_gemma4().to_dict()
    d["enable_moe_block"] = moe
    return ModelConfig.from_hf_dict(d, name="tiny-gemma4")


def _packed(seq_len: int = 256):
    groups = synthetic_groups(num_groups=2, rollouts_per_group=3, prompt_len=30, completion_len=12, vocab_size=512,
                              seed=4)
    res = list(tokenize_trajectory_groups(None, groups, False, True, rng=random.Random(0)))
    return packed_tensors_from_tokenized_results(res, seq_len, rng=random.Random(0))


def test_prefix_tree_row_equals_separate_sequences():
    torch.manual_seed(0)
    cfg = _cfg()
    m = Gemma4LM(cfg, LoRASpec(r=4, alpha=8), "cpu", seed=1)
    prompt = torch.randint(0, 512, (20,))
    seqs = [torch.cat([prompt, torch.randint(0, 512, (n,))]) for n in (10, 14)]
    pack = prefix_tree_pack(seqs, max_depth=4096, shareable_lengths=[20, 20])
    kend = visibility_ends(pack.group_ids, pack.parent_ids)[0]
    meta = fused.AttnMeta.build(pack.position_ids[0], kend, torch.device("cpu"))
    with torch.no_grad():
        h = m.forward(pack.tokens[0], meta, {})
        for s, where in zip(seqs, pack.positions_by_sequence):
            T = s.numel()
            alone = m.forward(s, fused.AttnMeta.build(torch.arange(T), torch.full((T,), T, dtype=torch.int32),
                                                      torch.device("cpu")), {})
            assert torch.allclose(h[where], alone, atol=1e-5, rtol=1e-4)


def test_grpo_steps_train_the_adapter():
    cfg = _cfg()
    tr = GRPOTrainer(cfg, LoRASpec(r=4, alpha=8), "cpu", seed=0)
    assert isinstance(tr.model, Gemma4LM)
    packed = _packed()
    before = tr.store.master.clone()
    for _ in range(2):
        m = tr.train_step(packed, 1e-3, {}).to_host()
    assert torch.isfinite(torch.tensor(m["loss/train"]))
    assert m["loss/grad_norm"] > 0
    assert not torch.equal(before, tr.store.master)
    with pytest.raises(ValueError):
        GRPOTrainer(cfg, LoRASpec(r=4, alpha=8), "cpu", seed=0, recompute=True)


def test_native_generation_refuses_gemma4():
    from art_mlx_b200.runtime.generate import GenerationEngine

    m = Gemma4LM(_cfg(), LoRASpec(r=4, alpha=8), "cpu", seed=0)
    with pytest.raises(NotImplementedError):
        GenerationEngine(m)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_gemma4_step_gpu_matches_cpu_fp32():
    """One GRPO step on the GPU (bf16 weights, LoRA projections through
    ops.fused) against the CPU fp32 step from the same weights (without the
    expert block: bf16 router scores can pick other experts on near ties)."""
    cfg = _cfg(moe=False)
    lora = LoRASpec(r=4, alpha=8)
    tg = GRPOTrainer(cfg, lora, torch.device("cuda", 0), seed=0)
    tc = GRPOTrainer(cfg, lora, "cpu", seed=0)
    sd = {k: v.float().cpu() for k, v in tg.model.hf_state_dict().items()}
    tc.model.load_hf_state_dict(sd)
    g = torch.Generator().manual_seed(0)
    vals = torch.randn(tc.store.numel, generator=g) * 0.05
    for t in (tc, tg):
        t.store.master.copy_(vals.to(t.store.master.device))
        t.store.sync_compute()
    packed = _packed()
    mg = tg.train_step(packed, 1e-3, {}).to_host()
    mc = tc.train_step(packed, 1e-3, {}).to_host()
    assert abs(mg["loss/train"] - mc["loss/train"]) < 5e-2 * max(1.0, abs(mc["loss/train"]))
    # the gradient (Adam's first update is close to its sign, too noisy a check in bf16)
    assert abs(mg["loss/grad_norm"] - mc["loss/grad_norm"]) < 0.1 * mc["loss/grad_norm"]
    assert torch.isfinite(tg.store.master).all()


def test_trainer_rank_outputs_use_the_soft_capped_logits():
    from art_mlx_b200.runtime.trainer_rank import ForwardInput, TrainerRank

    tr = GRPOTrainer(_cfg(), LoRASpec(r=4, alpha=8), "cpu", seed=0)
    rank = TrainerRank(tr)
    toks = torch.randint(0, 512, (20,)).tolist()
    out = rank.forward([ForwardInput(tokens=toks, top_k=3, logits=True)])[0]
    ref = torch.log_softmax(out.logits.detach(), -1)
    assert out.logits.abs().max() <= 30.0 + 1e-4  # capped
    assert torch.allclose(out.logprobs.detach(), ref.gather(-1, out.targets.unsqueeze(-1)).squeeze(-1), atol=1e-5)
    assert torch.allclose(out.top_k.logprobs, ref.topk(3, dim=-1).values, atol=1e-5)
