"""Generation engine on CPU: cached decoding equals recomputing the full
sequence, shared prompts, stop tokens, adapters."""

import torch

from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.models.transformer import DecoderLM
from art_mlx_b200.ops import fused
from art_mlx_b200.runtime.generate import GenerationEngine, SamplingParams


def _model():
    m = DecoderLM(get_config("tiny-qwen3"), LoRASpec(r=4, alpha=8), "cpu", seed=0)
    m.store.master.normal_(0, 0.05)  # non-trivial adapter
    m.store.compute.copy_(m.store.master)
    m.store.version += 1
    return m


def _full_logprobs(m, seq):
    T = len(seq)
    meta = fused.AttnMeta.build(torch.arange(T), torch.full((T,), T, dtype=torch.int32), m.device)
    with torch.no_grad():
        h = m.forward(torch.tensor(seq), meta, {})
        return torch.log_softmax((h @ m.lm_head.t()).float(), -1)


def test_greedy_decode_matches_full_recompute():
    m = _model()
    eng = GenerationEngine(m, max_len=256)
    prompts = [[1, 2, 3, 4, 5], [7, 8, 9], [1, 2, 3, 4, 5]]
    res = eng.generate(prompts, SamplingParams(max_tokens=6, temperature=0.0))
    assert res[0].token_ids == res[2].token_ids  # shared prompt, greedy
    for r in res:
        seq = r.prompt_token_ids + r.token_ids
        lp = _full_logprobs(m, seq)
        P = len(r.prompt_token_ids)
        for i, t in enumerate(r.token_ids):
            row = lp[P - 1 + i]
            assert int(row.argmax()) == t
            assert abs(float(row[t]) - r.logprobs[i]) < 1e-4


def test_stop_tokens_sampling_and_adapters():
    m = _model()
    eng = GenerationEngine(m, max_len=256)
    greedy = eng.generate([[3, 4, 5]], SamplingParams(max_tokens=5, temperature=0.0))[0]
    stop = greedy.token_ids[2]
    r = eng.generate([[3, 4, 5]], SamplingParams(max_tokens=5, temperature=0.0, stop_token_ids=[stop]))[0]
    assert r.finish_reason == "stop" and r.token_ids[-1] == stop and len(r.token_ids) <= 3
    a = eng.generate([[3, 4, 5]] * 4, SamplingParams(max_tokens=8, temperature=1.0, seed=3))
    b = eng.generate([[3, 4, 5]] * 4, SamplingParams(max_tokens=8, temperature=1.0, seed=3))
    assert [x.token_ids for x in a] == [x.token_ids for x in b]
    # base model (adapter off) and a registered adapter; the live store is restored
    before = m.store.compute.clone()
    base = eng.generate([[3, 4, 5]], SamplingParams(max_tokens=5, temperature=0.0), adapter="base")[0]
    eng.add_adapter("zero", torch.zeros_like(m.store.compute))
    zero = eng.generate([[3, 4, 5]], SamplingParams(max_tokens=5, temperature=0.0), adapter="zero")[0]
    assert torch.equal(m.store.compute, before) and m.lora_enabled
    assert base.token_ids == zero.token_ids  # B = 0 adapter == no adapter
    assert abs(base.logprobs[0] - zero.logprobs[0]) < 1e-5


def test_hybrid_gated_deltanet_generation_matches_full_recompute():
    """Hybrid model (gated DeltaNet + attention + MoE): recurrent decode of the
    linear-attention layers equals recomputing the whole sequence."""
    from art_mlx_b200.models.config import ModelConfig

    cfg = ModelConfig(
        name="hybrid-tiny", family="qwen3_next", vocab_size=512, hidden_size=64, num_hidden_layers=4,
        num_attention_heads=2, num_key_value_heads=1, head_dim=32, intermediate_size=0, qk_norm=True,
        full_attention_interval=2, num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32,
        shared_expert_intermediate_size=32, linear_num_key_heads=2, linear_num_value_heads=2,
        linear_key_head_dim=16, linear_value_head_dim=16, attn_output_gate=True,
    )
    m = DecoderLM(cfg, LoRASpec(r=4, alpha=8), "cpu", seed=0)
    eng = GenerationEngine(m, max_len=256)
    prompts = [[5, 6, 7, 8, 9, 10, 11, 12], [3, 2], [5, 6, 7, 8, 9, 10, 11, 12]]
    res = eng.generate(prompts, SamplingParams(max_tokens=6, temperature=0.0))
    assert res[0].token_ids == res[2].token_ids
    for r in res:
        seq = r.prompt_token_ids + r.token_ids
        lp = _full_logprobs(m, seq)
        P = len(r.prompt_token_ids)
        for i, t in enumerate(r.token_ids):
            assert int(lp[P - 1 + i].argmax()) == t
            assert abs(float(lp[P - 1 + i][t]) - r.logprobs[i]) < 1e-4
