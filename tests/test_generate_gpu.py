"""Decode kernels (ops/csrc/decode.cu) against the PyTorch reference, and the
generation engine on the GPU against a full recompute."""

import math

import pytest
import torch

from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.models.transformer import DecoderLM
from art_mlx_b200.ops import fused, native
from art_mlx_b200.runtime.generate import GenerationEngine, SamplingParams, _decode_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,L,Hq,Hkv", [(3, 300, 8, 2), (5, 1000, 28, 4), (1, 33, 4, 4), (8, 4096, 16, 1)])
def test_decode_attn_matches_reference(cuda, B, L, Hq, Hkv):
    torch.manual_seed(0)
    D = 128
    kc = torch.randn(B, L, Hkv, D, device=cuda, dtype=torch.bfloat16)
    vc = torch.randn(B, L, Hkv, D, device=cuda, dtype=torch.bfloat16)
    q = torch.randn(B, Hq, D, device=cuda, dtype=torch.bfloat16)
    lens = torch.randint(1, L + 1, (B,), device=cuda, dtype=torch.int32)
    C = native.lib()
    o = C.decode_attn(q, kc, vc, lens, 1 / math.sqrt(D))
    ref = _decode_ref(q, kc, vc, lens, 1 / math.sqrt(D))
    err = (o.float() - ref.float()).norm() / ref.float().norm()
    assert err < 1e-2, err


def test_kv_append(cuda):
    kc = torch.zeros(4, 16, 2, 128, device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    k = torch.randn(3, 256, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(3, 256, device=cuda, dtype=torch.bfloat16)
    slot = torch.tensor([2, 0, 3], device=cuda, dtype=torch.int32)
    pos = torch.tensor([5, 0, 15], device=cuda, dtype=torch.int32)
    native.lib().kv_append(k, v, slot, pos, kc, vc)
    for i in range(3):
        assert torch.equal(kc[slot[i], pos[i]].reshape(-1), k[i])
        assert torch.equal(vc[slot[i], pos[i]].reshape(-1), v[i])


def test_engine_greedy_matches_full_recompute(cuda):
    m = DecoderLM(get_config("small-qwen3"), LoRASpec(r=8, alpha=16), cuda, seed=0)
    eng = GenerationEngine(m, max_len=512)
    prompts = [[1, 2, 3, 4, 5, 6, 7], [9, 8, 7], [1, 2, 3, 4, 5, 6, 7]]
    res = eng.generate(prompts, SamplingParams(max_tokens=8, temperature=0.0))
    assert res[0].token_ids == res[2].token_ids
    for r in res:
        seq = r.prompt_token_ids + r.token_ids
        T = len(seq)
        meta = fused.AttnMeta.build(torch.arange(T), torch.full((T,), T, dtype=torch.int32), cuda)
        with torch.no_grad():
            h = m.forward(torch.tensor(seq, device=cuda), meta, {})
            lp = torch.log_softmax((h @ m.lm_head.t()).float(), -1)
        P = len(r.prompt_token_ids)
        got = torch.tensor(r.logprobs, device=cuda)
        want = lp[P - 1 : T - 1].gather(1, torch.tensor(r.token_ids, device=cuda)[:, None])[:, 0]
        assert torch.allclose(got, want, atol=5e-2), (got, want)


def test_engine_hybrid_gated_deltanet_on_gpu(cuda):
    from art_mlx_b200.models.config import ModelConfig

    cfg = ModelConfig(
        name="hybrid-small", family="qwen3_next", vocab_size=2048, hidden_size=256, num_hidden_layers=4,
        num_attention_heads=2, num_key_value_heads=1, head_dim=128, intermediate_size=0, qk_norm=True,
        full_attention_interval=2, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128,
        shared_expert_intermediate_size=128, linear_num_key_heads=2, linear_num_value_heads=2,
        linear_key_head_dim=64, linear_value_head_dim=64, attn_output_gate=True,
    )
    m = DecoderLM(cfg, LoRASpec(r=8, alpha=16), cuda, seed=0)
    eng = GenerationEngine(m, max_len=512)
    prompts = [[1, 2, 3, 4, 5, 6, 7, 8, 9], [9, 8, 7]]
    res = eng.generate(prompts, SamplingParams(max_tokens=6, temperature=0.0))
    for r in res:
        seq = r.prompt_token_ids + r.token_ids
        T = len(seq)
        meta = fused.AttnMeta.build(torch.arange(T), torch.full((T,), T, dtype=torch.int32), cuda)
        with torch.no_grad():
            h = m.forward(torch.tensor(seq, device=cuda), meta, {})
            lp = torch.log_softmax((h @ m.lm_head.t()).float(), -1)
        P = len(r.prompt_token_ids)
        got = torch.tensor(r.logprobs, device=cuda)
        want = lp[P - 1 : T - 1].gather(1, torch.tensor(r.token_ids, device=cuda)[:, None])[:, 0]
        assert torch.allclose(got, want, atol=5e-2), (got, want)
