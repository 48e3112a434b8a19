"""Tensor-parallel (+ sequence-parallel) decoder for dense Qwen models.

Weights are drawn with the same generator sequence as
:class:`~art_mlx_b200.models.transformer.DecoderLM` and then sliced, so a
tensor-parallel model is numerically the single-GPU model split across ranks.
Per rank: the q/k/v heads ``[rank*nq/tp, ...)``, the gate/up rows and the
o/down columns of its shard, the vocab rows ``[rank*V/tp, ...)`` of the LM
head, and transposed copies of the projection shards for the backward GEMMs.
"""

from __future__ import annotations

from typing import Any

import torch

from ..ops import fused
from ..ops.fused import AttnMeta, grad_anchor
from ..parallel.tp import (
    AllGatherSeq,
    ColumnParallelLoRA,
    RowParallelLoRA,
    ScatterSeq,
    TPContext,
    VocabParallelLogprobs,
)
from .config import LoRASpec, ModelConfig
from .lora import LoRAStore, peft_key
from .transformer import _randn, lora_specs_for


class _ColLoRA:
    """Column-parallel LoRA binding: replicated A, row slices of each B."""

    def __init__(self, store: LoRAStore, layer: int, block: str, projs: list[tuple[str, int, int, int]], r: int,
                 scale: float):
        # projs: (name, full_out, local_lo, local_hi) in output order
        names = [p for p, *_ in projs if peft_key(layer, block, p, "A") in store.entries]
        self.r, self.scale, self.store = r, scale, store
        self.A = self.gA = None
        self.blocks = []
        if not names:
            return
        off, n = store.contiguous_span([peft_key(layer, block, p, "A") for p in names])
        H = n // (len(names) * r)
        self.A = store.compute[off : off + n].view(len(names) * r, H)
        self.gA = store.grad[off : off + n].view(len(names) * r, H)
        local_start = 0
        k = 0
        for name, full_out, lo, hi in projs:
            width = hi - lo
            if name in names:
                kb = peft_key(layer, block, name, "B")
                self.blocks.append((k, local_start, width, store.param(kb)[lo:hi], store.grad_view(kb)[lo:hi]))
                k += 1
            local_start += width
        self.n_local = local_start
        self._bd = None
        self._v = -1

    def block_diag(self, version: int) -> torch.Tensor:
        if self._bd is None or self._v != version:
            nr = self.A.shape[0]
            bd = self.A.new_zeros(self.n_local, nr)
            for k, s0, w, B, _ in self.blocks:
                bd[s0 : s0 + w, k * self.r : (k + 1) * self.r] = B
            self._bd, self._v = bd, version
        return self._bd

    def grad_B(self, dy: torch.Tensor, u: torch.Tensor, s: float) -> None:
        for k, s0, w, _, gB in self.blocks:
            a = dy[:, s0 : s0 + w].t()
            b = u[:, k * self.r : (k + 1) * self.r]
            if gB.device.type == "cuda":
                gB.add_(torch.mm(a, b, out_dtype=torch.float32), alpha=s)
            else:
                gB.add_(a.to(gB.dtype) @ b.to(gB.dtype), alpha=s)


class TPDecoderLM:
    def __init__(self, cfg: ModelConfig, lora: LoRASpec, device: torch.device, tp: TPContext, seed: int = 0,
                 store: LoRAStore | None = None) -> None:
        assert not cfg.is_moe and cfg.full_attention_interval == 0, "tensor parallelism: dense models"
        W = tp.world
        assert cfg.num_attention_heads % W == 0 and cfg.num_key_value_heads % W == 0
        assert cfg.intermediate_size % W == 0 and cfg.vocab_size % W == 0
        self.cfg, self.lora_spec, self.device, self.tp = cfg, lora, torch.device(device), tp
        self.dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.store = store or LoRAStore(lora_specs_for(cfg, lora), self.device, self.dtype)
        if store is None:
            self.store.init_(seed + 1)
        dev, dt = self.device, self.dtype
        gen = torch.Generator(device=dev).manual_seed(seed)
        H, V, D, F = cfg.hidden_size, cfg.vocab_size, cfg.head_dim, cfg.intermediate_size
        nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.nq_l, self.nkv_l, self.F_l, self.V_l = nq // W, nkv // W, F // W, V // W
        r0 = tp.rank
        self.embed = _randn((V, H), gen, dev, dt)
        lm = self.embed if cfg.tie_word_embeddings else _randn((V, H), gen, dev, dt)
        self.v0 = r0 * self.V_l
        self.lm_head = lm[self.v0 : self.v0 + self.V_l].contiguous()
        self.final_norm = torch.ones(H, device=dev, dtype=dt)
        self.inv_freq = fused.rope_inv_freq(D, cfg.rope_theta, dev, dict(cfg.rope_scaling))
        r, sc = lora.r, lora.scale
        q_lo, q_hi = r0 * self.nq_l * D, (r0 + 1) * self.nq_l * D
        kv_lo, kv_hi = r0 * self.nkv_l * D, (r0 + 1) * self.nkv_l * D
        f_lo, f_hi = r0 * self.F_l, (r0 + 1) * self.F_l
        self.layers: list[dict[str, Any]] = []
        for i in range(cfg.num_hidden_layers):
            qkv = _randn((cfg.q_size + 2 * cfg.kv_size, H), gen, dev, dt)
            qkv_b = _randn((cfg.q_size + 2 * cfg.kv_size,), gen, dev, dt) if cfg.attention_bias else None
            o = _randn((H, cfg.q_size), gen, dev, dt)
            gu = _randn((2 * F, H), gen, dev, dt)
            down = _randn((H, F), gen, dev, dt)
            qs, ks = cfg.q_size, cfg.kv_size
            rows = torch.cat([torch.arange(q_lo, q_hi), qs + torch.arange(kv_lo, kv_hi),
                              qs + ks + torch.arange(kv_lo, kv_hi)]).to(dev)
            L: dict[str, Any] = {
                "in_norm": torch.ones(H, device=dev, dtype=dt),
                "post_norm": torch.ones(H, device=dev, dtype=dt),
                "qkv_w": qkv[rows].contiguous(),
                "qkv_b": qkv_b[rows].contiguous() if qkv_b is not None else None,
                "o_w": o[:, q_lo:q_hi].contiguous(),
                "gu_w": torch.cat([gu[f_lo:f_hi], gu[F + f_lo : F + f_hi]]).contiguous(),
                "down_w": down[:, f_lo:f_hi].contiguous(),
                "q_norm": torch.ones(D, device=dev, dtype=dt) if cfg.qk_norm else None,
                "k_norm": torch.ones(D, device=dev, dtype=dt) if cfg.qk_norm else None,
            }
            for name in ("qkv_w", "o_w", "gu_w", "down_w"):
                L[name + "_t"] = L[name].t().contiguous()
            st = self.store
            L["qkv_lora"] = _ColLoRA(st, i, "self_attn", [("q_proj", qs, q_lo, q_hi), ("k_proj", ks, kv_lo, kv_hi),
                                                           ("v_proj", ks, kv_lo, kv_hi)], r, sc)
            L["gu_lora"] = _ColLoRA(st, i, "mlp", [("gate_proj", F, f_lo, f_hi), ("up_proj", F, f_lo, f_hi)], r, sc)
            for name, block, lo, hi in (("o_proj", "self_attn", q_lo, q_hi), ("down_proj", "mlp", f_lo, f_hi)):
                ka, kb = peft_key(i, block, name, "A"), peft_key(i, block, name, "B")
                if ka in st.entries:
                    L[name] = (st.param(ka)[:, lo:hi], st.param(kb), st.grad_view(ka)[:, lo:hi], st.grad_view(kb))
                else:
                    L[name] = None
            self.layers.append(L)
            del qkv, o, gu, down
        self.lora_enabled = True

    # ------------------------------------------------------------------
    def _col(self, x_sh, W, Wt, bias, lora: _ColLoRA):
        en = self.lora_enabled and lora.A is not None
        return ColumnParallelLoRA.apply(
            x_sh, W, Wt, bias, lora.A if en else None, lora.block_diag(self.store.version) if en else None,
            lora.gA, lora.grad_B, lora.scale, self.tp, grad_anchor(x_sh.device) if en else None)

    def _row(self, x, W, Wt, lora):
        en = self.lora_enabled and lora is not None
        A, B, gA, gB = lora if en else (None, None, None, None)
        return RowParallelLoRA.apply(x, W, Wt, A, B, gA, gB, self.lora_spec.scale, self.tp,
                                     grad_anchor(x.device) if en else None)

    def forward_hidden(self, tokens: torch.Tensor, meta: AttnMeta) -> torch.Tensor:
        """Final-normed hidden states, token-sharded ``[T/tp, H]``."""
        cfg, tp = self.cfg, self.tp
        eps = cfg.rms_norm_eps
        x = ScatterSeq.apply(self.embed[tokens.clamp_min(0)], tp)
        resid = None
        out = x
        for L in self.layers:
            h, resid = fused.add_rmsnorm(out, resid, L["in_norm"], eps)
            qkv = self._col(h, L["qkv_w"], L["qkv_w_t"], L["qkv_b"], L["qkv_lora"])
            o = fused.rope_attention(qkv, meta, self.inv_freq, self.nq_l, self.nkv_l, cfg.head_dim,
                                     L["q_norm"], L["k_norm"], eps)
            a = self._row(o, L["o_w"], L["o_w_t"], L["o_proj"])
            h, resid = fused.add_rmsnorm(a, resid, L["post_norm"], eps)
            gu = self._col(h, L["gu_w"], L["gu_w_t"], None, L["gu_lora"])
            act = fused.swiglu(gu)
            out = self._row(act, L["down_w"], L["down_w_t"], L["down_proj"])
        h, _ = fused.add_rmsnorm(out, resid, self.final_norm, eps)
        return h

    def token_logprobs(self, tokens, meta, sel, targets, ctx, entropy: bool):
        h_sh = self.forward_hidden(tokens, meta)
        h = AllGatherSeq.apply(h_sh, self.tp)
        hs = h.index_select(0, sel)
        return VocabParallelLogprobs.apply(hs, self.lm_head, targets, self.v0, self.tp, entropy)
