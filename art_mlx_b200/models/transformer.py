"""Decoder-only LM (Qwen2 / Qwen3 dense, Qwen3-MoE) with LoRA adapters.

Layout choices for B200:

* tokens of one packed row are processed flat as ``[T, hidden]``;
* q/k/v and gate/up are fused projections (one GEMM each); their LoRA
  factors are applied as a block-diagonal rank-``n*r`` update;
* the residual add is fused into the following RMSNorm;
* RoPE (and Qwen3's per-head q/k RMSNorm) is fused into the attention op,
  whose mask is the prefix-tree interval ``kend`` (shared prompt attended
  once by every completion);
* all base weights are frozen; only the flat LoRA store is trained.

Random initialisation (N(0, 0.02) weights, unit norms) is seeded and
deterministic; :meth:`DecoderLM.load_hf_state_dict` maps Hugging Face
parameter names onto the fused layout when real weights are available.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import Any

import torch

from ..ops import fused
from ..ops.fused import AttnMeta, LoRABinding
from .config import LoRASpec, ModelConfig
from .lora import LoRAStore, peft_key
from .moe import MoEBlock


@dataclass
class DenseMLP:
    gu_w: torch.Tensor  # [2F, H] (gate rows then up rows)
    down_w: torch.Tensor  # [H, F]
    gu_lora: LoRABinding | None = None
    down_lora: LoRABinding | None = None


@dataclass
class Layer:
    index: int
    kind: str
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    qkv_w: torch.Tensor | None = None
    qkv_b: torch.Tensor | None = None
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None
    o_w: torch.Tensor | None = None
    qkv_lora: LoRABinding | None = None
    o_lora: LoRABinding | None = None
    o_b: torch.Tensor | None = None  # GPT-OSS: bias of o_proj
    sinks: torch.Tensor | None = None  # GPT-OSS: fp32 [heads] attention-sink logits
    window: int = 0  # sliding-window size (0: full attention)
    mlp: DenseMLP | None = None
    moe: MoEBlock | None = None
    gdn: Any = None


def recompute_enabled() -> bool:
    """``ART_B200_RECOMPUTE=full`` (or 1): recompute every layer's
    activations in the backward (the reference's Megatron provider default,
    uniform full recompute of one layer at a time)."""
    return os.environ.get("ART_B200_RECOMPUTE", "").strip().lower() in {"1", "full", "true", "yes", "on"}


def _randn(shape, gen, device, dtype, std=0.02) -> torch.Tensor:
    t = torch.empty(shape, device=device, dtype=torch.float32)
    t.normal_(0.0, std, generator=gen)
    return t.to(dtype)


def lora_specs_for(cfg: ModelConfig, spec: LoRASpec) -> list[tuple[str, tuple[int, ...], str]]:
    """Ordered (key, shape, kind) list of every LoRA factor of the model.

    Factors of one fused projection are stored back to back (all ``A`` then
    all ``B``) so the concatenated ``A`` is a single view.
    """
    if cfg.family == "gemma4":
        from .gemma4 import gemma4_lora_specs

        return gemma4_lora_specs(cfg, spec)
    r = spec.r
    H = cfg.hidden_size
    out: list[tuple[str, tuple[int, ...], str]] = []
    t = set(spec.target_modules)
    for i in range(cfg.num_hidden_layers):
        kind = cfg.layer_kind(i)
        if kind == "attention":
            qkv = [("q_proj", cfg.q_size * (2 if cfg.attn_output_gate else 1)), ("k_proj", cfg.kv_size), ("v_proj", cfg.kv_size)]
            sel = [(p, o) for p, o in qkv if p in t]
            for p, _ in sel:
                out.append((peft_key(i, "self_attn", p, "A"), (r, H), "A"))
            for p, o in sel:
                out.append((peft_key(i, "self_attn", p, "B"), (o, r), "B"))
            if "o_proj" in t:
                out.append((peft_key(i, "self_attn", "o_proj", "A"), (r, cfg.q_size), "A"))
                out.append((peft_key(i, "self_attn", "o_proj", "B"), (H, r), "B"))
        else:
            from .gdn import gdn_lora_specs

            out.extend(gdn_lora_specs(cfg, i, spec))
        if cfg.is_moe:
            from .moe import moe_lora_specs

            out.extend(moe_lora_specs(cfg, i, spec))
        else:
            F = cfg.intermediate_size
            gu = [(p, F) for p in ("gate_proj", "up_proj") if p in t]
            for p, _ in gu:
                out.append((peft_key(i, "mlp", p, "A"), (r, H), "A"))
            for p, o in gu:
                out.append((peft_key(i, "mlp", p, "B"), (o, r), "B"))
            if "down_proj" in t:
                out.append((peft_key(i, "mlp", "down_proj", "A"), (r, F), "A"))
                out.append((peft_key(i, "mlp", "down_proj", "B"), (H, r), "B"))
    return out


def make_binding(
    store: LoRAStore,
    layer: int,
    block: str,
    projs: list[tuple[str, int]],
    spec: LoRASpec,
    expert: int | None = None,
) -> LoRABinding | None:
    """Binding of a fused projection whose output slices are ``projs``
    (name, out_size) in order; slices without a LoRA target get no block."""
    names_a, blocks, gblocks, slices = [], [], [], []
    start = 0
    present = []
    for p, o in projs:
        ka = peft_key(layer, block, p, "A", expert)
        if ka in store.entries:
            present.append((p, o, start))
        start += o
    if not present:
        return None
    for p, o, s in present:
        names_a.append(peft_key(layer, block, p, "A", expert))
        blocks.append(store.param(peft_key(layer, block, p, "B", expert)))
        gblocks.append(store.grad_view(peft_key(layer, block, p, "B", expert)))
        slices.append((s, s + o))
    off, n = store.contiguous_span(names_a)
    r = spec.r
    in_features = n // (len(names_a) * r)
    A = store.compute[off : off + n].view(len(names_a) * r, in_features)
    gA = store.grad[off : off + n].view(len(names_a) * r, in_features)
    return LoRABinding(
        A=A, B_blocks=blocks, gA=gA, gB_blocks=gblocks, slices=slices, r=r,
        scale=spec.scale, out_features=start,
    )


class DecoderLM:
    def __init__(
        self,
        cfg: ModelConfig,
        lora: LoRASpec,
        device: torch.device | str = "cpu",
        dtype: torch.dtype | None = None,
        seed: int = 0,
        store: LoRAStore | None = None,
        init_weights: bool = True,
        ep: Any = None,
        etp: Any = None,
    ) -> None:
        self.cfg = cfg
        self.ep = ep  # expert-parallel context (MoE models on several ranks)
        self.etp = etp  # expert-tensor-parallel context (experts' FFN split over ranks)
        self.lora_spec = lora
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        self.store = store or LoRAStore(lora_specs_for(cfg, lora), self.device, self.dtype)
        if store is None:
            self.store.init_(seed + 1)
        gen = torch.Generator(device=self.device).manual_seed(seed)
        H, V = cfg.hidden_size, cfg.vocab_size
        dev, dt = self.device, self.dtype
        self.embed = _randn((V, H), gen, dev, dt)
        self.final_norm = torch.ones(H, device=dev, dtype=dt)
        self.lm_head = self.embed if cfg.tie_word_embeddings else _randn((V, H), gen, dev, dt)
        self.rope_perm = None
        if cfg.rotary_dim and cfg.rotary_dim < cfg.head_dim:  # partial rotary (Qwen3-Next / Qwen3.5)
            self.inv_freq, perm = fused.partial_rotary(cfg.head_dim, cfg.rotary_dim, cfg.rope_theta, dev,
                                                       dict(cfg.rope_scaling))
            self.rope_perm = perm.to(torch.int16)
        else:
            self.inv_freq = fused.rope_inv_freq(cfg.head_dim, cfg.rope_theta, dev, dict(cfg.rope_scaling))
        # a RoPE that scales cos / sin (YaRN) scales q and k: the scores carry its square
        self.attn_scale = fused.rope_attention_factor(dict(cfg.rope_scaling)) ** 2 / math.sqrt(cfg.head_dim)
        self.layers: list[Layer] = []
        for i in range(cfg.num_hidden_layers):
            self.layers.append(self._build_layer(i, gen))
        self.lora_enabled = True
        # full activation recompute per layer (the training forward keeps each
        # layer's inputs only); off by default
        self.recompute = recompute_enabled()
        self.streamer = None  # runtime.weight_stream.LayerWeightStreamer when streaming

    def enable_weight_streaming(self, slots: int = 2) -> None:
        """Keep the layers' base weights in pinned host memory and stream
        them in one layer at a time (``slots`` device buffers); turns on
        activation recompute, which brings each layer back for its backward."""
        from ..runtime.weight_stream import LayerWeightStreamer

        if self.ep is not None or self.etp is not None:
            raise NotImplementedError("weight streaming runs without expert parallelism")
        self.recompute = True
        self.streamer = LayerWeightStreamer(self, slots)

    # ------------------------------------------------------------------
    def _build_layer(self, i: int, gen: torch.Generator) -> Layer:
        cfg, dev, dt, spec, st = self.cfg, self.device, self.dtype, self.lora_spec, self.store
        H = cfg.hidden_size
        layer = Layer(
            index=i,
            kind=cfg.layer_kind(i),
            in_norm=torch.ones(H, device=dev, dtype=dt),
            post_norm=torch.ones(H, device=dev, dtype=dt),
        )
        if layer.kind == "attention":
            qo = cfg.q_size * (2 if cfg.attn_output_gate else 1)
            nqkv = qo + 2 * cfg.kv_size
            layer.qkv_w = _randn((nqkv, H), gen, dev, dt)
            if cfg.attention_bias:
                layer.qkv_b = _randn((nqkv,), gen, dev, dt)
            if cfg.qk_norm:
                layer.q_norm = torch.ones(cfg.head_dim, device=dev, dtype=dt)
                layer.k_norm = torch.ones(cfg.head_dim, device=dev, dtype=dt)
            layer.o_w = _randn((H, cfg.q_size), gen, dev, dt)
            if cfg.o_bias:
                layer.o_b = _randn((H,), gen, dev, dt)
            if cfg.attn_sinks:
                layer.sinks = torch.zeros(cfg.num_attention_heads, device=dev, dtype=torch.float32)
            layer.window = cfg.layer_window(i)
            layer.qkv_lora = make_binding(
                st, i, "self_attn", [("q_proj", qo), ("k_proj", cfg.kv_size), ("v_proj", cfg.kv_size)], spec
            )
            layer.o_lora = make_binding(st, i, "self_attn", [("o_proj", H)], spec)
        else:
            from .gdn import GatedDeltaNet

            layer.gdn = GatedDeltaNet(cfg, i, gen, dev, dt, st, spec)
        if cfg.is_moe:
            layer.moe = MoEBlock(cfg, i, gen, dev, dt, st, spec, ep=self.ep, etp=self.etp)
        else:
            F = cfg.intermediate_size
            layer.mlp = DenseMLP(
                gu_w=_randn((2 * F, H), gen, dev, dt),
                down_w=_randn((H, F), gen, dev, dt),
                gu_lora=make_binding(st, i, "mlp", [("gate_proj", F), ("up_proj", F)], spec),
                down_lora=make_binding(st, i, "mlp", [("down_proj", H)], spec),
            )
        return layer

    # ------------------------------------------------------------------
    def attention(self, layer: Layer, h: torch.Tensor, meta: AttnMeta, ctx: dict[str, Any] | None = None) -> torch.Tensor:
        cfg = self.cfg
        v = self.store.version
        en = self.lora_enabled
        qkv = fused.lora_linear(h, layer.qkv_w, layer.qkv_b, layer.qkv_lora, v, en)
        nq, nkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        gate = None
        if cfg.attn_output_gate:
            # Qwen3-Next: q projection carries [q | gate] per head
            T = qkv.shape[0]
            qg = qkv[:, : 2 * cfg.q_size].view(T, nq, 2 * D)
            gate = qg[..., D:].reshape(T, cfg.q_size)
            qkv = torch.cat([qg[..., :D].reshape(T, cfg.q_size), qkv[:, 2 * cfg.q_size :]], dim=1)
        if ctx is not None and ctx.get("cp_plan") is not None:
            if layer.window or layer.sinks is not None:
                raise NotImplementedError("context parallelism with sliding windows or attention sinks")
            from ..parallel.cp import cp_rope_attention

            o = cp_rope_attention(qkv, ctx["cp_plan"], ctx["cp"], self.inv_freq, nq, nkv, D,
                                  layer.q_norm, layer.k_norm, cfg.rms_norm_eps, self.rope_perm, self.attn_scale)
        else:
            o = fused.rope_attention(
                qkv, meta.windowed(layer.window), self.inv_freq, nq, nkv, D, layer.q_norm, layer.k_norm,
                cfg.rms_norm_eps, sinks=layer.sinks, scale=self.attn_scale, perm=self.rope_perm,
            )
        if gate is not None:
            o = o * torch.sigmoid(gate)
        return fused.lora_linear(o, layer.o_w, layer.o_b, layer.o_lora, v, en)

    def mlp(self, layer: Layer, h: torch.Tensor, ctx: dict[str, Any]) -> torch.Tensor:
        if layer.moe is not None:
            return layer.moe(h, self.store.version, self.lora_enabled, ctx)
        m = layer.mlp
        assert m is not None
        v, en = self.store.version, self.lora_enabled
        gu = fused.lora_linear(h, m.gu_w, None, m.gu_lora, v, en)
        a = fused.swiglu(gu)
        return fused.lora_linear(a, m.down_w, None, m.down_lora, v, en)

    def _layer(self, layer: Layer, out: torch.Tensor, resid: torch.Tensor | None, meta: AttnMeta,
               ctx: dict[str, Any]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """One decoder layer on the residual stream: ``(mlp out, residual,
        mixer out)``."""
        if self.streamer is not None:  # base weights streamed in from the host
            self.streamer.ensure(layer.index)
        eps = self.cfg.rms_norm_eps
        h, resid = fused.add_rmsnorm(out, resid, layer.in_norm, eps)
        if layer.kind == "attention":
            a = self.attention(layer, h, meta, ctx)
        elif ctx.get("cp_plan") is not None:
            from ..parallel.cp import cp_gdn

            a = cp_gdn(layer.gdn, h, ctx["cp_plan"], ctx["cp"], self.store.version, self.lora_enabled)
        else:
            a = layer.gdn(h, meta, self.store.version, self.lora_enabled, ctx)
        h, resid = fused.add_rmsnorm(a, resid, layer.post_norm, eps)
        return self.mlp(layer, h, ctx), resid, a

    def forward(
        self, tokens: torch.Tensor, meta: AttnMeta, ctx: dict[str, Any] | None = None
    ) -> torch.Tensor:
        """Final-normed hidden states ``[T, hidden]`` for one packed row."""
        ctx = ctx if ctx is not None else {}
        cfg = self.cfg
        eps = cfg.rms_norm_eps
        x = self.embed[tokens.clamp_min(0)]
        resid = None
        out = x
        trace = ctx.get("trace")  # utils.trace.ForwardTraceCapture: per-layer outputs by token UID
        uids = None
        if trace is not None or ctx.get("token_uids") is not None:
            uids = ctx.get("token_uids")
            if uids is None:  # the row's global token indices (a CP rank holds a contiguous slice)
                plan = ctx.get("cp_plan")
                start = plan.a if plan is not None else 0
                uids = torch.arange(start, start + tokens.shape[0])
        # full activation recompute: a layer keeps only its inputs and runs
        # its forward again in the backward (every rank in the same order, so
        # the collectives inside a layer stay matched)
        recompute = self.recompute and torch.is_grad_enabled() and trace is None
        for layer in self.layers:
            if recompute:
                from torch.utils.checkpoint import checkpoint

                out, resid, a = checkpoint(self._layer, layer, out, resid, meta, ctx, use_reentrant=False,
                                           preserve_rng_state=False)
            else:
                out, resid, a = self._layer(layer, out, resid, meta, ctx)
            if trace is not None:
                trace.record(layer.index, "mixer", a, uids)
                trace.record(layer.index, "mlp", out, uids)
        h, _ = fused.add_rmsnorm(out, resid, self.final_norm, eps)
        if trace is not None:
            trace.record(len(self.layers), "hidden", h, uids)
        return h

    # ------------------------------------------------------------------
    def num_parameters(self) -> int:
        n = self.embed.numel() + (0 if self.cfg.tie_word_embeddings else self.lm_head.numel())
        for layer in self.layers:
            for t in (layer.qkv_w, layer.o_w, layer.qkv_b):
                if t is not None:
                    n += t.numel()
            if layer.mlp is not None:
                n += layer.mlp.gu_w.numel() + layer.mlp.down_w.numel()
            if layer.moe is not None:
                n += layer.moe.num_parameters()
            if layer.gdn is not None:
                n += layer.gdn.num_parameters()
        return n

    def hf_state_dict(self) -> dict[str, torch.Tensor]:
        """Base weights under Hugging Face names (the fused q/k/v and gate/up
        projections split back), inverse of :meth:`load_hf_state_dict`."""
        cfg = self.cfg
        out: dict[str, torch.Tensor] = {"model.embed_tokens.weight": self.embed, "model.norm.weight": self.final_norm}
        if not cfg.tie_word_embeddings:
            out["lm_head.weight"] = self.lm_head
        q, kv = cfg.q_size * (2 if cfg.attn_output_gate else 1), cfg.kv_size
        for i, layer in enumerate(self.layers):
            p = f"model.layers.{i}."
            out[p + "input_layernorm.weight"] = layer.in_norm
            out[p + "post_attention_layernorm.weight"] = layer.post_norm
            if layer.kind == "attention":
                a = p + "self_attn."
                out[a + "q_proj.weight"], out[a + "k_proj.weight"], out[a + "v_proj.weight"] = (
                    layer.qkv_w[:q], layer.qkv_w[q : q + kv], layer.qkv_w[q + kv :])
                if layer.qkv_b is not None:
                    out[a + "q_proj.bias"], out[a + "k_proj.bias"], out[a + "v_proj.bias"] = (
                        layer.qkv_b[:q], layer.qkv_b[q : q + kv], layer.qkv_b[q + kv :])
                if layer.q_norm is not None:
                    out[a + "q_norm.weight"], out[a + "k_norm.weight"] = layer.q_norm, layer.k_norm
                out[a + "o_proj.weight"] = layer.o_w
            if layer.mlp is not None:
                m = p + "mlp."
                F = cfg.intermediate_size
                out[m + "gate_proj.weight"], out[m + "up_proj.weight"] = layer.mlp.gu_w[:F], layer.mlp.gu_w[F:]
                out[m + "down_proj.weight"] = layer.mlp.down_w
        return out

    def load_hf_state_dict(self, sd: dict[str, torch.Tensor]) -> None:
        """Copy Hugging Face weights (``model.layers.{i}.self_attn.q_proj.weight``
        etc.) into the fused layout."""
        cfg = self.cfg
        if "model.embed_tokens.weight" not in sd and "model.language_model.embed_tokens.weight" in sd:
            # multimodal checkpoints (Qwen3.5): the language model under model.language_model.
            pre = "model.language_model."
            sd = {("model." + k[len(pre):]) if k.startswith(pre) else k: v for k, v in sd.items()}
        g = lambda k: sd[k].to(device=self.device, dtype=self.dtype)  # noqa: E731
        # Qwen3-Next / Qwen3.5 store RMSNorm weights as offsets from one
        nz = (lambda k: sd[k].to(device=self.device, dtype=torch.float32).add(1.0).to(self.dtype)) \
            if cfg.norm_zero_centered else g
        self.embed.copy_(g("model.embed_tokens.weight"))
        self.final_norm.copy_(nz("model.norm.weight"))
        if not cfg.tie_word_embeddings and "lm_head.weight" in sd:
            self.lm_head.copy_(g("lm_head.weight"))
        for i, layer in enumerate(self.layers):
            p = f"model.layers.{i}."
            layer.in_norm.copy_(nz(p + "input_layernorm.weight"))
            layer.post_norm.copy_(nz(p + "post_attention_layernorm.weight"))
            if layer.kind == "attention":
                a = p + "self_attn."
                layer.qkv_w.copy_(torch.cat([g(a + "q_proj.weight"), g(a + "k_proj.weight"), g(a + "v_proj.weight")]))
                if layer.qkv_b is not None:
                    layer.qkv_b.copy_(torch.cat([g(a + "q_proj.bias"), g(a + "k_proj.bias"), g(a + "v_proj.bias")]))
                if layer.q_norm is not None:
                    layer.q_norm.copy_(nz(a + "q_norm.weight"))
                    layer.k_norm.copy_(nz(a + "k_norm.weight"))
                layer.o_w.copy_(g(a + "o_proj.weight"))
                if layer.o_b is not None:
                    layer.o_b.copy_(g(a + "o_proj.bias"))
                if layer.sinks is not None:
                    layer.sinks.copy_(sd[a + "sinks"].to(device=self.device, dtype=torch.float32))
            if layer.mlp is not None:
                m = p + "mlp."
                layer.mlp.gu_w.copy_(torch.cat([g(m + "gate_proj.weight"), g(m + "up_proj.weight")]))
                layer.mlp.down_w.copy_(g(m + "down_proj.weight"))
            if layer.moe is not None:
                layer.moe.load_hf(sd, p + "mlp.", g)
            if layer.gdn is not None:
                layer.gdn.load_hf(sd, p + "linear_attn.", g)
