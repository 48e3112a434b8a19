"""Gemma-4 text decoder (dense and with the MoE block) for training.

Architecture as in the Hugging Face ``gemma4_text`` model: sandwich
RMSNorms around attention and MLP (plain weights, eps inside the mean),
sliding-window layers with their own head size and default RoPE, full
attention layers with a wider head, proportional (partial) RoPE and, with
``attention_k_eq_v``, values taken from the key projection; q / k / v
RMSNorms (the value one without a weight) and attention scale 1; the last
``num_kv_shared_layers`` layers reuse the keys and values of the last
non-shared layer of their kind; per-layer input embeddings (PLE) gated into
the residual after the MLP; an optional expert block beside the dense MLP
(router on the RMS-normed residual with a learned scale and per-expert
output scales); a per-layer scalar; tied, soft-capped logits.

Reference: the reference registers Gemma-4 dense / MoE through its model
support handler (``src/art/megatron/model_support/handlers/gemma4.py``).

This family runs on PyTorch operations plus the LoRA projections of
``ops.fused`` (which use the CTA-pair GEMM where the shapes allow): the
tcgen05 attention kernels take head_dim <= 128 and a pre-norm layer, and
Gemma-4's full-attention heads are 512 wide, so attention here is the dense
prefix-tree attention of ``fused.attention_ref`` (fp32 math, O(T^2) memory
per head).  Adapters target q / k / v / o and gate / up / down (the
projections that exist in each layer); the experts, the router and the PLE
projections stay frozen.  One process or data parallelism only.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.nn.functional as F

from ..ops import fused
from ..ops.fused import AttnMeta
from .config import LoRASpec, ModelConfig
from .lora import LoRAStore, peft_key


def _kinds(cfg: ModelConfig) -> list[str]:
    return list(cfg.layer_types)


def _first_shared(cfg: ModelConfig) -> int:
    n = cfg.ex.get("num_kv_shared_layers", 0)
    return cfg.num_hidden_layers - n if n else cfg.num_hidden_layers


def _layer_dims(cfg: ModelConfig, i: int) -> tuple[bool, int, int, bool, bool, int]:
    """(full attention, head size, kv heads, values = keys, kv shared, MLP width) of layer ``i``."""
    ex = cfg.ex
    full = cfg.layer_types[i] != "sliding_attention"
    D = ex["global_head_dim"] if full and ex["global_head_dim"] else cfg.head_dim
    k_eq_v = bool(ex["attention_k_eq_v"]) and full
    nkv = ex["num_global_key_value_heads"] if k_eq_v else cfg.num_key_value_heads
    shared = i >= _first_shared(cfg) > 0
    Fm = cfg.intermediate_size * (2 if ex["use_double_wide_mlp"] and shared else 1)
    return full, D, nkv, k_eq_v, shared, Fm


def _share_source(cfg: ModelConfig, i: int) -> int:
    """The last non-shared layer of layer ``i``'s kind (keys / values it reuses)."""
    first = _first_shared(cfg)
    kinds = _kinds(cfg)[:first]
    return len(kinds) - 1 - kinds[::-1].index(cfg.layer_types[i])


def gemma4_lora_specs(cfg: ModelConfig, spec: LoRASpec) -> list[tuple[str, tuple[int, ...], str]]:
    r, H = spec.r, cfg.hidden_size
    t = set(spec.target_modules)
    out: list[tuple[str, tuple[int, ...], str]] = []
    for i in range(cfg.num_hidden_layers):
        _, D, nkv, k_eq_v, shared, Fm = _layer_dims(cfg, i)
        projs = [("q_proj", cfg.num_attention_heads * D)]
        if not shared:
            projs.append(("k_proj", nkv * D))
            if not k_eq_v:
                projs.append(("v_proj", nkv * D))
        for p, o in projs:
            if p in t:
                out.append((peft_key(i, "self_attn", p, "A"), (r, H), "A"))
                out.append((peft_key(i, "self_attn", p, "B"), (o, r), "B"))
        if "o_proj" in t:
            out.append((peft_key(i, "self_attn", "o_proj", "A"), (r, cfg.num_attention_heads * D), "A"))
            out.append((peft_key(i, "self_attn", "o_proj", "B"), (H, r), "B"))
        gu = [p for p in ("gate_proj", "up_proj") if p in t]
        for p in gu:
            out.append((peft_key(i, "mlp", p, "A"), (r, H), "A"))
        for p in gu:
            out.append((peft_key(i, "mlp", p, "B"), (Fm, r), "B"))
        if "down_proj" in t:
            out.append((peft_key(i, "mlp", "down_proj", "A"), (r, Fm), "A"))
            out.append((peft_key(i, "mlp", "down_proj", "B"), (H, r), "B"))
    return out


def _rms(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    """Gemma-4 RMSNorm: ``x (mean(x^2) + eps)^-1/2 [* w]`` in fp32, cast back."""
    xf = x.float()
    y = xf * torch.pow(xf.pow(2).mean(-1, keepdim=True) + eps, -0.5)
    if w is not None:
        y = y * w.float()
    return y.to(x.dtype)


def _rope(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE of ``x [T, heads, D]`` at positions ``pos`` (zero frequencies leave dims alone)."""
    ang = pos.float().unsqueeze(-1) * inv_freq.float().unsqueeze(0)  # [T, D/2]
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(x.dtype).unsqueeze(1), emb.sin().to(x.dtype).unsqueeze(1)
    d = x.shape[-1] // 2
    rot = torch.cat([-x[..., d:], x[..., :d]], -1)
    return x * cos + rot * sin


def _inv_freq(kind: str, cfg: ModelConfig, device: torch.device) -> torch.Tensor:
    ex = cfg.ex
    if kind == "sliding":
        typ, base, factor = ex["rope_sliding_type"], ex["rope_sliding_theta"], ex["rope_sliding_factor"]
        partial, D = 1.0, cfg.head_dim
    else:
        typ, base, factor = ex["rope_full_type"], ex["rope_full_theta"], ex["rope_full_factor"]
        partial = ex["rope_full_partial"]
        D = ex["global_head_dim"] if typ == "proportional" else cfg.head_dim
    if typ == "proportional":
        # the first int(partial * D / 2) frequencies rotate, the rest are zero
        angles = int(partial * D // 2)
        rot = 1.0 / (base ** (torch.arange(0, 2 * angles, 2, dtype=torch.int64).float() / D))
        inv = torch.cat([rot, torch.zeros(D // 2 - angles)]) if D // 2 > angles else rot
        return (inv / factor).to(device)
    if typ != "default":
        raise NotImplementedError(f"Gemma-4 RoPE type {typ!r}")
    return (1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))).to(device)


class _G4Layer:
    pass


class Gemma4LM:
    """The training model of the Gemma-4 family (same interface as
    :class:`~art_mlx_b200.models.transformer.DecoderLM` for the trainer)."""

    def __init__(self, cfg: ModelConfig, lora: LoRASpec, device: torch.device | str = "cpu",
                 dtype: torch.dtype | None = None, seed: int = 0, store: LoRAStore | None = None,
                 ep: Any = None, etp: Any = None) -> None:
        from .transformer import _randn, make_binding

        if ep is not None or etp is not None:
            raise NotImplementedError("Gemma-4 trains on one GPU or with data parallelism only")
        self.cfg, self.lora_spec = cfg, lora
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        self.store = store or LoRAStore(gemma4_lora_specs(cfg, lora), self.device, self.dtype)
        if store is None:
            self.store.init_(seed + 1)
        gen = torch.Generator(device=self.device).manual_seed(seed)
        dev, dt, ex = self.device, self.dtype, cfg.ex
        H, V, L = cfg.hidden_size, cfg.vocab_size, cfg.num_hidden_layers
        ones = lambda n: torch.ones(n, device=dev, dtype=dt)  # noqa: E731
        self.embed = _randn((V, H), gen, dev, dt)
        self.lm_head = self.embed if cfg.tie_word_embeddings else _randn((V, H), gen, dev, dt)
        self.final_norm = ones(H)
        self.softcap = float(ex.get("final_logit_softcapping", 0.0) or 0.0)
        self.Hp = int(ex.get("hidden_size_per_layer_input", 0) or 0)
        if self.Hp:
            self.ple_embed = _randn((ex["vocab_size_per_layer_input"], L * self.Hp), gen, dev, dt)
            self.ple_proj = _randn((L * self.Hp, H), gen, dev, dt)
            self.ple_norm = ones(self.Hp)
        self.inv_freq = {"sliding": _inv_freq("sliding", cfg, dev), "full": _inv_freq("full", cfg, dev)}
        st, spec = self.store, lora
        self.layers: list[_G4Layer] = []
        for i in range(L):
            full, D, nkv, k_eq_v, shared, Fm = _layer_dims(cfg, i)
            ly = _G4Layer()
            ly.index, ly.kind, ly.full, ly.D = i, "attention", full, D
            ly.nkv, ly.k_eq_v, ly.shared = nkv, k_eq_v, shared
            ly.window = 0 if full else int(cfg.sliding_window or 0)
            ly.src = _share_source(cfg, i) if shared else i
            nq = cfg.num_attention_heads
            ly.q_w = _randn((nq * D, H), gen, dev, dt)
            ly.k_w = _randn((nkv * D, H), gen, dev, dt)
            ly.v_w = None if k_eq_v else _randn((nkv * D, H), gen, dev, dt)
            ly.o_w = _randn((H, nq * D), gen, dev, dt)
            ly.q_norm, ly.k_norm = ones(D), ones(D)
            ly.in_norm, ly.post_attn_norm, ly.pre_ff_norm, ly.post_ff_norm = ones(H), ones(H), ones(H), ones(H)
            ly.gu_w = _randn((2 * Fm, H), gen, dev, dt)
            ly.down_w = _randn((H, Fm), gen, dev, dt)
            ly.scalar = ones(1)
            ly.q_lora = make_binding(st, i, "self_attn", [("q_proj", nq * D)], spec)
            ly.k_lora = make_binding(st, i, "self_attn", [("k_proj", nkv * D)], spec)
            ly.v_lora = make_binding(st, i, "self_attn", [("v_proj", nkv * D)], spec)
            ly.o_lora = make_binding(st, i, "self_attn", [("o_proj", H)], spec)
            ly.gu_lora = make_binding(st, i, "mlp", [("gate_proj", Fm), ("up_proj", Fm)], spec)
            ly.down_lora = make_binding(st, i, "mlp", [("down_proj", H)], spec)
            if self.Hp:
                ly.ple_gate = _randn((self.Hp, H), gen, dev, dt)
                ly.ple_up = _randn((H, self.Hp), gen, dev, dt)
                ly.ple_post_norm = ones(H)
            ly.moe = None
            if ex.get("enable_moe_block"):
                E, Fe = ex["moe_num_experts"], ex["moe_intermediate_size"]
                ly.moe = dict(
                    router_w=_randn((E, H), gen, dev, dt), router_scale=ones(H), expert_scale=ones(E),
                    gu=_randn((E, 2 * Fe, H), gen, dev, dt), down=_randn((E, H, Fe), gen, dev, dt),
                    post1=ones(H), pre2=ones(H), post2=ones(H),
                )
            self.layers.append(ly)
        self.lora_enabled = True  # (no per-layer activation recompute in this family)

    # ------------------------------------------------------------------ pieces
    def _act(self, x: torch.Tensor) -> torch.Tensor:
        a = self.cfg.ex.get("hidden_activation", "gelu_pytorch_tanh")
        if a in ("gelu_pytorch_tanh", "gelu_tanh", "gelu_new"):
            return F.gelu(x, approximate="tanh")
        if a == "gelu":
            return F.gelu(x)
        if a == "silu":
            return F.silu(x)
        raise NotImplementedError(f"activation {a!r}")

    def _per_layer_inputs(self, tokens: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        T, L, Hp, H = tokens.shape[0], self.cfg.num_hidden_layers, self.Hp, self.cfg.hidden_size
        ple = self.ple_embed[tokens.clamp_min(0)] * torch.tensor(Hp ** 0.5, dtype=self.dtype, device=x.device)
        proj = (x @ self.ple_proj.t()) * (H ** -0.5)
        proj = _rms(proj.view(T, L, Hp), self.ple_norm, self.cfg.rms_norm_eps)
        return (proj + ple.view(T, L, Hp)) * (2.0 ** -0.5)

    def _attention(self, ly: _G4Layer, h: torch.Tensor, meta: AttnMeta, pos: torch.Tensor,
                   kv: dict[int, tuple[torch.Tensor, torch.Tensor]]) -> torch.Tensor:
        cfg, v, en, eps = self.cfg, self.store.version, self.lora_enabled, self.cfg.rms_norm_eps
        T, nq, D = h.shape[0], cfg.num_attention_heads, ly.D
        inv = self.inv_freq["full" if ly.full else "sliding"]
        q = fused.lora_linear(h, ly.q_w, None, ly.q_lora, v, en).view(T, nq, D)
        q = _rope(_rms(q, ly.q_norm, eps), pos, inv)
        if ly.shared:
            k, val = kv[ly.src]
        else:
            kr = fused.lora_linear(h, ly.k_w, None, ly.k_lora, v, en).view(T, ly.nkv, D)
            vr = kr if ly.v_w is None else fused.lora_linear(h, ly.v_w, None, ly.v_lora, v, en).view(T, ly.nkv, D)
            k = _rope(_rms(kr, ly.k_norm, eps), pos, inv)
            val = _rms(vr, None, eps)
            kv[ly.index] = (k, val)
        o, _ = fused.attention_ref(q, k, val, meta.kend, 1.0, positions=meta.positions, window=ly.window)
        return fused.lora_linear(o.reshape(T, nq * D), ly.o_w, None, ly.o_lora, v, en)

    def _experts(self, ly: _G4Layer, resid: torch.Tensor, ctx: dict[str, Any]) -> torch.Tensor:
        m, ex, eps, H = ly.moe, self.cfg.ex, self.cfg.rms_norm_eps, self.cfg.hidden_size
        hn = _rms(resid, None, eps) * m["router_scale"] * (H ** -0.5)
        probs = torch.softmax((hn @ m["router_w"].t()).float(), dim=-1)
        replay = ctx.get("replay_routes")
        if replay is not None:
            idx = replay[:, ly.index].long()
            w = probs.gather(1, idx)
        else:
            w, idx = probs.topk(ex["moe_top_k"], dim=-1)
        rec = ctx.get("record_routes")
        if rec is not None:
            rec[ly.index] = idx.detach().to(torch.int32)
        w = w / w.sum(-1, keepdim=True)
        w = (w * m["expert_scale"].float()[idx]).to(resid.dtype)
        x = _rms(resid, m["pre2"], eps)
        out = torch.zeros_like(x)
        for e in torch.unique(idx).tolist():
            tok, slot = torch.where(idx == e)
            g, u = (x[tok] @ m["gu"][e].t()).chunk(2, dim=-1)
            y = (self._act(g) * u) @ m["down"][e].t()
            out = out.index_add(0, tok, y * w[tok, slot].unsqueeze(-1))
        return out

    def _layer(self, ly: _G4Layer, x: torch.Tensor, meta: AttnMeta, pos: torch.Tensor, ple: torch.Tensor | None,
               kv: dict, ctx: dict[str, Any]) -> torch.Tensor:
        eps, v, en = self.cfg.rms_norm_eps, self.store.version, self.lora_enabled
        a = self._attention(ly, _rms(x, ly.in_norm, eps), meta, pos, kv)
        x = x + _rms(a, ly.post_attn_norm, eps)
        resid = x
        h = _rms(x, ly.pre_ff_norm, eps)
        g, u = fused.lora_linear(h, ly.gu_w, None, ly.gu_lora, v, en).chunk(2, dim=-1)
        m = fused.lora_linear(self._act(g) * u, ly.down_w, None, ly.down_lora, v, en)
        if ly.moe is not None:
            m = _rms(m, ly.moe["post1"], eps) + _rms(self._experts(ly, resid, ctx), ly.moe["post2"], eps)
        x = resid + _rms(m, ly.post_ff_norm, eps)
        if ple is not None:
            p = self._act(x @ ly.ple_gate.t()) * ple[:, ly.index]
            x = x + _rms(p @ ly.ple_up.t(), ly.ple_post_norm, eps)
        return x * ly.scalar

    # ------------------------------------------------------------------ model
    def forward(self, tokens: torch.Tensor, meta: AttnMeta, ctx: dict[str, Any] | None = None) -> torch.Tensor:
        """Final-normed hidden states ``[T, hidden]`` for one packed row."""
        ctx = ctx if ctx is not None else {}
        if ctx.get("cp_plan") is not None:
            raise NotImplementedError("Gemma-4 runs without context parallelism")
        H = self.cfg.hidden_size
        x = self.embed[tokens.clamp_min(0)] * torch.tensor(H ** 0.5, dtype=self.dtype, device=tokens.device)
        ple = self._per_layer_inputs(tokens, x) if self.Hp else None
        pos = meta.positions.to(tokens.device).long()
        kv: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        for ly in self.layers:
            x = self._layer(ly, x, meta, pos, ple, kv, ctx)
        return _rms(x, self.final_norm, self.cfg.rms_norm_eps)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """Soft-capped logits ``cap * tanh(h W^T / cap)`` (fp32)."""
        z = (h @ self.lm_head.t()).float()
        return torch.tanh(z / self.softcap) * self.softcap if self.softcap else z

    def token_logprobs_hidden(self, h: torch.Tensor, targets: torch.Tensor, chunk: int = 4096,
                              entropy: bool = True) -> tuple[torch.Tensor, torch.Tensor | None]:
        """``log softmax(softcap(h W^T))[target]`` per row (fp32) and the
        entropy; each row chunk's logits are recomputed in the backward
        instead of kept."""
        from torch.utils.checkpoint import checkpoint

        cap, W = self.softcap, self.lm_head

        def part(hc: torch.Tensor, tc: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
            z = (hc @ W.t()).float()
            if cap:
                z = torch.tanh(z / cap) * cap
            lse = torch.logsumexp(z, dim=-1)
            lp = z.gather(-1, tc.clamp_min(0).unsqueeze(-1)).squeeze(-1) - lse
            with torch.no_grad():
                logp = z - lse.unsqueeze(-1)
                ent = -(logp.exp() * logp).sum(-1)
            return lp, ent

        lps, ents = [], []
        step = max(1, min(chunk, 1024))
        for s in range(0, h.shape[0], step):
            hc, tc = h[s : s + step], targets[s : s + step]
            if torch.is_grad_enabled() and hc.requires_grad:
                lp, ent = checkpoint(part, hc, tc, use_reentrant=False)
            else:
                lp, ent = part(hc, tc)
            lps.append(lp)
            ents.append(ent)
        lp = torch.cat(lps) if lps else h.new_zeros(0, dtype=torch.float32)
        ent = (torch.cat(ents) if ents else h.new_zeros(0, dtype=torch.float32)) if entropy else None
        return lp, ent

    # ------------------------------------------------------------------ weights
    def _hf_map(self) -> dict[str, tuple[Any, str]]:
        """HF name -> (holder, attribute or key) of every base tensor."""
        m: dict[str, tuple[Any, str]] = {"model.embed_tokens.weight": (self, "embed"),
                                         "model.norm.weight": (self, "final_norm")}
        if not self.cfg.tie_word_embeddings:
            m["lm_head.weight"] = (self, "lm_head")
        if self.Hp:
            m["model.embed_tokens_per_layer.weight"] = (self, "ple_embed")
            m["model.per_layer_model_projection.weight"] = (self, "ple_proj")
            m["model.per_layer_projection_norm.weight"] = (self, "ple_norm")
        for ly in self.layers:
            p = f"model.layers.{ly.index}."
            m.update({p + "self_attn.q_proj.weight": (ly, "q_w"), p + "self_attn.k_proj.weight": (ly, "k_w"),
                      p + "self_attn.o_proj.weight": (ly, "o_w"), p + "self_attn.q_norm.weight": (ly, "q_norm"),
                      p + "self_attn.k_norm.weight": (ly, "k_norm"), p + "input_layernorm.weight": (ly, "in_norm"),
                      p + "post_attention_layernorm.weight": (ly, "post_attn_norm"),
                      p + "pre_feedforward_layernorm.weight": (ly, "pre_ff_norm"),
                      p + "post_feedforward_layernorm.weight": (ly, "post_ff_norm"),
                      p + "mlp.down_proj.weight": (ly, "down_w"), p + "layer_scalar": (ly, "scalar")})
            if ly.v_w is not None:
                m[p + "self_attn.v_proj.weight"] = (ly, "v_w")
            if self.Hp:
                m.update({p + "per_layer_input_gate.weight": (ly, "ple_gate"),
                          p + "per_layer_projection.weight": (ly, "ple_up"),
                          p + "post_per_layer_input_norm.weight": (ly, "ple_post_norm")})
            if ly.moe is not None:
                d = ly.moe
                m.update({p + "router.proj.weight": (d, "router_w"), p + "router.scale": (d, "router_scale"),
                          p + "router.per_expert_scale": (d, "expert_scale"),
                          p + "experts.gate_up_proj": (d, "gu"), p + "experts.down_proj": (d, "down"),
                          p + "post_feedforward_layernorm_1.weight": (d, "post1"),
                          p + "pre_feedforward_layernorm_2.weight": (d, "pre2"),
                          p + "post_feedforward_layernorm_2.weight": (d, "post2")})
        return m

    @staticmethod
    def _get(holder: Any, key: str) -> torch.Tensor:
        return holder[key] if isinstance(holder, dict) else getattr(holder, key)

    @staticmethod
    def _set(holder: Any, key: str, t: torch.Tensor) -> None:
        if isinstance(holder, dict):
            holder[key] = t
        else:
            setattr(holder, key, t)

    def load_hf_state_dict(self, sd: dict[str, torch.Tensor]) -> None:
        """Base weights from a Hugging Face Gemma-4 checkpoint (text model, or
        the language model of the multimodal one)."""
        norm = {}
        for k, t in sd.items():
            if k.startswith("model.language_model."):
                k = "model." + k[len("model.language_model."):]
            norm[k] = t
        missing = []
        for name, (holder, key) in self._hf_map().items():
            src = norm.get(name)
            if src is None:
                missing.append(name)
                continue
            cur = self._get(holder, key)
            self._set(holder, key, src.to(cur.device, cur.dtype).reshape(cur.shape).contiguous())
        for ly in self.layers:
            p = f"model.layers.{ly.index}.mlp."
            g, u = norm.get(p + "gate_proj.weight"), norm.get(p + "up_proj.weight")
            if g is None or u is None:
                missing.append(p + "gate_proj/up_proj")
                continue
            ly.gu_w = torch.cat([g, u]).to(ly.gu_w.device, ly.gu_w.dtype).contiguous()
        if self.cfg.tie_word_embeddings:
            self.lm_head = self.embed
        if missing:
            raise KeyError(f"Gemma-4 checkpoint lacks {missing[:4]}{' ...' if len(missing) > 4 else ''}")

    def hf_state_dict(self) -> dict[str, torch.Tensor]:
        out = {name: self._get(h, k) for name, (h, k) in self._hf_map().items()}
        for ly in self.layers:
            F2 = ly.gu_w.shape[0] // 2
            out[f"model.layers.{ly.index}.mlp.gate_proj.weight"] = ly.gu_w[:F2]
            out[f"model.layers.{ly.index}.mlp.up_proj.weight"] = ly.gu_w[F2:]
        return out

    def num_parameters(self) -> int:
        seen, n = set(), 0
        for name, (h, k) in self._hf_map().items():
            t = self._get(h, k)
            if id(t) not in seen:
                seen.add(id(t))
                n += t.numel()
        return n + sum(ly.gu_w.numel() for ly in self.layers)

