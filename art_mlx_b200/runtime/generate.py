"""Token generation on the training model (rollouts without a separate server).

The reference samples rollouts from vLLM (``src/art/vllm_runtime.py``,
``src/art/unsloth/service.py:585``) or, in the MLX fork, from an in-process
generator (``src/art/mlx/backend.py:163`` ``create_chat_completion``).
Here generation runs on the same :class:`DecoderLM` (and the same LoRA
store) the trainer updates, so a colocated policy needs no weight sync:

* **prefill**: every distinct prompt once (requests that share a prompt,
  e.g. the rollouts of one GRPO group, share its prefill), packed into one
  row of independent segments and run through the prefix-tree attention
  kernel; the rotated K and V of every attention layer are copied into the
  per-sequence KV cache;
* **decode**: one token per sequence per step: projections for the batch,
  ``kv_append`` + ``decode_attn`` (split-K decode kernel, ops/csrc/decode.cu)
  against the cache, LM head, sampling (temperature / top-p / greedy);
* the log-probability returned for each sampled token is the model's
  (temperature-free) log-softmax, the quantity the GRPO loss compares with;
* adapters: ``None`` samples from the live training adapter; a name selects
  an adapter registered with :meth:`add_adapter` (copied into the store's
  compute buffer for the call and restored afterwards); ``"base"`` disables
  LoRA.

Gated DeltaNet layers (hybrid models) run recurrently: the prefill runs the
chunked delta rule over each prompt and keeps its final state and the last
conv inputs per sequence; every decode step updates them with one token.

On CPU the same loop runs the PyTorch reference ops (tests).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

import torch

from ..ops import fused, native


@dataclass
class SamplingParams:
    max_tokens: int = 256
    temperature: float = 1.0
    top_p: float = 1.0
    stop_token_ids: Sequence[int] = ()
    seed: int | None = None


@dataclass
class GenerationResult:
    prompt_token_ids: list[int]
    token_ids: list[int] = field(default_factory=list)
    logprobs: list[float] = field(default_factory=list)
    finish_reason: str = "length"


class GenerationEngine:
    def __init__(self, model, max_len: int = 8192, max_batch: int = 256) -> None:
        if getattr(getattr(model, "cfg", None), "family", "") == "gemma4":
            raise NotImplementedError("the native rollout engine does not run Gemma-4; serve it with vLLM "
                                      "(LocalBackend(inference='vllm'))")
        cfg = model.cfg
        self.model, self.cfg = model, cfg
        self.device = model.device
        self.max_len = max_len  # KV-cache length per sequence (engine_args.max_model_len)
        self.max_batch = max(1, max_batch)  # sequences decoded together (engine_args.max_num_seqs)
        self.adapters: dict[str, torch.Tensor] = {}
        self._cache: tuple[list[torch.Tensor], list[torch.Tensor]] | None = None

    # ------------------------------------------------------------------ adapters
    def add_adapter(self, name: str, source: str | torch.Tensor) -> None:
        """Register an adapter from a checkpoint directory or a flat compute
        vector of the model's LoRA store."""
        st = self.model.store
        if isinstance(source, torch.Tensor):
            flat = source.to(device=st.compute.device, dtype=st.compute.dtype).clone()
        else:
            import os

            from safetensors.torch import load_file

            sd = load_file(os.path.join(source, "adapter_model.safetensors"))
            flat = torch.zeros_like(st.compute)
            for key, e in st.entries.items():
                if key in sd:
                    flat[e.offset : e.offset + e.numel].copy_(sd[key].reshape(-1).to(flat.dtype))
        self.adapters[name] = flat

    def remove_adapter(self, name: str) -> None:
        self.adapters.pop(name, None)

    # ------------------------------------------------------------------ model pieces
    def _qkv(self, layer, h):
        m, cfg = self.model, self.cfg
        v, en = m.store.version, m.lora_enabled
        qkv = fused.lora_linear(h, layer.qkv_w, layer.qkv_b, layer.qkv_lora, v, en)
        gate = None
        if cfg.attn_output_gate:
            T, nq, D = qkv.shape[0], cfg.num_attention_heads, cfg.head_dim
            qg = qkv[:, : 2 * cfg.q_size].view(T, nq, 2 * D)
            gate = qg[..., D:].reshape(T, cfg.q_size)
            qkv = torch.cat([qg[..., :D].reshape(T, cfg.q_size), qkv[:, 2 * cfg.q_size :]], dim=1).contiguous()
        return qkv, gate

    def _rope(self, layer, qkv, positions):
        """Rotated (and, for Qwen3, RMS-normed) q [T, nq, D], k [T, nkv, D], and v [T, nkv, D]."""
        cfg, m = self.cfg, self.model
        nq, nkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        T = qkv.shape[0]
        v = qkv[:, (nq + nkv) * D : (nq + 2 * nkv) * D].view(T, nkv, D)
        perm = getattr(m, "rope_perm", None)  # partial rotary: q / k in the kernels' dim order
        if qkv.is_cuda:
            qk, _ = native.lib().rope_fwd(qkv, positions, m.inv_freq, nq, nkv, D, layer.q_norm, layer.k_norm,
                                          cfg.rms_norm_eps, None if perm is None else perm.to(qkv.device))
            return qk[:, : nq * D].view(T, nq, D), qk[:, nq * D :].view(T, nkv, D), v
        q = qkv[:, : nq * D].view(T, nq, D)
        k = qkv[:, nq * D : (nq + nkv) * D].view(T, nkv, D)
        if layer.q_norm is not None:
            q = fused._rmsnorm_ref(q, layer.q_norm, cfg.rms_norm_eps)
            k = fused._rmsnorm_ref(k, layer.k_norm, cfg.rms_norm_eps)
        if perm is not None:
            q, k = q[..., perm.long()], k[..., perm.long()]
        return fused._rope_ref(q, positions, m.inv_freq), fused._rope_ref(k, positions, m.inv_freq), v

    def _layers(self, tokens: torch.Tensor, positions: torch.Tensor, attend, linear=None) -> torch.Tensor:
        m, cfg = self.model, self.cfg
        eps = cfg.rms_norm_eps
        out = m.embed[tokens]
        resid = None
        for li, layer in enumerate(m.layers):
            h, resid = fused.add_rmsnorm(out, resid, layer.in_norm, eps)
            if layer.kind != "attention":  # gated DeltaNet
                a = linear(li, layer, h)
                h, resid = fused.add_rmsnorm(a, resid, layer.post_norm, eps)
                out = m.mlp(layer, h, {})
                continue
            qkv, gate = self._qkv(layer, h)
            q, k, v = self._rope(layer, qkv, positions)
            o = attend(li, q, k, v).reshape(q.shape[0], -1)
            if gate is not None:
                o = o * torch.sigmoid(gate)
            a = fused.lora_linear(o, layer.o_w, None, layer.o_lora, m.store.version, m.lora_enabled)
            h, resid = fused.add_rmsnorm(a, resid, layer.post_norm, eps)
            out = m.mlp(layer, h, {})
        h, _ = fused.add_rmsnorm(out, resid, m.final_norm, eps)
        return h

    def _logits(self, h: torch.Tensor) -> torch.Tensor:
        return (h @ self.model.lm_head.t()).float()

    # ------------------------------------------------------------------ sampling
    @staticmethod
    def _sample(logits: torch.Tensor, p: SamplingParams, gen: torch.Generator | None):
        logp = torch.log_softmax(logits, dim=-1)
        if p.temperature <= 0:
            tok = logits.argmax(-1)
        else:
            probs = torch.softmax(logits / p.temperature, dim=-1)
            if p.top_p < 1.0:
                sp, si = probs.sort(-1, descending=True)
                keep = sp.cumsum(-1) - sp < p.top_p
                sp = sp * keep
                probs = torch.zeros_like(probs).scatter_(-1, si, sp)
            tok = torch.multinomial(probs, 1, generator=gen).squeeze(-1)
        return tok, logp.gather(-1, tok.unsqueeze(-1)).squeeze(-1)

    # ------------------------------------------------------------------ cache
    def _kv(self, B: int, L: int):
        cfg = self.cfg
        first = None if self._cache is None else next((c for c in self._cache[0] if c is not None), None)
        if self._cache is None or (first is not None and (first.shape[0] < B or first.shape[1] < L)):
            shape = (B, L, cfg.num_key_value_heads, cfg.head_dim)
            n = len(self.model.layers)
            dt = self.model.embed.dtype
            att = [layer.kind == "attention" for layer in self.model.layers]  # gated DeltaNet layers keep no KV
            self._cache = ([torch.empty(shape, device=self.device, dtype=dt) if a else None for a in att],
                           [torch.empty(shape, device=self.device, dtype=dt) if a else None for a in att])
        return self._cache

    # ------------------------------------------------------------------ generate
    @torch.no_grad()
    def generate(self, prompts: Sequence[Sequence[int]], params: SamplingParams | None = None,
                 adapter: str | None = None) -> list[GenerationResult]:
        p = params or SamplingParams()
        m = self.model
        st = m.store
        saved = None
        prev_enabled = m.lora_enabled
        if adapter == "base":
            m.lora_enabled = False
        elif adapter is not None:
            saved = st.compute.clone()
            st.compute.copy_(self.adapters[adapter])
            st.version += 1
        try:
            ps = [list(x) for x in prompts]
            out: list[GenerationResult] = []
            for a in range(0, len(ps), self.max_batch):
                out.extend(self._generate(ps[a : a + self.max_batch], p))
            return out
        finally:
            m.lora_enabled = prev_enabled
            if saved is not None:
                st.compute.copy_(saved)
                st.version += 1

    def _generate(self, prompts: list[list[int]], p: SamplingParams) -> list[GenerationResult]:
        B = len(prompts)
        if B == 0:
            return []
        dev = self.device
        cfg = self.cfg
        D = cfg.head_dim
        scale = 1.0 / math.sqrt(D)
        longest = max(len(x) for x in prompts)
        L = min(self.max_len, longest + p.max_tokens)
        if longest >= L:
            raise ValueError(f"prompt of {longest} tokens leaves no room under max_len={self.max_len}")
        kc, vc = self._kv(B, L)
        gen = None
        if p.seed is not None:
            gen = torch.Generator(device=dev)
            gen.manual_seed(p.seed)
        # ---- prefill: distinct prompts once, packed as independent segments
        uniq: dict[tuple[int, ...], int] = {}
        for x in prompts:
            uniq.setdefault(tuple(x), len(uniq))
        order = list(uniq)
        starts, toks, pos, kend = [], [], [], []
        for u in order:
            s = len(toks)
            starts.append(s)
            toks.extend(u)
            pos.extend(range(len(u)))
            kend.extend([s + len(u)] * len(u))
        T = len(toks)
        tok_t = torch.tensor(toks, dtype=torch.long).to(dev)
        pos_t = torch.tensor(pos, dtype=torch.int32).to(dev)
        kend_t = torch.tensor(kend, dtype=torch.int32)
        meta = fused.AttnMeta.build(pos_t, kend_t, dev)
        # cache fill map: (packed row, sequence slot, position) of every prompt token of every sequence
        rows_l, slot_l, posl = [], [], []
        for b, x in enumerate(prompts):
            s0 = starts[uniq[tuple(x)]]
            rows_l.extend(range(s0, s0 + len(x)))
            slot_l.extend([b] * len(x))
            posl.extend(range(len(x)))
        fill_rows = torch.tensor(rows_l, dtype=torch.long).to(dev)
        fill_slot = torch.tensor(slot_l, dtype=torch.int32).to(dev)
        fill_pos = torch.tensor(posl, dtype=torch.int32).to(dev)

        def attend_prefill(li, q, k, v):
            ks = k.index_select(0, fill_rows)
            vs = v.index_select(0, fill_rows)
            if q.is_cuda:
                C = native.lib()
                o, _ = C.attn_fwd_tc(q, k, v, meta.kend, meta.tile_kmax, meta.tile_kmin, scale)
                C.kv_append(ks.reshape(ks.shape[0], -1), vs.reshape(vs.shape[0], -1), fill_slot, fill_pos,
                            kc[li], vc[li])
                return o
            o, _ = fused.attention_ref(q, k, v, meta.kend, scale)
            kc[li][fill_slot.long(), fill_pos.long()] = ks.to(kc[li].dtype)
            vc[li][fill_slot.long(), fill_pos.long()] = vs.to(vc[li].dtype)
            return o

        # gated DeltaNet prefill: each distinct prompt is a root segment
        seg = torch.tensor([u + 1 for u, x in enumerate(order) for _ in x], dtype=torch.long)
        gdn_ctx = {"group_ids": seg, "parent_ids": seg, "gdn_finals": {}}
        K = cfg.linear_conv_kernel_dim - 1
        states: dict[int, dict[str, torch.Tensor]] = {}
        seq_u = [uniq[tuple(x)] for x in prompts]

        def linear_prefill(li, layer, h):
            a = layer.gdn(h, meta, self.model.store.version, self.model.lora_enabled, gdn_ctx)
            finals, qkv = gdn_ctx["gdn_finals"][layer.gdn.index]
            S = torch.stack([finals[u] for u in seq_u])
            tail = qkv.new_zeros(B, K, qkv.shape[1])
            for b, u in enumerate(seq_u):
                e = starts[u] + len(order[u])
                lo = max(starts[u], e - K)
                tail[b, K - (e - lo):] = qkv[lo:e]
            states[li] = {"S": S, "tail": tail}
            return a

        def linear_decode(li, layer, h):
            return layer.gdn.decode_step(h, states[li], self.model.store.version, self.model.lora_enabled)

        h = self._layers(tok_t, pos_t, attend_prefill, linear_prefill)
        last = torch.tensor([starts[uniq[tuple(x)]] + len(x) - 1 for x in prompts]).to(dev)
        tok, lp = self._sample(self._logits(h.index_select(0, last)), p, gen)
        lens = torch.tensor([len(x) for x in prompts], dtype=torch.int32, device=dev)
        results = [GenerationResult(prompt_token_ids=list(x)) for x in prompts]
        done = [False] * B
        stop = set(int(t) for t in p.stop_token_ids)
        slots = torch.arange(B, dtype=torch.int32, device=dev)
        for step in range(p.max_tokens):
            tl, ll = tok.tolist(), lp.tolist()
            for b in range(B):
                if done[b]:
                    continue
                results[b].token_ids.append(int(tl[b]))
                results[b].logprobs.append(float(ll[b]))
                if int(tl[b]) in stop:
                    done[b] = True
                    results[b].finish_reason = "stop"
                elif len(results[b].token_ids) >= p.max_tokens or int(lens[b]) + 1 >= L:
                    done[b] = True
                    results[b].finish_reason = "length"
            if all(done):
                break
            positions = lens.clone()  # the new token's position = current length
            lens = lens + 1

            def attend_decode(li, q, k, v):
                if q.is_cuda:
                    C = native.lib()
                    C.kv_append(k.reshape(B, -1), v.reshape(B, -1), slots, positions, kc[li], vc[li])
                    return C.decode_attn(q, kc[li], vc[li], lens, scale)
                kc[li][slots.long(), positions.long()] = k.to(kc[li].dtype)
                vc[li][slots.long(), positions.long()] = v.to(vc[li].dtype)
                return _decode_ref(q, kc[li][:B], vc[li][:B], lens, scale)

            h = self._layers(tok, positions, attend_decode, linear_decode)
            tok, lp = self._sample(self._logits(h), p, gen)
        return results


def _decode_ref(q, kc, vc, lens, scale):
    """One query per sequence against its first ``lens[b]`` cached keys."""
    B, Hq, D = q.shape
    Hkv = kc.shape[2]
    G = Hq // Hkv
    k = kc.float().repeat_interleave(G, dim=2)  # [B, L, Hq, D]
    v = vc.float().repeat_interleave(G, dim=2)
    s = torch.einsum("bhd,blhd->bhl", q.float(), k) * scale
    mask = torch.arange(kc.shape[1], device=q.device).view(1, 1, -1) < lens.view(B, 1, 1).to(q.device)
    s = s.masked_fill(~mask, float("-inf"))
    # cache rows past each length are unwritten memory: keep them out of the sum
    v = v.masked_fill(~mask.view(B, 1, -1).transpose(1, 2).unsqueeze(-1), 0.0)
    return torch.einsum("bhl,blhd->bhd", torch.softmax(s, -1), v).to(q.dtype)
