"""Gated DeltaNet linear-attention layer (Qwen3-Next-style hybrid models).

Per head, with state ``S`` [dk, dv]:

    S_t = exp(g_t) (I - beta_t k_t k_t^T) S_{t-1} + beta_t k_t v_t^T,   o_t = S_t^T q_t

(q, k L2-normalised, q scaled by 1/sqrt(dk); beta = sigmoid(b);
g = -exp(A_log) * softplus(a + dt_bias)).  Layer: in_proj_qkvz and in_proj_ba
projections, depthwise causal conv (width 4) + SiLU over q/k/v, the delta
rule, gated RMSNorm ``rmsnorm(o) * w * silu(z)``, out_proj.

Chunked form (chunk C = 64, following the WY representation of the delta
rule).  With G the in-chunk cumulative log decay, gamma = exp(G),
L_ij = beta_i exp(G_i - G_j) k_i.k_j (j < i) and T = (I + L)^{-1}:

    W = T (beta gamma * K),  U0 = T (beta * V),  U = U0 - W S_in
    O = (gamma * Q) S_in + ((Q K^T) * M) U,  M_ij = exp(G_i - G_j) (j <= i)
    S_out = gamma_C S_in + (exp(G_C - G) * K)^T U  =  A S_in + B

with A = gamma_C I - Kd^T W and B = Kd^T U0.  Everything except the scan
``S_{c+1} = A_c S_c + B_c`` is batched over all chunks; a span of chunks
collapses into one affine summary (A, B) — the quantity context
parallelism exchanges between ranks (reference ``gdn/fla_cp.py:315-580``).

Prefix trees: a segment starts from its parent's final state (zero for
roots); siblings of one parent are batched.  The causal conv reads each
token's sequence predecessors, crossing into the parent segment at the start
of a branch.
"""

from __future__ import annotations

import math
from typing import Any

import torch

from ..ops import fused
from ..ops import gdn as gdn_ops
from ..ops.fused import AttnMeta, LoRABinding
from .config import LoRASpec, ModelConfig
from .lora import LoRAStore, peft_key

CHUNK = 64


def gdn_lora_specs(cfg: ModelConfig, i: int, spec: LoRASpec) -> list[tuple[str, tuple[int, ...], str]]:
    """LoRA on the GDN input projection (q|k|v|z) and output projection when
    the attention projections are targeted."""
    r, H = spec.r, cfg.hidden_size
    kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
    vd = cfg.linear_num_value_heads * cfg.linear_value_head_dim
    t = set(spec.target_modules)
    out: list[tuple[str, tuple[int, ...], str]] = []
    if cfg.gdn_split_proj:  # Qwen3.5: in_proj_qkv and in_proj_z are separate modules (adapter keys too)
        sel = [(p, o) for p, o in (("in_proj_qkv", 2 * kd + vd), ("in_proj_z", vd))
               if p in t or t & {"q_proj", "k_proj", "v_proj"}]
        for p, _ in sel:
            out.append((peft_key(i, "linear_attn", p, "A"), (r, H), "A"))
        for p, o in sel:
            out.append((peft_key(i, "linear_attn", p, "B"), (o, r), "B"))
    elif t & {"q_proj", "k_proj", "v_proj", "in_proj_qkvz"}:
        out.append((peft_key(i, "linear_attn", "in_proj_qkvz", "A"), (r, H), "A"))
        out.append((peft_key(i, "linear_attn", "in_proj_qkvz", "B"), (2 * kd + 2 * vd, r), "B"))
    if t & {"o_proj", "out_proj"}:
        out.append((peft_key(i, "linear_attn", "out_proj", "A"), (r, vd), "A"))
        out.append((peft_key(i, "linear_attn", "out_proj", "B"), (H, r), "B"))
    return out


# ---------------------------------------------------------------------------
# core math
# ---------------------------------------------------------------------------


def chunk_parts(q, k, v, g, beta, C: int = CHUNK):
    """Intra-chunk operands of the scan for sequences ``[N, L, H, d]`` (L a
    multiple of C), all batched over chunks.  Returns (shapes ``[N, H, nc,
    ...]``) gq = gamma*Q, W, U0, QKM = (Q K^T)*M, Kd = exp(G_C - G)*K and
    gC = gamma_C ``[N, H, nc]``."""
    N, L, Hh, dk = k.shape
    dv = v.shape[-1]
    nc = L // C
    f = lambda t, d: t.reshape(N, nc, C, Hh, d).permute(0, 3, 1, 2, 4)  # noqa: E731  [N,H,nc,C,d]
    Q, K, V = f(q, dk), f(k, dk), f(v, dv)
    G = torch.cumsum(g.reshape(N, nc, C, Hh).permute(0, 3, 1, 2), dim=-1)  # [N,H,nc,C]
    bt = beta.reshape(N, nc, C, Hh).permute(0, 3, 1, 2)
    gamma = torch.exp(G)
    diff = G.unsqueeze(-1) - G.unsqueeze(-2)  # G_i - G_j
    tril_strict = torch.ones(C, C, dtype=torch.bool, device=k.device).tril(-1)
    tril = torch.ones(C, C, dtype=torch.bool, device=k.device).tril()
    decay = torch.exp(torch.where(tril, diff, torch.full_like(diff, -float("inf"))))
    KK = K @ K.transpose(-1, -2)
    Lm = torch.where(tril_strict, bt.unsqueeze(-1) * decay * KK, torch.zeros_like(KK))
    eye = torch.eye(C, dtype=k.dtype, device=k.device)
    Tinv = torch.linalg.solve_triangular(eye + Lm, eye.expand_as(Lm), upper=False, unitriangular=True)
    W = Tinv @ ((bt * gamma).unsqueeze(-1) * K)
    U0 = Tinv @ (bt.unsqueeze(-1) * V)
    QKM = (Q @ K.transpose(-1, -2)) * decay
    Kd = torch.exp(G[..., -1:] - G).unsqueeze(-1) * K  # [N,H,nc,C,dk]
    return gamma.unsqueeze(-1) * Q, W, U0, QKM, Kd, gamma[..., -1]


def chunk_summaries(q, k, v, g, beta, C: int = CHUNK):
    """:func:`chunk_parts` with each chunk's affine map instead of (Kd, gC):
    returns gq, W, U0, QKM, A = gamma_C I - Kd^T W, B = Kd^T U0."""
    gq, W, U0, QKM, Kd, gC = chunk_parts(q, k, v, g, beta, C)
    dk = W.shape[-1]
    A = gC[..., None, None] * torch.eye(dk, dtype=W.dtype, device=W.device) - Kd.transpose(-1, -2) @ W
    B = Kd.transpose(-1, -2) @ U0
    return gq, W, U0, QKM, A, B


def delta_rule(q, k, v, g, beta, S0=None, C: int = CHUNK):
    """Chunked gated delta rule.  Inputs ``[N, L, H, d]``, ``g``/``beta``
    ``[N, L, H]``, optional initial state ``[N, H, dk, dv]``.  Returns
    ``(o [N, L, H, dv], S_end)``.  Lengths are padded to ``C`` internally
    (padded steps: g=0, beta=0, k=0, which leave the state unchanged).  The
    intra-chunk operands are batched GEMMs; the chunk recurrence is the
    ``gdn_scan`` kernel on CUDA."""
    N, L, Hh, dk = k.shape
    dv = v.shape[-1]
    pad = (-L) % C
    if pad:
        P = lambda t: torch.nn.functional.pad(t, (0, 0, 0, 0, 0, pad)) if t.dim() == 4 else torch.nn.functional.pad(t, (0, 0, 0, pad))  # noqa: E731
        q, k, v, g, beta = P(q), P(k), P(v), P(g), P(beta)
    gq, W, U0, QKM, Kd, gC = chunk_parts(q, k, v, g, beta, C)
    nc = gq.shape[2]
    o, S = gdn_ops.scan(gq, W, U0, QKM, Kd, gC, S0)
    o = o.permute(0, 2, 3, 1, 4).reshape(N, nc * C, Hh, dv)[:, :L]
    return o, S


def delta_rule_reference(q, k, v, g, beta, S0=None):
    """Token-by-token recurrence (test oracle)."""
    N, L, Hh, dk = k.shape
    dv = v.shape[-1]
    S = S0.clone() if S0 is not None else q.new_zeros(N, Hh, dk, dv)
    outs = []
    for t in range(L):
        S = S * torch.exp(g[:, t]).view(N, Hh, 1, 1)
        kt = k[:, t]
        pred = torch.einsum("nhk,nhkv->nhv", kt, S)
        delta = (v[:, t] - pred) * beta[:, t].unsqueeze(-1)
        S = S + kt.unsqueeze(-1) * delta.unsqueeze(-2)
        outs.append(torch.einsum("nhk,nhkv->nhv", q[:, t], S))
    return torch.stack(outs, 1), S


# ---------------------------------------------------------------------------
# prefix-tree plan
# ---------------------------------------------------------------------------


def sequence_predecessors(segs: list[tuple[int, int, int]], T: int, width: int) -> torch.Tensor:
    """Conv predecessor table of a packed tree row: ``prev[i, m]`` is the
    packed index of the token ``m+1`` positions before ``i`` in its sequence
    (walking from a segment's start into its ancestors), -1 before the
    sequence start.  ``segs`` = (start, end, parent segment or -1)."""
    prev = torch.full((T, width - 1), -1, dtype=torch.int64)
    for n, (s, e, p) in enumerate(segs):
        for m in range(1, width):
            if e - s > m:  # inside the segment
                prev[s + m : e, m - 1] = torch.arange(s, e - m)
            for i in range(s, min(e, s + m)):  # first m tokens: into the ancestors
                need = m - (i - s)
                anc, pos = p, None
                while anc >= 0:
                    a_s, a_e, a_p = segs[anc]
                    if a_e - a_s >= need:
                        pos = a_e - need
                        break
                    need -= a_e - a_s
                    anc = a_p
                prev[i, m - 1] = pos if pos is not None else -1
    return prev


class TreePlan:
    """Segments of one packed row grouped by depth, plus the conv
    predecessor table (``prev[i, m]`` = packed index of the token ``m+1``
    positions before ``i`` in its sequence, -1 before the sequence start)."""

    def __init__(self, meta: AttnMeta, group_ids: torch.Tensor | None, parent_ids: torch.Tensor | None, T: int,
                 width: int = 4) -> None:
        from ..preprocessing.prefix_tree import parse_prefix_tree_row

        if group_ids is None:
            segs = [(0, T, -1)]
        else:
            parsed = parse_prefix_tree_row(group_ids[:T], parent_ids[:T])
            idx = {s.group_id: n for n, s in enumerate(parsed)}
            segs = [(s.start, s.end, idx[s.parent_id] if s.parent_id != s.group_id else -1) for s in parsed]
            covered = parsed[-1].end if parsed else 0
            if covered < T:  # trailing padding: its own root segment
                segs.append((covered, T, -1))
        self.segs = segs
        depth = []
        for s, e, p in segs:
            depth.append(0 if p < 0 else depth[p] + 1)
        self.levels: list[list[int]] = []
        for n, d in enumerate(depth):
            while len(self.levels) <= d:
                self.levels.append([])
            self.levels[d].append(n)
        prev = sequence_predecessors(segs, T, width)
        dev = meta.kend.device
        self.prev = prev.to(dev, non_blocking=True)
        # inverse table for the conv backward kernel (CUDA only)
        self.succ = gdn_ops.successors(prev, dev) if dev.type == "cuda" else None


def causal_conv(x: torch.Tensor, w: torch.Tensor, prev: torch.Tensor) -> torch.Tensor:
    """Depthwise causal conv along sequences: y_i = w[:, -1] x_i +
    sum_m w[:, -1-m] x_{prev_m(i)};  x [T, Cc], w [Cc, width]."""
    y = x * w[:, -1]
    for m in range(prev.shape[1]):
        idx = prev[:, m]
        valid = (idx >= 0).unsqueeze(1).to(x.dtype)
        y = y + x.index_select(0, idx.clamp_min(0)) * valid * w[:, -2 - m]
    return y


def tree_delta_rule(q, k, v, g, beta, plan: TreePlan, finals_out: dict | None = None):
    """Delta rule over a packed prefix-tree row: ``[T, H, d]`` inputs.
    ``finals_out`` (optional) receives each segment's final state."""
    T, Hh, dk = k.shape
    dv = v.shape[-1]
    out = q.new_zeros(T, Hh, dv)
    finals: dict[int, torch.Tensor] = {}
    outs = []
    for level in plan.levels:
        Lmax = max(plan.segs[n][1] - plan.segs[n][0] for n in level)
        idx = torch.full((len(level), Lmax), -1, dtype=torch.int64)
        for row, n in enumerate(level):
            s, e, _ = plan.segs[n]
            idx[row, : e - s] = torch.arange(s, e)
        idx = idx.to(q.device)
        valid = (idx >= 0)
        gi = idx.clamp_min(0)
        take = lambda t: t[gi] * valid.view(*valid.shape, *([1] * (t.dim() - 1))).to(t.dtype)  # noqa: E731
        S0 = torch.stack([
            finals[plan.segs[n][2]] if plan.segs[n][2] >= 0 else q.new_zeros(Hh, dk, dv) for n in level
        ])
        o, S = delta_rule(take(q), take(k), take(v), take(g), take(beta), S0)
        for row, n in enumerate(level):
            finals[n] = S[row]
        outs.append((idx, valid, o))
    for idx, valid, o in outs:
        sel = valid.reshape(-1)
        out = out.index_copy(0, idx.reshape(-1)[sel], o.reshape(-1, Hh, dv)[sel])
    if finals_out is not None:
        finals_out.update(finals)
    return out


# ---------------------------------------------------------------------------
# the layer
# ---------------------------------------------------------------------------


class GatedDeltaNet:
    def __init__(self, cfg: ModelConfig, i: int, gen, dev, dt, store: LoRAStore, spec: LoRASpec) -> None:
        from .transformer import _randn, make_binding

        self.cfg, self.index = cfg, i
        H = cfg.hidden_size
        self.nk, self.nv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        kd, vd = self.nk * self.dk, self.nv * self.dv
        self.kd, self.vd = kd, vd
        self.qkvz_w = _randn((2 * kd + 2 * vd, H), gen, dev, dt)
        self.ba_w = _randn((2 * self.nv, H), gen, dev, dt)
        self.conv_w = _randn((2 * kd + vd, cfg.linear_conv_kernel_dim), gen, dev, dt, std=0.2)
        self.dt_bias = torch.ones(self.nv, device=dev, dtype=torch.float32)
        self.A_log = torch.log(torch.arange(1, self.nv + 1, device=dev, dtype=torch.float32))
        self.norm_w = torch.ones(self.dv, device=dev, dtype=dt)
        self.out_w = _randn((H, vd), gen, dev, dt)
        projs = ([("in_proj_qkv", 2 * kd + vd), ("in_proj_z", vd)] if cfg.gdn_split_proj
                 else [("in_proj_qkvz", 2 * kd + 2 * vd)])
        self.qkvz_lora = make_binding(store, i, "linear_attn", projs, spec)
        self.out_lora = make_binding(store, i, "linear_attn", [("out_proj", H)], spec)

    def num_parameters(self) -> int:
        return sum(t.numel() for t in (self.qkvz_w, self.ba_w, self.conv_w, self.out_w, self.norm_w))

    def load_hf(self, sd: dict[str, torch.Tensor], prefix: str, g) -> None:
        """Hugging Face weights into the [q | k | v | z] and [b | a] layouts:
        Qwen3.5 stores the projections split (``in_proj_qkv``, ``in_proj_z``,
        ``in_proj_b``, ``in_proj_a``), Qwen3-Next grouped per key head
        (``in_proj_qkvz`` rows ``[q | k | v_group | z_group]`` per key head,
        ``in_proj_ba`` rows ``[b_group | a_group]``)."""
        nk, nv, dk, dv, H = self.nk, self.nv, self.dk, self.dv, self.cfg.hidden_size
        rep = nv // nk
        if prefix + "in_proj_qkv.weight" in sd:
            self.qkvz_w.copy_(torch.cat([g(prefix + "in_proj_qkv.weight"), g(prefix + "in_proj_z.weight")]))
            self.ba_w.copy_(torch.cat([g(prefix + "in_proj_b.weight"), g(prefix + "in_proj_a.weight")]))
        else:
            w = g(prefix + "in_proj_qkvz.weight").view(nk, 2 * dk + 2 * rep * dv, H)
            q, k = w[:, :dk], w[:, dk : 2 * dk]
            v, z = w[:, 2 * dk : 2 * dk + rep * dv], w[:, 2 * dk + rep * dv :]
            self.qkvz_w.copy_(torch.cat([t.reshape(-1, H) for t in (q, k, v, z)]))
            ba = g(prefix + "in_proj_ba.weight").view(nk, 2 * rep, H)
            self.ba_w.copy_(torch.cat([ba[:, :rep].reshape(nv, H), ba[:, rep:].reshape(nv, H)]))
        self.conv_w.copy_(g(prefix + "conv1d.weight").reshape(self.conv_w.shape))
        self.dt_bias.copy_(sd[prefix + "dt_bias"].to(self.dt_bias.device, torch.float32))
        self.A_log.copy_(sd[prefix + "A_log"].to(self.A_log.device, torch.float32))
        self.norm_w.copy_(g(prefix + "norm.weight"))
        self.out_w.copy_(g(prefix + "out_proj.weight"))

    def mix(self, h: torch.Tensor, version: int, enabled: bool):
        """Projections + conv inputs: returns (qkv_pre_conv, z, g, beta)."""
        kd, vd = self.kd, self.vd
        qkvz = fused.lora_linear(h, self.qkvz_w, None, self.qkvz_lora, version, enabled)
        ba = h @ self.ba_w.t()
        b, a = ba[:, : self.nv].float(), ba[:, self.nv :].float()
        beta = torch.sigmoid(b)
        g = -torch.exp(self.A_log) * torch.nn.functional.softplus(a + self.dt_bias)
        return qkvz[:, : 2 * kd + vd], qkvz[:, 2 * kd + vd :], g, beta

    def core_inputs(self, qkv, plan_prev, succ=None):
        """Tree causal conv + SiLU (one kernel on CUDA), then the head split."""
        return self.split_heads(gdn_ops.conv_silu(qkv, self.conv_w, plan_prev, succ))

    def post_conv(self, x):
        """SiLU after the causal conv, split into q, k, v heads, L2-normalised q / k."""
        return self.split_heads(torch.nn.functional.silu(x.float()))

    def split_heads(self, x):
        """Split the activated conv output into q, k, v heads; L2-normalised q / k."""
        kd, T = self.kd, x.shape[0]
        q = x[:, :kd].view(T, self.nk, self.dk)
        k = x[:, kd : 2 * kd].view(T, self.nk, self.dk)
        v = x[:, 2 * kd :].view(T, self.nv, self.dv)
        # L2 normalisation with the eps inside the root (x / sqrt(|x|^2 + 1e-6)),
        # as the published gated-DeltaNet kernels and Qwen3-Next do
        q = q * torch.rsqrt(q.float().pow(2).sum(-1, keepdim=True) + 1e-6).to(q.dtype) / math.sqrt(self.dk)
        k = k * torch.rsqrt(k.float().pow(2).sum(-1, keepdim=True) + 1e-6).to(k.dtype)
        return q, k, v

    def expand_heads(self, q, k):
        if self.nv != self.nk:  # grouped value heads
            rep = self.nv // self.nk
            q = q.repeat_interleave(rep, dim=1)
            k = k.repeat_interleave(rep, dim=1)
        return q, k

    def decode_step(self, h: torch.Tensor, state: dict[str, torch.Tensor], version: int, enabled: bool) -> torch.Tensor:
        """One token per sequence: ``h`` [B, hidden]; ``state`` holds the
        delta-rule state ``S`` [B, H, dk, dv] and the conv tail ``tail``
        [B, width-1, C] (oldest first), both updated in place."""
        qkv, z, g, beta = self.mix(h, version, enabled)
        tail = state["tail"]
        K = tail.shape[1]
        w = self.conv_w
        y = qkv * w[:, -1]
        for m in range(K):  # the token m+1 positions back sits at tail[:, K-1-m]
            y = y + tail[:, K - 1 - m].to(qkv.dtype) * w[:, -2 - m]
        state["tail"] = torch.cat([tail[:, 1:], qkv.unsqueeze(1).to(tail.dtype)], dim=1)
        q, k, v = self.post_conv(y)
        q, k = self.expand_heads(q, k)
        o, S = delta_rule_reference(q.unsqueeze(1), k.unsqueeze(1), v.float().unsqueeze(1), g.unsqueeze(1),
                                    beta.unsqueeze(1), state["S"])
        state["S"] = S
        return self.finish(o[:, 0], z, version, enabled, h.dtype)

    def finish(self, o, z, version: int, enabled: bool, out_dtype):
        T = o.shape[0]
        of = o.float()
        r = torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps)
        zf = z.float().view(T, self.nv, self.dv)
        y = (of * r) * self.norm_w.float() * torch.nn.functional.silu(zf)
        y = y.reshape(T, self.vd).to(out_dtype)
        return fused.lora_linear(y, self.out_w, None, self.out_lora, version, enabled)

    def __call__(self, h: torch.Tensor, meta: AttnMeta, version: int, enabled: bool, ctx: dict[str, Any]) -> torch.Tensor:
        plan: TreePlan = ctx.get("gdn_plan")
        if plan is None:
            plan = TreePlan(meta, ctx.get("group_ids"), ctx.get("parent_ids"), h.shape[0],
                            self.cfg.linear_conv_kernel_dim)
            ctx["gdn_plan"] = plan
        qkv, z, g, beta = self.mix(h, version, enabled)
        q, k, v = self.core_inputs(qkv, plan.prev, plan.succ)
        q, k = self.expand_heads(q, k)
        finals = ctx.get("gdn_finals")
        out_finals = {} if finals is not None else None
        o = tree_delta_rule(q, k, v.float(), g, beta, plan, out_finals)
        if finals is not None:  # generation prefill: per-segment final states and conv inputs
            finals[self.index] = (out_finals, qkv)
        return self.finish(o, z, version, enabled, h.dtype)
