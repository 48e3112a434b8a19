"""Context parallelism for long packed prefix-tree rows.

Reference behaviour: planner-driven all-to-all-v context parallelism for
attention plus a cross-rank affine-summary scan for the gated DeltaNet layers
(``src/art/megatron/context_parallel/*``, ``src/art/megatron/gdn/fla_cp.py``).

Here every rank of the CP group takes one contiguous slice ``[a, b)`` of the
packed row (``T`` padded to a multiple of ``cp * 128``):

* projections, norms, MLP/MoE and the LM head run on local tokens only;
* attention: keys/values are all-gathered (backward: dK/dV partial sums are
  reduce-scattered to their owners) and the prefix-tree kernel runs the local
  queries (global offset ``a``) against every key, with work units planned
  for the local query range;
* gated DeltaNet: each local piece of a tree segment collapses into one
  affine state map (A, B) (``models/gdn.py``); the maps of all ranks are
  all-gathered and every rank resolves the tree recurrence in pre-order
  (a piece starts from the previous piece of its segment or from its parent
  segment's final state), then finishes its local outputs.  The causal conv
  gets its cross-rank predecessors from an all-gathered table of each piece's
  last tokens.

All exchanges are differentiable (all-gather forward, reduce-scatter
backward), so autograd runs the mirrored communication in the backward.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops import fused, native
from . import mutation


CP_BARRIER_TIMEOUT_NS = 60 * 10**9


class CPContext:
    """Context-parallel group.  Transport ``"p2p"`` (CUDA, world > 1): the
    gated DeltaNet summary exchange is fused into the summary scan, whose
    epilogue stores each piece's ``[A | B]`` into every rank's peer-mapped
    receive slot; ``"nccl"``: an all-gather (also the gloo CPU path)."""

    def __init__(self, group: dist.ProcessGroup | None, device: torch.device, transport: str | None = None) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.device = device
        if transport is None:
            transport = "p2p" if device.type == "cuda" and self.world > 1 else "nccl"
        self.transport = transport
        self.arena = None
        self._turn_bytes = 0
        self._turn = 0
        self.epoch = 0
        self.status = torch.zeros(1, dtype=torch.int32, device=device) if transport == "p2p" else None

    def exchange_region(self, nbytes: int) -> int:
        """Byte offset of this call's receive region (two regions alternate, so
        a fast rank never overwrites data a slow rank has yet to read: it
        must pass the barrier of the call in between first).  Collective:
        every rank calls it in the same order with the same size."""
        from .dp import PeerArena, _round

        need = _round(nbytes)
        if self.arena is None or need > self._turn_bytes:
            if self.arena is not None:
                torch.cuda.current_stream(self.device).synchronize()
                dist.barrier(group=self.group)
                self.arena.close()
            self._turn_bytes = need
            self.arena = PeerArena(2 * need + 256, self.group, self.device)
            self.flag_tab = self.arena.table(2 * need)
            self.arena.buf[2 * need :].zero_()
            self.epoch = 0
            dist.barrier(group=self.group)
        off = self._turn * self._turn_bytes
        self._turn ^= 1
        return off

    def barrier(self) -> None:
        self.epoch += 1
        native.lib().peer_barrier(self.flag_tab, self.rank, self.world, self.epoch, CP_BARRIER_TIMEOUT_NS,
                                  self.status)

    def check(self) -> None:
        if self.status is not None and int(self.status.item()) != 0:
            raise RuntimeError("context-parallel peer barrier timed out")

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x
        out = x.new_empty(x.shape[0] * self.world, *x.shape[1:])
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x
        rows = x.shape[0] // self.world
        if x.device.type == "cuda":
            out = x.new_empty(rows, *x.shape[1:])
            dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
            return out
        y = x.clone()
        dist.all_reduce(y, group=self.group)
        return y[self.rank * rows : (self.rank + 1) * rows].clone()


class _Gather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cp):
        ctx.cp = cp
        return cp.all_gather(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.cp.reduce_scatter(g.contiguous()), None


def gather(x: torch.Tensor, cp: CPContext) -> torch.Tensor:
    """Differentiable all-gather along dim 0 (backward: reduce-scatter)."""
    return _Gather.apply(x, cp)


class _ArenaGather(torch.autograd.Function):
    """The receive side of the fused summary exchange: the scan epilogues have
    already stored every rank's rows into this rank's arena region; after the
    peer barrier the region is the all-gathered stack.  Backward: the
    reduce-scatter of the gathered gradient, as for :func:`gather`."""

    @staticmethod
    def forward(ctx, local, cp, off):
        ctx.cp = cp
        cp.barrier()
        n = local.numel() * cp.world
        return cp.arena.view(off, n, torch.float32).view(-1, *local.shape[1:]).clone()

    @staticmethod
    def backward(ctx, g):
        return ctx.cp.reduce_scatter(g.contiguous()), None, None


@dataclass
class Piece:
    seg: int
    start: int
    end: int
    rank: int
    pred: int  # index of the piece whose final state starts this one (-1: zero state)


class CPPlan:
    """Per-row plan for one rank: local range, attention metadata with global
    keys, GDN pieces and the conv boundary table."""

    def __init__(self, cp: CPContext, kend_full: torch.Tensor, positions_full: torch.Tensor,
                 group_ids: torch.Tensor | None, parent_ids: torch.Tensor | None, conv_width: int = 4,
                 linear_layers: bool = True) -> None:
        T = int(kend_full.numel())
        W = cp.world
        assert T % W == 0
        self.T, self.rows = T, T // W
        self.a = cp.rank * self.rows
        self.b = self.a + self.rows
        dev = cp.device
        k_cpu = kend_full.to("cpu", torch.int32)
        self.meta = fused.AttnMeta.build(positions_full[self.a : self.b], k_cpu, dev)
        pin = dev.type == "cuda"
        units = fused.attention_bwd_units_tc(k_cpu, self.a, self.rows)
        self.meta.bwd_units = (units.pin_memory() if pin else units).to(dev, non_blocking=True)
        self.K = conv_width - 1
        if linear_layers:
            self._plan_linear(cp, group_ids, parent_ids, conv_width)

    def _plan_linear(self, cp: CPContext, group_ids, parent_ids, conv_width: int) -> None:
        """Pieces of the tree segments per rank and the conv boundary table
        (only needed by the gated DeltaNet layers)."""
        from ..models.gdn import sequence_predecessors
        from ..preprocessing.prefix_tree import parse_prefix_tree_row

        T, W, dev = self.T, cp.world, cp.device
        if group_ids is None:
            segs = [(0, T, -1)]
        else:
            parsed = parse_prefix_tree_row(group_ids[:T], parent_ids[:T])
            idx = {s.group_id: n for n, s in enumerate(parsed)}
            segs = [(s.start, s.end, idx[s.parent_id] if s.parent_id != s.group_id else -1) for s in parsed]
            cov = parsed[-1].end if parsed else 0
            if cov < T:  # trailing padding: its own root segment
                segs.append((cov, T, -1))
        self.segs = segs
        pieces: list[Piece] = []
        last_piece_of_seg: dict[int, int] = {}
        for n, (s, e, p) in enumerate(segs):
            for r in range(W):
                lo, hi = max(s, r * self.rows), min(e, (r + 1) * self.rows)
                if lo >= hi:
                    continue
                if n in last_piece_of_seg:
                    pred = last_piece_of_seg[n]
                else:
                    pred = last_piece_of_seg.get(p, -1) if p >= 0 else -1
                pieces.append(Piece(n, lo, hi, r, pred))
                last_piece_of_seg[n] = len(pieces) - 1
        self.pieces = pieces
        self.local = [i for i, pc in enumerate(pieces) if pc.rank == cp.rank]
        self.max_local = max(sum(1 for pc in pieces if pc.rank == r) for r in range(W))
        # slot of every piece in the gathered summary stack (rank-major, padded)
        self.slot_of: dict[int, int] = {}
        K = self.K
        gtab = torch.full((T,), -1, dtype=torch.int64)  # global token -> row of the gathered tail table
        tail_rows = torch.full((self.max_local * K,), -1, dtype=torch.int64)
        for r in range(W):
            k = 0
            for i, pc in enumerate(pieces):
                if pc.rank != r:
                    continue
                slot = r * self.max_local + k
                self.slot_of[i] = slot
                for m in range(K):
                    t = pc.end - 1 - m
                    if t >= pc.start:
                        gtab[t] = slot * K + m
                        if r == cp.rank:
                            tail_rows[k * K + m] = t - self.a
                k += 1
        self.tail_rows = tail_rows.to(dev)
        # conv predecessors of the local tokens: local rows, or rows of the
        # gathered table of each piece's last tokens (offset by ``rows``)
        loc = sequence_predecessors(segs, T, conv_width)[self.a : self.b]
        inside = (loc >= self.a) & (loc < self.b)
        prev = torch.where(inside, loc - self.a, self.rows + gtab[loc.clamp_min(0)])
        prev = torch.where(loc < 0, torch.full_like(loc, -1), prev)
        assert bool((prev[(loc >= 0) & ~inside] >= self.rows).all()), "conv predecessor outside every piece tail"
        self.conv_prev = prev.to(dev)
        # predecessor table of [local rows | gathered tails] and its inverse
        ext_prev = torch.cat([prev, torch.full((W * self.max_local * K, K), -1, dtype=torch.int64)])
        self.ext_prev = ext_prev.to(dev)
        if dev.type == "cuda":
            from ..ops.gdn import successors

            self.ext_succ = successors(ext_prev, dev)
        else:
            self.ext_succ = None


# ---------------------------------------------------------------------------
# attention under CP
# ---------------------------------------------------------------------------


class _CPRopeAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, plan, cp, inv_freq, nq, nkv, D, qn_w, kn_w, eps, scale, perm):
        C = native.lib()
        meta = plan.meta
        T = qkv.shape[0]
        qk, rstd = C.rope_fwd(qkv, meta.positions, inv_freq, nq, nkv, D, qn_w, kn_w, eps, perm)
        q = qk[:, : nq * D].view(T, nq, D)
        k_loc = qk[:, nq * D :].reshape(T, nkv, D)
        v_loc = qkv[:, (nq + nkv) * D : (nq + 2 * nkv) * D].reshape(T, nkv, D)
        k_full = cp.all_gather(k_loc)
        v_full = cp.all_gather(v_loc)
        o, lse = C.attn_fwd_tc(q, k_full, v_full, meta.kend, meta.tile_kmax, meta.tile_kmin, scale, plan.a)
        ctx.save_for_backward(qkv, qk, k_full, v_full, o, lse, inv_freq,
                              qn_w if qn_w is not None else qkv.new_empty(0),
                              kn_w if kn_w is not None else qkv.new_empty(0),
                              rstd if rstd is not None and rstd.numel() else qkv.new_empty(0, dtype=torch.float32))
        ctx.plan, ctx.cp, ctx.dims = plan, cp, (nq, nkv, D, scale, qn_w is not None)
        ctx.perm = perm
        return o.view(T, nq * D)

    @staticmethod
    def backward(ctx, do):
        C = native.lib()
        qkv, qk, k_full, v_full, o, lse, inv_freq, qn_w, kn_w, rstd = ctx.saved_tensors
        nq, nkv, D, scale, has_norm = ctx.dims
        plan, cp = ctx.plan, ctx.cp
        T = qkv.shape[0]
        do = do.contiguous().view(T, nq, D)
        q = qk[:, : nq * D].view(T, nq, D)
        dq, dk_full, dv_full, _ = C.attn_bwd_tc(do, q, k_full, v_full, o, lse, plan.meta.kend, plan.meta.bwd_units,
                                             scale, plan.a)
        dk = cp.reduce_scatter(dk_full)
        dv = cp.reduce_scatter(dv_full)
        dqkv = torch.empty_like(qkv)
        dqk = torch.empty_like(qk)
        dqk[:, : nq * D].copy_(dq.view(T, nq * D))
        dqk[:, nq * D :].copy_(dk.view(T, nkv * D))
        dqkv[:, (nq + nkv) * D : (nq + 2 * nkv) * D].copy_(dv.view(T, nkv * D))
        C.rope_bwd(dqk, qkv, plan.meta.positions, inv_freq, nq, nkv, D,
                   qn_w if has_norm else None, kn_w if has_norm else None, rstd if has_norm else None, dqkv,
                   ctx.perm)
        return dqkv, None, None, None, None, None, None, None, None, None, None, None


def cp_rope_attention(qkv, plan: CPPlan, cp: CPContext, inv_freq, nq, nkv, D, qn_w, kn_w, eps,
                      perm=None, scale=None):
    """``perm``: partial-rotary dim order (see ``ops.fused.partial_rotary``)."""
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if qkv.device.type == "cuda":
        if perm is not None:
            perm = perm.to(device=qkv.device, dtype=torch.int16).contiguous()
        return _CPRopeAttention.apply(qkv, plan, cp, inv_freq, nq, nkv, D, qn_w, kn_w, eps, scale, perm)
    # CPU: the same exchange around the dense-mask oracle
    T = qkv.shape[0]
    q = qkv[:, : nq * D].view(T, nq, D)
    k = qkv[:, nq * D : (nq + nkv) * D].view(T, nkv, D)
    v = qkv[:, (nq + nkv) * D :].reshape(T, nkv, D)
    if qn_w is not None:
        q = fused._rmsnorm_ref(q, qn_w, eps)
        k = fused._rmsnorm_ref(k, kn_w, eps)
    pos = plan.meta.positions
    if perm is not None:
        q, k = q[..., perm.long()], k[..., perm.long()]
    q = fused._rope_ref(q, pos, inv_freq)
    k = fused._rope_ref(k, pos, inv_freq)
    k_full = gather(k.contiguous(), cp)
    v_full = gather(v.contiguous(), cp)
    o = _dense_cp_attention(q, k_full, v_full, plan.meta.kend, plan.a, scale)
    return o.reshape(T, nq * D)


def _dense_cp_attention(q, k, v, kend, q_off, scale):
    Tq, Hq, D = q.shape
    Tk = k.shape[0]
    G = Hq // k.shape[1]
    acc = fused._acc
    kx = acc(k).repeat_interleave(G, dim=1)
    vx = acc(v).repeat_interleave(G, dim=1)
    s = torch.einsum("ihd,jhd->hij", acc(q), kx) * scale
    i = (torch.arange(Tq, device=q.device) + q_off).view(Tq, 1)
    j = torch.arange(Tk, device=q.device).view(1, Tk)
    mask = (j <= i) & (i < kend.to(q.device).long().view(1, Tk))
    s = s.masked_fill(~mask.unsqueeze(0), float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hij,jhd->ihd", p, vx).to(q.dtype)


# ---------------------------------------------------------------------------
# gated DeltaNet under CP
# ---------------------------------------------------------------------------


def compose(A: torch.Tensor, B: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Compose per-chunk maps ``S -> A_c S + B_c`` over the chunk axis (dim 2)
    (a plain-PyTorch oracle of :func:`art_mlx_b200.ops.gdn.summary_scan`)."""
    Acc, Bcc = A[:, :, 0], B[:, :, 0]
    for c in range(1, A.shape[2]):
        Acc = A[:, :, c] @ Acc
        Bcc = A[:, :, c] @ Bcc + B[:, :, c]
    return Acc, Bcc


def cp_gdn(layer, h: torch.Tensor, plan: CPPlan, cp: CPContext, version: int, enabled: bool) -> torch.Tensor:
    """Gated DeltaNet over this rank's slice of a packed row (reference
    ``src/art/megatron/gdn/fla_cp.py:315-580``): local pieces of every tree
    segment collapse into affine summaries ``[A | B]`` (the summary scan),
    the summaries are exchanged (fused into the scan epilogue over NVLink on
    the p2p transport), the tree recurrence is resolved in pre-order, and
    each local piece is scanned from its true initial state."""
    from ..models.gdn import CHUNK, chunk_parts
    from ..ops import gdn as gdn_ops

    qkv, z, g, beta = layer.mix(h, version, enabled)
    T = qkv.shape[0]
    # cross-rank conv predecessors: every rank publishes its pieces' last tokens
    tr = plan.tail_rows
    tails = qkv.index_select(0, tr.clamp_min(0)) * (tr >= 0).unsqueeze(1).to(qkv.dtype)
    ext = torch.cat([qkv, gather(tails.contiguous(), cp)], dim=0)
    q, k, v = layer.core_inputs(ext, plan.ext_prev, plan.ext_succ)
    q, k, v = q[:T], k[:T], v[:T].float()
    if layer.nv != layer.nk:
        rep = layer.nv // layer.nk
        q, k = q.repeat_interleave(rep, dim=1), k.repeat_interleave(rep, dim=1)
    Hh, dk, dv = k.shape[1], k.shape[2], v.shape[2]
    fused_x = cp.transport == "p2p"
    slot_numel = Hh * dk * (dk + dv)
    off = cp.exchange_region(cp.world * plan.max_local * slot_numel * 4) if fused_x else 0
    # local pieces: intra-chunk operands and their affine summaries
    local_data = []
    summs = []
    for j, gi in enumerate(plan.local):
        pc = plan.pieces[gi]
        s, e = pc.start - plan.a, pc.end - plan.a
        pad = (-(e - s)) % CHUNK

        def cut(t: torch.Tensor) -> torch.Tensor:
            t = t[s:e]
            t = torch.nn.functional.pad(t, (0, 0) * (t.dim() - 1) + (0, pad))
            return t.unsqueeze(0)

        parts = chunk_parts(cut(q), cut(k), cut(v), cut(g), cut(beta), CHUNK)
        _, Wm, U0, _, Kd, gC = parts
        peer_out = cp.arena.table(off + (cp.rank * plan.max_local + j) * slot_numel * 4) if fused_x else None
        summs.append(gdn_ops.summary_scan(Wm, U0, Kd, gC, peer_out)[0])
        local_data.append((s, e, parts))
    while len(summs) < plan.max_local:  # padding slots (never read)
        summs.append(q.new_zeros(Hh, dk, dk + dv))
    summ = torch.stack(summs)  # [P, H, dk, dk+dv]
    allsumm = _ArenaGather.apply(summ, cp, off) if fused_x else gather(summ.contiguous(), cp)
    # resolve the tree recurrence over all pieces in pre-order
    S_out: list[torch.Tensor] = []
    S_in: list[torch.Tensor] = []
    for i, pc in enumerate(plan.pieces):
        handoff = pc.pred >= 0 and not mutation.active("cp_skip_state_handoff")
        sin = S_out[pc.pred] if handoff else q.new_zeros(Hh, dk, dv)
        row = allsumm[plan.slot_of[i]]
        S_in.append(sin)
        S_out.append(row[..., :dk] @ sin + row[..., dk:])
    # local outputs
    out = q.new_zeros(T, Hh, dv)
    for (s, e, parts), gi in zip(local_data, plan.local):
        o, _ = gdn_ops.scan(*parts, S_in[gi].unsqueeze(0))
        o = o.permute(0, 2, 3, 1, 4).reshape(-1, Hh, dv)[: e - s]
        out = out.index_copy(0, torch.arange(s, e, device=q.device), o)
    return layer.finish(out, z, version, enabled, h.dtype)
