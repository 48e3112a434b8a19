"""Tensor parallelism with sequence parallelism (Megatron layout).

Activations between blocks are sharded by tokens (``[T/tp, H]`` per rank);
column-parallel projections (QKV, gate/up) consume the all-gathered input and
produce a column shard; row-parallel projections (O, down) produce partial
sums that are reduce-scattered back to token shards.  Attention runs on the
rank's heads over all tokens; the LM head is vocab-parallel.

Communication-fused kernels (``ops/csrc/gemm_tc.cu``, transport ``"p2p"``):

* AG -> GEMM: each rank publishes its token shard in a peer-mapped arena;
  every peer shard crosses NVLink once, pulled by the copy engine into a local
  buffer on a side stream, while the tcgen05 GEMM runs on the shards that
  have already arrived (own shard first).  No kernel reads peer memory
  through TMA on this path, and nothing uses multicast;
* GEMM -> RS: the GEMM epilogue stores each row block of the partial product
  into the owning rank's staging slot over NVLink (whole 128-byte lines from
  the CTA-pair kernel's staged epilogue); the owner sums its slots.

The NCCL transport (``"nccl"``) is the baseline: ``all_gather_into_tensor``
and ``reduce_scatter_tensor`` around cuBLAS GEMMs (also the gloo CPU path).

LoRA under TP: factors stay full-size in every rank's flat store.  Column-
parallel ``A`` and row-parallel ``B`` are replicated; their gradients are
built from local shards after tiny ``[T, r]`` all-reduces, so each rank's
gradient buffer holds its share and the data-parallel reduction over all
ranks completes the tensor-parallel gradient sync (reference:
``src/art/megatron/lora.py:1084-1128`` and ``training/finalize_grads.py``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import native
from . import mutation

TP_BARRIER_TIMEOUT_NS = 60 * 10**9


class TPContext:
    def __init__(self, group: dist.ProcessGroup | None, device: torch.device, max_tokens: int, hidden: int,
                 transport: str | None = None) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.device = device
        if transport is None:
            transport = "p2p" if device.type == "cuda" and self.world > 1 else "nccl"
        self.transport = transport
        self.max_tokens = max_tokens
        self.hidden = hidden
        self.arena = None
        if transport == "p2p":
            from .dp import PeerArena

            rows = max_tokens // self.world
            self.shard_bytes = (rows * hidden * 2 + 255) // 256 * 256
            self.stage_bytes = (max_tokens * hidden * 2 + 255) // 256 * 256
            self.off_ag = 0  # 2 x shard
            self.off_rs = 2 * self.shard_bytes  # 2 x staging
            self.off_flags = self.off_rs + 2 * self.stage_bytes
            self.arena = PeerArena(self.off_flags + 256, group, device)
            self.flag_tab = self.arena.table(self.off_flags)
            self.status = torch.zeros(1, dtype=torch.int32, device=device)
            self.epoch = 0
            self._ag_turn = 0
            self._rs_turn = 0

    # ---------------------------------------------------------------- helpers
    def shard_rows(self, T: int) -> int:
        assert T % self.world == 0
        return T // self.world

    def barrier(self) -> None:
        self.epoch += 1
        native.lib().peer_barrier(self.flag_tab, self.rank, self.world, self.epoch, TP_BARRIER_TIMEOUT_NS, self.status)

    def check(self) -> None:
        if self.arena is not None and int(self.status.item()) != 0:
            raise RuntimeError("tensor-parallel peer barrier timed out")

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """[T/tp, ...] -> [T, ...] (collective)."""
        if self.world == 1:
            return x
        out = x.new_empty(x.shape[0] * self.world, *x.shape[1:])
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        """[T, ...] partial sums -> [T/tp, ...] (collective)."""
        if self.world == 1:
            return x
        rows = x.shape[0] // self.world
        if x.device.type == "cuda":
            out = x.new_empty(rows, *x.shape[1:])
            dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
            return out
        y = x.clone()
        if not mutation.active("tp_skip_reduce_scatter"):
            dist.all_reduce(y, group=self.group)
        return y[self.rank * rows : (self.rank + 1) * rows].clone()

    # ---------------------------------------------------------------- fused
    def _ag_slot(self):
        turn = self._ag_turn
        self._ag_turn ^= 1
        off = self.off_ag + turn * self.shard_bytes
        return off

    def ag_gemm(self, x_sh: torch.Tensor, W: torch.Tensor, a2: torch.Tensor | None = None,
                b2: torch.Tensor | None = None, bias: torch.Tensor | None = None) -> torch.Tensor:
        """``AG(x_sh) @ W^T (+ a2 @ b2^T) (+ bias)`` with the gather overlapped.

        Every rank publishes its shard into its peer arena; then each peer
        shard crosses NVLink exactly once, pulled by the copy engine into a
        local buffer on a side stream, while the tcgen05 GEMM runs on the
        shard that arrived before it (the own shard first).  Reading the peer
        rows straight from the GEMM's TMA would fetch every remote A tile
        once per output column band."""
        rows, H = x_sh.shape
        if self.transport != "p2p":
            y = self.all_gather(x_sh) @ W.t()
            if a2 is not None:
                y = y + a2 @ b2.t()
            return y if bias is None else y + bias
        C = native.lib()
        off = self._ag_slot()
        slot = self.arena.view(off, rows * H, x_sh.dtype).view(rows, H)
        slot.copy_(x_sh)
        self.barrier()  # every rank's shard is published
        T, N = rows * self.world, W.shape[0]
        out = torch.empty(T, N, device=x_sh.device, dtype=x_sh.dtype)
        gathered = self._gather_buffer(T, H, x_sh.dtype)
        main = torch.cuda.current_stream()
        side = self._side_stream()
        side.wait_stream(main)
        order = [(self.rank + i) % self.world for i in range(self.world)]
        events = {}
        with torch.cuda.stream(side):
            for q in order[1:]:
                C.peer_copy(gathered[q * rows : (q + 1) * rows], self.arena.bases[q] + off, rows * H * x_sh.element_size())
                ev = torch.cuda.Event()
                ev.record(side)
                events[q] = ev
        for q in order:
            src = x_sh if q == self.rank else gathered[q * rows : (q + 1) * rows]
            if q != self.rank:
                main.wait_event(events[q])
            r = slice(q * rows, (q + 1) * rows)
            if _pair(rows, W):
                C.gemm_pair(src.contiguous(), W, None if a2 is None else a2[r].contiguous(), b2, bias, out[r])
            else:
                C.gemm_tc(src, W, None if a2 is None else a2[r], b2, bias, out[r], False)
        gathered.record_stream(side)
        return out

    def _side_stream(self) -> torch.cuda.Stream:
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=self.device)
        return self._side

    def _gather_buffer(self, T: int, H: int, dtype: torch.dtype) -> torch.Tensor:
        buf = getattr(self, "_gbuf", None)
        if buf is None or buf.numel() < T * H or buf.dtype != dtype:
            buf = torch.empty(T * H, device=self.device, dtype=dtype)
            self._gbuf = buf
        return buf[: T * H].view(T, H)

    def gemm_rs(self, x: torch.Tensor, W: torch.Tensor, a2: torch.Tensor | None = None,
                b2: torch.Tensor | None = None) -> torch.Tensor:
        """``RS(x @ W^T (+ a2 @ b2^T))`` with the scatter inside the GEMM epilogue."""
        T = x.shape[0]
        N = W.shape[0]
        if self.transport != "p2p":
            y = x @ W.t()
            if a2 is not None:
                y = y + a2 @ b2.t()
            return self.reduce_scatter(y)
        rows = T // self.world
        turn = self._rs_turn
        self._rs_turn ^= 1
        off = self.off_rs + turn * self.stage_bytes
        ptrs = [b + off for b in self.arena.bases]
        if _pair(T, W):
            native.lib().gemm_pair_rs(x.contiguous(), W, a2, b2, ptrs, rows, N, self.rank)
        else:
            native.lib().gemm_tc_rs(x.contiguous(), W, a2, b2, ptrs, rows, N, self.rank)
        self.barrier()  # every rank's partial rows have landed in the owners' slots
        staging = self.arena.view(off, T * N, x.dtype).view(T, N)
        return native.lib().slot_sum(staging, self.world, rows, None)


def _pair(rows: int, W: torch.Tensor) -> bool:
    """The CTA-pair tcgen05 GEMM for a TP product (else the 1-CTA kernel):
    bf16, at least a full tile of rows, 128-multiple widths."""
    from ..ops import fused

    return (fused.PAIR_GEMM and W.dtype == torch.bfloat16 and rows >= 256 and W.shape[0] % 128 == 0
            and W.shape[1] % 128 == 0 and W.is_contiguous())


# ---------------------------------------------------------------------------
# autograd ops
# ---------------------------------------------------------------------------


def _acc_into(slot: torch.Tensor, a: torch.Tensor, b: torch.Tensor, alpha: float) -> None:
    """slot += alpha * a @ b (fp32 accumulate; slot may be a strided view)."""
    if slot.device.type == "cuda" and a.dtype != torch.float32:
        slot.add_(torch.mm(a, b, out_dtype=torch.float32), alpha=alpha)
    else:
        slot.add_((a.to(slot.dtype) @ b.to(slot.dtype)), alpha=alpha)


class ColumnParallelLoRA(torch.autograd.Function):
    """y[T, N_local] = AG(x_sh) W_local^T + b_local + s * (AG(x_sh) A^T) B_local^T.

    ``A`` [n*r, H] is replicated, ``B_bd`` [N_local, n*r] is this rank's
    (block-diagonal) rows.  Backward returns the token-shard gradient."""

    @staticmethod
    def forward(ctx, x_sh, W, Wt, bias, A, B_bd, gA, gB_fn, scale, tp, anchor):
        rows = x_sh.shape[0]
        u_sh = x_sh @ A.t() if A is not None else None  # [T/tp, n*r]
        u = tp.all_gather(u_sh) if u_sh is not None else None
        y = tp.ag_gemm(x_sh, W, u, (B_bd * scale).to(x_sh.dtype) if u is not None else None, bias)
        ctx.save_for_backward(x_sh, u if u is not None else x_sh.new_empty(0))
        ctx.W, ctx.Wt, ctx.A, ctx.B_bd, ctx.gA, ctx.gB_fn, ctx.scale, ctx.tp = W, Wt, A, B_bd, gA, gB_fn, scale, tp
        return y

    @staticmethod
    def backward(ctx, dy):
        x_sh, u = ctx.saved_tensors
        tp, s, A, B_bd = ctx.tp, ctx.scale, ctx.A, ctx.B_bd
        dy = dy.contiguous()
        rows = x_sh.shape[0]
        lo = tp.rank * rows
        dx_sh = tp.gemm_rs(dy, ctx.Wt)  # RS(dy_local W_local)
        if A is not None:
            dyB = dy @ B_bd  # partial over tp ranks: [T, n*r]
            tp.all_reduce_(dyB)
            # dA (replicated A): this rank's token rows; the cross-rank sum completes it
            _acc_into(ctx.gA, dyB[lo : lo + rows].t(), x_sh, s)
            # dB (local rows): s * dy^T u over all tokens
            ctx.gB_fn(dy, u, s)
            dx_sh = dx_sh + (s * (dyB[lo : lo + rows] @ A)).to(dx_sh.dtype)
        return dx_sh, None, None, None, None, None, None, None, None, None, None


class RowParallelLoRA(torch.autograd.Function):
    """y_sh[T/tp, H] = RS(x_local W_local^T + s * (x_local A_local^T) B^T).

    ``A_local`` [r, K_local] is this rank's column slice, ``B`` [H, r] is
    replicated."""

    @staticmethod
    def forward(ctx, x, W, Wt, A_loc, B, gA_loc, gB, scale, tp, anchor):
        u_part = x @ A_loc.t() if A_loc is not None else None  # [T, r] partial
        y_sh = tp.gemm_rs(x, W, u_part, (B * scale).to(x.dtype) if u_part is not None else None)
        u_full = tp.all_reduce_(u_part.clone()) if u_part is not None else None
        ctx.save_for_backward(x, u_full if u_full is not None else x.new_empty(0))
        ctx.W, ctx.Wt, ctx.A, ctx.B, ctx.gA, ctx.gB, ctx.scale, ctx.tp = W, Wt, A_loc, B, gA_loc, gB, scale, tp
        return y_sh

    @staticmethod
    def backward(ctx, dy_sh):
        x, u_full = ctx.saved_tensors
        tp, s = ctx.tp, ctx.scale
        dy_sh = dy_sh.contiguous()
        rows = dy_sh.shape[0]
        lo = tp.rank * rows
        dx = tp.ag_gemm(dy_sh, ctx.Wt)  # AG(dy) W_local
        if ctx.A is not None:
            dyB_sh = dy_sh @ ctx.B  # [T/tp, r]
            dyB = tp.all_gather(dyB_sh)  # [T, r]
            _acc_into(ctx.gA, dyB.t(), x, s)  # local A slice: all tokens
            _acc_into(ctx.gB, dy_sh.t(), u_full[lo : lo + rows], s)  # replicated B: own rows
            dx = dx + (s * (dyB @ ctx.A)).to(dx.dtype)
        return dx, None, None, None, None, None, None, None, None, None


class AllGatherSeq(torch.autograd.Function):
    """Token shards -> full sequence (backward: reduce-scatter)."""

    @staticmethod
    def forward(ctx, x_sh, tp):
        ctx.tp = tp
        return tp.all_gather(x_sh)

    @staticmethod
    def backward(ctx, dy):
        return ctx.tp.reduce_scatter(dy.contiguous()), None


class ScatterSeq(torch.autograd.Function):
    """Full (replicated) sequence -> this rank's token shard (backward: all-gather)."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        rows = x.shape[0] // tp.world
        return x[tp.rank * rows : (tp.rank + 1) * rows].contiguous()

    @staticmethod
    def backward(ctx, dy_sh):
        return ctx.tp.all_gather(dy_sh.contiguous()), None


class VocabParallelLogprobs(torch.autograd.Function):
    """Log-softmax gather over a vocab-sharded LM head (rows = selected
    positions, replicated on every tp rank).  lse = logsumexp over ranks of the
    local lse; the target logit comes from the owning shard."""

    @staticmethod
    def forward(ctx, h, W_loc, targets, v0, tp, want_entropy):
        logits = (h @ W_loc.t())
        V_loc = W_loc.shape[0]
        local_t = targets - v0
        in_shard = (local_t >= 0) & (local_t < V_loc)
        lt = torch.where(in_shard, local_t, torch.full_like(local_t, -1))
        if h.device.type == "cuda":
            lse_l, tgt_l, ent_l = native.lib().logits_stats(logits, lt.contiguous(), want_entropy)
        else:
            lf = logits.float()
            lse_l = torch.logsumexp(lf, -1)
            tgt_l = torch.where(in_shard, lf.gather(1, lt.clamp_min(0)[:, None])[:, 0], torch.zeros_like(lse_l))
            p = torch.softmax(lf, -1)
            ent_l = lse_l - (p * lf).sum(-1)
        tgt_l = torch.where(in_shard, tgt_l, torch.zeros_like(tgt_l))
        if tp.world > 1:
            allv = torch.empty(tp.world * lse_l.numel(), device=h.device, dtype=torch.float32)
            dist.all_gather_into_tensor(allv, lse_l.float().contiguous(), group=tp.group)
            lses = allv.view(tp.world, -1)
            lse = torch.logsumexp(lses, 0)
            tp.all_reduce_(tgt_l)
        else:
            lses = lse_l.view(1, -1)
            lse = lse_l
        lp = tgt_l - lse
        ent = None
        if want_entropy and ent_l is not None:
            ex = (lse_l - ent_l) * torch.exp(lse_l - lse)  # this shard's share of E[x]
            ex = tp.all_reduce_(ex.clone())
            ent = lse - ex
        ctx.save_for_backward(logits, W_loc, lt, lse)
        ctx.tp = tp
        return lp, ent

    @staticmethod
    def backward(ctx, glp, gent):
        logits, W_loc, lt, lse = ctx.saved_tensors
        tp = ctx.tp
        g = glp.float().contiguous()
        if logits.device.type == "cuda":
            native.lib().logits_grad_(logits, lt.contiguous(), lse.contiguous(), g)
            dlog = logits
        else:
            p = torch.exp(logits.float() - lse[:, None])
            onehot = torch.zeros_like(p)
            m = lt >= 0
            onehot[m, lt[m]] = 1.0
            dlog = (g[:, None] * (onehot - p)).to(logits.dtype)
        # partial over vocab shards; the reduce-scatter of the sequence
        # all-gather upstream sums the shards' contributions
        dh = dlog @ W_loc
        return dh, None, None, None, None, None
