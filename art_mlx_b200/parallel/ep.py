"""Expert parallelism: token dispatch / combine for MoE layers.

Reference behaviour: Megatron MoE with the DeepEP flex dispatcher and expert
LoRA through a grouped GEMM (``src/art/megatron/provider.py:416-434``,
``lora.py:1464-1572``), routing replay forcing the rollout's expert ids.

Here expert ``e`` lives on rank ``e // (E / world)``.  For one MoE layer:

plan      every rank histograms its (token, slot) -> expert assignments; the
          ``[world, E]`` count matrix is all-gathered (tiny); from it each
          origin computes, for each of its slots, the destination rank and the
          row in that rank's receive buffer.  Receive buffers are laid out
          expert-contiguous (expert, then origin rank, then token order), which
          is exactly the grouped-GEMM input order: no permute pass.
dispatch  origin ranks store their token rows straight into the owners'
          receive buffers (P2P stores over NVLink, ``scatter_rows``).
experts   grouped base + LoRA GEMMs on the receive buffer (``models/moe.py``).
combine   origin ranks load their slots' expert outputs from the owners
          (P2P loads, ``gather_rows``) and reduce them with the routing
          weights (``combine_rows``).
backward  mirrors it: weighted output gradients are pushed to the owners,
          expert backward runs there, input gradients are pulled back.

Barriers between phases are the bounded peer flag barriers of the DP layer.
A second transport, :class:`AllToAllTransport`, moves the same rows with
``torch.distributed.all_to_all_single`` (the NCCL baseline; also the gloo
path used by the CPU tests).
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops import native


@dataclass
class EPPlan:
    T: int
    k: int
    dest_rank: torch.Tensor  # [T*k] int32
    dest_row: torch.Tensor  # [T*k] int64
    src_idx: torch.Tensor  # [T*k] int64 (= slot // k)
    local_counts: list[int]  # rows per local expert on this rank (receiver)
    n_recv: int
    counts_all: torch.Tensor  # [world, E] int64 (device)
    # all-to-all transport bookkeeping
    send_order: torch.Tensor | None = None
    send_splits: list[int] | None = None
    recv_splits: list[int] | None = None
    recv_rows: torch.Tensor | None = None  # receive-buffer row of each received slot


class EPContext:
    def __init__(self, group: dist.ProcessGroup | None, num_experts: int, hidden: int, device: torch.device,
                 capacity_rows: int, transport: str | None = None) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        assert num_experts % self.world == 0, "experts must divide evenly over ranks"
        self.E = num_experts
        self.E_local = num_experts // self.world
        self.H = hidden
        self.device = device
        if transport is None:
            transport = "p2p" if device.type == "cuda" and self.world > 1 else "a2a"
        self.transport = P2PTransport(self, capacity_rows) if transport == "p2p" else AllToAllTransport(self)
        # the exchange fused into the expert GEMMs (parallel/ep_fused.py), used
        # when every rank's route counts are known on the host (routing replay)
        self.fused = None
        if transport == "p2p" and os.environ.get("ART_B200_EP_FUSED", "1") != "0" and self.world <= 8:
            from .ep_fused import FusedEP

            self.fused = FusedEP(group, num_experts, hidden, device, capacity_rows, capacity_rows // 2)

    @property
    def first_expert(self) -> int:
        return self.rank * self.E_local

    def plan(self, idx: torch.Tensor) -> EPPlan:
        T, k = idx.shape
        flat = idx.reshape(-1).to(torch.int64)
        E, W = self.E, self.world
        counts = torch.bincount(flat, minlength=E)
        if W > 1:
            allc = torch.empty(W * E, dtype=counts.dtype, device=counts.device)
            dist.all_gather_into_tensor(allc, counts, group=self.group)
            allc = allc.view(W, E)
        else:
            allc = counts.view(1, E)
        per_expert = allc.sum(0)  # [E]
        # expert base inside its owner's buffer: exclusive cumsum within each owner's block
        blk = per_expert.view(W, self.E_local)
        expert_base = (torch.cumsum(blk, 1) - blk).reshape(E)
        origin_base = (torch.cumsum(allc, 0) - allc)[self.rank]  # [E]
        my_start = expert_base + origin_base
        order = torch.argsort(flat, stable=True)
        first = torch.cumsum(counts, 0) - counts
        pos_sorted = torch.arange(flat.numel(), device=flat.device) - first[flat[order]]
        dest_row = torch.empty_like(flat)
        dest_row[order] = my_start[flat[order]] + pos_sorted
        dest_rank = (flat // self.E_local).to(torch.int32)
        local = per_expert.view(W, self.E_local)[self.rank].tolist()  # host sync: receive sizes
        plan = EPPlan(T=T, k=k, dest_rank=dest_rank, dest_row=dest_row,
                      src_idx=torch.arange(T * k, device=flat.device) // k, local_counts=local,
                      n_recv=int(sum(local)), counts_all=allc)
        self.transport.prepare(plan)
        return plan


class P2PTransport:
    """Receive / output buffers in a CUDA-IPC arena shared by the EP group."""

    def __init__(self, ctx: EPContext, capacity_rows: int) -> None:
        from .dp import PeerArena

        self.ctx = ctx
        H = ctx.H
        self.cap = capacity_rows
        row_bytes = H * 2
        self.nbuf = 4  # recv_x, recv_out, d_recv, d_recv_x
        self.buf_bytes = (capacity_rows * row_bytes + 255) // 256 * 256
        self.off_flags = self.nbuf * self.buf_bytes
        total = self.off_flags + 256
        self.arena = PeerArena(total, ctx.group, ctx.device)
        self.tabs = [self.arena.table(i * self.buf_bytes) for i in range(self.nbuf)]
        self.views = [self.arena.view(i * self.buf_bytes, capacity_rows * H, torch.bfloat16).view(capacity_rows, H)
                      for i in range(self.nbuf)]
        self.flag_tab = self.arena.table(self.off_flags)
        self.status = torch.zeros(1, dtype=torch.int32, device=ctx.device)
        self.epoch = 0

    def barrier(self) -> None:
        from .dp import BARRIER_TIMEOUT_NS

        self.epoch += 1
        native.lib().peer_barrier(self.flag_tab, self.ctx.rank, self.ctx.world, self.epoch, BARRIER_TIMEOUT_NS,
                                  self.status)

    def prepare(self, plan: EPPlan) -> None:
        if plan.n_recv > self.cap:
            raise RuntimeError(f"expert-parallel receive capacity {self.cap} rows exceeded ({plan.n_recv})")

    def push(self, plan: EPPlan, src: torch.Tensor, scale: torch.Tensor | None, buf: int) -> torch.Tensor:
        """Rows ``src[slot // k] * scale[slot]`` to their owners' buffer ``buf``;
        returns this rank's received rows ``[n_recv, H]`` (a view)."""
        C = native.lib()
        C.scatter_rows_idx(src.contiguous(), plan.src_idx, plan.dest_rank, plan.dest_row, scale,
                           self.tabs[buf], self.ctx.H)
        self.barrier()
        return self.views[buf][: plan.n_recv]

    def publish(self, rows: torch.Tensor, buf: int) -> None:
        self.views[buf][: rows.shape[0]].copy_(rows)
        self.barrier()

    def pull(self, plan: EPPlan, buf: int) -> torch.Tensor:
        """Each slot's row from its owner's buffer ``buf``: ``[T*k, H]``."""
        out = torch.empty(plan.T * plan.k, self.ctx.H, device=self.ctx.device, dtype=torch.bfloat16)
        native.lib().gather_rows(out, plan.dest_rank, plan.dest_row, None, self.tabs[buf], self.ctx.H)
        return out

    def check(self) -> None:
        if int(self.status.item()) != 0:
            raise RuntimeError("expert-parallel peer barrier timed out")


class AllToAllTransport:
    """The same exchange with ``all_to_all_single`` (NCCL baseline / gloo)."""

    def __init__(self, ctx: EPContext) -> None:
        self.ctx = ctx
        self._published: dict[int, torch.Tensor] = {}

    def prepare(self, plan: EPPlan) -> None:
        ctx = self.ctx
        order = torch.argsort(plan.dest_rank.to(torch.int64), stable=True)
        send = torch.bincount(plan.dest_rank.to(torch.int64), minlength=ctx.world)
        plan.send_order = order
        plan.send_splits = send.tolist()
        if ctx.world > 1:
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=ctx.group)
            plan.recv_splits = recv.tolist()
            rows = torch.empty(sum(plan.recv_splits), dtype=torch.int64, device=send.device)
            dist.all_to_all_single(rows, plan.dest_row[order].contiguous(), plan.recv_splits, plan.send_splits,
                                   group=ctx.group)
        else:
            plan.recv_splits = plan.send_splits
            rows = plan.dest_row[order]
        plan.recv_rows = rows

    def _a2a(self, x: torch.Tensor, in_splits: list[int], out_splits: list[int]) -> torch.Tensor:
        if self.ctx.world == 1:
            return x
        out = x.new_empty(sum(out_splits), *x.shape[1:])
        dist.all_to_all_single(out, x.contiguous(), out_splits, in_splits, group=self.ctx.group)
        return out

    def push(self, plan: EPPlan, src: torch.Tensor, scale: torch.Tensor | None, buf: int) -> torch.Tensor:
        rows = src[plan.src_idx[plan.send_order]]
        if scale is not None:
            rows = (rows.float() * scale[plan.send_order].unsqueeze(1)).to(src.dtype)
        got = self._a2a(rows, plan.send_splits, plan.recv_splits)
        out = src.new_zeros(plan.n_recv, src.shape[1])
        out[plan.recv_rows] = got
        return out

    def publish(self, rows: torch.Tensor, buf: int) -> None:
        self._published[buf] = rows

    def pull(self, plan: EPPlan, buf: int) -> torch.Tensor:
        rows = self._published.pop(buf)
        send_back = rows[plan.recv_rows]
        got = self._a2a(send_back, plan.recv_splits, plan.send_splits)
        out = rows.new_empty(plan.T * plan.k, rows.shape[1])
        out[plan.send_order] = got
        return out

    def barrier(self) -> None:
        pass

    def check(self) -> None:
        pass
