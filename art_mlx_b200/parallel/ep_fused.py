"""Expert parallelism with the exchange fused into the expert GEMMs.

Reference behaviour: Megatron MoE with the DeepEP dispatcher around the
grouped expert GEMMs and grouped LoRA (``src/art/megatron/provider.py:
416-434``, ``lora.py:1464-1572``), routing replay forcing the rollout's
expert ids.  B200 design (kernels in ``ops/csrc/ep_gemm.cu``):

forward of one MoE layer on every rank of the EP group
  1. plan     -- with replayed routes every rank knows, on the host, how many
                 slots each rank sends to each expert (the per-layer count
                 matrices are exchanged once per step, not per layer), so the
                 receive layout, the GEMM tile table and the arrival targets
                 are built without a device sync or a count all-gather; only
                 the slot -> row map is computed on the device;
  2. the rank-side LoRA rows ``u = x A_e^T`` of this rank's slots are computed
     here, at the origin, so they travel with the token rows;
  3. peer barrier (no rank writes a buffer a slower rank still reads);
  4. ``ep_gemm`` dispatch + gate/up: one persistent kernel pushes the rows
     into the owners' receive buffers (P2P stores) while its GEMM warps run
     each expert's tiles as soon as that expert's rows have landed;
  5. SwiGLU, the down-projection LoRA rows, then ``ep_gemm`` down with the
     combine fused into its epilogue: each output row goes straight into its
     origin rank's slot buffer;
  6. ``ep_wait_combine``: the origin waits for its slots and reduces them
     with the routing weights.
backward mirrors it: the weighted output gradients (and their rank-side rows
``w dy B_e``) are dispatched into the down input-gradient GEMM, the expert
LoRA gradients are taken on the owner with the low-rank kernels, and the
gate/up input-gradient GEMM scatters its rows back to the origins.

Every wait is bounded; counters only grow and the host tracks cumulative
targets.  The ranks must call the layers in the same order (they do: the
micro steps and layers are lock-step).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch
import torch.distributed as dist

from ..ops import lowrank, native

BARRIER_TIMEOUT_NS = 60 * 10**9
EXT_COLS = 64  # receive-buffer columns for the rank-side LoRA rows (2r <= 64)
N_TILE = 256  # GEMM tile width: the epilogue reports each row once per column tile


def _round(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


def _h2d(a: np.ndarray, device: torch.device) -> torch.Tensor:
    """Host array -> device through pinned memory: queued like a kernel (a
    copy from pageable memory would first wait for the stream to drain)."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if device.type == "cuda":
        return t.pin_memory().to(device, non_blocking=True)
    return t.to(device)


@dataclass
class FusedPlan:
    T: int
    k: int
    n_recv: int
    offs: list[int]  # local experts' row offsets in the receive buffer
    local_counts: list[int]
    push_tok: torch.Tensor
    push_rank: torch.Tensor
    push_row: torch.Tensor
    push_expert: torch.Tensor
    push_meta: torch.Tensor
    push_order: torch.Tensor  # slot index of each push (push order)
    push_counts: list[int]  # this rank's slots per (local expert j, owner) segment, push order
    push_groups: list[int]  # global expert of each push segment
    arrive_target: torch.Tensor = field(default=None)  # device int32 [E_local]


class FusedEP:
    """Peer buffers and counters of the fused expert-parallel exchange."""

    def __init__(self, group: dist.ProcessGroup | None, num_experts: int, hidden: int, device: torch.device,
                 capacity_rows: int, max_slots: int) -> None:
        from .dp import PeerArena

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        if self.world > 8:
            raise ValueError("the fused expert-parallel exchange supports up to 8 ranks per group")
        self.E, self.H, self.device = num_experts, hidden, device
        self.E_local = num_experts // self.world
        self.cap = capacity_rows
        self.max_slots = max_slots
        H = hidden
        self.off_x = 0
        self.off_ext = _round(self.off_x + capacity_rows * H * 2)
        self.off_meta = _round(self.off_ext + capacity_rows * EXT_COLS * 2)
        self.off_slots = _round(self.off_meta + capacity_rows * 8)
        self.off_arrive = _round(self.off_slots + max_slots * H * 2)
        self.off_slotcnt = _round(self.off_arrive + self.E_local * 4)
        self.off_flags = _round(self.off_slotcnt + 4)
        total = self.off_flags + 256
        if self.world > 1:
            self.arena = PeerArena(total, group, device)
            bases = self.arena.bases
            buf = self.arena.buf
        else:
            self.arena = None
            buf = torch.zeros(total, dtype=torch.uint8, device=device)
            bases = [buf.data_ptr()]
        self._buf = buf
        self.bases = bases
        self.recv_x = buf[self.off_x : self.off_x + capacity_rows * H * 2].view(torch.bfloat16).view(capacity_rows, H)
        self.recv_ext = buf[self.off_ext : self.off_ext + capacity_rows * EXT_COLS * 2].view(torch.bfloat16).view(
            capacity_rows, EXT_COLS)
        self.recv_meta = buf[self.off_meta : self.off_meta + capacity_rows * 8].view(torch.int64)
        self.slots = buf[self.off_slots : self.off_slots + max_slots * H * 2].view(torch.bfloat16).view(max_slots, H)
        self.arrive = buf[self.off_arrive : self.off_arrive + self.E_local * 4].view(torch.int32)
        self.slot_count = buf[self.off_slotcnt : self.off_slotcnt + 4].view(torch.int32)
        self.ptr_x = [b + self.off_x for b in bases]
        self.ptr_ext = [b + self.off_ext for b in bases]
        self.ptr_meta = [b + self.off_meta for b in bases]
        self.ptr_slots = [b + self.off_slots for b in bases]
        self.ptr_arrive = [b + self.off_arrive for b in bases]
        self.ptr_slotcnt = [b + self.off_slotcnt for b in bases]
        self.flag_tab = torch.tensor([b + self.off_flags for b in bases], dtype=torch.int64, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.epoch = 0
        # cumulative counter targets (counters only grow)
        self.arrive_total = np.zeros(self.E_local, dtype=np.int64)
        self.slot_total = 0
        if self.world > 1:
            torch.cuda.synchronize(device)
            dist.barrier(group=group)

    # ------------------------------------------------------------------
    def barrier(self) -> None:
        if self.world == 1:
            return
        self.epoch += 1
        native.lib().peer_barrier(self.flag_tab, self.rank, self.world, self.epoch, BARRIER_TIMEOUT_NS, self.status)

    def plan(self, idx: torch.Tensor, counts_all: np.ndarray) -> FusedPlan:
        """Plan of one exchange.  ``counts_all`` [world, E]: slots each rank
        routes to each expert in this layer (host, identical on every rank)."""
        T, k = idx.shape
        W, E, El, me = self.world, self.E, self.E_local, self.rank
        ca = np.asarray(counts_all, dtype=np.int64).reshape(W, E)
        mine = ca[me]
        if int(mine.sum()) != T * k:
            raise RuntimeError(f"host route counts ({int(mine.sum())} slots) disagree with the routes ({T * k})")
        per_expert = ca.sum(0)  # rows each expert receives
        blk = per_expert.reshape(W, El)
        expert_base = (np.cumsum(blk, 1) - blk).reshape(E)  # expert start in its owner's buffer
        origin_base = np.cumsum(ca, 0) - ca  # [W, E] start of rank q's rows inside expert e
        base_mine = expert_base + origin_base[me]
        local_counts = blk[me].tolist()
        n_recv = int(sum(local_counts))
        if n_recv > self.cap:
            raise RuntimeError(f"expert-parallel receive capacity {self.cap} rows exceeded ({n_recv})")
        if T * k > self.max_slots:
            raise RuntimeError(f"expert-parallel slot capacity {self.max_slots} exceeded ({T * k})")
        offs = [0]
        for c in local_counts:
            offs.append(offs[-1] + int(c))
        dev = idx.device
        flat = idx.reshape(-1).to(torch.int64)
        # slot -> row in the owner's buffer: stable rank of the slot among this
        # rank's slots of the same expert, plus the expert's base
        order = torch.argsort(flat, stable=True)
        first = np.cumsum(mine) - mine
        first_d = _h2d(first, dev)
        base_d = _h2d(base_mine, dev)
        fs = flat[order]
        dest_row = torch.empty_like(flat)
        dest_row[order] = base_d[fs] + torch.arange(flat.numel(), device=dev) - first_d[fs]
        # push order: by (local expert j, owner) so the grid sweeps every
        # owner's experts in the same order
        key = (flat % El) * W + flat // El
        push_order = torch.argsort(key, stable=True)
        fp = flat[push_order]
        seg_counts, seg_groups = [], []
        for j in range(El):
            for o in range(W):
                seg_counts.append(int(mine[o * El + j]))
                seg_groups.append(o * El + j)
        # arrival targets of this rank's experts
        self.arrive_total += blk[me]
        tgt = (self.arrive_total & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
        plan = FusedPlan(
            T=T, k=k, n_recv=n_recv, offs=offs, local_counts=local_counts,
            push_tok=push_order // k,
            push_rank=(fp // El).to(torch.int32),
            push_row=dest_row[push_order],
            push_expert=(fp % El).to(torch.int32),
            push_meta=(push_order | (me << 40)),
            push_order=push_order,
            push_counts=seg_counts, push_groups=seg_groups,
        )
        plan.arrive_target = _h2d(tgt, dev)
        return plan

    def next_arrive_target(self, plan: FusedPlan) -> torch.Tensor:
        """Targets for a second exchange over the same plan (the backward)."""
        self.arrive_total += np.asarray(plan.local_counts, dtype=np.int64)
        tgt = (self.arrive_total & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
        return _h2d(tgt, self.device)

    def combine_target(self, plan: FusedPlan) -> int:
        self.slot_total += plan.T * plan.k * ((self.H + N_TILE - 1) // N_TILE)
        return self.slot_total & 0xFFFFFFFF

    def check(self) -> None:
        if int(self.status.item()) != 0:
            raise RuntimeError("fused expert-parallel peer barrier timed out")

    # ------------------------------------------------------------------
    def gemm(self, x, w, plan: FusedPlan, N: int, w_transposed: bool, a2=None, b2=None, *, push: dict | None = None,
             arrive_target=None, out=None, row_dst=None) -> None:
        C = native.lib()
        if push is not None:
            C.ep_gemm(x, w, plan.offs, N, w_transposed, a2, b2,
                      push["src"], push.get("ext"), plan.push_tok, push.get("scale"), plan.push_rank, plan.push_row,
                      plan.push_expert, push.get("meta"), self.ptr_x, self.ptr_ext, self.ptr_meta, self.ptr_arrive,
                      self.arrive, arrive_target, out, row_dst, [], [])
        else:
            C.ep_gemm(x, w, plan.offs, N, w_transposed, a2, b2,
                      None, None, None, None, None, None, None, None, [], [], [], [], None, None,
                      out, row_dst, self.ptr_slots if row_dst is not None else [],
                      self.ptr_slotcnt if row_dst is not None else [])


def _bd_gu(B_gu: torch.Tensor, s: float) -> torch.Tensor:
    """Per expert block-diagonal ``s * [B_gate, B_up]`` as ``[E*2F, 2r]``."""
    E, _, F, r = B_gu.shape
    bd = B_gu.new_zeros(E, 2 * F, 2 * r)
    bd[:, :F, :r] = s * B_gu[:, 0]
    bd[:, F:, r:] = s * B_gu[:, 1]
    return bd.view(E * 2 * F, 2 * r)


class FusedEPExperts(torch.autograd.Function):
    """Dispatch -> experts -> combine with the exchanges fused into the expert
    GEMMs (``ops/csrc/ep_gemm.cu``)."""

    @staticmethod
    def forward(ctx, h, w, idx, fep: FusedEP, params, lora: bool, counts_all, anchor):
        C = native.lib()
        h = h.contiguous()
        plan = fep.plan(idx, counts_all)
        p = params
        s = p.scale
        E_l, H, F2 = p.gu_w_t.shape
        F = F2 // 2
        use_lora = lora and p.A_gu is not None
        u_push = b2 = None
        if use_lora:
            r = p.B_gu.shape[-1]
            # rank-side rows of this rank's slots at the origin: x A_e^T, push order
            A_all = p.A_all_gu  # [E, 2r, H] every expert's A (the origin routes to any expert)
            u_push = lowrank.rows(h, A_all, (A_all.stride(0), A_all.stride(1), A_all.stride(2)), 2 * r, H,
                                  counts=plan.push_counts, groups=plan.push_groups, src=plan.push_tok)
            b2 = _bd_gu(p.B_gu, s)
        fep.barrier()
        gu = torch.empty(max(plan.n_recv, 1), F2, device=h.device, dtype=torch.bfloat16)
        x_recv = fep.recv_x
        a2 = fep.recv_ext[:, : 2 * r] if use_lora else None
        fep.gemm(x_recv, p.gu_w_t.view(E_l * H, F2), plan, F2, True, a2, b2,
                 push={"src": h, "ext": u_push, "meta": plan.push_meta}, arrive_target=plan.arrive_target, out=gu)
        n = plan.n_recv
        gu = gu[:n]
        act = C.swiglu_fwd(gu) if n else gu[:, :F]
        u_d = a2d = b2d = None
        if lora and p.A_d is not None:
            rd = p.A_d.shape[1]
            u_d = lowrank.rows(act, p.A_d, (p.A_d.stride(0), p.A_d.stride(1), p.A_d.stride(2)), rd, F,
                               counts=plan.local_counts) if n else act.new_zeros(0, rd)
            a2d, b2d = u_d, (s * p.B_d).reshape(E_l * H, -1).contiguous()
        row_dst = fep.recv_meta[:n].clone()
        xs = x_recv[:n].clone()
        u_gu = fep.recv_ext[:n, : 2 * r].clone() if use_lora else None
        if n:
            fep.gemm(act, p.down_w_t.view(E_l * F, H), plan, H, True, a2d, b2d, row_dst=row_dst)
        target = fep.combine_target(plan)
        y = C.ep_wait_combine(fep.slots[: plan.T * plan.k], w.reshape(-1).float().contiguous(), plan.k,
                              fep.slot_count, target)
        slots = fep.slots[: plan.T * plan.k].clone()
        ctx.fep, ctx.plan, ctx.p, ctx.lora = fep, plan, p, lora
        # through save_for_backward, so that activation recompute can drop them
        ctx.save_for_backward(w, xs, gu, act, u_gu, u_d, row_dst, slots)
        return y

    @staticmethod
    def backward(ctx, dy):
        C = native.lib()
        w, xs, gu, act, u_gu, u_d, row_dst, slots = ctx.saved_tensors
        fep, plan, p, lora = ctx.fep, ctx.plan, ctx.p, ctx.lora
        dy = dy.contiguous()
        T, k = plan.T, plan.k
        s = p.scale
        E_l, H, F2 = p.gu_w_t.shape
        F = F2 // 2
        n = plan.n_recv
        dw = (slots.view(T, k, -1).float() * dy.view(T, 1, -1).float()).sum(-1)
        wf = w.reshape(-1).float().contiguous()
        push_scale = wf[plan.push_order].contiguous()
        use_d = lora and p.A_d is not None
        ext = a2 = b2 = None
        if use_d:
            rd = p.B_d.shape[-1]
            B_all = p.B_all_d  # [E, H, r] every expert's B of the down projection
            # w * dy B_e at the origin, push order
            ext = lowrank.rows(dy, B_all, (B_all.stride(0), B_all.stride(2), B_all.stride(1)), rd, H,
                               counts=plan.push_counts, groups=plan.push_groups, src=plan.push_tok, scale=push_scale)
            a2 = fep.recv_ext[:, :rd]
            b2 = (s * p.A_d.transpose(1, 2)).reshape(E_l * F, -1).contiguous()
        tgt = fep.next_arrive_target(plan)
        fep.barrier()
        dact = torch.empty(max(n, 1), F, device=dy.device, dtype=torch.bfloat16)
        fep.gemm(fep.recv_x, p.down_w_t.view(E_l * F, H), plan, F, False, a2, b2,
                 push={"src": dy, "ext": ext, "scale": push_scale}, arrive_target=tgt, out=dact)
        dact = dact[:n]
        d_recv = fep.recv_x[:n]
        if use_d and n:
            rd = p.B_d.shape[-1]
            lowrank.wgrad(u_d, d_recv, p.g_B_d, (p.g_B_d.stride(0), p.g_B_d.stride(2), p.g_B_d.stride(1)), rd, H, s,
                          counts=plan.local_counts)  # dB_d += s d_recv^T u_d
            lowrank.wgrad(fep.recv_ext[:n, :rd], act, p.g_A_d, (p.g_A_d.stride(0), p.g_A_d.stride(1),
                                                                 p.g_A_d.stride(2)), rd, F, s,
                          counts=plan.local_counts)  # dA_d += s dyB^T act
        dgu = C.swiglu_bwd(dact.contiguous(), gu) if n else gu
        a2 = b2 = None
        if lora and p.A_gu is not None and n:
            r = p.B_gu.shape[-1]
            dyB = dgu.new_empty(n, 2 * r)
            Bg, Bu = p.B_gu[:, 0], p.B_gu[:, 1]
            lowrank.rows(dgu[:, :F], Bg, (Bg.stride(0), Bg.stride(2), Bg.stride(1)), r, F, counts=plan.local_counts,
                         out=dyB[:, :r])
            lowrank.rows(dgu[:, F:], Bu, (Bu.stride(0), Bu.stride(2), Bu.stride(1)), r, F, counts=plan.local_counts,
                         out=dyB[:, r:])
            for half, g in ((0, p.g_B_gu[:, 0]), (1, p.g_B_gu[:, 1])):
                lowrank.wgrad(u_gu[:, half * r : (half + 1) * r], dgu[:, half * F : (half + 1) * F], g,
                              (g.stride(0), g.stride(2), g.stride(1)), r, F, s, counts=plan.local_counts)
            lowrank.wgrad(dyB, xs, p.g_A_gu, (p.g_A_gu.stride(0), p.g_A_gu.stride(1), p.g_A_gu.stride(2)), 2 * r, H,
                          s, counts=plan.local_counts)
            a2, b2 = dyB, (s * p.A_gu.transpose(1, 2)).reshape(E_l * H, -1).contiguous()
        if n:
            fep.gemm(dgu, p.gu_w_t.view(E_l * H, F2), plan, H, False, a2, b2, row_dst=row_dst)
        target = fep.combine_target(plan)
        dh = C.ep_wait_combine(fep.slots[: T * k], None, k, fep.slot_count, target)
        return dh, dw.to(w.dtype), None, None, None, None, None, None
