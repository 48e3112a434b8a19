"""Data parallelism: the fused LoRA-gradient reduce-scatter + AdamW + all-gather.

The reference reduces LoRA gradients with a coalesced fp32 NCCL all-reduce
(``src/art/megatron/training/finalize_grads.py:63-171``) and then runs the
full optimizer on every rank.  Here each rank owns one contiguous shard of
the flat LoRA buffers:

1. barrier A (every rank finished its backward);
2. ``dp_reduce_sumsq``: rank r sums shard r of all ranks' fp32 gradients with
   peer loads over NVLink and takes the shard's sum of squares;
3. the partial norm is stored into every peer's norm table; barrier B;
4. ``dp_adamw_allgather``: global-norm clip + AdamW on the shard, bf16
   parameters stored into every rank's compute buffer; own gradient zeroed;
5. barrier C (parameters published).

Remote traffic per step: (N-1)/N of the fp32 gradient read + (N-1)/N of the
bf16 parameters written, instead of an all-reduce (2x the gradient) plus N
redundant optimizer passes.  The master weights and moments of other shards
are refreshed from their owners (NCCL all-gather) only when a checkpoint is
written (:meth:`FusedDataParallel.gather_full_state`).

The peer buffers are one CUDA-IPC arena per rank (``ops/csrc/comm.cu``);
barriers are bounded flag waits that record a status code instead of hanging.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..ops import native

ALIGN = 64
BARRIER_TIMEOUT_NS = 60 * 10**9


class PeerArena:
    """A local cudaMalloc arena, mapped by every rank of ``group``."""

    def __init__(self, nbytes: int, group: dist.ProcessGroup | None, device: torch.device) -> None:
        C = native.lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        self.nbytes = nbytes
        self.buf, handle = C.ipc_alloc(nbytes)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle.tolist(), group=group)
        self.bases: list[int] = []
        self._opened: list[int] = []
        for k, h in enumerate(handles):
            if k == self.rank:
                self.bases.append(self.buf.data_ptr())
            else:
                ptr = C.ipc_open(torch.tensor(h, dtype=torch.uint8))
                self._opened.append(ptr)
                self.bases.append(ptr)

    def view(self, offset_bytes: int, numel: int, dtype: torch.dtype) -> torch.Tensor:
        es = torch.empty(0, dtype=dtype).element_size()
        assert offset_bytes % 256 == 0 and offset_bytes + numel * es <= self.nbytes
        return self.buf[offset_bytes : offset_bytes + numel * es].view(dtype)

    def table(self, offset_bytes: int, with_local: bool = False) -> torch.Tensor:
        ptrs = [b + offset_bytes for b in self.bases]
        if with_local:
            ptrs.append(self.bases[self.rank] + offset_bytes)
        return torch.tensor(ptrs, dtype=torch.int64, device=self.device)

    def close(self) -> None:
        C = native.lib()
        for p in self._opened:
            C.ipc_close(p)
        self._opened = []


def _round(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class FusedDataParallel:
    """Owns the peer arena holding the LoRA gradient and compute buffers."""

    def __init__(self, numel: int, compute_dtype: torch.dtype, group: dist.ProcessGroup | None,
                 device: torch.device) -> None:
        self.numel = numel
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        es = torch.empty(0, dtype=compute_dtype).element_size()
        self.off_grad = 0
        self.off_comp = _round(numel * 4)
        self.off_flags = _round(self.off_comp + numel * es)
        self.off_norms = self.off_flags + 256
        total = self.off_norms + 256
        self.arena = PeerArena(total, group, device)
        self.grad = self.arena.view(self.off_grad, numel, torch.float32)
        self.compute = self.arena.view(self.off_comp, numel, compute_dtype)
        self.norms = self.arena.view(self.off_norms, 64, torch.float32)
        self.grad_tab = self.arena.table(self.off_grad, with_local=True)
        self.comp_tab = self.arena.table(self.off_comp)
        self.flag_tab = self.arena.table(self.off_flags)
        self.norm_tab = self.arena.table(self.off_norms)
        per = (numel + self.world - 1) // self.world
        per = (per + ALIGN - 1) // ALIGN * ALIGN
        self.shards = [(min(r * per, numel), max(0, min(per, numel - r * per))) for r in range(self.world)]
        self.partial = torch.zeros(1, dtype=torch.float32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.epoch = 0
        self._hp = torch.zeros(8, dtype=torch.float32, device=device)

    # ------------------------------------------------------------------
    def barrier(self) -> None:
        self.epoch += 1
        native.lib().peer_barrier(self.flag_tab, self.rank, self.world, self.epoch, BARRIER_TIMEOUT_NS, self.status)

    def check(self) -> None:
        """Raise if a bounded wait gave up (call at a point that syncs anyway)."""
        if int(self.status.item()) != 0:
            raise RuntimeError("data-parallel peer barrier timed out (a rank stopped participating)")

    def reduce_and_step(self, optim, lr: float, stats: torch.Tensor | None = None) -> torch.Tensor:
        """Fused reduce-scatter + clipped AdamW + all-gather over the store."""
        C = native.lib()
        st = optim.store
        st.step += 1
        off, n = self.shards[self.rank]
        hp = optim._hparams(lr, 1.0, st.step)
        self._hp.copy_(torch.tensor(hp, dtype=torch.float32), non_blocking=True)
        self.barrier()  # A: all ranks' gradients complete
        C.dp_reduce_sumsq(self.grad_tab, self.world, off, n, self.partial)
        C.dp_publish_norm(self.norm_tab, self.rank, self.world, self.partial)
        self.barrier()  # B: reduced shards and partial norms visible
        sl = slice(off, off + n)
        C.dp_adamw_allgather(self.comp_tab, self.world, off, n, st.grad[sl], st.master[sl],
                             st.exp_avg[sl], st.exp_avg_sq[sl], self._hp, self.norms, optim.grad_norm)
        st.grad.zero_()
        self.barrier()  # C: parameters published to every rank
        st.version += 1
        if stats is not None:
            dist.all_reduce(stats, group=self.group)
        return optim.grad_norm

    def gather_full_state(self, store, moments: bool = True) -> None:
        """All-gather the master weights (and, with ``moments``, the AdamW
        moments) of every shard, before a checkpoint is written (cold path
        over NCCL).  Without ``moments`` each rank keeps only its own moment
        shard current and writes it itself (sharded optimizer state)."""
        per = self.shards[0][1]
        off, n = self.shards[self.rank]
        bufs = (store.master, store.exp_avg, store.exp_avg_sq) if moments else (store.master,)
        for buf in bufs:
            mine = torch.zeros(per, dtype=buf.dtype, device=buf.device)
            mine[:n].copy_(buf[off : off + n])
            out = torch.empty(per * self.world, dtype=buf.dtype, device=buf.device)
            dist.all_gather_into_tensor(out, mine, group=self.group)
            for r, (o, m) in enumerate(self.shards):
                buf[o : o + m].copy_(out[r * per : r * per + m])


def numel_of_specs(specs) -> int:
    return sum((math.prod(s) + ALIGN - 1) // ALIGN * ALIGN for _, s, _ in specs)
