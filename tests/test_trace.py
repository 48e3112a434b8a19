"""Forward traces keyed by token UID: a context-parallel run (2 gloo ranks,
each its slice of every packed row) merged and compared layer by layer with
the one-process trace of the same model and rows (the reference's topology
oracle on forward traces)."""

import os
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from art_mlx_b200.models.config import LoRASpec
from art_mlx_b200.runtime.trainer import GRPOTrainer
from art_mlx_b200.utils.trace import ForwardTraceCapture, diff_traces
from test_distributed import HYBRID_CPU, _packed, _shape


def _trace(tr, mbs) -> list[dict]:
    out = []
    for mb in mbs:
        cap = ForwardTraceCapture()
        ctx = {"trace": cap, "group_ids": mb.group_ids, "parent_ids": mb.parent_ids}
        if mb.cp_plan is not None:
            ctx["cp_plan"], ctx["cp"] = mb.cp_plan, tr.cp
        with torch.no_grad():
            tr.model.forward(mb.tokens, mb.meta, ctx)
        out.append(cap.state())
    return out


def _worker(rank, world, init_file, out_dir):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        packed = _packed(*_shape("gloo", HYBRID_CPU))
        tr = GRPOTrainer(HYBRID_CPU, LoRASpec(r=8, alpha=16), torch.device("cpu"), seed=0, group=dist.group.WORLD,
                         cp_size=world)
        torch.save(_trace(tr, tr.stage(packed)), os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_cp_trace_matches_single_process_by_token_uid():
    d = tempfile.mkdtemp()
    mp.start_processes(_worker, args=(2, os.path.join(d, "init"), d), nprocs=2, start_method="spawn")
    ranks = [torch.load(os.path.join(d, f"rank{r}.pt")) for r in range(2)]
    packed = _packed(*_shape("gloo", HYBRID_CPU))
    tr = GRPOTrainer(HYBRID_CPU, LoRASpec(r=8, alpha=16), torch.device("cpu"), seed=0)
    single = _trace(tr, tr.stage(packed))
    assert len(single) == len(ranks[0])
    for row, ref in enumerate(single):
        merged = ForwardTraceCapture.merge([ranks[0][row], ranks[1][row]])
        ref_t = ForwardTraceCapture.merge([ref])
        # the two ranks hold disjoint slices that together cover the row
        k = next(iter(ref_t))
        assert torch.equal(merged[k][0], ref_t[k][0])
        d = diff_traces(merged, ref_t)
        assert len(d) == 2 * HYBRID_CPU.num_hidden_layers + 1
        assert max(d.values()) < 1e-5, d
