#!/usr/bin/env python
"""Headline benchmark: trained tokens/sec per GRPO step.

Config (the data-parallel benchmark configuration): Qwen2.5-7B-shape dense
model, random init, bf16; LoRA rank 16 on q/k/v/o/gate/up/down; 8 groups x 16
rollouts per step, each group a shared 1024-token prompt + 16 completions of
512 tokens packed into one prefix-tree row; uniform token ids; Bernoulli(0.5)
rewards.  The global batch is fixed (strong scaling): with N GPUs each rank
trains 8/N rows per step, then gradients are reduced and one AdamW step runs.

``value`` = trainable tokens per step (65,536) / device step time (CUDA events,
max over ranks).  ``e2e`` times the same step through the public API
(``LocalBackend.train`` on ``TrajectoryGroup`` objects: tokenize, pack, pinned
H2D copy of the packed batch, train, D2H read of the metrics, checkpoint).

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Multi-GPU: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
"""

from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import subprocess
import sys
import tempfile
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", choices=sorted(CONFIGS), default="dense7b",
                   help="benchmark configuration (the BASELINE configs); flags below override its fields")
    p.add_argument("--model", default=None)
    p.add_argument("--groups", type=int, default=None)
    p.add_argument("--rollouts", type=int, default=None)
    p.add_argument("--prompt-len", type=int, default=None)
    p.add_argument("--completion-len", type=int, default=None)
    p.add_argument("--lora-rank", type=int, default=None)
    p.add_argument("--kl", type=float, default=None, help="KL penalty coefficient against the frozen base")
    p.add_argument("--layers", type=int, default=0, help="override layer count (debug only; invalid for the headline)")
    p.add_argument("--tp", type=int, default=None, help="tensor-parallel size (dense models)")
    p.add_argument("--cp", type=int, default=None, help="context-parallel size")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--e2e-steps", type=int, default=2)
    p.add_argument("--unfused", action="store_true",
                   help="the unfused baseline of this framework: cuBLAS projections and LM head, NCCL all-reduce "
                        "of the LoRA gradients and a replicated AdamW (the comparison point of the fused kernels)")
    p.add_argument("--recompute", default=None, choices=["none", "full"],
                   help="activation recompute per layer (default: the config's choice; the hybrid config "
                        "recomputes, as its 65,536-token row does not leave room for every layer's activations)")
    p.add_argument("--kernel-table", default=None,
                   help="write the device time per kernel of one profiled (untimed) step to this file, per rank")
    a = p.parse_args()
    c = CONFIGS[a.config]
    for key in ("model", "groups", "rollouts", "prompt_len", "completion_len", "lora_rank", "kl"):
        if getattr(a, key) is None:
            setattr(a, key, c[key])
    n = max(a.gpus, 1)
    if a.tp is None:
        a.tp = n if c["par"] == "tp" else 1
    if a.cp is None:
        if c["par"] == "cp":
            a.cp = n
        elif c["par"] == "ep":
            # one packed row per group: the rows are spread over data-parallel
            # groups and each row over the context-parallel ranks of its group
            a.cp = max(1, n // min(n, a.groups))
        else:
            a.cp = 1
    return a


# The GPU benchmark configurations (model shape, data per step, adapter, how
# the GPUs split the work).  "dense7b" is the headline.
CONFIGS = {
    "dense7b": dict(model="qwen2.5-7b", groups=8, rollouts=16, prompt_len=1024, completion_len=512,
                    lora_rank=16, kl=0.0, par="dp"),
    "moe30b": dict(model="qwen3-30b-a3b", groups=4, rollouts=8, prompt_len=2048, completion_len=1024,
                   lora_rank=8, kl=0.0, par="ep"),
    "hybrid": dict(model="qwen3-next-hybrid", groups=1, rollouts=8, prompt_len=8192, completion_len=7168,
                   lora_rank=16, kl=0.0, par="cp", recompute=True),
    "dense32b": dict(model="qwen3-32b", groups=16, rollouts=8, prompt_len=4096, completion_len=1024,
                     lora_rank=32, kl=0.01, par="tp"),
}


def write_kernel_table(path: str, events, rank: int) -> None:
    """Device time per kernel name of one profiled step (torch.profiler CUDA
    activity: every launch, no replay), with the span from the first kernel's
    start to the last one's end, so idle device time shows as the gap."""
    tot: dict[str, list] = {}
    t0, t1 = float("inf"), 0.0
    for e in events:
        d = e.device_time_total if hasattr(e, "device_time_total") else e.cuda_time_total
        r = tot.setdefault(e.name, [0.0, 0])
        r[0] += d
        r[1] += 1
        if e.time_range is not None:
            t0 = min(t0, e.time_range.start)
            t1 = max(t1, e.time_range.end)
    busy = sum(v[0] for v in tot.values())
    span = (t1 - t0) if t1 > t0 else float("nan")
    root, ext = os.path.splitext(path)
    with open(f"{root}.rank{rank}{ext or '.txt'}", "w") as f:
        f.write(f"# busy {busy / 1e3:.1f} ms of a {span / 1e3:.1f} ms span ({len(events)} launches)\n")
        f.write("share_pct\tms\tlaunches\tkernel\n")
        for name, (d, n) in sorted(tot.items(), key=lambda kv: -kv[1][0]):
            f.write(f"{100 * d / busy:.2f}\t{d / 1e3:.2f}\t{n}\t{name[:160]}\n")


BASELINE_VALUE = None  # the reference publishes no GPU number for this metric
METRIC = "trained tokens/sec per GRPO step (whole box, device-timed, max over ranks) 1/2/4/8 B200"


def reference_arm(args: argparse.Namespace) -> None:
    """The reference's own trainer cannot run here; say why in one line."""
    ref = os.path.join(HERE, "baseline", "_ref")
    reason = None
    if not os.path.isdir(os.path.join(ref, "art")):
        reason = (
            "reference not installable offline: its build backend 'hatchling' is not in "
            "/opt/wheelhouse, and its trainers need unsloth/peft/trl (LocalBackend) or "
            "megatron-core/transformer-engine (MegatronBackend), none of which are installed"
        )
    else:
        sys.path.insert(0, ref)
        try:
            import art  # noqa: F401
            from art.megatron import backend  # noqa: F401
        except Exception as exc:  # pragma: no cover - depends on the box
            reason = f"reference import failed: {type(exc).__name__}: {str(exc)[:160]}"
    if reason is None:
        reason = "reference Megatron trainer requires megatron-core, which is not installed"
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons in the background."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self) -> None:
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except Exception:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self, gpu_indices: list[int]) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if gpu_indices and idx not in gpu_indices:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                pass
            for name, val in zip(names, parts[5:9]):
                if val.lower() in ("active", "1", "yes"):
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return

    if args.unfused:  # read at import time by the op wrappers
        os.environ["ART_B200_PAIR_GEMM"] = "0"
        os.environ["ART_B200_LMHEAD_LIBRARY"] = "1"
        os.environ["ART_B200_EP_FUSED"] = "0"
    import torch
    import torch.distributed as dist

    sys.path.insert(0, HERE)
    from art_mlx_b200.models.config import LoRASpec, get_config
    from art_mlx_b200.preprocessing.pack import packed_tensors_from_tokenized_results
    from art_mlx_b200.preprocessing.synthetic import synthetic_groups
    from art_mlx_b200.preprocessing.tokenize import tokenize_trajectory_groups
    from art_mlx_b200.runtime.trainer import GRPOTrainer, _route_counts

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch one rank per GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=300))

    cfg = get_config(args.model)
    if args.layers:
        cfg = cfg.scaled(num_hidden_layers=args.layers)
    lora = LoRASpec(r=args.lora_rank, alpha=2 * args.lora_rank)
    random.seed(1234)
    torch.manual_seed(1234)
    groups = synthetic_groups(
        num_groups=args.groups, rollouts_per_group=args.rollouts, prompt_len=args.prompt_len,
        completion_len=args.completion_len, vocab_size=cfg.vocab_size, seed=1234, reward="bernoulli",
    )
    results = list(tokenize_trajectory_groups(None, groups, False, True, rng=random.Random(1)))
    row_len = args.prompt_len + args.rollouts * (args.completion_len + 1)
    seq_len = (row_len + 127) // 128 * 128
    packed = packed_tensors_from_tokenized_results(results, seq_len, rng=random.Random(2))
    n_rows = int(packed["tokens"].shape[0])
    train_tokens = float(packed["assistant_mask"][:, 1:].sum())
    packed_tokens = int((packed["group_ids"] >= 0).sum())

    # tokens a rank holds: a context-parallel row is padded to 128 tokens per rank
    rank_tokens = max(16384, -(-seq_len // (128 * args.cp)) * 128)
    recompute = args.recompute == "full" if args.recompute else bool(CONFIGS[args.config].get("recompute"))
    trainer = GRPOTrainer(cfg, lora, device, seed=0, group=dist.group.WORLD if world > 1 else None,
                          tp_size=args.tp, cp_size=args.cp, max_tokens_per_rank=rank_tokens,
                          recompute=recompute,
                          fused_dp=not args.unfused)
    lr = 1e-5
    loss_cfg: dict = {"kl_penalty_coef": args.kl} if args.kl else {}
    staged = trainer.stage(packed)
    if cfg.is_moe:
        # routing replay: the top-k experts of every token and layer are
        # recorded in a seeded forward pass and replayed by the training pass
        for mb in staged:
            rec: dict = {}
            with torch.no_grad():
                trainer.model.forward(mb.tokens, mb.meta, {"record_routes": rec, "group_ids": mb.group_ids,
                                                           "parent_ids": mb.parent_ids, "cp_plan": mb.cp_plan,
                                                           "cp": trainer.cp})
            mb.routes = torch.stack([rec[i] for i in sorted(rec)], dim=1)
            # as for routes that arrive from the rollout side, the per-layer
            # expert group sizes are counted on the host while staging
            mb.route_counts = _route_counts(mb.routes.cpu())
    l2_flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)

    def step() -> None:
        l2_flush.fill_(1)  # evict L2 between timed iterations
        trainer.train_step(packed, lr, loss_cfg, micro_batches=staged)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    parallelism = f"dp{world // (args.tp * args.cp)}" + (f"_tp{args.tp}" if args.tp > 1 else "") + (
        f"_cp{args.cp}" if args.cp > 1 else "") + (f"_ep{world}" if cfg.is_moe and world > 1 else "")
    ms = start.elapsed_time(end) / args.steps
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    clocks = sampler.stop(list(range(world))) if rank == 0 else {}
    metrics = trainer.train_step(packed, lr, loss_cfg, micro_batches=staged).to_host()

    # kernel launch count of one step (separate, untimed step under the profiler)
    launches = None
    try:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize()
        events = [e for e in prof.events() if e.device_type.name == "CUDA"]
        names = [e.name for e in events]
        ours = [n for n in names if "art::" in n]
        launches = len(ours) * args.steps
        lib_kernels = len(names) - len(ours)
        if args.kernel_table:
            try:
                write_kernel_table(args.kernel_table, events, rank)
            except Exception as exc:  # the table is a diagnostic: never fail the bench line
                print(f"kernel table not written: {exc!r}", file=sys.stderr)
    except Exception:
        lib_kernels = None

    # end-to-end through the public API
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, cfg, lora, groups, trainer, device, world, rank, train_tokens)

    value = train_tokens / (ms / 1000.0)
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "trained tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None if BASELINE_VALUE is None else value / BASELINE_VALUE,
            "dtype": "bf16",
            "data": "synthetic (uniform token ids, Bernoulli(0.5) rewards, random-init weights)",
            "config": {
                "model": cfg.name + ("" if not args.layers else f"-{args.layers}L(INVALID)"),
                "global_batch": f"{args.groups} groups x {args.rollouts} rollouts",
                "seq_len": seq_len,
                "prompt_len": args.prompt_len,
                "completion_len": args.completion_len,
                "lora_rank": args.lora_rank,
                "parallelism": parallelism,
                "activation_recompute": "full" if recompute else "none",
                "rows_per_step": n_rows,
                "trained_tokens_per_step": int(train_tokens),
                "packed_tokens_per_step": packed_tokens,
                "packed_tokens_per_s": round(packed_tokens / (ms / 1000.0), 1),
                "l2": "256 MiB buffer written before every step; the per-GPU weights exceed L2",
                "loss": "cispo (default)" + (f", KL {args.kl} against the frozen base" if args.kl else ""),
                "bench_config": args.config,
                "library_kernels_per_step": lib_kernels,
                "final_metrics": metrics,
            },
            "clocks": clocks,
            "gpu_launches": launches,
            "impl": "ours-unfused" if args.unfused else "ours",
        }
        if e2e is not None:
            out["e2e"] = e2e
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, cfg, lora, groups, trainer, device, world, rank, train_tokens) -> dict | None:
    """Time the public ``LocalBackend.train`` call (tokenize, pack, pinned H2D,
    train, D2H metrics, checkpoint) on the already-built trainer."""
    import asyncio

    import torch
    import torch.distributed as dist

    try:
        from art_mlx_b200 import TrainableModel
        from art_mlx_b200.backends.local import LocalBackend
    except Exception as exc:  # pragma: no cover
        return {"value": None, "unavailable": f"{type(exc).__name__}: {exc}"}

    # one model directory for the whole job: rank 0 publishes the adapter
    # there and every rank adds its optimizer shard
    tmp = [tempfile.mkdtemp(prefix="artb200_bench_") if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(tmp, src=0)
    tmp = tmp[0]
    backend = LocalBackend(path=tmp, trainer=trainer)
    model = TrainableModel(
        name="bench", project="bench", base_model=cfg.name,
        _internal_config={"peft_args": {"r": lora.r, "lora_alpha": lora.alpha}},
    )

    async def go():
        await model.register(backend)
        times = []
        h2d = d2h = 0
        breakdown: dict = {}
        for i in range(args.e2e_steps + 1):
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            res = await backend.train(model, groups, learning_rate=1e-5, packed_sequence_length=None)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            if i > 0:  # first call is warm-up
                times.append(dt)
                breakdown = {k.split("/", 1)[1]: round(float(v), 4) for k, v in res.metrics.items()
                             if k.startswith("time/step_")}
            h2d = backend.last_h2d_bytes
            d2h = backend.last_d2h_bytes
        return times, h2d, d2h, breakdown

    times, h2d, d2h, breakdown = asyncio.run(go())
    dt = max(times) if times else float("nan")
    t = torch.tensor([dt], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dt = float(t.item())
    return {
        "value": round(train_tokens / dt, 1),
        "unit": "trained tokens/s",
        "seconds_per_step": round(dt, 4),
        "steps": len(times),
        "h2d_bytes_per_step": int(h2d),
        "d2h_bytes_per_step": int(d2h),
        "api": "LocalBackend.train(model, groups)",
        "breakdown_s": breakdown,
    }


if __name__ == "__main__":
    main()
