"""Persistent training worker: one process per GPU, launched by
``torch.distributed.run`` and driven by job files (runtime/jobs.py).

Reference behaviour: the torchrun worker loop of the Megatron service
(``src/art/megatron/train.py:334`` ``build_training_runtime``,
``run_megatron_worker_loop``; job handling ``service.py:971``).  Here every
rank builds a :class:`GRPOTrainer` with the requested topology once, then
loops: poll the jobs directory, run the next job collectively (train / SFT /
load / shutdown), rank 0 publishes the adapter and the result records.

Usage (what ``MultiGPUBackend`` runs)::

    python -m torch.distributed.run --nnodes 1 --nproc-per-node N \\
        --master-addr 127.0.0.1 --master-port P \\
        -m art_mlx_b200.runtime.worker --jobs-dir D --model qwen2.5-7b \\
        --lora '{"r": 16, "alpha": 32}' --tp 1 --cp 1 --etp 1 --init-checkpoint C
"""

from __future__ import annotations

import argparse
import json
import os
import threading
import time
import traceback
from datetime import timedelta

import torch
import torch.distributed as dist

from . import jobs as J


def _beat(path: str, stop: threading.Event) -> None:
    while not stop.is_set():
        with open(path, "a"):
            os.utime(path, None)
        stop.wait(1.0)


def _load_adapter_into(tr, ck: str) -> None:
    from .checkpoint import load_adapter

    opt = load_adapter(ck, tr.store)
    if opt is not None:
        tr.optim.load_state_dict(opt)


def _save(tr, out: str, base_model: str, rank: int) -> None:
    from .checkpoint import save_adapter

    tr.prepare_checkpoint()  # collective
    if rank == 0:
        save_adapter(out, tr.store, base_model, tr.model.lora_spec, tr.optim.state_dict())


def _injected_exit(rank: int, kind: str) -> None:
    """Host-side failure injection for tests: ``ART_B200_WORKER_EXIT=<rank>:<kind>``
    makes that rank's process exit when it picks up a job of that kind,
    before any collective of the job (a rank that leaves between steps)."""
    spec = os.environ.get("ART_B200_WORKER_EXIT")
    if spec:
        r, k = spec.split(":")
        if int(r) == rank and k == kind:
            os._exit(3)


def run_job(tr, job, state: dict) -> list[dict]:
    """Run one job on every rank (collective); returns rank 0's records."""
    rank = tr.rank
    _injected_exit(rank, job.kind)
    if job.kind == "load":
        _load_adapter_into(tr, job.checkpoint_dir)
        state["loaded"] = job.checkpoint_dir
        return [{"loaded": job.checkpoint_dir}]
    if job.kind == "train":
        from ..preprocessing.pack import packed_tensors_from_dir

        if state.get("loaded") != job.checkpoint_dir:
            _load_adapter_into(tr, job.checkpoint_dir)
        packed = packed_tensors_from_dir(dir=job.packed_dir, num_sequences=job.num_sequences,
                                         sequence_length=job.sequence_length)
        ref = None
        if float(job.config.get("kl_penalty_coef", 0.0) or 0.0) > 0 and job.kl_ref_adapter_path:
            from safetensors.torch import load_file

            ref = load_file(os.path.join(job.kl_ref_adapter_path, "adapter_model.safetensors"))
        tr.set_reference_adapter(ref)
        tr.logprob_chunk = job.logprob_chunk
        t0 = time.monotonic()
        steps = [m.to_host() for m in tr.train_steps(packed, job.learning_rate, job.config,
                                                     job.grad_accumulation_sequences)]
        metrics = {k: sum(m[k] for m in steps) / len(steps) for k in steps[0]}
        for k in ("data/step_trainer_tokens", "data/step_packed_tokens"):
            metrics[k] = sum(m[k] for m in steps)
        metrics["data/step_num_gradient_steps"] = float(len(steps))
        metrics["time/step_trainer_s"] = time.monotonic() - t0
        if job.output_dir is not None:
            _save(tr, job.output_dir, job.base_model, rank)
            state["loaded"] = job.output_dir
        return [metrics]
    if job.kind == "sft":
        if state.get("loaded") != job.checkpoint_dir:
            _load_adapter_into(tr, job.checkpoint_dir)
        with open(job.batches_path) as f:
            batches = json.load(f)
        out = []
        for i, batch in enumerate(batches):
            lr = job.learning_rates[min(i, len(job.learning_rates) - 1)]
            out.append(tr.sft_step([(ids, labels) for ids, labels in batch], lr))
        if job.output_dir is not None:
            _save(tr, job.output_dir, job.base_model, rank)
            state["loaded"] = job.output_dir
        return out
    return []


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs-dir", required=True)
    ap.add_argument("--model", required=True, help="architecture preset name")
    ap.add_argument("--lora", default="{}", help="LoRA spec as PEFT-style JSON")
    ap.add_argument("--adamw", default="{}", help="AdamW settings as JSON")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--cp", type=int, default=1)
    ap.add_argument("--etp", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--device", choices=["cuda", "cpu"], default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--init-checkpoint", required=True, help="adapter to load, written first if missing")
    ap.add_argument("--base-model", default=None)
    ap.add_argument("--timeout-s", type=float, default=600.0)
    ap.add_argument("--poll-s", type=float, default=0.02)
    args = ap.parse_args(argv)

    from ..models.config import LoRASpec, get_config
    from .optimizer import AdamWConfig
    from .trainer import GRPOTrainer

    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.device == "cuda":
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=args.timeout_s))
    else:
        device = torch.device("cpu")
        dist.init_process_group("gloo", timeout=timedelta(seconds=args.timeout_s))
    rank, world = dist.get_rank(), dist.get_world_size()
    stop = threading.Event()
    threading.Thread(target=_beat, args=(J.heartbeat_path(args.jobs_dir, rank), stop), daemon=True).start()
    tr = None
    try:
        cfg = get_config(args.model)
        lora = LoRASpec.from_peft(json.loads(args.lora)) if json.loads(args.lora) else LoRASpec()
        adamw = AdamWConfig(**json.loads(args.adamw))
        tr = GRPOTrainer(cfg, lora, device, seed=args.seed, adamw=adamw, group=dist.group.WORLD,
                         tp_size=args.tp, cp_size=args.cp, etp_size=args.etp)
        if args.base_model and hasattr(tr.model, "load_hf_state_dict"):
            from ..models.weights import maybe_load_base_weights

            maybe_load_base_weights(tr.model, args.base_model)
        state: dict = {}
        if os.path.exists(os.path.join(args.init_checkpoint, "adapter_model.safetensors")):
            _load_adapter_into(tr, args.init_checkpoint)
        else:
            _save(tr, args.init_checkpoint, args.base_model or args.model, rank)
        state["loaded"] = args.init_checkpoint
        dist.barrier()
        if rank == 0:
            with open(os.path.join(args.jobs_dir, "ready"), "w") as f:
                f.write(str(world))
        last = 0
        while True:
            todo = J.pending_jobs(args.jobs_dir, last)
            if not todo:
                time.sleep(args.poll_s)
                continue
            seq, path = todo[0]
            job = J.load_job(open(path, encoding="utf-8").read())
            last = seq
            if job.kind == "shutdown":
                dist.barrier()
                if rank == 0:
                    J.append_log(job.log_path, J.DONE)
                break
            try:
                records = run_job(tr, job, state)
                err = None
            except Exception:  # the job fails on this rank; tell the client
                records, err = [], traceback.format_exc()
            # every rank learns whether any rank failed before the next job
            flag = torch.tensor([1.0 if err else 0.0], device=device)
            dist.all_reduce(flag)
            if rank == 0 or err:
                for r in records if rank == 0 else []:
                    J.append_log(job.log_path, r)
                if err:
                    J.append_log(job.log_path, {"error": f"rank {rank}: {err}"})
            dist.barrier()
            if rank == 0:
                J.append_log(job.log_path, J.DONE)
            if flag.item() > 0:
                raise SystemExit(1)  # state may be inconsistent across ranks: stop the group
    finally:
        stop.set()
        if tr is not None and tr.grad_sync is not None:
            tr.grad_sync = None
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
