"""``MultiGPUBackend``: trains on every GPU of this host through a persistent
worker group (one process per GPU, ``torch.distributed`` over NCCL).

Reference behaviour: ``MegatronBackend`` / ``MegatronService``
(``src/art/megatron/backend.py:15-81``, ``service.py:188-1000``): the client
process tokenizes and packs, writes the packed tensors to disk and submits a
job; a torchrun worker group that stays alive across steps trains on them and
publishes the adapter; the client streams the results.

Here:

* the topology (``TopologyConfig``: ``tp`` or ``cp`` inside a data-parallel
  job, expert parallelism over all ranks for MoE models) is fixed when the
  worker group starts (``runtime_config`` or the constructor);
* the worker group is ``python -m torch.distributed.run ... -m
  art_mlx_b200.runtime.worker`` in its own process group; ``close()`` sends a
  shutdown job, then stops the process group it started if it lingers;
* tokenization, advantages, packing, checkpoint directories, metrics and the
  result type are the ``LocalBackend`` ones (inherited).
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
import time
from typing import Any, AsyncIterator, Iterable

from .. import dev
from ..runtime import jobs as J
from ..trajectories import Trajectory
from ..types import RuntimeConfig, TopologyConfig, TrainSFTConfig
from ..utils import managed_process
from ..utils.output_dirs import get_step_checkpoint_dir, get_step_from_dir
from .local import LocalBackend

_RUNTIME_CONFIG: RuntimeConfig | None = None


def init_runtime_config(
    config: RuntimeConfig | dict | None = None,
    *,
    topology: TopologyConfig | dict | None = None,
    packed_sequence_length: int | None = None,
) -> RuntimeConfig:
    """Process-wide runtime configuration (reference
    ``src/art/megatron/runtime_config.py:11-40``): set once, re-setting it
    to a different value is an error."""
    global _RUNTIME_CONFIG
    if config is None:
        config = {"topology": topology or TopologyConfig(), "packed_sequence_length": packed_sequence_length}
    rc = RuntimeConfig.model_validate(config)
    if _RUNTIME_CONFIG is None:
        _RUNTIME_CONFIG = rc
    elif _RUNTIME_CONFIG != rc:
        raise ValueError(f"runtime config already initialised with {_RUNTIME_CONFIG.model_dump(mode='json')}")
    return _RUNTIME_CONFIG


def get_runtime_config() -> RuntimeConfig | None:
    return _RUNTIME_CONFIG


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _WorkerGroup:
    def __init__(self, jobs_dir: str, proc: subprocess.Popen, world: int, log_path: str) -> None:
        self.jobs_dir, self.proc, self.world, self.log_path = jobs_dir, proc, world, log_path

    def alive(self) -> bool:
        return self.proc.poll() is None


class MultiGPUBackend(LocalBackend):
    def __init__(
        self,
        *,
        path: str | None = None,
        num_gpus: int | None = None,
        topology: TopologyConfig | dict | None = None,
        packed_sequence_length: int | None = None,
        device: str = "auto",
        seed: int = 0,
        startup_timeout_s: float = 600.0,
        heartbeat_limit_s: float | None = 120.0,
        worker_timeout_s: float = 600.0,
    ) -> None:
        import torch

        dev_type = ("cuda" if torch.cuda.is_available() else "cpu") if device == "auto" else device
        super().__init__(path=path, device="cpu", seed=seed)
        rc = get_runtime_config()
        if topology is None and rc is not None:
            topology = rc.topology
        if packed_sequence_length is None and rc is not None:
            packed_sequence_length = rc.packed_sequence_length
        self._world = num_gpus or (torch.cuda.device_count() if dev_type == "cuda" else 2)
        topo = TopologyConfig.model_validate(topology) if isinstance(topology, dict) else topology
        self._topology = topo  # None: the default layout policy, resolved per model
        self._packed_len = packed_sequence_length
        self._dev_type = dev_type
        self._groups: dict[str, _WorkerGroup] = {}
        self._startup_timeout = startup_timeout_s
        self._heartbeat_limit = heartbeat_limit_s
        self._worker_timeout = worker_timeout_s
        self.last_h2d_bytes = 0

    # ------------------------------------------------------------------
    def _worker_group(self, model: Any) -> _WorkerGroup:
        g = self._groups.get(model.name)
        if g is not None and g.alive():
            return g
        d = self._model_dir(model)
        jobs_dir = os.path.join(d, "jobs")
        os.makedirs(jobs_dir, exist_ok=True)
        for f in os.listdir(jobs_dir):  # a fresh group starts from an empty queue
            if os.path.isfile(os.path.join(jobs_dir, f)):
                os.remove(os.path.join(jobs_dir, f))
        step = get_step_from_dir(d)
        init_ck = get_step_checkpoint_dir(d, step)
        internal = getattr(model, "_internal_config", None) or {}
        preset = internal.get("model_preset") or model.base_model
        targs = dict(dev.default_trainer_args())
        targs.update(internal.get("trainer_args") or {})
        adamw = {
            "beta1": targs.get("adam_beta1", 0.9), "beta2": targs.get("adam_beta2", 0.99),
            "eps": targs.get("adam_epsilon", 1e-8), "weight_decay": targs.get("weight_decay", 0.1),
            "max_grad_norm": targs.get("max_grad_norm", 0.1),
        }
        peft = dict(internal.get("peft_args") or {})
        peft.update(getattr(model, "lora_config", None) or {})
        topo = self._topology
        if topo is None:  # no layout named: the default policy for this model and GPU count
            from ..models.config import get_config
            from ..parallel.topology import default_topology

            layout = default_topology(get_config(preset), self._world,
                                      row_tokens=self._packed_len if getattr(self, "_packed_len", None) else None)
            topo = TopologyConfig(tp=layout["tp"], cp=layout["cp"], ep=layout["ep"])
        tp = topo.tp if topo.tp > 1 else 1
        cp = topo.cp if (topo.cp > 1 and topo.cp <= self._world and tp == 1) else 1
        etp = topo.etp if (topo.etp > 1 and self._world % topo.etp == 0) else 1
        cmd = [
            sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(self._world),
            "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
            "-m", "art_mlx_b200.runtime.worker", "--jobs-dir", jobs_dir, "--model", preset,
            "--base-model", model.base_model, "--lora", json.dumps(peft), "--adamw", json.dumps(adamw),
            "--tp", str(tp), "--cp", str(cp), "--etp", str(etp), "--seed", str(self._seed),
            "--device", self._dev_type,
            "--init-checkpoint", init_ck, "--timeout-s", str(self._worker_timeout),
        ]
        log_path = os.path.join(d, "logs", "workers.log")
        os.makedirs(os.path.dirname(log_path), exist_ok=True)
        env = dict(os.environ)
        pkg_root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        env["PYTHONPATH"] = pkg_root + os.pathsep + env.get("PYTHONPATH", "")
        with open(log_path, "a") as logf:
            # own session + parent-death signal: the worker group never outlives this process
            proc = managed_process.popen(cmd, stdout=logf, stderr=subprocess.STDOUT, env=env)
        g = _WorkerGroup(jobs_dir, proc, self._world, log_path)
        deadline = time.monotonic() + self._startup_timeout
        while not os.path.exists(os.path.join(jobs_dir, "ready")):
            if proc.poll() is not None:
                raise RuntimeError(f"worker group exited with code {proc.returncode}; see {log_path}")
            if time.monotonic() > deadline:
                self._stop(g)
                raise TimeoutError(f"worker group not ready after {self._startup_timeout}s; see {log_path}")
            time.sleep(0.05)
        self._groups[model.name] = g
        return g

    async def _submit(self, model: Any, job_factory) -> AsyncIterator[dict[str, Any]]:
        g = self._worker_group(model)
        path = J.next_job_path(g.jobs_dir)
        job = job_factory(path[:-5] + ".log")
        J.write_job(job, path)
        async for rec in J.stream_job(job, path, process=g.proc, jobs_dir=g.jobs_dir, world=g.world,
                                      heartbeat_limit_s=self._heartbeat_limit):
            yield rec

    def _stop(self, g: _WorkerGroup, grace_s: float = 60.0) -> None:
        if g.alive():
            try:
                path = J.next_job_path(g.jobs_dir)
                J.write_job(J.ShutdownJob(log_path=path[:-5] + ".log"), path)
                g.proc.wait(timeout=grace_s)
            except subprocess.TimeoutExpired:
                managed_process.stop_group(g.proc)  # the process group this backend started

    async def close(self) -> None:
        for g in self._groups.values():
            self._stop(g)
        self._groups.clear()
        await super().close()

    # ------------------------------------------------------------------
    async def _prepare_backend_for_training(self, model: Any, config: dev.OpenAIServerConfig | None = None):
        self._worker_group(model)
        cfg = config or {}
        host, port = cfg.get("host", "127.0.0.1"), int(cfg.get("port", 8000))
        return f"http://{host}:{port}/v1", cfg.get("server_args", {}).get("api_key", "default")

    def _pack(self, results, packed_sequence_length, advantage_balance, model=None):
        # the client packs every row: the worker ranks read the rows they train from disk
        return super()._pack(results, packed_sequence_length or self._packed_len, advantage_balance)

    async def _train_packed(self, model, packed, lr, dev_config, kl_ref_adapter_path, logprob_chunk, out_dir,
                            grad_accumulation_sequences=None):
        from ..preprocessing.pack import packed_tensors_to_dir

        d = self._model_dir(model)
        step = get_step_from_dir(d)
        g = self._worker_group(model)
        pdir = os.path.join(g.jobs_dir, "packed")
        disk = packed_tensors_to_dir(packed, pdir)
        self.last_h2d_bytes = sum(int(packed[k].numel() * packed[k].element_size())
                                  for k in ("tokens", "group_ids", "parent_ids", "input_pos", "assistant_mask",
                                            "logprobs", "advantages", "weights"))
        out = None
        async for rec in self._submit(model, lambda log: J.TrainJob(
            packed_dir=pdir, num_sequences=disk["num_sequences"], sequence_length=disk["sequence_length"],
            checkpoint_dir=get_step_checkpoint_dir(d, step), output_dir=out_dir, base_model=model.base_model,
            learning_rate=lr, config=dict(dev_config), kl_ref_adapter_path=kl_ref_adapter_path,
            logprob_chunk=logprob_chunk, grad_accumulation_sequences=grad_accumulation_sequences, log_path=log,
        )):
            out = rec
        if out is None:
            raise RuntimeError("worker group returned no metrics")
        return out

    async def _train_sft(
        self,
        model: Any,
        trajectories: Iterable[Trajectory],
        config: TrainSFTConfig,
        dev_config: dev.TrainSFTConfig,
        verbose: bool = False,
    ) -> AsyncIterator[dict[str, float]]:
        from ..runtime.sft import sft_batches_from_trajectories

        trajs = list(trajectories)
        bs = config.batch_size if isinstance(config.batch_size, int) else max(2, 2 * self._world)
        batches = sft_batches_from_trajectories(trajs, bs)
        lrs = config.learning_rate if isinstance(config.learning_rate, list) else [config.learning_rate]
        d = self._model_dir(model)
        g = self._worker_group(model)
        bpath = os.path.join(g.jobs_dir, "sft_batches.json")
        with open(bpath, "w") as f:
            json.dump([[list(x) for x in b] for b in batches], f)
        step = get_step_from_dir(d)
        async for rec in self._submit(model, lambda log: J.SFTJob(
            batches_path=bpath, checkpoint_dir=get_step_checkpoint_dir(d, step),
            output_dir=get_step_checkpoint_dir(d, step + 1), base_model=model.base_model,
            learning_rates=[float(x) for x in lrs], log_path=log,
        )):
            yield rec

    async def _experimental_fork_checkpoint(self, model: Any, from_model: str, from_project: str | None = None,
                                            not_after_step: int | None = None) -> int:
        import shutil

        from ..utils.output_dirs import get_output_dir_from_model_properties, list_checkpoint_steps

        src = get_output_dir_from_model_properties(from_project or model.project, from_model, self._path)
        steps = [s for s in list_checkpoint_steps(src) if not_after_step is None or s <= not_after_step]
        if not steps:
            raise FileNotFoundError(f"no checkpoints under {src}")
        s = max(steps)
        dst = get_step_checkpoint_dir(self._model_dir(model), s)
        if os.path.exists(dst):
            shutil.rmtree(dst)
        shutil.copytree(get_step_checkpoint_dir(src, s), dst)
        async for _ in self._submit(model, lambda log: J.LoadJob(checkpoint_dir=dst, log_path=log)):
            pass
        return s
