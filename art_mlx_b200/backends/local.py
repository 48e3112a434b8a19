"""``LocalBackend``: trains LoRA adapters on this host's GPUs.

Behaviour of the reference ``src/art/local/backend.py:192-1713`` re-designed
for one process per GPU:

* ``register`` creates ``{path}/{project}/models/{name}/`` and ``model.json``;
* ``_prepare_backend_for_training`` builds the trainer for
  ``model.base_model`` (a preset architecture, random-init unless real
  weights are loaded), resumes from the latest checkpoint or writes the
  step-0 adapter, and (optionally) starts the rollout server;
* ``train(model, groups, ...)`` = tokenize (token ids from the rollout
  server) → group advantages → prefix-tree pack → stage rows on the device
  (pinned host memory) → GRPO step → read metrics back → publish
  ``checkpoints/{step+1:04d}`` atomically → ``LocalTrainResult``;
* when nothing in the batch is trainable the step still advances by
  copying the previous checkpoint (reference ``:1035-1090``);
* under ``torch.distributed`` (one rank per GPU) every rank calls ``train``
  with the same groups; rows are interleaved across data-parallel ranks and
  rank 0 writes the checkpoint.
"""

from __future__ import annotations

import contextlib
import json
import os
import random
import shutil
import time
from typing import Any, AsyncIterator, Iterable, Literal

import torch
import torch.distributed as dist

from .. import dev
from ..backend import aggregate_rl_training_metrics, build_rl_train_configs
from ..metrics import MetricsBuilder
from ..models.config import LoRASpec, get_config
from ..preprocessing.pack import packed_tensors_from_tokenized_results, packed_tensors_to_dir
from ..preprocessing.tokenize import TokenizedResult, tokenize_trajectory_groups
from ..runtime.checkpoint import AsyncCheckpointWriter, load_adapter, save_adapter
from ..runtime.trainer import GRPOTrainer
from ..trajectories import Trajectory, TrajectoryGroup
from ..types import LocalTrainResult, TrainSFTConfig
from ..utils.output_dirs import get_model_dir, get_step_checkpoint_dir, get_step_from_dir


def _rank() -> int:
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def _barrier() -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


class LocalBackend:
    def __init__(
        self,
        *,
        in_process: bool = True,
        path: str | None = None,
        trainer: GRPOTrainer | None = None,
        device: str | torch.device | None = None,
        seed: int = 0,
        inference: Literal["none", "native", "vllm"] = "none",
        vllm_gpus: str | None = None,
        vllm_engine_args: dict | None = None,
    ) -> None:
        self._path = path or os.path.join(os.getcwd(), ".art")
        os.makedirs(self._path, exist_ok=True)
        self._in_process = in_process
        self._trainers: dict[str, GRPOTrainer] = {}
        self._given_trainer = trainer
        self._device = torch.device(device) if device is not None else self._default_device()
        self._seed = seed
        self._inference = inference
        # inference="vllm": a vLLM OpenAI server (runtime/vllm_runtime.py) on the GPUs
        # named by vllm_gpus (dedicated mode); each published step is hot-loaded
        # as the adapter "{model}@{step}"
        self._vllm_gpus = vllm_gpus
        self._vllm_engine_args = dict(vllm_engine_args or {})
        self._vllm: dict[str, Any] = {}
        self._servers: dict[str, Any] = {}
        self._engines: dict[str, Any] = {}
        # step checkpoints are written in the background (the write of step n
        # overlaps step n+1); everything that reads checkpoints waits first
        self._writer = AsyncCheckpointWriter()
        self._leases: dict[str, Any] = {}
        self._metrics: dict[str, MetricsBuilder] = {}
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0

    @staticmethod
    def _default_device() -> torch.device:
        if torch.cuda.is_available():
            return torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        return torch.device("cpu")

    async def __aenter__(self) -> "LocalBackend":
        return self

    async def __aexit__(self, *exc: Any) -> None:
        await self.close()

    def _flush(self) -> None:
        """Wait until every submitted optimizer-state write is on disk (adapters
        are published synchronously by the writer)."""
        self._writer.wait()

    async def close(self) -> None:
        self._flush()
        for server in self._servers.values():
            server.stop()
        self._servers.clear()
        for rt in self._vllm.values():
            rt.close()
        self._vllm.clear()

    # ------------------------------------------------------------------
    def _model_dir(self, model: Any) -> str:
        return get_model_dir(model, self._path)

    def _model_inference_name(self, model: Any, step: int | None = None) -> str:
        from ..adapter_leases import pinned_inference_step

        self._flush()
        if step is None:
            step = pinned_inference_step(model.name)
        if step is None:
            step = get_step_from_dir(self._model_dir(model)) if getattr(model, "trainable", False) else None
        base = model.name
        return f"{base}@{step}" if step is not None else base

    async def register(self, model: Any) -> None:
        # the model's own logs (history, trajectories) live next to its checkpoints
        model.base_path = self._path
        d = self._model_dir(model)
        os.makedirs(d, exist_ok=True)
        if _rank() == 0:
            with open(os.path.join(d, "model.json"), "w") as f:
                json.dump(model.model_dump(mode="json"), f, indent=2, default=str)

    async def _get_step(self, model: Any) -> int:
        return get_step_from_dir(self._model_dir(model))

    def adapter_leases(self, model: Any):
        """Lease manager of the model's checkpoints: leased steps survive cleanup."""
        from ..adapter_leases import AdapterLeaseManager

        return self._leases.setdefault(model.name, AdapterLeaseManager())

    async def _delete_checkpoint_files(self, model: Any, steps_to_keep: list[int]) -> None:
        self._flush()
        steps_to_keep = sorted(set(steps_to_keep) | self.adapter_leases(model).active_steps())
        if _rank() != 0:
            return
        ck = os.path.join(self._model_dir(model), "checkpoints")
        if not os.path.isdir(ck):
            return
        for d in os.listdir(ck):
            if d.isdigit() and int(d) not in steps_to_keep:
                shutil.rmtree(os.path.join(ck, d), ignore_errors=True)

    # ------------------------------------------------------------------
    def _lora_spec(self, model: Any) -> LoRASpec:
        internal = getattr(model, "_internal_config", None) or {}
        peft = dict(internal.get("peft_args") or {})
        peft.update(getattr(model, "lora_config", None) or {})
        spec = LoRASpec.from_peft(peft) if peft else LoRASpec()
        return spec

    def _get_trainer(self, model: Any) -> GRPOTrainer:
        key = model.name
        if key in self._trainers:
            return self._trainers[key]
        if self._given_trainer is not None:
            tr = self._given_trainer
        else:
            internal = getattr(model, "_internal_config", None) or {}
            cfg = get_config(internal.get("model_preset") or model.base_model)
            targs = dict(dev.default_trainer_args())
            targs.update(internal.get("trainer_args") or {})
            from ..runtime.optimizer import AdamWConfig

            adamw = AdamWConfig(
                beta1=targs.get("adam_beta1", 0.9), beta2=targs.get("adam_beta2", 0.99),
                eps=targs.get("adam_epsilon", 1e-8), weight_decay=targs.get("weight_decay", 0.1),
                max_grad_norm=targs.get("max_grad_norm", 0.1),
            )
            group = dist.group.WORLD if dist.is_available() and dist.is_initialized() else None
            tr = GRPOTrainer(cfg, self._lora_spec(model), self._device, seed=self._seed, adamw=adamw, group=group)
            from ..models.weights import maybe_load_base_weights

            if hasattr(tr.model, "load_hf_state_dict"):
                maybe_load_base_weights(tr.model, model.base_model)
        self._trainers[key] = tr
        return tr

    async def _prepare_backend_for_training(
        self, model: Any, config: dev.OpenAIServerConfig | None = None
    ) -> tuple[str, str]:
        self._flush()
        _barrier()  # every rank's optimizer shard of the last step is on disk
        tr = self._get_trainer(model)
        d = self._model_dir(model)
        step = get_step_from_dir(d)
        ck = get_step_checkpoint_dir(d, step)
        if os.path.exists(os.path.join(ck, "adapter_model.safetensors")):
            opt = load_adapter(ck, tr.store)
            if opt is not None:
                tr.optim.load_state_dict(opt)
        elif _rank() == 0:
            save_adapter(ck, tr.store, model.base_model, tr.model.lora_spec, tr.optim.state_dict())
        _barrier()
        cfg = config or {}
        host = cfg.get("host", "127.0.0.1")
        port = int(cfg.get("port", 8000))
        api_key = cfg.get("server_args", {}).get("api_key", "default")
        if self._inference == "native" and _rank() == 0 and model.name not in self._servers:
            from .inference import RolloutServer

            server = RolloutServer(self._engine(model), self._tokenizer(model), served_name=model.name,
                                   resolve_adapter=lambda name: self._resolve_adapter(model, name),
                                   host=host, port=port, api_key=api_key)
            server.start()
            self._servers[model.name] = server
        if self._inference == "vllm":
            if _rank() == 0 and model.name not in self._vllm:
                from ..runtime.vllm_runtime import ManagedVllmRuntime, VllmRuntimeConfig

                rt = ManagedVllmRuntime(
                    VllmRuntimeConfig(base_model=model.base_model, served_model_name=model.name, host=host,
                                      port=port, gpus=self._vllm_gpus, api_key=api_key,
                                      max_lora_rank=max(8, self._lora_spec(model).r),
                                      engine_args=self._vllm_engine_args),
                    log_path=os.path.join(self._model_dir(model), "logs", "vllm.log"))
                await rt.start()
                self._vllm[model.name] = rt
                await rt.load_lora(f"{model.name}@{step}", ck)
            _barrier()
        return f"http://{host}:{port}/v1", api_key

    async def _publish_to_vllm(self, model: Any, step: int, path: str) -> None:
        """Hot-load a published checkpoint into the model's vLLM server."""
        rt = self._vllm.get(model.name)
        if rt is not None:
            await rt.load_lora(f"{model.name}@{step}", path)

    # ------------------------------------------------------------------ generation
    def _engine(self, model: Any):
        """Generation engine on the trainer's own model: rollouts sample from
        the live adapter the trainer updates (no weight transfer)."""
        eng = self._engines.get(model.name)
        if eng is None:
            from ..runtime.generate import GenerationEngine

            # the resolved engine arguments (dev.get_model_config) size the engine
            ea = dev.get_model_config(model.base_model, self._model_dir(model),
                                      getattr(model, "_internal_config", None) or {})["engine_args"]
            eng = GenerationEngine(self._get_trainer(model).model, max_len=int(ea.get("max_model_len", 8192)),
                                   max_batch=int(ea.get("max_num_seqs", 256)))
            self._engines[model.name] = eng
        return eng

    def _tokenizer(self, model: Any):
        from ..tokenizer import get_tokenizer

        return get_tokenizer(model.base_model)

    def _resolve_adapter(self, model: Any, name: str) -> str | None:
        """Served model name -> engine adapter: the base model, a saved step
        ``{name}@{step}`` other than the current one (loaded on first use), or
        the live policy (``None``)."""
        if name == model.base_model:
            return "base"
        if "@" in name:
            _, step = name.rsplit("@", 1)
            d = self._model_dir(model)
            if step.isdigit() and int(step) != get_step_from_dir(d):
                eng = self._engine(model)
                if name not in eng.adapters:
                    eng.add_adapter(name, get_step_checkpoint_dir(d, int(step)))
                return name
        return None

    async def create_chat_completion(self, model: Any, messages: list[dict[str, Any]], **kwargs: Any) -> dict[str, Any]:
        """One chat completion from the in-process engine, without HTTP
        (the MLX fork's ``MLXBackend.create_chat_completion``); the response is
        the OpenAI JSON the rollout server returns, token ids included."""
        from .inference import RolloutServer

        server = self._servers.get(model.name)
        if server is None:
            server = RolloutServer(self._engine(model), self._tokenizer(model), served_name=model.name,
                                   resolve_adapter=lambda name: self._resolve_adapter(model, name))
            import threading

            server._worker = threading.Thread(target=server._work, name="rollout-engine", daemon=True)
            server._worker.start()
            self._servers[f"{model.name}#inproc"] = server
        body = {"model": kwargs.pop("model", model.name), "messages": messages, **kwargs}
        return await server.chat_completions(body)

    # ------------------------------------------------------------------
    def _pack(
        self,
        results: list[TokenizedResult],
        packed_sequence_length: int | None,
        advantage_balance: float,
        model: Any = None,
    ) -> dict[str, Any]:
        if packed_sequence_length is None:
            from ..preprocessing.prefix_tree import _plan_segments

            # one prompt group per row at least: the row length is the largest
            # prefix-tree-packed group, rounded up to 128
            by_prompt: dict[int, list[TokenizedResult]] = {}
            for r in results:
                by_prompt.setdefault(r.prompt_id, []).append(r)
            longest = 0
            for rs in by_prompt.values():
                segs = _plan_segments([r.token_ids for r in rs], 1 << 30,
                                      [max(0, min(r.prompt_length, len(r.token_ids))) for r in rs])
                longest = max(longest, sum(s.end - s.start for s in segs))
            packed_sequence_length = max(128, (longest + 127) // 128 * 128)
        # with several data-parallel ranks each fills only the rows it trains
        rows_needed = None
        tr = self._get_trainer(model) if model is not None else None
        if tr is not None and tr.world > 1:
            rows_needed = tr.rows_needed
        return packed_tensors_from_tokenized_results(
            results, packed_sequence_length, advantage_balance=advantage_balance,
            rng=random.Random(self._seed + 7), rows_needed=rows_needed,
        )

    async def train(
        self,
        model: Any,
        trajectory_groups: Iterable[TrajectoryGroup],
        *,
        learning_rate: float = 5e-6,
        loss_fn: Literal["cispo", "ppo"] = "cispo",
        loss_fn_config: dict | None = None,
        normalize_advantages: bool = True,
        adam_params: object | None = None,
        kl_penalty_coef: float = 0.0,
        kl_penalty_reference_step: int | None = None,
        kl_ref_adapter_path: str | None = None,
        kl_penalty_source: Literal["current_learner", "sample"] = "current_learner",
        epsilon: float | None = None,
        epsilon_high: float | None = None,
        advantage_balance: float = 0.0,
        scale_rewards: bool = True,
        importance_sampling_level: Literal["token", "sequence", "average", "geometric_average"] = "token",
        max_negative_advantage_importance_sampling_weight: float | None = None,
        mask_prob_ratio: bool = False,
        kimi_k2_tau: float | None = None,
        precalculate_logprobs: bool = False,
        allow_training_without_logprobs: bool = False,
        plot_tensors: bool = False,
        truncated_importance_sampling: float | None = None,
        scale_learning_rate_by_reward_std_dev: bool = False,
        logprob_calculation_chunk_size: int = 4096,
        packed_sequence_length: int | None = None,
        grad_accumulation_sequences: int | None = None,
        num_trajectories_learning_rate_multiplier_power: float = 0.0,
        save_checkpoint: bool = True,
        verbose: bool = False,
    ) -> LocalTrainResult:
        if loss_fn not in ("cispo", "ppo"):
            raise ValueError("LocalBackend supports loss_fn='cispo' or 'ppo'")
        if loss_fn_config is not None or adam_params is not None:
            raise ValueError("LocalBackend requires loss_fn_config=None and adam_params=None")
        if not normalize_advantages:
            scale_rewards = False
        started = time.monotonic()
        groups = list(trajectory_groups)
        d = self._model_dir(model)
        if kl_ref_adapter_path is None and kl_penalty_reference_step is not None:
            kl_ref_adapter_path = get_step_checkpoint_dir(d, kl_penalty_reference_step)
        config, dev_config = build_rl_train_configs(
            learning_rate=learning_rate, advantage_balance=advantage_balance, scale_rewards=scale_rewards,
            importance_sampling_level=importance_sampling_level, mask_prob_ratio=mask_prob_ratio,
            ppo=loss_fn == "ppo", precalculate_logprobs=precalculate_logprobs, epsilon=epsilon,
            epsilon_high=epsilon_high,
            max_negative_advantage_importance_sampling_weight=max_negative_advantage_importance_sampling_weight,
            kimi_k2_tau=kimi_k2_tau, kl_penalty_coef=kl_penalty_coef, kl_penalty_source=kl_penalty_source,
            allow_training_without_logprobs=allow_training_without_logprobs,
            truncated_importance_sampling=truncated_importance_sampling,
            scale_learning_rate_by_reward_std_dev=scale_learning_rate_by_reward_std_dev,
            logprob_calculation_chunk_size=logprob_calculation_chunk_size,
            packed_sequence_length=packed_sequence_length,
            num_trajectories_learning_rate_multiplier_power=num_trajectories_learning_rate_multiplier_power,
            kl_ref_adapter_path=kl_ref_adapter_path,
        )
        # adapters are published synchronously; only the optimizer state of
        # the previous step may still be in flight, and nothing here reads it
        step = get_step_from_dir(d)
        results = list(
            tokenize_trajectory_groups(
                None, groups, allow_training_without_logprobs, scale_rewards,
                rng=random.Random(self._seed + step),
            )
        )
        lr = learning_rate
        if num_trajectories_learning_rate_multiplier_power:
            n_traj = len({id(r.trajectory) for r in results})
            lr *= max(n_traj, 1) ** num_trajectories_learning_rate_multiplier_power
        if scale_learning_rate_by_reward_std_dev:
            rewards = [t.reward for g in groups for t in g]
            if rewards:
                m = sum(rewards) / len(rewards)
                lr *= (sum((r - m) ** 2 for r in rewards) / len(rewards)) ** 0.5
        base_metrics: dict[str, float] = {}
        if not results:
            # nothing trainable: advance the step with an unchanged adapter
            new_step = step + 1
            ck = get_step_checkpoint_dir(d, new_step)
            if save_checkpoint:
                self._flush()  # the copy includes the previous optimizer state (every rank's shard)
                _barrier()
            if save_checkpoint and _rank() == 0:
                prev = get_step_checkpoint_dir(d, step)
                if os.path.exists(ck):
                    shutil.rmtree(ck)
                if os.path.exists(prev):
                    shutil.copytree(prev, ck)
                else:
                    tr = self._get_trainer(model)
                    save_adapter(ck, tr.store, model.base_model, tr.model.lora_spec, tr.optim.state_dict())
            _barrier()
            base_metrics.update({"data/step_num_groups_trainable": 0.0, "data/step_trainer_tokens": 0.0})
            return LocalTrainResult(step=new_step, metrics=base_metrics, checkpoint_path=ck if save_checkpoint else None)

        packed = self._pack(results, packed_sequence_length, advantage_balance, model)
        t_prepared = time.monotonic()
        if plot_tensors and _rank() == 0:
            packed_tensors_to_dir(packed, os.path.join(d, "tensors"))
        new_step = step + 1
        ck = get_step_checkpoint_dir(d, new_step)
        metrics = await self._train_packed(
            model, packed, lr, dev_config, kl_ref_adapter_path if kl_penalty_coef > 0 else None,
            logprob_calculation_chunk_size, ck if save_checkpoint else None, grad_accumulation_sequences,
        )
        metrics["time/step_trainer_s"] = time.monotonic() - started
        metrics["time/step_prepare_s"] = t_prepared - started
        metrics.setdefault("data/step_num_gradient_steps", 1.0)
        builder = self._metrics.setdefault(model.name, MetricsBuilder())
        metrics = builder.update(metrics)
        metrics = aggregate_rl_training_metrics([metrics], groups)
        if save_checkpoint and _rank() == 0:
            await self._publish_to_vllm(model, new_step, ck)
        return LocalTrainResult(step=new_step, metrics=metrics, checkpoint_path=ck if save_checkpoint else None)

    async def _train_packed(
        self,
        model: Any,
        packed: dict[str, Any],
        lr: float,
        dev_config: dict[str, Any],
        kl_ref_adapter_path: str | None,
        logprob_chunk: int,
        out_dir: str | None,
        grad_accumulation_sequences: int | None = None,
    ) -> dict[str, float]:
        """GRPO optimizer step(s) on packed rows (one, or one per
        ``grad_accumulation_sequences`` rows); publishes the adapter to ``out_dir``."""
        tr = self._get_trainer(model)
        # reference adapter for the KL penalty (default: the frozen base)
        ref_state = None
        if kl_ref_adapter_path:
            from safetensors.torch import load_file

            ref_state = load_file(os.path.join(kl_ref_adapter_path, "adapter_model.safetensors"))
        tr.set_reference_adapter(ref_state)
        tr.logprob_chunk = logprob_chunk
        server = self._servers.get(model.name) or self._servers.get(f"{model.name}#inproc")
        lock = server.engine_lock if server is not None else contextlib.nullcontext()
        n_rows = int(packed["tokens"].shape[0])
        with lock:  # colocated rollouts: no generation batch during the update
            if grad_accumulation_sequences is not None and grad_accumulation_sequences < n_rows:
                steps = [m.to_host() for m in tr.train_steps(packed, lr, dev_config, grad_accumulation_sequences)]
                metrics = {k: sum(m[k] for m in steps) / len(steps) for k in steps[0]}
                for k in ("data/step_trainer_tokens", "data/step_packed_tokens"):
                    metrics[k] = sum(m[k] for m in steps)
                metrics["data/step_num_gradient_steps"] = float(len(steps))
                self.last_h2d_bytes = 0
            else:
                t0 = time.monotonic()
                mbs = tr.stage(packed)
                self.last_h2d_bytes = sum(mb.h2d_bytes for mb in mbs)
                t1 = time.monotonic()
                metrics = tr.train_step(packed, lr, dev_config, micro_batches=mbs).to_host()
                metrics["time/step_stage_s"] = t1 - t0
                metrics["time/step_compute_s"] = time.monotonic() - t1
        self.last_d2h_bytes = 5 * 4
        t2 = time.monotonic()
        shard = tr.optimizer_shard() if out_dir is not None else None
        if out_dir is not None:
            # sharded optimizer: only the master weights are gathered (the
            # adapter rank 0 publishes); every rank writes its own moments
            tr.prepare_checkpoint(moments=shard is None)
            if _rank() == 0:
                self._writer.submit(out_dir, tr.store, model.base_model, tr.model.lora_spec,
                                    with_optimizer=shard is None)
        _barrier()  # the adapter directory is published
        if shard is not None:
            self._writer.submit_optimizer_shard(out_dir, tr.store, *shard)
        metrics["time/step_checkpoint_s"] = time.monotonic() - t2
        return metrics

    # ------------------------------------------------------------------
    async def _train_sft(
        self,
        model: Any,
        trajectories: Iterable[Trajectory],
        config: TrainSFTConfig,
        dev_config: dev.TrainSFTConfig,
        verbose: bool = False,
    ) -> AsyncIterator[dict[str, float]]:
        """Supervised fine-tuning on trajectories whose assistant turns carry
        token ids (or on ``input_ids``/``labels`` produced by a tokenizer)."""
        from ..runtime.sft import sft_batches_from_trajectories

        tr = self._get_trainer(model)
        trajs = list(trajectories)
        bs = config.batch_size if isinstance(config.batch_size, int) else max(2, 2 * tr.world)
        lrs = config.learning_rate
        batches = sft_batches_from_trajectories(trajs, bs)
        d = self._model_dir(model)
        for i, batch in enumerate(batches):
            lr = lrs[i] if isinstance(lrs, list) else lrs
            m = tr.sft_step(batch, lr)
            yield m
        self._flush()
        step = get_step_from_dir(d) + 1
        tr.prepare_checkpoint()  # collective: every shard's master and moments on every rank
        if _rank() == 0:
            save_adapter(get_step_checkpoint_dir(d, step), tr.store, model.base_model, tr.model.lora_spec,
                         tr.optim.state_dict())
        _barrier()

    # ------------------------------------------------------------------ S3
    async def _experimental_push_to_s3(self, model: Any, *, s3_bucket: str | None = None, prefix: str | None = None,
                                       verbose: bool = False, delete: bool = False) -> None:
        """Upload the model directory (checkpoints, logs, trajectories) to S3
        (reference ``local/backend.py:1520``; layout in ``utils/s3.py``)."""
        from ..utils.s3 import push_model_to_s3

        self._flush()
        await push_model_to_s3(model.name, model.project, s3_bucket, prefix, verbose, delete, self._path)

    async def _experimental_pull_from_s3(self, model: Any, *, s3_bucket: str | None = None, prefix: str | None = None,
                                         verbose: bool = False, delete: bool = False,
                                         only_step: int | str | None = None, exclude: list | None = None) -> None:
        """Download the model directory, or one step (``only_step``: a step or
        ``"latest"``), from S3 into this backend's storage."""
        from ..utils.s3 import get_latest_checkpoint_step_from_s3, pull_model_from_s3

        step = None
        if only_step == "latest":
            step = await get_latest_checkpoint_step_from_s3(model.name, model.project, s3_bucket, prefix)
            if step is None:
                return
        elif only_step is not None:
            step = int(only_step)
        await pull_model_from_s3(model.name, model.project, step, s3_bucket, prefix, verbose, delete, self._path,
                                 exclude)

    async def _experimental_pull_model_checkpoint(self, model: Any, *, step: int | str | None = None,
                                                  local_path: str | None = None, s3_bucket: str | None = None,
                                                  prefix: str | None = None, verbose: bool = False) -> str:
        """Path of a local copy of a checkpoint: the local one when present
        (for ``"latest"`` the newer of local and S3, local on a tie), else
        pulled from S3; copied to ``local_path`` when given."""
        from ..utils.output_dirs import list_checkpoint_steps
        from ..utils.s3 import get_latest_checkpoint_step_from_s3, pull_model_from_s3

        d = self._model_dir(model)
        local_steps = list_checkpoint_steps(d) if os.path.isdir(d) else []
        if step in (None, "latest"):
            s3_step = (await get_latest_checkpoint_step_from_s3(model.name, model.project, s3_bucket, prefix)
                       if s3_bucket else None)
            cands = [x for x in (max(local_steps) if local_steps else None, s3_step) if x is not None]
            if not cands:
                raise FileNotFoundError(f"no checkpoint of {model.name} locally or in S3")
            step = max(cands)
        step = int(step)
        ck = get_step_checkpoint_dir(d, step)
        if not os.path.isdir(ck):
            if not s3_bucket:
                raise FileNotFoundError(ck)
            ck = await pull_model_from_s3(model.name, model.project, step, s3_bucket, prefix, verbose, False,
                                          self._path)
        if local_path is not None:
            if os.path.exists(local_path):
                shutil.rmtree(local_path)
            shutil.copytree(ck, local_path)
            return local_path
        return ck

    # ------------------------------------------------------------------
    async def _experimental_fork_checkpoint(self, model: Any, from_model: str, from_project: str | None = None,
                                            not_after_step: int | None = None) -> int:
        """Copy another model's latest (or bounded) checkpoint into this model
        as its current step (reference ``local/backend.py:1540``)."""
        from ..utils.output_dirs import get_output_dir_from_model_properties, list_checkpoint_steps

        self._flush()
        src = get_output_dir_from_model_properties(from_project or model.project, from_model, self._path)
        steps = [s for s in list_checkpoint_steps(src) if not_after_step is None or s <= not_after_step]
        if not steps:
            raise FileNotFoundError(f"no checkpoints under {src}")
        s = max(steps)
        dst = get_step_checkpoint_dir(self._model_dir(model), s)
        if _rank() == 0:
            if os.path.exists(dst):
                shutil.rmtree(dst)
            shutil.copytree(get_step_checkpoint_dir(src, s), dst)
        _barrier()
        tr = self._get_trainer(model)
        opt = load_adapter(dst, tr.store)
        if opt is not None:
            tr.optim.load_state_dict(opt)
        return s
