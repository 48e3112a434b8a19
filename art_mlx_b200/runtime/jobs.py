"""Job protocol between a backend (client) and its persistent worker group.

Same shape as the reference's trainer job protocol
(``src/art/megatron/runtime/jobs.py:20-88``, ``client.py:12-67``): the client
writes one JSON job file, the workers run it collectively, rank 0 appends one
JSON line per result to the job's log file and finally the line
``all done``; the client streams that log and deletes both files.

Differences, chosen for one host with one process per GPU:

* job files are numbered (``{seq:08d}.json``) and written atomically
  (temporary file + rename); every rank polls the directory itself and runs
  jobs in sequence order, so idle workers issue no collective (no
  process-group timeout while waiting for work);
* a failed job writes ``{"error": ...}`` before ``all done`` and the client
  raises; a worker group that died is detected from its launcher's exit code;
* every rank refreshes a heartbeat file once a second from a side thread;
  the client reports a worker whose heartbeat is older than its limit.
"""

from __future__ import annotations

import asyncio
import json
import os
import time
from typing import Annotated, Any, AsyncIterator, Literal, Union

from pydantic import BaseModel, Field, TypeAdapter

DONE = "all done"


class TrainJob(BaseModel):
    kind: Literal["train"] = "train"
    packed_dir: str  # packed tensors on disk (preprocessing.pack.packed_tensors_to_dir)
    num_sequences: int
    sequence_length: int
    checkpoint_dir: str  # adapter (+ optimizer state) the step starts from
    output_dir: str | None  # where to publish the new adapter (None: keep in memory)
    base_model: str
    learning_rate: float
    config: dict[str, Any] = Field(default_factory=dict)  # loss knobs (dev.TrainConfig)
    kl_ref_adapter_path: str | None = None
    logprob_chunk: int = 4096
    grad_accumulation_sequences: int | None = None
    log_path: str


class SFTJob(BaseModel):
    kind: Literal["sft"] = "sft"
    batches_path: str  # JSON: list of batches, each a list of [input_ids, labels]
    checkpoint_dir: str
    output_dir: str | None
    base_model: str
    learning_rates: list[float]
    log_path: str


class LoadJob(BaseModel):
    """Load an adapter (and optimizer state) into the workers' trainer."""

    kind: Literal["load"] = "load"
    checkpoint_dir: str
    log_path: str


class ShutdownJob(BaseModel):
    kind: Literal["shutdown"] = "shutdown"
    log_path: str


Job = Annotated[Union[TrainJob, SFTJob, LoadJob, ShutdownJob], Field(discriminator="kind")]
_ADAPTER = TypeAdapter(Job)


def dump_job(job: Job) -> str:
    return _ADAPTER.dump_json(job).decode()


def load_job(raw: str | bytes) -> Job:
    return _ADAPTER.validate_json(raw)


def next_job_path(jobs_dir: str) -> str:
    os.makedirs(jobs_dir, exist_ok=True)
    seqs = [int(f[:-5]) for f in os.listdir(jobs_dir) if f.endswith(".json") and f[:-5].isdigit()]
    counter = os.path.join(jobs_dir, "last_seq")
    last = int(open(counter).read() or 0) if os.path.exists(counter) else 0
    seq = max([last, *seqs]) + 1
    with open(counter, "w") as f:
        f.write(str(seq))
    return os.path.join(jobs_dir, f"{seq:08d}.json")


def write_job(job: Job, job_path: str) -> None:
    tmp = job_path + ".tmp"
    with open(tmp, "w", encoding="utf-8") as f:
        f.write(dump_job(job))
    os.replace(tmp, job_path)


def pending_jobs(jobs_dir: str, after: int) -> list[tuple[int, str]]:
    """``(seq, path)`` of the job files with ``seq > after``, in order."""
    if not os.path.isdir(jobs_dir):
        return []
    out = []
    for f in os.listdir(jobs_dir):
        if f.endswith(".json") and f[:-5].isdigit() and int(f[:-5]) > after:
            out.append((int(f[:-5]), os.path.join(jobs_dir, f)))
    return sorted(out)


def append_log(log_path: str, record: dict[str, Any] | str) -> None:
    line = record if isinstance(record, str) else json.dumps(record)
    with open(log_path, "a", encoding="utf-8") as f:
        f.write(line + "\n")
        f.flush()
        os.fsync(f.fileno())


def heartbeat_path(jobs_dir: str, rank: int) -> str:
    return os.path.join(jobs_dir, f"heartbeat-{rank}")


def stale_heartbeats(jobs_dir: str, world: int, limit_s: float) -> list[int]:
    now = time.time()
    out = []
    for r in range(world):
        p = heartbeat_path(jobs_dir, r)
        if not os.path.exists(p) or now - os.path.getmtime(p) > limit_s:
            out.append(r)
    return out


async def stream_job(
    job: Job,
    job_path: str,
    *,
    process: Any | None = None,
    jobs_dir: str | None = None,
    world: int = 0,
    heartbeat_limit_s: float | None = None,
    poll_interval: float = 0.05,
) -> AsyncIterator[dict[str, Any]]:
    """Yield the job's result records until ``all done``; raise if the job
    failed, the worker group exited or a rank stopped beating."""
    n = 0
    try:
        while True:
            await asyncio.sleep(poll_interval)
            lines: list[str] = []
            if os.path.exists(job.log_path):
                with open(job.log_path, encoding="utf-8") as f:
                    lines = f.readlines()[n:]
            for line in lines:
                n += 1
                line = line.strip()
                if not line:
                    continue
                if line == DONE:
                    return
                rec = json.loads(line)
                if "error" in rec:
                    raise RuntimeError(f"worker job failed: {rec['error']}")
                yield rec
            if process is not None and process.poll() is not None:
                raise RuntimeError(f"worker group exited with code {process.returncode}")
            if heartbeat_limit_s is not None and jobs_dir is not None and world:
                stale = stale_heartbeats(jobs_dir, world, heartbeat_limit_s)
                if stale:
                    raise RuntimeError(f"worker ranks {stale} stopped beating for > {heartbeat_limit_s}s")
    finally:
        for p in (job_path, job.log_path):
            if os.path.exists(p):
                os.remove(p)
