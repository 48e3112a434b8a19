"""Supervised fine-tuning helpers: learning-rate schedules, chunked dataset
iteration and streaming from JSONL files.

Interfaces and schedule values follow the reference's ``src/art/utils/sft.py``
(``create_lr_schedule``, ``create_sft_dataset_iterator``, ``iterate_file``,
``get_file_row_count``, ``train_sft_from_file``) so a schedule or a resumed
run lines up step for step with one started there:

* warm-up: ``warmup_steps`` linear steps from ``min_lr`` towards ``peak_lr``
  (step ``s`` gets fraction ``(s+1)/warmup_steps``);
* decay: progress ``(s - warmup) / (decay_steps - 1)`` from 0 to 1, cosine
  (``min + (peak-min)(1+cos(pi p))/2``), linear (``peak - (peak-min) p``) or
  constant;
* datasets are consumed in chunks of ``chunk_size`` batches, each chunk one
  ``train_sft`` call with its slice of the global schedule; epoch ``e``
  shuffles with ``random.Random(seed + e)``.
"""

from __future__ import annotations

import itertools
import json
import math
import random
from typing import TYPE_CHECKING, Any, Generator, Iterator, Literal, NamedTuple

if TYPE_CHECKING:  # pragma: no cover
    from ..trajectories import Trajectory

Schedule = Literal["cosine", "linear", "constant"]


class SFTChunk(NamedTuple):
    trajectories: list
    config: Any  # TrainSFTConfig
    step: int
    epoch: int
    epoch_step: int


def resolve_sft_batch_size(*, batch_size: int | Literal["auto"], default_batch_size: int) -> int:
    return default_batch_size if batch_size == "auto" else int(batch_size)


def create_lr_schedule(total_steps: int, peak_lr: float, method: Schedule = "linear", warmup_steps: int = 0,
                       min_lr: float = 0.0) -> list[float]:
    if total_steps <= 0:
        return []
    if method not in ("cosine", "linear", "constant"):
        raise ValueError(f"Unknown method: {method}. Choose from: cosine, linear, constant")
    decay = total_steps - warmup_steps
    span = peak_lr - min_lr
    out: list[float] = []
    for s in range(total_steps):
        if s < warmup_steps:
            out.append(min_lr + span * (s + 1) / warmup_steps)
            continue
        p = (s - warmup_steps) / (decay - 1) if decay > 1 else 0.0
        if method == "cosine":
            out.append(min_lr + span * 0.5 * (1.0 + math.cos(math.pi * p)))
        elif method == "linear":
            out.append(peak_lr - span * p)
        else:
            out.append(peak_lr)
    return out


def create_sft_dataset_iterator(
    trajectories: list,
    chunk_size: int = 10,
    epochs: int = 1,
    batch_size: int = 2,
    peak_lr: float = 2e-4,
    schedule_type: Schedule = "linear",
    warmup_ratio: float = 0.1,
    shuffle: bool = True,
    seed: int = 42,
    initial_step: int = 0,
    show_progress: bool = True,
) -> Generator[SFTChunk, None, None]:
    """Chunks of ``chunk_size`` batches, each with its slice of one schedule
    computed over all epochs; ``initial_step`` (in batches) skips whole chunks."""
    from ..types import TrainSFTConfig

    if chunk_size < 1:
        raise ValueError(f"chunk_size must be >= 1, got {chunk_size}")
    n = len(trajectories)
    if n == 0:
        return
    per_epoch = math.ceil(n / batch_size)
    total = per_epoch * epochs
    lrs = create_lr_schedule(total, peak_lr, schedule_type, int(total * warmup_ratio))
    items = batch_size * chunk_size
    chunks_per_epoch = math.ceil(n / items)
    first_chunk = initial_step // chunk_size
    bar = None
    if show_progress:
        try:
            from tqdm.auto import tqdm

            bar = tqdm(initial=initial_step, total=total, desc="SFT Training", unit="step")
        except Exception:  # pragma: no cover
            bar = None
    try:
        for epoch in range(epochs):
            order = list(trajectories)
            if shuffle:
                random.Random(seed + epoch).shuffle(order)
            for c in range(chunks_per_epoch):
                if epoch * chunks_per_epoch + c < first_chunk:
                    continue
                part = order[c * items : min((c + 1) * items, n)]
                nb = math.ceil(len(part) / batch_size)
                epoch_step = (c * items) // batch_size
                step = epoch * per_epoch + epoch_step
                yield SFTChunk(part, TrainSFTConfig(learning_rate=lrs[step : step + nb], batch_size=batch_size),
                               step, epoch, epoch_step)
                if bar is not None:
                    bar.update(nb)
    finally:
        if bar is not None:
            bar.close()


def _trajectory_from_line(line: str) -> "Trajectory":
    from ..trajectories import Trajectory

    d = json.loads(line)
    return Trajectory(messages_and_choices=d.get("messages", []), tools=d.get("tools"))


def get_file_row_count(file_path: str) -> int:
    """Non-empty lines of a JSONL file."""
    if not file_path.endswith(".jsonl"):
        raise ValueError(f"Only JSONL files are supported. Got: {file_path}")
    with open(file_path, "rb") as f:
        return sum(1 for line in f if line.strip())


def iterate_file(file_path: str, epochs: int = 1, shuffle_buffer_size: int = 10000, seed: int = 42,
                 initial_skip: int = 0) -> Iterator["Trajectory"]:
    """Stream trajectories from a JSONL file with a bounded shuffle buffer:
    once the buffer holds ``shuffle_buffer_size`` items a random one is
    emitted per line read; the rest is shuffled and emitted at the end of the
    epoch.  The first ``initial_skip`` emitted items (over all epochs) are
    dropped (resume)."""
    if not file_path.endswith(".jsonl"):
        raise ValueError(f"Only JSONL files are supported. Got: {file_path}")
    to_skip = initial_skip

    def emit(t):
        nonlocal to_skip
        if to_skip > 0:
            to_skip -= 1
            return None
        return t

    for epoch in range(epochs):
        rng = random.Random(seed + epoch)
        buf: list = []
        with open(file_path) as f:
            for line in f:
                if not line.strip():
                    continue
                buf.append(_trajectory_from_line(line))
                if len(buf) >= shuffle_buffer_size:
                    t = emit(buf.pop(rng.randint(0, len(buf) - 1)))
                    if t is not None:
                        yield t
        rng.shuffle(buf)
        for t in buf:
            t = emit(t)
            if t is not None:
                yield t


async def train_sft_from_file(
    model: Any,
    file_path: str,
    epochs: int = 1,
    batch_size: int = 2,
    peak_lr: float = 2e-4,
    schedule_type: Schedule = "linear",
    warmup_ratio: float = 0.1,
    initial_step: int = 0,
    final_step: int | None = None,
    _config: Any = None,
    verbose: bool = False,
    shuffle_buffer_size: int = 10000,
    log_metrics: bool = True,
) -> None:
    """Supervised fine-tuning of ``model`` on a JSONL file without loading it:
    one schedule over ``ceil(rows * epochs / batch_size)`` batches, sliced to
    ``[initial_step, final_step)``, the stream capped to that many batches."""
    from ..types import TrainSFTConfig

    rows = get_file_row_count(file_path)
    if rows == 0:
        return
    total_items = rows * epochs
    skip = initial_step * batch_size
    if skip >= total_items:
        return
    total = math.ceil(total_items / batch_size)
    if final_step is not None:
        final_step = min(final_step, total)
    lrs = create_lr_schedule(total, peak_lr, schedule_type, int(total * warmup_ratio))[initial_step:final_step]
    if verbose:
        print(f"SFT from {file_path}: {rows} rows, {len(lrs)} batches of {batch_size}, {schedule_type} peak {peak_lr}")
    stream = itertools.islice(iterate_file(file_path, epochs, shuffle_buffer_size, initial_skip=skip),
                              len(lrs) * batch_size)
    # log_metrics: the SFT metrics are always appended to the model's history
    await model.train_sft(stream, TrainSFTConfig(learning_rate=lrs, batch_size=batch_size), _config=_config,
                          verbose=verbose)
