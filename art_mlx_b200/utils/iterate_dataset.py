"""Epoch-wise batching of a scenario list with deterministic shuffling.

Interface of the reference's ``src/art/utils/iterate_dataset.py``: batches of
``groups_per_step`` items, each epoch shuffled with ``random.Random(epoch)``
(so a resumed run sees the same order), global steps below ``initial_step``
skipped, an optional tqdm progress bar.
"""

from __future__ import annotations

import math
import random
from dataclasses import dataclass
from typing import Generator, Generic, List, TypeVar

T = TypeVar("T")


@dataclass
class DatasetBatch(Generic[T]):
    items: List[T]
    step: int  # global step across epochs
    epoch: int
    epoch_step: int


def iterate_dataset(
    dataset: List[T],
    groups_per_step: int = 1,
    num_epochs: int = 1,
    initial_step: int = 0,
    use_tqdm: bool = True,
) -> Generator[DatasetBatch[T], None, None]:
    n = len(dataset)
    if n == 0:
        return
    if groups_per_step < 1:
        raise ValueError("groups_per_step must be >= 1")
    per_epoch = math.ceil(n / groups_per_step)
    bar = None
    if use_tqdm:
        try:
            from tqdm.auto import tqdm

            bar = tqdm(initial=initial_step, total=per_epoch * num_epochs, desc="Iterating dataset", unit="batch")
        except Exception:  # pragma: no cover - tqdm missing
            bar = None
    try:
        for epoch in range(num_epochs):
            order = list(range(n))
            random.Random(epoch).shuffle(order)
            for epoch_step in range(per_epoch):
                step = epoch * per_epoch + epoch_step
                if step < initial_step:
                    continue
                idx = order[epoch_step * groups_per_step : (epoch_step + 1) * groups_per_step]
                yield DatasetBatch(items=[dataset[i] for i in idx], step=step, epoch=epoch, epoch_step=epoch_step)
                if bar is not None:
                    bar.update(1)
    finally:
        if bar is not None:
            bar.close()
