"""Parquet logging of trajectory groups (one file per split and step),
the format of the reference ``src/art/utils/trajectory_logging.py:59-251``:
one row per trajectory with its group index, reward, metrics, metadata and
the chat messages as JSON."""

from __future__ import annotations

import json
import os
from typing import Any

from ..trajectories import Trajectory, TrajectoryGroup


def _row(group_index: int, t: Trajectory) -> dict[str, Any]:
    d = t.for_logging()
    return {
        "group_index": group_index,
        "reward": float(t.reward),
        "metrics": json.dumps(d["metrics"]),
        "metadata": json.dumps(d["metadata"], default=str),
        "messages": json.dumps(d["messages"], default=str),
        "tools": json.dumps(d["tools"], default=str),
        "logs": json.dumps(d["logs"]),
    }


def write_trajectory_groups_parquet(groups: list[TrajectoryGroup], path: str) -> None:
    import pyarrow as pa
    import pyarrow.parquet as pq

    os.makedirs(os.path.dirname(path), exist_ok=True)
    rows = [_row(i, t) for i, g in enumerate(groups) for t in g]
    table = pa.Table.from_pylist(rows) if rows else pa.table({"group_index": pa.array([], pa.int64())})
    pq.write_table(table, path)


def read_trajectory_groups_parquet(path: str) -> list[TrajectoryGroup]:
    import pyarrow.parquet as pq

    table = pq.read_table(path).to_pylist()
    groups: dict[int, list[Trajectory]] = {}
    for r in table:
        msgs = [
            {k: v for k, v in m.items() if k != "trainable"} for m in json.loads(r.get("messages") or "[]")
        ]
        groups.setdefault(int(r["group_index"]), []).append(
            Trajectory(
                messages_and_choices=msgs,
                reward=float(r["reward"]),
                metrics=json.loads(r.get("metrics") or "{}"),
                metadata=json.loads(r.get("metadata") or "{}"),
                logs=json.loads(r.get("logs") or "[]"),
            )
        )
    return [TrajectoryGroup(v) for _, v in sorted(groups.items())]
