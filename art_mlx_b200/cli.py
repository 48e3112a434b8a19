"""Command line: ``python -m art_mlx_b200 <command>`` (or the ``art-b200``
console script).

Commands (the reference's ``src/art/cli.py:58-330`` surface):

* ``init [PATH]``      - a project skeleton: ``.art/`` and a runnable
  ``train.py`` (synthetic rollouts, LocalBackend, a few GRPO steps);
* ``migrate PATH``     - convert trajectory logs written as JSON lines (one
  trajectory group per line) into the parquet layout
  (``trajectories/{split}/{step:04d}.parquet``); PATH is a ``.jsonl`` file, a
  trajectories directory, a model directory or a project directory;
* ``run``              - serve a ``LocalBackend`` over HTTP for
  :class:`art_mlx_b200.backends.remote.RemoteBackend` clients (register,
  step, prepare, train, delete checkpoints, close, health check);
* ``help``             - this overview.
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import sys
from dataclasses import dataclass, field
from pathlib import Path

_TRAIN_TEMPLATE = '''"""GRPO on synthetic rollouts: replace `rollout` with your agent."""

import asyncio

import art_mlx_b200 as art
from art_mlx_b200.preprocessing.synthetic import synthetic_groups


async def main() -> None:
    backend = art.LocalBackend(path=".art")
    model = art.TrainableModel(name="my-agent", project="my-project", base_model="tiny-qwen3")
    await model.register(backend)
    for step in range(3):
        groups = synthetic_groups(num_groups=4, rollouts_per_group=8, prompt_len=64, completion_len=32,
                                  vocab_size=1024, seed=step)
        result = await backend.train(model, groups, learning_rate=1e-5)
        print(result.step, result.metrics["loss/train"])


if __name__ == "__main__":
    asyncio.run(main())
'''


def cmd_init(path: str) -> int:
    root = Path(path)
    root.mkdir(parents=True, exist_ok=True)
    (root / ".art").mkdir(exist_ok=True)
    target = root / "train.py"
    if not target.exists():
        target.write_text(_TRAIN_TEMPLATE)
    print(f"initialised {root.resolve()} (.art/, train.py)")
    return 0


@dataclass
class MigrationResult:
    files_migrated: int = 0
    files_skipped: int = 0
    bytes_before: int = 0
    bytes_after: int = 0
    errors: list[str] = field(default_factory=list)

    def add(self, other: "MigrationResult") -> None:
        self.files_migrated += other.files_migrated
        self.files_skipped += other.files_skipped
        self.bytes_before += other.bytes_before
        self.bytes_after += other.bytes_after
        self.errors += other.errors


def _message_of(item: dict) -> dict:
    if "finish_reason" in item and isinstance(item.get("message"), dict):  # a serialized Choice
        m = dict(item["message"])
        m["trainable"] = True
        return m
    return item


def migrate_jsonl_file(path: Path, keep_original: bool = False, dry_run: bool = False) -> MigrationResult:
    """One ``.jsonl`` file (a trajectory group per line) -> ``.parquet`` beside it."""
    from .trajectories import Trajectory, TrajectoryGroup
    from .utils.trajectory_logging import write_trajectory_groups_parquet

    res = MigrationResult()
    if path.suffix != ".jsonl":
        res.files_skipped = 1
        return res
    res.bytes_before = path.stat().st_size
    if dry_run:
        res.files_migrated = 1
        return res
    try:
        groups = []
        for line in path.read_text().splitlines():
            if not line.strip():
                continue
            g = json.loads(line)
            trajs = []
            for t in g.get("trajectories", []):
                trajs.append(Trajectory(
                    messages_and_choices=[_message_of(m) for m in t.get("messages_and_choices", [])],
                    reward=float(t.get("reward", 0.0)), metrics=t.get("metrics") or {},
                    metadata=t.get("metadata") or {}, logs=t.get("logs") or [],
                ))
            groups.append(TrajectoryGroup(trajs))
        out = path.with_suffix(".parquet")
        write_trajectory_groups_parquet(groups, str(out))
        res.bytes_after = out.stat().st_size
        res.files_migrated = 1
        if not keep_original:
            path.unlink()
    except Exception as exc:  # reported, the other files continue
        res.errors.append(f"{path}: {type(exc).__name__}: {exc}")
    return res


def migrate(path: str, dry_run: bool = False, keep_jsonl: bool = False, verbose: bool = False) -> MigrationResult:
    p = Path(path)
    total = MigrationResult()
    if not p.exists():
        total.errors.append(f"path does not exist: {p}")
        return total
    files = [p] if p.is_file() else sorted(p.rglob("*.jsonl"))
    for f in files:
        if f.name == "history.jsonl" or f.parent.name == "jobs":
            continue  # metric history and job logs stay JSON lines
        r = migrate_jsonl_file(f, keep_original=keep_jsonl, dry_run=dry_run)
        if verbose and r.files_migrated:
            print(f"  {f}")
        total.add(r)
    return total


def cmd_migrate(args: argparse.Namespace) -> int:
    r = migrate(args.path, args.dry_run, args.keep_jsonl, args.verbose)
    verb = "would migrate" if args.dry_run else "migrated"
    print(f"{verb} {r.files_migrated} files ({r.bytes_before} -> {r.bytes_after} bytes), skipped {r.files_skipped}")
    for e in r.errors[:10]:
        print(f"  error: {e}", file=sys.stderr)
    return 1 if r.errors else 0


def build_server_app(backend):
    """FastAPI app exposing a backend's methods to RemoteBackend clients."""
    from fastapi import Body, FastAPI

    from .trajectories import TrajectoryGroup
    from .types import TrainSFTConfig
    from .model import TrainableModel

    app = FastAPI()

    def groups_of(items: list[dict]) -> list[TrajectoryGroup]:
        from openai.types.chat.chat_completion import Choice

        from .trajectories import Trajectory

        out = []
        for g in items:
            trajs = []
            for t in g.get("trajectories", []):
                t = dict(t)
                t["messages_and_choices"] = [
                    Choice.model_validate(m) if isinstance(m, dict) and "finish_reason" in m else m
                    for m in t.get("messages_and_choices", [])
                ]
                trajs.append(Trajectory(**t))
            out.append(TrajectoryGroup(trajs, metadata=g.get("metadata"), metrics=g.get("metrics"),
                                       logs=g.get("logs")))
        return out

    def model_of(d: dict) -> TrainableModel:
        internal = d.pop("_internal_config", None)
        return TrainableModel(_internal_config=internal, **d)

    @app.get("/healthcheck")
    async def health():
        return {"status": "ok"}

    @app.post("/register")
    async def register(model: dict = Body(..., embed=True)):
        await backend.register(model_of(model))
        return {}

    @app.post("/_get_step")
    async def get_step(model: dict = Body(..., embed=True)):
        return await backend._get_step(model_of(model))

    @app.post("/_prepare_backend_for_training")
    async def prepare(model: dict = Body(...), config: dict | None = Body(None)):
        m = model_of(model)
        await backend.register(m)
        return list(await backend._prepare_backend_for_training(m, config))

    @app.post("/_delete_checkpoint_files")
    async def delete(model: dict = Body(...), steps_to_keep: list[int] = Body(...)):
        await backend._delete_checkpoint_files(model_of(model), steps_to_keep)
        return {}

    @app.post("/train")
    async def train(model: dict = Body(...), trajectory_groups: list[dict] = Body(...), kwargs: dict = Body({})):
        m = model_of(model)
        groups = groups_of(trajectory_groups)
        res = await backend.train(m, groups, **kwargs)
        return {"step": res.step, "metrics": res.metrics, "checkpoint_path": res.checkpoint_path}

    @app.post("/_train_sft")
    async def train_sft(model: dict = Body(...), trajectories: list[dict] = Body(...), config: dict = Body({})):
        from .trajectories import Trajectory

        m = model_of(model)
        out = []
        async for row in backend._train_sft(m, [Trajectory.model_validate(t) for t in trajectories],
                                            TrainSFTConfig(**config), {}):
            out.append(row)
        return out

    @app.post("/close")
    async def close():
        await backend.close()
        return {}

    return app


def cmd_run(args: argparse.Namespace) -> int:
    import uvicorn

    from .backends.local import LocalBackend

    with socket.socket() as s:
        if s.connect_ex(("127.0.0.1", args.port)) == 0:
            print(f"port {args.port} is already in use (is the server already running?)")
            return 1
    backend = LocalBackend(path=args.path)
    uvicorn.run(build_server_app(backend), host=args.host, port=args.port, log_level="warning")
    return 0


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="art-b200", description="B200-native GRPO trainer for LLM agents")
    sub = ap.add_subparsers(dest="cmd")
    p = sub.add_parser("init", help="create a project skeleton")
    p.add_argument("path", nargs="?", default=".")
    p = sub.add_parser("migrate", help="convert JSON-lines trajectory logs to parquet")
    p.add_argument("path")
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("--keep-jsonl", action="store_true")
    p.add_argument("--verbose", "-v", action="store_true")
    p = sub.add_parser("run", help="serve a LocalBackend over HTTP")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=7999)
    p.add_argument("--path", default=os.path.join(os.getcwd(), ".art"))
    sub.add_parser("help", help="show this overview")
    args = ap.parse_args(argv)
    if args.cmd == "init":
        return cmd_init(args.path)
    if args.cmd == "migrate":
        return cmd_migrate(args)
    if args.cmd == "run":
        return cmd_run(args)
    ap.print_help()
    print(__doc__)
    return 0


if __name__ == "__main__":
    sys.exit(main())
