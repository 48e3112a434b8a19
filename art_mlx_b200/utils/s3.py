"""Model directories to and from S3 through the AWS CLI.

Same layout and entry points as the reference's ``src/art/utils/s3.py`` and
``s3_checkpoint_utils.py`` so a bucket written by either is readable by the
other: ``s3://{bucket}/{prefix/}{project}/models/{name}`` mirrors the local
model directory, a step lives under ``checkpoints/{step:04d}``, zipped steps
under ``zipped-steps/{step:04d}.zip``; the bucket defaults to
``$BACKUP_BUCKET``.  Transfers run ``aws s3 sync`` (directories) or
``aws s3 cp`` (files) as subprocesses without blocking the event loop.
"""

from __future__ import annotations

import asyncio
import os
import re
import shutil
import tempfile
from asyncio.subprocess import DEVNULL, PIPE
from typing import Literal, Optional

from .limit_concurrency import limit_concurrency
from .output_dirs import get_output_dir_from_model_properties

ExcludableOption = Literal["checkpoints", "logs", "trajectories"]


class S3SyncError(RuntimeError):
    """An ``aws s3`` command exited with a non-zero status."""


def _bucket(s3_bucket: str | None) -> str:
    if s3_bucket:
        return s3_bucket
    b = os.environ.get("BACKUP_BUCKET")
    if not b:
        raise ValueError("no S3 bucket given and BACKUP_BUCKET is not set")
    return b


def build_s3_path(*, model_name: str, project: str, step: int | None = None, s3_bucket: str | None = None,
                  prefix: str | None = None) -> str:
    pre = f"{prefix.strip('/')}/" if prefix else ""
    path = f"s3://{_bucket(s3_bucket)}/{pre}{project}/models/{model_name}"
    return path if step is None else f"{path}/checkpoints/{step:04d}"


def build_s3_zipped_step_path(*, model_name: str, project: str, step: int, s3_bucket: str | None = None,
                              prefix: str | None = None) -> str:
    base = build_s3_path(model_name=model_name, project=project, s3_bucket=s3_bucket, prefix=prefix)
    return f"{base}/zipped-steps/{step:04d}.zip"


async def _aws(args: list[str], profile: str | None, verbose: bool, capture: bool = False) -> str:
    cmd = ["aws"] + (["--profile", profile] if profile else []) + args
    out = PIPE if capture else (None if verbose else DEVNULL)
    proc = await asyncio.create_subprocess_exec(*cmd, stdout=out, stderr=None if verbose else DEVNULL)
    data, _ = await proc.communicate()
    if proc.returncode != 0:
        raise S3SyncError(f"{' '.join(cmd)} exited with status {proc.returncode}")
    return (data or b"").decode()


@limit_concurrency(1)
async def s3_sync(source: str, destination: str, *, profile: Optional[str] = None, verbose: bool = False,
                  delete: bool = False, exclude: list[ExcludableOption] | None = None) -> None:
    """``aws s3 cp`` for a file, ``aws s3 sync`` for a directory; either side
    may be an ``s3://`` URI.  Raises :class:`S3SyncError` on failure."""
    args = ["s3", "cp" if os.path.isfile(source) else "sync"]
    if delete:
        args.append("--delete")
    for d in exclude or []:
        args += ["--exclude", f"{d}/*"]
    await _aws(args + [source, destination], profile, verbose)


async def ensure_bucket_exists(s3_bucket: str | None = None, profile: str | None = None, verbose: bool = False) -> None:
    bucket = _bucket(s3_bucket)
    try:
        await _aws(["s3api", "head-bucket", "--bucket", bucket], profile, verbose)
    except S3SyncError:
        await _aws(["s3", "mb", f"s3://{bucket}"], profile, verbose)


async def list_checkpoint_steps(model_name: str, project: str, s3_bucket: str | None = None,
                                prefix: str | None = None, profile: str | None = None) -> list[int]:
    """Steps present under the model's ``checkpoints/`` prefix (sorted)."""
    base = build_s3_path(model_name=model_name, project=project, s3_bucket=s3_bucket, prefix=prefix)
    try:
        listing = await _aws(["s3", "ls", f"{base}/checkpoints/"], profile, False, capture=True)
    except S3SyncError:
        return []
    steps = {int(m.group(1)) for m in re.finditer(r"PRE (\d+)/", listing)}
    return sorted(steps)


async def get_latest_checkpoint_step_from_s3(model_name: str, project: str, s3_bucket: str | None = None,
                                             prefix: str | None = None) -> int | None:
    steps = await list_checkpoint_steps(model_name, project, s3_bucket, prefix)
    return steps[-1] if steps else None


async def get_checkpoint_step_not_after_from_s3(model_name: str, project: str, not_after: int,
                                                s3_bucket: str | None = None, prefix: str | None = None) -> int | None:
    steps = [s for s in await list_checkpoint_steps(model_name, project, s3_bucket, prefix) if s <= not_after]
    return steps[-1] if steps else None


async def pull_model_from_s3(model_name: str, project: str, step: int | None = None, s3_bucket: str | None = None,
                             prefix: str | None = None, verbose: bool = False, delete: bool = False,
                             art_path: str | None = None, exclude: list[ExcludableOption] | None = None) -> str:
    """Sync the model directory (or one step's checkpoint) from S3 into the
    local ``.art`` tree; returns the local directory."""
    local = get_output_dir_from_model_properties(project, model_name, art_path or ".art")
    src = build_s3_path(model_name=model_name, project=project, step=step, s3_bucket=s3_bucket, prefix=prefix)
    dst = local if step is None else os.path.join(local, "checkpoints", f"{step:04d}")
    os.makedirs(dst, exist_ok=True)
    await s3_sync(src, dst, verbose=verbose, delete=delete, exclude=exclude)
    return dst


async def push_model_to_s3(model_name: str, project: str, s3_bucket: str | None = None, prefix: str | None = None,
                           verbose: bool = False, delete: bool = False, art_path: str | None = None) -> None:
    local = get_output_dir_from_model_properties(project, model_name, art_path or ".art")
    dst = build_s3_path(model_name=model_name, project=project, s3_bucket=s3_bucket, prefix=prefix)
    await s3_sync(local, dst, verbose=verbose, delete=delete)


async def archive_and_presign_step_url(model_name: str, project: str, step: int, s3_bucket: str | None = None,
                                       prefix: str | None = None, verbose: bool = False, delete: bool = False,
                                       art_path: str | None = None, checkpoint_path: str | None = None) -> str:
    """Zip one step's checkpoint, upload it to ``zipped-steps/`` and return a
    presigned download URL."""
    if checkpoint_path is None:
        local = get_output_dir_from_model_properties(project, model_name, art_path or ".art")
        checkpoint_path = os.path.join(local, "checkpoints", f"{step:04d}")
    if not os.path.isdir(checkpoint_path):
        raise FileNotFoundError(checkpoint_path)
    dst = build_s3_zipped_step_path(model_name=model_name, project=project, step=step, s3_bucket=s3_bucket,
                                    prefix=prefix)
    with tempfile.TemporaryDirectory() as tmp:
        archive = shutil.make_archive(os.path.join(tmp, f"{step:04d}"), "zip", checkpoint_path)
        await s3_sync(archive, dst, verbose=verbose, delete=delete)
    return (await _aws(["s3", "presign", dst, "--expires-in", "86400"], None, verbose, capture=True)).strip()
