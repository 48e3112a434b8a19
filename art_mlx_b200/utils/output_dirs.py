"""Directory layout of a model's artefacts (same layout as the reference's
``src/art/utils/output_dirs.py`` / ``get_model_step.py``):

``{art_path}/{project}/models/{name}/``
    ``checkpoints/{step:04d}/adapter_model.safetensors`` + ``adapter_config.json``
    ``trajectories/{split}/{step:04d}.parquet``
    ``history.jsonl``, ``model.json``, ``tensors/`` (packed batch mmap files)
"""

from __future__ import annotations

import os


def get_models_dir(project: str, art_path: str) -> str:
    return f"{art_path}/{project}/models"


def get_model_dir(model, art_path: str) -> str:
    return f"{art_path}/{model.project}/models/{model.name}"


def get_output_dir_from_model_properties(project: str, name: str, art_path: str) -> str:
    return f"{art_path}/{project}/models/{name}"


def get_step_checkpoint_dir(model_output_dir: str, step: int) -> str:
    return f"{model_output_dir}/checkpoints/{step:04d}"


def get_trajectories_dir(model_output_dir: str) -> str:
    return f"{model_output_dir}/trajectories"


def get_trajectories_split_dir(model_output_dir: str, split: str) -> str:
    return f"{model_output_dir}/trajectories/{split}"


def get_step_from_dir(output_dir: str) -> int:
    """Latest step = the largest numeric directory under ``checkpoints/``."""
    ckpt = os.path.join(output_dir, "checkpoints")
    if not os.path.isdir(ckpt):
        return 0
    steps = [int(d) for d in os.listdir(ckpt) if d.isdigit() and os.path.isdir(os.path.join(ckpt, d))]
    return max(steps, default=0)


def list_checkpoint_steps(output_dir: str) -> list[int]:
    ckpt = os.path.join(output_dir, "checkpoints")
    if not os.path.isdir(ckpt):
        return []
    return sorted(int(d) for d in os.listdir(ckpt) if d.isdigit())
