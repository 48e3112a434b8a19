"""art_mlx_b200: a Blackwell-native (B200 / sm_100a) GRPO trainer for LLM agents.

Public API (same names and call shapes as OpenPipe ART):

    import art_mlx_b200 as art
    model = art.TrainableModel(name=..., project=..., base_model=...)
    await model.register(art.LocalBackend())
    groups = await art.gather_trajectory_groups(...)
    result = await backend.train(model, groups, learning_rate=5e-6)
"""

from . import dev
from .auto_trajectory import auto_trajectory, capture_auto_trajectory
from .yield_trajectory import capture_yielded_trajectory, yield_trajectory
from .backend import Backend
from .gather import gather_trajectories, gather_trajectory_groups, trajectory_group_batches
from .model import Model, TrainableModel
from .trajectories import History, Trajectory, TrajectoryGroup
from .types import (
    LocalTrainResult,
    MegatronRuntimeConfig,
    MegatronTopologyConfig,
    Messages,
    MessagesAndChoices,
    RuntimeConfig,
    ServerlessTrainResult,
    TopologyConfig,
    Tools,
    TrainConfig,
    TrainResult,
    TrainSFTConfig,
)

__version__ = "0.1.0"


def __getattr__(name: str):
    # heavy submodules (torch models, kernels) load on first use
    if name == "LocalBackend":
        from .backends.local import LocalBackend

        return LocalBackend
    if name == "ServerlessBackend":
        from .backends.serverless import ServerlessBackend

        return ServerlessBackend
    if name in ("MultiGPUBackend", "MegatronBackend"):
        from .backends.multigpu import MultiGPUBackend

        return MultiGPUBackend
    if name in ("init_runtime_config", "init_megatron_runtime_config"):
        from .backends.multigpu import init_runtime_config

        return init_runtime_config
    if name == "PipelineTrainer":
        from .pipeline_trainer.trainer import PipelineTrainer

        return PipelineTrainer
    raise AttributeError(name)


__all__ = [
    "auto_trajectory",
    "capture_auto_trajectory",
    "capture_yielded_trajectory",
    "yield_trajectory",
    "Backend",
    "History",
    "LocalBackend",
    "LocalTrainResult",
    "MegatronRuntimeConfig",
    "MegatronTopologyConfig",
    "Messages",
    "MessagesAndChoices",
    "Model",
    "MegatronBackend",
    "MultiGPUBackend",
    "ServerlessBackend",
    "PipelineTrainer",
    "RuntimeConfig",
    "ServerlessTrainResult",
    "TopologyConfig",
    "Tools",
    "TrainConfig",
    "TrainResult",
    "TrainSFTConfig",
    "TrainableModel",
    "Trajectory",
    "TrajectoryGroup",
    "dev",
    "gather_trajectories",
    "gather_trajectory_groups",
    "init_megatron_runtime_config",
    "init_runtime_config",
    "trajectory_group_batches",
]
