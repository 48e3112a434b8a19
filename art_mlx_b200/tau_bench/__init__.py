"""tau-bench environments over HTTP: scenario listing, environment
create / step / delete, and an agent rollout loop that turns an episode
into a :class:`~art_mlx_b200.trajectories.Trajectory` (reference:
``src/art/tau_bench/``)."""

from .client import (DeleteEnvironmentResponse, EnvironmentResponse, Scenario, StepEnvironmentResponse, Task,
                     TauBenchClient, default_client, get_scenarios)
from .rollout import default_user_llm_args, rollout, tool_call_action

__all__ = [
    "DeleteEnvironmentResponse", "EnvironmentResponse", "Scenario", "StepEnvironmentResponse", "Task",
    "TauBenchClient", "default_client", "default_user_llm_args", "get_scenarios", "rollout", "tool_call_action",
]
