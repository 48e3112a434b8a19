"""Guided completions for distillation: constrain a student's sampling to a
teacher's answer.

Reference: ``src/art/guided_completion.py:33`` (``get_guided_completion_params``,
``freeze_tool_schema``).  Given a teacher's chat completion, returns
``(guided_choice, tool_choice, tools)``: for a text answer the one allowed
output string; for a tool call the forced tool and a copy of its schema whose
parameters accept exactly the teacher's arguments (an ``enum`` of one value
per field, all required, nothing else), which a structured-output engine
then enforces.
"""

from __future__ import annotations

import copy
import json
from typing import Any, Iterable


def _get(o: Any, key: str) -> Any:
    return o.get(key) if isinstance(o, dict) else getattr(o, key, None)


def freeze_tool_schema(tool: dict, fixed_args: dict) -> dict:
    """A copy of ``tool`` whose parameters admit only ``fixed_args``."""
    locked = copy.deepcopy(tool)
    locked["function"]["parameters"] = {
        "type": "object",
        "title": f"{tool['function']['name'].title()}FrozenArgs",
        "properties": {k: {"enum": [v], "title": k.replace("_", " ").title()} for k, v in fixed_args.items()},
        "required": list(fixed_args),
        "additionalProperties": False,
    }
    return locked


def get_guided_completion_params(completion: Any, base_tools: Iterable[dict] | None = None
                                 ) -> tuple[list[str] | None, dict | None, list[dict] | None]:
    msg = _get(_get(completion, "choices")[0], "message")
    calls = _get(msg, "tool_calls") or []
    if calls:
        call = calls[0]
        if _get(call, "type") not in (None, "function"):
            raise ValueError("only function tool calls can be guided")
        if base_tools is None:
            raise ValueError("No base tools provided")
        fn = _get(call, "function")
        name = _get(fn, "name")
        tool = next((t for t in base_tools if t["function"]["name"] == name), None)
        if tool is None:
            raise ValueError(f"the teacher called {name!r}, which is not among the base tools")
        args = json.loads(_get(fn, "arguments") or "{}")
        return None, {"type": "function", "function": {"name": name}}, [freeze_tool_schema(tool, args)]
    return [_get(msg, "content")], None, None
