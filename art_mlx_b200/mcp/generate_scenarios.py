"""Training scenarios for an MCP server's tools, written by an LLM.

Behaviour of the reference ``src/art/mcp/generate_scenarios.py:27``: the
server's tools and resources are described to a generator model, which
returns ``num_scenarios`` realistic tasks with a difficulty from 1 to 5 as
JSON; invalid answers raise.  The generator is any OpenAI-compatible chat
endpoint (``client``; by default one built from ``generator_base_url`` /
``generator_api_key``, or ``OPENROUTER_API_KEY``).
"""

from __future__ import annotations

import json
import os
from typing import Any

from .types import GeneratedScenarioCollection, MCPResource, MCPTool


def _as_dicts(items: list[Any], kind: type) -> list[dict[str, Any]]:
    out = []
    for it in items or []:
        if isinstance(it, kind):
            out.append(it.to_dict())
        elif isinstance(it, dict):
            out.append(it)
        else:  # objects of the mcp SDK (Tool / Resource)
            out.append(kind.from_dict(it.model_dump() if hasattr(it, "model_dump") else vars(it)).to_dict())
    return out


def scenario_prompt(tools: list[dict], resources: list[dict], num_scenarios: int,
                    custom_instructions: str | None = None) -> str:
    text = (
        f"You write test tasks for an AI agent that works through the tools of an MCP server.\n\n"
        f"Tools:\n{json.dumps(tools, indent=2)}\n\n"
        f"Resources:\n{json.dumps(resources, indent=2) if resources else 'none'}\n\n"
        f"Write {num_scenarios} different, realistic tasks a user could ask the agent to do with these tools. "
        "Mix simple tasks (one tool call) with multi-step ones, cover different tools and combinations without "
        "naming the tools in the task, and ask for a short written summary of the outcome in every task. "
        "Rate each task's difficulty from 1 (one call) to 5 (long multi-step analysis).\n\n"
        'Answer with JSON only: {"scenarios": [{"task": "...", "difficulty": 1}, ...]} with exactly '
        f"{num_scenarios} entries."
    )
    if custom_instructions:
        text += "\n\nAlso follow these instructions:\n" + custom_instructions
    return text


async def generate_scenarios(
    tools: list[MCPTool] | list[dict[str, Any]],
    resources: list[MCPResource] | list[dict[str, Any]] | None = None,
    num_scenarios: int = 24,
    show_preview: bool = True,
    custom_instructions: str | None = None,
    generator_model: str = "openai/gpt-4.1-mini",
    generator_api_key: str | None = None,
    generator_base_url: str = "https://openrouter.ai/api/v1",
    *,
    client: Any | None = None,
) -> GeneratedScenarioCollection:
    tools_d = _as_dicts(list(tools or []), MCPTool)
    res_d = _as_dicts(list(resources or []), MCPResource)
    if not tools_d and not res_d:
        raise ValueError("at least one tool or resource is required")
    if client is None:
        from openai import AsyncOpenAI

        key = generator_api_key or os.getenv("OPENROUTER_API_KEY")
        if not key:
            raise ValueError("generator_api_key (or OPENROUTER_API_KEY) is required without a client")
        client = AsyncOpenAI(api_key=key, base_url=generator_base_url)
    resp = await client.chat.completions.create(
        model=generator_model,
        messages=[{"role": "user", "content": scenario_prompt(tools_d, res_d, num_scenarios, custom_instructions)}],
        response_format={"type": "json_object"},
    )
    content = resp.choices[0].message.content or "{}"
    coll = GeneratedScenarioCollection.from_json(content)
    if len(coll) != num_scenarios:
        raise ValueError(f"expected {num_scenarios} scenarios, the generator returned {len(coll)}")
    if show_preview:
        coll.preview()
    return coll
