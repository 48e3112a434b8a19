"""Tool / resource descriptions of an MCP server and generated scenarios
(same fields as the reference ``src/art/mcp/types.py``)."""

from __future__ import annotations

import json
import random
from collections import Counter
from dataclasses import asdict, dataclass, field
from typing import Any, Iterator


@dataclass
class MCPTool:
    name: str
    description: str = ""
    parameters: dict[str, Any] = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "MCPTool":
        return cls(d.get("name", ""), d.get("description", ""), d.get("parameters") or d.get("inputSchema") or {})

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    def to_tool_schema(self) -> dict[str, Any]:
        """OpenAI function-tool schema (the ``tools=`` entry of a chat request)."""
        return {"type": "function", "function": {"name": self.name, "description": self.description,
                                                 "parameters": self.parameters or {"type": "object", "properties": {}}}}


@dataclass
class MCPResource:
    uri: str
    name: str = ""
    description: str = ""
    mime_type: str | None = None

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "MCPResource":
        return cls(d.get("uri", ""), d.get("name", ""), d.get("description", ""), d.get("mimeType") or d.get("mime_type"))

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


@dataclass
class GeneratedScenario:
    task: str
    difficulty: int

    def __post_init__(self) -> None:
        if not 1 <= int(self.difficulty) <= 5:
            raise ValueError(f"difficulty must be in 1..5, got {self.difficulty}")
        self.difficulty = int(self.difficulty)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "GeneratedScenario":
        return cls(str(d["task"]), int(d["difficulty"]))

    def to_dict(self) -> dict[str, Any]:
        return {"task": self.task, "difficulty": self.difficulty}

    def preview(self, max_length: int = 120) -> str:
        t = self.task if len(self.task) <= max_length else self.task[:max_length] + "..."
        return f"[{self.difficulty}/5] {t}"


class GeneratedScenarioCollection:
    def __init__(self, scenarios: list[GeneratedScenario]) -> None:
        self.scenarios = list(scenarios)

    @classmethod
    def from_dicts(cls, data: list[dict[str, Any]]) -> "GeneratedScenarioCollection":
        return cls([GeneratedScenario.from_dict(d) for d in data])

    @classmethod
    def from_json(cls, text: str) -> "GeneratedScenarioCollection":
        data = json.loads(text)
        return cls.from_dicts(data["scenarios"] if isinstance(data, dict) else data)

    def to_dicts(self) -> list[dict[str, Any]]:
        return [s.to_dict() for s in self.scenarios]

    def to_json(self, indent: int | None = None) -> str:
        return json.dumps({"scenarios": self.to_dicts()}, indent=indent)

    def __len__(self) -> int:
        return len(self.scenarios)

    def __iter__(self) -> Iterator[GeneratedScenario]:
        return iter(self.scenarios)

    def __getitem__(self, i):
        return self.scenarios[i]

    def shuffle(self, seed: int | None = None) -> "GeneratedScenarioCollection":
        s = list(self.scenarios)
        random.Random(seed).shuffle(s)
        return GeneratedScenarioCollection(s)

    def split(self, train_size: int | float = 0.8, seed: int | None = None
              ) -> tuple["GeneratedScenarioCollection", "GeneratedScenarioCollection"]:
        s = self.shuffle(seed).scenarios if seed is not None else list(self.scenarios)
        n = int(round(train_size * len(s))) if isinstance(train_size, float) else int(train_size)
        return GeneratedScenarioCollection(s[:n]), GeneratedScenarioCollection(s[n:])

    def filter_by_difficulty(self, min_difficulty: int = 1, max_difficulty: int = 5) -> "GeneratedScenarioCollection":
        return GeneratedScenarioCollection([s for s in self.scenarios if min_difficulty <= s.difficulty <= max_difficulty])

    def get_difficulty_distribution(self) -> Counter:
        return Counter(s.difficulty for s in self.scenarios)

    def get_summary(self) -> dict[str, Any]:
        d = self.get_difficulty_distribution()
        n = len(self.scenarios)
        return {"total": n, "difficulty_distribution": dict(sorted(d.items())),
                "avg_difficulty": (sum(k * v for k, v in d.items()) / n) if n else 0.0}

    def preview(self, n: int = 5, max_task_length: int = 120) -> None:
        for i, s in enumerate(self.scenarios[:n], 1):
            print(f"{i}. {s.preview(max_task_length)}")
