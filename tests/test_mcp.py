import asyncio
import json
from types import SimpleNamespace

import pytest

from art_mlx_b200.mcp import GeneratedScenarioCollection, MCPTool, generate_scenarios


class FakeGen:
    def __init__(self, n):
        self.n = n
        self.chat = SimpleNamespace(completions=SimpleNamespace(create=self.create))

    async def create(self, model, messages, **kw):
        body = {"scenarios": [{"task": f"task {i}", "difficulty": 1 + i % 5} for i in range(self.n)]}
        return SimpleNamespace(choices=[SimpleNamespace(message=SimpleNamespace(content=json.dumps(body)))])


def test_generate_and_split():
    tools = [MCPTool("search", "search docs", {"type": "object", "properties": {"q": {"type": "string"}}}),
             {"name": "read", "description": "read a file"}]
    coll = asyncio.run(generate_scenarios(tools, num_scenarios=10, client=FakeGen(10), show_preview=False))
    assert len(coll) == 10 and coll.get_summary()["total"] == 10
    train, val = coll.split(0.8, seed=0)
    assert len(train) == 8 and len(val) == 2
    assert len(coll.filter_by_difficulty(4, 5)) == 4
    again = GeneratedScenarioCollection.from_json(coll.to_json())
    assert [s.task for s in again] == [s.task for s in coll]
    assert tools[0].to_tool_schema()["function"]["name"] == "search"
    with pytest.raises(ValueError, match="expected 5"):
        asyncio.run(generate_scenarios(tools, num_scenarios=5, client=FakeGen(3), show_preview=False))
