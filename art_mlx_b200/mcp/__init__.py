"""MCP (Model Context Protocol) helpers: tool / resource descriptions and
LLM-generated training scenarios (reference ``src/art/mcp/``)."""

from .generate_scenarios import generate_scenarios
from .types import GeneratedScenario, GeneratedScenarioCollection, MCPResource, MCPTool

__all__ = ["GeneratedScenario", "GeneratedScenarioCollection", "MCPResource", "MCPTool", "generate_scenarios"]
