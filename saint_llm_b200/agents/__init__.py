"""Agents: messages, tools, policies (incl. one backed by this framework's model), the agent
loop and multi-agent runtime, tool-call parsing, MCP and A2A over JSON-RPC, Code Mode,
skills and memory."""

from saint_llm_b200.agents.code_mode import (
    CodeModePolicy,
    ExecutionResult,
    InProcessExecutor,
    SandboxExecutor,
    generate_api_stub,
)
from saint_llm_b200.agents.core import (
    Agent,
    CallablePolicy,
    FunctionTool,
    Message,
    MockPolicy,
    Policy,
    Runtime,
    TextLMPolicy,
    Tool,
    ToolCall,
    ToolRegistry,
    ToolSpec,
)
from saint_llm_b200.agents.jsonrpc import (
    A2AClient,
    A2AServer,
    InMemoryJsonRpcChannel,
    JsonRpcChannel,
    MCPServer,
    StdioJsonRpcChannel,
    mcp_client_tools,
    mcp_list_tools,
    pair_channels,
    send_to_agent,
)
from saint_llm_b200.agents.memory import FileMemoryStore, InMemoryMemoryStore, MemoryStore, register_memory_tools
from saint_llm_b200.agents.model_policy import ModelPolicy
from saint_llm_b200.agents.parsing import format_tool_call, parse_tool_calls
from saint_llm_b200.agents.skills import (
    Skill,
    SkillRegistry,
    load_skill,
    load_skills,
    register_skill_scripts,
    register_skills_as_tools,
)

__all__ = [n for n in dir() if not n.startswith("_") and n[0].isupper() or n in (
    "generate_api_stub", "mcp_client_tools", "mcp_list_tools", "pair_channels", "send_to_agent",
    "register_memory_tools", "format_tool_call", "parse_tool_calls", "load_skill", "load_skills",
    "register_skill_scripts", "register_skills_as_tools")]
