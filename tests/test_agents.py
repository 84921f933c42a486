"""Agents, protocols, Code Mode, skills, memory and the sandbox (CPU)."""

import threading

import pytest
import torch

from saint_llm_b200.agents import (
    A2AClient,
    A2AServer,
    Agent,
    CodeModePolicy,
    FileMemoryStore,
    FunctionTool,
    InMemoryMemoryStore,
    InProcessExecutor,
    MCPServer,
    Message,
    MockPolicy,
    ModelPolicy,
    Runtime,
    SandboxExecutor,
    SkillRegistry,
    TextLMPolicy,
    ToolCall,
    ToolRegistry,
    ToolSpec,
    format_tool_call,
    generate_api_stub,
    load_skills,
    mcp_client_tools,
    pair_channels,
    parse_tool_calls,
    register_memory_tools,
    register_skill_scripts,
    register_skills_as_tools,
    send_to_agent,
)
from saint_llm_b200.sandbox import ContainerSandbox, FunctionCallSandbox, SandboxConfig


def _registry():
    r = ToolRegistry()
    r.register(FunctionTool(ToolSpec("add", "add two ints", {"type": "object", "properties": {
        "a": {"type": "integer"}, "b": {"type": "integer"}}, "required": ["a", "b"]}), lambda a, b: a + b))
    r.register(FunctionTool(ToolSpec("boom", "fails"), lambda: 1 / 0))
    return r


def test_registry_and_agent_loop():
    r = _registry()
    assert r.execute(ToolCall("c1", "add", {"a": 2, "b": 3})).content == "5"
    assert r.execute(ToolCall("c2", "boom")).content.startswith("ERROR: ZeroDivisionError")
    with pytest.raises(ValueError):
        r.register(FunctionTool(ToolSpec("add", "dup"), lambda: 0))
    pol = MockPolicy([Message("assistant", "", (ToolCall("c1", "add", {"a": 1, "b": 2}),)),
                      Message("assistant", "the answer is 3")])
    agent = Agent(name="bot", policy=pol, system="be helpful", tools=r)
    hist = agent.run(user_message="1+2?")
    assert [m.role for m in hist] == ["system", "user", "assistant", "tool", "assistant"]
    assert hist[3].content == "3" and hist[-1].name == "bot" and pol.remaining == 0
    with pytest.raises(ValueError):
        Message("user", "x", (ToolCall("c", "add"),))


def test_runtime_round_robin():
    a = Agent(name="a", policy=MockPolicy([Message("assistant", "ping"), Message("assistant", "ping2")]))
    b = Agent(name="b", policy=MockPolicy([Message("assistant", "pong")]))
    rt = Runtime([a, b])
    rt.send(to="a", content="start")
    rt.tick()
    assert rt.inbox_for("b")[0].content == "ping" and rt.cursor == 1
    rt.tick()
    assert rt.inbox_for("a")[0].name == "b"
    assert len(rt.transcript) == 3


def test_parser_formats():
    text = ('<tool_call name="add" id="x1">{"a": 1, "b": 2}</tool_call>\n'
            '```json\n[{"name": "add", "arguments": {"a": 1, "b": 2}}, {"name": "mul", "arguments": {"x": 3}}]\n```')
    calls = parse_tool_calls(text)
    assert [(c.name, c.id) for c in calls][:1] == [("add", "x1")] and [c.name for c in calls] == ["add", "mul"]
    assert parse_tool_calls('<tool_call name="x">not json</tool_call>') == []
    with pytest.raises(ValueError):
        parse_tool_calls('<tool_call name="x">not json</tool_call>', strict=True)
    c = ToolCall("id9", "add", {"a": 1})
    assert parse_tool_calls(format_tool_call(c), fmt="xml")[0] == c
    pol = TextLMPolicy(lambda h: format_tool_call(c))
    assert pol.act([Message("user", "hi")]).tool_calls == (c,)


def _serve(server, channel):
    t = threading.Thread(target=server.serve, args=(channel,), daemon=True)
    t.start()
    return t


def test_mcp_roundtrip():
    client_ch, server_ch = pair_channels()
    _serve(MCPServer(_registry()), server_ch)
    tools = {t.spec.name: t for t in mcp_client_tools(client_ch, name_prefix="remote.")}
    assert set(tools) == {"remote.add", "remote.boom"}
    assert tools["remote.add"](a=4, b=5) == "9"
    assert tools["remote.boom"]().startswith("ERROR:")
    client_ch.close()


def test_a2a_roundtrip():
    pol = MockPolicy([Message("assistant", "", (ToolCall("c", "add", {"a": 2, "b": 2}),)),
                      Message("assistant", "four")])
    ch, sch = pair_channels()
    _serve(A2AServer(Agent(name="math", policy=pol, tools=_registry())), sch)
    c = A2AClient(ch)
    assert c.agent_info()["name"] == "math"
    task = c.send_task("2+2?", task_id="t1")
    assert task["status"] == "completed" and task["artifacts"][0]["text"] == "four"
    assert c.get_task("t1")["status"] == "completed" and c.cancel_task("t1")["status"] == "completed"
    with pytest.raises(RuntimeError):
        c.get_task("missing")
    ch.close()


@pytest.mark.parametrize("executor", [InProcessExecutor(), SandboxExecutor(timeout_s=20)])
def test_code_mode(executor):
    r = _registry()
    stub = generate_api_stub(list(r.specs()))
    assert "def add(**kwargs)" in stub.source and stub.names == ("add", "boom")
    pol = CodeModePolicy(MockPolicy([Message("assistant", "RESULT = tools.add(a=20, b=22)")]), r, executor)
    out = pol.act([Message("user", "add")])
    assert out.content.startswith("Code Mode result:") and "42" in out.content


def test_skills_and_scripts(tmp_path):
    d = tmp_path / "skills" / "greet"
    (d / "scripts").mkdir(parents=True)
    (d / "SKILL.md").write_text("---\nname: greet\ndescription: say hello\nallowed-tools: a, b\n---\n# Hi\nBe kind.")
    (d / "scripts" / "hello.py").write_text("import sys; print('hello', *sys.argv[1:])")
    skills = load_skills(tmp_path / "skills")
    assert skills[0].name == "greet" and skills[0].allowed_tools == ("a", "b")
    reg = SkillRegistry(skills)
    assert "greet: say hello" in reg.catalog()
    tools = ToolRegistry()
    register_skills_as_tools(tools, reg)
    assert tools.get("use_greet")() == "# Hi\nBe kind."
    assert register_skill_scripts(tools, skills[0]) == 1
    assert tools.get("greet_hello")(name="bob", loud=True).strip() == "hello --name bob --loud"


@pytest.mark.parametrize("kind", ["mem", "file"])
def test_memory(tmp_path, kind):
    store = InMemoryMemoryStore() if kind == "mem" else FileMemoryStore(tmp_path)
    reg = ToolRegistry()
    register_memory_tools(reg, store)
    assert reg.get("memory_store")(key="k1", value="likes tea") == "ok"
    assert reg.get("memory_view")(key="k1") == "likes tea"
    assert reg.get("memory_recall")(query="TEA") == "k1: likes tea"
    assert reg.get("memory_delete")(key="k1") == "deleted" and reg.get("memory_view")(key="k1") == "no entry"
    with pytest.raises(ValueError):
        store.store("../x", "y")


def test_model_policy_and_send_to_agent():
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.data import CharTokenizer
    from saint_llm_b200.models import SaintLLM

    torch.manual_seed(0)
    model = SaintLLM(ModelConfig.tiny())
    pol = ModelPolicy(model, CharTokenizer(base_vocab=16, unicode_max=496), max_new_tokens=6)
    out = pol.act([Message("user", "hi")], tools=list(_registry().specs()))
    assert out.role == "assistant" and isinstance(out.content, str)
    ch, sch = pair_channels()
    _serve(A2AServer(Agent(name="m", policy=pol)), sch)
    assert isinstance(send_to_agent(ch, "hello"), str)
    ch.close()


def test_sandbox():
    sb = FunctionCallSandbox()
    assert sb.run_python("print(6*7)").stdout.strip() == "42"
    r = sb.run_python("import time; time.sleep(10)", config=SandboxConfig(timeout_s=0.5))
    assert not r.ok and "timeout" in r.error
    r = sb.run(["/nonexistent/binary"])
    assert not r.ok and r.exit_code == -1
    with pytest.raises(NotImplementedError):
        ContainerSandbox().run_python("1")
