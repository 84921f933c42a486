"""Agent protocols and plumbing on CPU: JSON-RPC error paths, MCP tool calls over a channel,
A2A task lifecycle, tool-call parsing edge cases, the multi-agent runtime contract, memory
stores and skill front matter."""

import threading

import pytest

from saint_llm_b200.agents import (
    A2AClient,
    A2AServer,
    Agent,
    FileMemoryStore,
    FunctionTool,
    InMemoryMemoryStore,
    MCPServer,
    Message,
    MockPolicy,
    Runtime,
    ToolCall,
    ToolRegistry,
    ToolSpec,
    format_tool_call,
    mcp_client_tools,
    pair_channels,
    parse_tool_calls,
)
from saint_llm_b200.agents.jsonrpc import (
    A2AClientError,
    JsonRpcClient,
    MCPClientError,
    RpcError,
    final_response,
    mcp_list_tools,
)


def _serve(server, channel):
    t = threading.Thread(target=server.serve, args=(channel,), daemon=True)
    t.start()
    return t


def _registry():
    r = ToolRegistry()
    r.register(FunctionTool(ToolSpec("echo", "echo text", {"type": "object", "properties": {"text": {"type": "string"}}}),
                            lambda text="": text))
    r.register(FunctionTool(ToolSpec("fail", "always raises"), lambda: (_ for _ in ()).throw(KeyError("nope"))))
    return r


# ----------------------------------------------------------------- JSON-RPC
def test_jsonrpc_unknown_method_and_notifications():
    a, b = pair_channels()
    srv = MCPServer(_registry())
    t = _serve(srv, b)
    c = JsonRpcClient(a, MCPClientError)
    with pytest.raises(MCPClientError, match="method not found"):
        c.request("no/such/method", {})
    c.notify("ping")  # a notification gets no reply, and the next request still pairs up
    assert c.request("ping") == {}
    a.close()
    t.join(timeout=5)


def test_jsonrpc_handler_crash_is_reported_not_fatal():
    class Crashy(MCPServer):
        def __init__(self):
            super().__init__(ToolRegistry())
            self.methods["boom"] = lambda p: 1 / 0

    a, b = pair_channels()
    t = _serve(Crashy(), b)
    c = JsonRpcClient(a, RuntimeError)
    with pytest.raises(RuntimeError, match="internal error: ZeroDivisionError"):
        c.request("boom")
    assert c.request("ping") == {}  # still serving
    a.close()
    t.join(timeout=5)


def test_rpc_error_carries_code():
    e = RpcError(-32602, "bad")
    assert e.code == -32602 and e.message == "bad"


# ---------------------------------------------------------------------- MCP
def test_mcp_tools_round_trip_and_errors():
    a, b = pair_channels()
    t = _serve(MCPServer(_registry()), b)
    specs = mcp_list_tools(a)
    assert [s.name for s in specs] == ["echo", "fail"]
    assert specs[0].parameters["properties"]["text"]["type"] == "string"
    a.close()
    t.join(timeout=5)

    a, b = pair_channels()
    t = _serve(MCPServer(_registry()), b)
    tools = {tl.spec.name: tl for tl in mcp_client_tools(a, name_prefix="remote_")}
    assert set(tools) == {"remote_echo", "remote_fail"}
    local = ToolRegistry()
    for tl in tools.values():
        local.register(tl)
    assert local.execute(ToolCall("1", "remote_echo", {"text": "hi"})).content == "hi"
    assert "KeyError" in local.execute(ToolCall("2", "remote_fail", {})).content
    client = JsonRpcClient(a, MCPClientError)
    res = client.request("tools/call", {"name": "missing", "arguments": {}})
    assert res["isError"] and "unknown tool" in res["content"][0]["text"]
    with pytest.raises(MCPClientError, match="string 'name'"):
        client.request("tools/call", {"name": 3})
    with pytest.raises(MCPClientError, match="must be an object"):
        client.request("tools/call", {"name": "echo", "arguments": [1, 2]})
    a.close()
    t.join(timeout=5)


# ---------------------------------------------------------------------- A2A
def test_a2a_task_lifecycle():
    pol = MockPolicy([Message("assistant", "", (ToolCall("c", "echo", {"text": "x"}),)),
                      Message("assistant", "done: x"), Message("assistant", "second")])
    agent = Agent(name="worker", policy=pol, tools=_registry())
    a, b = pair_channels()
    t = _serve(A2AServer(agent), b)
    c = A2AClient(a)
    info = c.agent_info()
    assert info["name"] == "worker" and {x["name"] for x in info["tools"]} == {"echo", "fail"}
    task = c.send_task("please echo", session_id="s1", task_id="t1")
    assert task["status"] == "completed" and task["artifacts"][0]["text"] == "done: x"
    assert task["sessionId"] == "s1"
    assert c.get_task("t1")["status"] == "completed"
    assert c.cancel_task("t1")["status"] == "completed"  # finished tasks stay finished
    with pytest.raises(A2AClientError, match="task not found"):
        c.get_task("nope")
    with pytest.raises(A2AClientError, match="non-empty 'message'"):
        c.send_task("")
    a.close()
    t.join(timeout=5)


def test_a2a_failing_agent_fails_the_task():
    class Broken:
        def act(self, messages, *, tools=()):
            raise RuntimeError("model offline")

    a, b = pair_channels()
    t = _serve(A2AServer(Agent(name="x", policy=Broken())), b)
    task = A2AClient(a).send_task("hello")
    assert task["status"] == "failed" and "model offline" in task["error"]
    a.close()
    t.join(timeout=5)


def test_final_response_prefers_plain_assistant_text():
    hist = [Message("user", "q"), Message("assistant", "thinking", (ToolCall("1", "echo", {}),)),
            Message("tool", "r", tool_call_id="1"), Message("assistant", "answer")]
    assert final_response(hist) == "answer"
    assert final_response([Message("assistant", "only", (ToolCall("1", "e", {}),))]) == "only"
    assert final_response([]) == ""


# ------------------------------------------------------------------ parsing
def test_parse_tags_fences_and_dedup():
    call = ToolCall("c9", "echo", {"text": "a"})
    text = format_tool_call(call) + '\n```json\n[{"name": "echo", "arguments": {"text": "a"}}, ' \
        '{"name": "other", "arguments": {"n": 1}, "id": "z"}]\n```'
    got = parse_tool_calls(text)
    assert [(c.name, c.arguments) for c in got] == [("echo", {"text": "a"}), ("other", {"n": 1})]
    assert got[0].id == "c9" and got[1].id == "z"
    assert [c.name for c in parse_tool_calls(text, fmt="xml")] == ["echo"]
    assert [c.name for c in parse_tool_calls(text, fmt="json")] == ["echo", "other"]


@pytest.mark.parametrize("bad", ['<tool_call id="1">{}</tool_call>', '<tool_call name="x">{oops</tool_call>',
                                 '<tool_call name="x">[1, 2]</tool_call>', '```json\n{"arguments": {}}\n```',
                                 '```json\nnot json\n```'])
def test_parse_malformed_skips_or_raises(bad):
    assert parse_tool_calls(bad) == []
    with pytest.raises(ValueError):
        parse_tool_calls(bad, strict=True)


def test_parse_unknown_format_and_generated_ids():
    with pytest.raises(ValueError, match="unknown parser format"):
        parse_tool_calls("", fmt="yaml")  # type: ignore[arg-type]
    a = parse_tool_calls('<tool_call name="t">{}</tool_call>')[0]
    assert a.id.startswith("call_") and a.arguments == {}


# ------------------------------------------------------------------ runtime
def _talker(name, lines):
    return Agent(name=name, policy=MockPolicy([Message("assistant", s) for s in lines]))


def test_runtime_round_robin_passes_spoken_text():
    rt = Runtime([_talker("a", ["a1", "a2"]), _talker("b", ["b1", "b2"])])
    rt.send(to="a", content="start")
    assert [m.content for m in rt.inbox_for("a")] == ["start"]
    rt.run(max_ticks=3)
    assert rt.cursor == 1
    said = [(m.name, m.content) for m in rt.transcript if m.role == "assistant"]
    assert said == [("a", "a1"), ("b", "b1"), ("a", "a2")]
    # b heard a's second line and nothing else is pending for a
    assert [m.content for m in rt.inbox_for("b")] == ["a2"] and rt.inbox_for("a") == []
    # each agent saw the other's text as a user message from that agent
    b_user = [m for m in rt.agents[1].history if m.role == "user"]
    assert [(m.name, m.content) for m in b_user] == [("a", "a1")]


def test_runtime_tool_traffic_stays_private():
    r = ToolRegistry()
    r.register(FunctionTool(ToolSpec("t", "tool"), lambda: "secret"))
    a = Agent(name="a", policy=MockPolicy([Message("assistant", "", (ToolCall("1", "t", {}),))]), tools=r)
    rt = Runtime([a, _talker("b", ["ok"])])
    rt.tick()
    assert rt.inbox_for("b") == []  # no spoken text: nothing forwarded
    assert any(m.role == "tool" and m.content == "secret" for m in rt.transcript)


@pytest.mark.parametrize("agents,err", [(1, "two or more"), (0, "two or more")])
def test_runtime_rejects_too_few_agents(agents, err):
    with pytest.raises(ValueError, match=err):
        Runtime([_talker(f"x{i}", ["."]) for i in range(agents)])


def test_runtime_rejects_duplicates_unknown_names_and_zero_ticks():
    with pytest.raises(ValueError, match="share the name"):
        Runtime([_talker("a", ["."]), _talker("a", ["."])])
    rt = Runtime([_talker("a", ["."]), _talker("b", ["."])])
    with pytest.raises(KeyError, match="no agent named"):
        rt.send(to="zed", content="hi")
    with pytest.raises(ValueError, match="at least one turn"):
        rt.run(max_ticks=0)


def test_agent_rejects_non_assistant_policy_and_bad_steps():
    class Wrong:
        def act(self, messages, *, tools=()):
            return Message("user", "??")

    with pytest.raises(ValueError, match="must be 'assistant'"):
        Agent(name="w", policy=Wrong()).step()
    with pytest.raises(ValueError, match="max_steps"):
        _talker("x", ["."]).run(user_message="hi", max_steps=0)


def test_agent_stops_after_max_steps_of_tool_calls():
    loop = [Message("assistant", "", (ToolCall(str(i), "echo", {"text": str(i)}),)) for i in range(10)]
    agent = Agent(name="x", policy=MockPolicy(loop), tools=_registry())
    hist = agent.run(user_message="go", max_steps=3)
    assert sum(1 for m in hist if m.role == "tool") == 3


# ------------------------------------------------------------------- memory
@pytest.mark.parametrize("store_kind", ["mem", "file"])
def test_memory_store_contract(tmp_path, store_kind):
    s = InMemoryMemoryStore() if store_kind == "mem" else FileMemoryStore(tmp_path / "m")
    s.store("alpha", "the Quick brown fox")
    s.store("beta.notes", "lazy dog")
    assert s.view("alpha").value == "the Quick brown fox"
    assert s.view("missing") is None
    assert [e.key for e in s.recall("quick")] == ["alpha"]
    assert [e.key for e in s.recall("NOTES")] == ["beta.notes"]
    assert s.recall("") == ()
    s.store("alpha", "replaced")
    assert s.view("alpha").value == "replaced" and len(s.list()) == 2
    assert s.delete("alpha") and not s.delete("alpha")
    s.clear()
    assert s.list() == ()
    for bad in ["", "..", "a/b", "sp ace", "x\\y"]:
        with pytest.raises(ValueError, match="invalid memory key"):
            s.store(bad, "v")


def test_file_memory_persists_across_instances(tmp_path):
    FileMemoryStore(tmp_path / "m").store("k", "v1")
    again = FileMemoryStore(tmp_path / "m")
    assert again.view("k").value == "v1"
    assert [e.key for e in again.list()] == ["k"]


# --------------------------------------------------------------- Code Mode
def test_api_stub_documents_every_tool():
    from saint_llm_b200.agents.code_mode import generate_api_stub

    stub = generate_api_stub([ToolSpec("add", "add ints", {"type": "object", "properties": {
        "a": {"type": "integer", "description": "left"}, "b": {"type": "integer"}}, "required": ["a"]}),
        ToolSpec("noop", "nothing")], namespace="api")
    assert stub.names == ("add", "noop")
    assert "class api:" in stub.source and "a (integer) (required): left" in stub.source
    assert "No parameters." in stub.source
    compile(stub.source, "<stub>", "exec")  # valid Python
    assert generate_api_stub([]).names == ()


def test_in_process_executor_logs_calls_and_reports_errors():
    from saint_llm_b200.agents.code_mode import InProcessExecutor

    ex = InProcessExecutor()
    ok = ex.execute("x = tools.echo(text='hi')\nprint(x)\nRESULT = x * 2", registry=_registry())
    assert ok.ok and ok.stdout.strip() == "hi" and ok.return_value == "hihi"
    assert ok.tool_calls == [{"name": "echo", "arguments": {"text": "hi"}}]
    bad = ex.execute("1 / 0", registry=_registry())
    assert not bad.ok and bad.error_type == "ZeroDivisionError" and "ZeroDivisionError" in bad.stderr
    missing = ex.execute("tools.nope()", registry=_registry())
    assert not missing.ok and missing.error_type == "AttributeError"


# ------------------------------------------------------------------ skills
def test_skill_front_matter_and_loading(tmp_path):
    from saint_llm_b200.agents.skills import SkillLoadError, load_skill, load_skills, parse_front_matter

    meta = parse_front_matter("name: demo\n# comment\ntags:\n  - a\n  - 'b c'\ndescription: \"quoted\"\n")
    assert meta == {"name": "demo", "tags": ["a", "b c"], "description": "quoted"}
    with pytest.raises(SkillLoadError):
        parse_front_matter("no colon here")
    root = tmp_path / "skills"
    (root / "one").mkdir(parents=True)
    (root / "one" / "SKILL.md").write_text("---\nname: one\ndescription: first\nallowed-tools: a, b\n---\nDo it.\n")
    (root / "two").mkdir()
    (root / "two" / "SKILL.md").write_text("---\nname: two\n---\nbody\n")
    (root / ".hidden").mkdir()
    (root / "notaskill").mkdir()
    skills = load_skills(root)
    assert [s.name for s in skills] == ["one", "two"]
    assert skills[0].allowed_tools == ("a", "b") and skills[0].instructions == "Do it."
    (root / "bad").mkdir()
    (root / "bad" / "SKILL.md").write_text("---\nname: bad\n")
    with pytest.raises(SkillLoadError, match="unterminated"):
        load_skill(root / "bad")
    with pytest.raises(SkillLoadError):
        load_skills(tmp_path / "missing")


def test_history_rendering_for_the_model_policy():
    from saint_llm_b200.agents.core import Message, ToolSpec
    from saint_llm_b200.agents.model_policy import TOOL_FORMAT_HINT, to_chat_turns, tools_prompt

    assert tools_prompt(()) == ""
    spec = ToolSpec("add", "adds", {"type": "object"})
    cat = tools_prompt([spec])
    assert cat.startswith(TOOL_FORMAT_HINT) and '- add: adds parameters={"type": "object"}' in cat
    msgs = [Message(role="system", content="rule one"), Message(role="user", content="hi"),
            Message(role="assistant", content="calling"), Message(role="tool", content="3", tool_call_id="c1"),
            Message(role="system", content="rule two")]
    turns = to_chat_turns(msgs, [spec])
    # every system message is folded into one leading system turn, followed by the catalogue
    assert turns[0].role == "system" and turns[0].content == "rule one\n\nrule two\n\n" + cat
    assert [(t.role, t.content) for t in turns[1:]] == [("user", "hi"), ("assistant", "calling"),
                                                         ("user", "[tool c1] 3")]
    assert to_chat_turns([Message(role="user", content="x")], [])[0].role == "user"
