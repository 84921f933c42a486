"""JSON-RPC 2.0 transports and the two agent protocols built on them:

* MCP (Model Context Protocol, version ``2024-11-05``): a server exposing a
  :class:`ToolRegistry` (``initialize``, ``tools/list``, ``tools/call``, ...) and a client that
  turns a remote server's tools into local tools;
* A2A (agent-to-agent, version ``2025-04-01``): a server running an :class:`Agent` per task
  (``tasks/send``, ``tasks/get``, ``tasks/cancel``, ``agent/info``) and its client.

Method names, payload shapes and error codes are the protocols' (reference:
``saint_llm_agents/mcp/*.py``, ``a2a/*.py``); one dispatch core serves both servers.
"""

from __future__ import annotations

import json
import logging
import queue
import sys
import uuid
from abc import ABC, abstractmethod
from collections.abc import Callable, Mapping
from dataclasses import dataclass, field
from typing import IO, Any, Literal

from saint_llm_b200.agents.core import Agent, FunctionTool, Message, Tool, ToolCall, ToolRegistry, ToolSpec

log = logging.getLogger(__name__)

MCP_PROTOCOL_VERSION = "2024-11-05"
A2A_PROTOCOL_VERSION = "2025-04-01"
PARSE_ERROR, INVALID_REQUEST, METHOD_NOT_FOUND, INVALID_PARAMS, INTERNAL_ERROR = -32700, -32600, -32601, -32602, -32603
TASK_NOT_FOUND = -32001


# ------------------------------------------------------------------ transports
class JsonRpcChannel(ABC):
    @abstractmethod
    def send(self, message: Mapping[str, Any]) -> None: ...

    @abstractmethod
    def receive(self) -> Mapping[str, Any] | None: ...

    def close(self) -> None:  # noqa: B027 - optional for transports without state
        pass


class InMemoryJsonRpcChannel(JsonRpcChannel):
    def __init__(self, inbox: queue.Queue, outbox: queue.Queue) -> None:
        self._in, self._out, self._closed = inbox, outbox, False

    def send(self, message: Mapping[str, Any]) -> None:
        if self._closed:
            raise RuntimeError("channel is closed")
        self._out.put(dict(message))

    def receive(self) -> Mapping[str, Any] | None:
        if self._closed:
            return None
        msg = self._in.get()
        if msg is None:
            self._closed = True
        return msg

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            self._out.put(None)


def pair_channels() -> tuple[InMemoryJsonRpcChannel, InMemoryJsonRpcChannel]:
    """(client side, server side) connected back to back."""
    a, b = queue.Queue(), queue.Queue()
    return InMemoryJsonRpcChannel(b, a), InMemoryJsonRpcChannel(a, b)


class StdioJsonRpcChannel(JsonRpcChannel):
    """One JSON object per line (MCP's local stdio transport)."""

    def __init__(self, reader: IO[str] | None = None, writer: IO[str] | None = None) -> None:
        self._r, self._w = reader or sys.stdin, writer or sys.stdout

    def send(self, message: Mapping[str, Any]) -> None:
        self._w.write(json.dumps(message, separators=(",", ":")) + "\n")
        self._w.flush()

    def receive(self) -> Mapping[str, Any] | None:
        line = self._r.readline()
        return json.loads(line) if line else None


# ------------------------------------------------------------------ server / client cores
class RpcError(Exception):
    def __init__(self, code: int, message: str) -> None:
        super().__init__(message)
        self.code, self.message = code, message


class JsonRpcServer:
    """Dispatch table server; subclasses fill ``self.methods``."""

    methods: dict[str, Callable[[Mapping[str, Any]], Any]]

    def serve(self, channel: JsonRpcChannel) -> None:
        while (msg := channel.receive()) is not None:
            self.handle_one(msg, channel)

    def handle_one(self, msg: Mapping[str, Any], channel: JsonRpcChannel) -> None:
        method, mid = msg.get("method"), msg.get("id")
        if method is None:
            return
        try:
            fn = self.methods.get(method)
            if fn is None:
                raise RpcError(METHOD_NOT_FOUND, f"method not found: {method}")
            result = fn(msg.get("params") or {})
        except RpcError as e:
            if mid is not None:
                channel.send({"jsonrpc": "2.0", "id": mid, "error": {"code": e.code, "message": e.message}})
            return
        except Exception as e:  # noqa: BLE001 - report, keep serving
            log.exception("json-rpc handler crashed for %s", method)
            if mid is not None:
                channel.send({"jsonrpc": "2.0", "id": mid,
                              "error": {"code": INTERNAL_ERROR, "message": f"internal error: {type(e).__name__}"}})
            return
        if mid is not None:
            channel.send({"jsonrpc": "2.0", "id": mid, "result": result})


class JsonRpcClient:
    def __init__(self, channel: JsonRpcChannel, error_type: type[Exception] = RuntimeError) -> None:
        self._ch, self._next, self._err = channel, 1, error_type

    def request(self, method: str, params: Mapping[str, Any] | None = None) -> Any:
        mid, self._next = self._next, self._next + 1
        msg: dict[str, Any] = {"jsonrpc": "2.0", "id": mid, "method": method}
        if params is not None:
            msg["params"] = dict(params)
        self._ch.send(msg)
        while True:
            reply = self._ch.receive()
            if reply is None:
                raise self._err(f"channel closed while waiting for {method}")
            if reply.get("id") != mid:
                continue
            if "error" in reply:
                err = reply["error"]
                raise self._err(f"{method} failed: [{err.get('code')}] {err.get('message')}")
            return reply.get("result")

    def notify(self, method: str, params: Mapping[str, Any] | None = None) -> None:
        msg: dict[str, Any] = {"jsonrpc": "2.0", "method": method}
        if params is not None:
            msg["params"] = dict(params)
        self._ch.send(msg)


# ------------------------------------------------------------------ MCP
class MCPClientError(RuntimeError):
    pass


class MCPServer(JsonRpcServer):
    def __init__(self, registry: ToolRegistry, *, server_name: str = "saint-llm-b200",
                 server_version: str = "0.1.0") -> None:
        self.registry, self.server_name, self.server_version = registry, server_name, server_version
        self._initialized = False
        self.methods = {
            "initialize": lambda p: {"protocolVersion": MCP_PROTOCOL_VERSION,
                                     "capabilities": {"tools": {}, "resources": {}, "prompts": {}},
                                     "serverInfo": {"name": self.server_name, "version": self.server_version}},
            "initialized": self._mark_init, "notifications/initialized": self._mark_init,
            "ping": lambda p: {},
            "tools/list": lambda p: {"tools": [{"name": s.name, "description": s.description,
                                                "inputSchema": dict(s.parameters) or {"type": "object",
                                                                                      "properties": {}}}
                                               for s in self.registry.specs()]},
            "tools/call": self._call,
            "resources/list": lambda p: {"resources": []},
            "prompts/list": lambda p: {"prompts": []},
        }

    def _mark_init(self, params: Mapping[str, Any]) -> None:
        self._initialized = True

    def _call(self, params: Mapping[str, Any]) -> dict[str, Any]:
        name, args = params.get("name"), params.get("arguments") or {}
        if not isinstance(name, str):
            raise RpcError(INVALID_PARAMS, "tools/call requires a string 'name'")
        if not isinstance(args, Mapping):
            raise RpcError(INVALID_PARAMS, "tools/call 'arguments' must be an object")
        if name not in self.registry:
            return {"content": [{"type": "text", "text": f"unknown tool: {name}"}], "isError": True}
        out = self.registry.execute(ToolCall(id="mcp", name=name, arguments=dict(args)))
        return {"content": [{"type": "text", "text": out.content}], "isError": out.content.startswith("ERROR:")}


def _mcp_connect(channel: JsonRpcChannel) -> tuple[JsonRpcClient, list[Mapping[str, Any]]]:
    c = JsonRpcClient(channel, MCPClientError)
    c.request("initialize", {"protocolVersion": MCP_PROTOCOL_VERSION, "capabilities": {},
                             "clientInfo": {"name": "saint-llm-b200", "version": "0.1.0"}})
    c.notify("notifications/initialized", {})
    res = c.request("tools/list", {})
    return c, list(res.get("tools", [])) if isinstance(res, Mapping) else []


def mcp_list_tools(channel: JsonRpcChannel) -> tuple[ToolSpec, ...]:
    _, raw = _mcp_connect(channel)
    return tuple(ToolSpec(r["name"], r.get("description", ""), r.get("inputSchema", {})) for r in raw)


def mcp_client_tools(channel: JsonRpcChannel, *, name_prefix: str = "") -> tuple[Tool, ...]:
    """Remote tools as local ones; ``isError`` results come back as text for the agent to read."""
    client, raw = _mcp_connect(channel)

    def caller(remote: str) -> Callable[..., str]:
        def call(**kwargs: Any) -> str:
            res = client.request("tools/call", {"name": remote, "arguments": kwargs})
            items = res.get("content", []) if isinstance(res, Mapping) else []
            return "\n".join(str(i.get("text", "")) for i in items
                             if isinstance(i, Mapping) and i.get("type") == "text")
        return call

    return tuple(FunctionTool(ToolSpec(f"{name_prefix}{r['name']}", r.get("description", ""),
                                       r.get("inputSchema", {})), caller(r["name"])) for r in raw)


# ------------------------------------------------------------------ A2A
TaskStatus = Literal["submitted", "working", "completed", "failed", "canceled"]


@dataclass
class A2ATask:
    id: str
    sessionId: str | None  # noqa: N815 - protocol field name
    status: TaskStatus
    message: str
    artifacts: list[dict[str, Any]] = field(default_factory=list)
    error: str | None = None

    def to_dict(self) -> dict[str, Any]:
        return {"id": self.id, "sessionId": self.sessionId, "status": self.status, "message": self.message,
                "artifacts": list(self.artifacts), "error": self.error}


class InMemoryTaskStore:
    def __init__(self) -> None:
        self._tasks: dict[str, A2ATask] = {}

    def put(self, task: A2ATask) -> None:
        self._tasks[task.id] = task

    def get(self, task_id: str) -> A2ATask | None:
        return self._tasks.get(task_id)

    def __len__(self) -> int:
        return len(self._tasks)


def final_response(history: list[Message]) -> str:
    """Last assistant message without tool calls, else the last assistant message."""
    asst = [m for m in history if m.role == "assistant"]
    done = [m for m in asst if not m.tool_calls]
    return (done or asst or [Message(role="assistant", content="")])[-1].content


class A2AServer(JsonRpcServer):
    def __init__(self, agent: Agent, *, store: InMemoryTaskStore | None = None, max_steps: int = 8,
                 server_name: str = "saint-llm-b200-a2a", server_version: str = "0.1.0") -> None:
        self.agent, self.store = agent, store or InMemoryTaskStore()
        self.max_steps, self.server_name, self.server_version = max_steps, server_name, server_version
        self.methods = {"ping": lambda p: {}, "agent/info": self._info, "tasks/send": self._send,
                        "tasks/get": self._get, "tasks/cancel": self._cancel}

    def _info(self, params: Mapping[str, Any]) -> dict[str, Any]:
        return {"name": self.agent.name,
                "tools": [{"name": s.name, "description": s.description} for s in self.agent.tools.specs()],
                "protocolVersion": A2A_PROTOCOL_VERSION,
                "serverInfo": {"name": self.server_name, "version": self.server_version}}

    def _send(self, params: Mapping[str, Any]) -> dict[str, Any]:
        text = params.get("message")
        if not isinstance(text, str) or not text:
            raise RpcError(INVALID_PARAMS, "tasks/send requires non-empty 'message'")
        sid = params.get("sessionId")
        task = A2ATask(str(params.get("id") or uuid.uuid4()), sid if isinstance(sid, str) else None, "working", text)
        self.store.put(task)
        try:
            hist = self.agent.run(user_message=text, max_steps=self.max_steps)
        except Exception as e:  # noqa: BLE001 - a failing agent fails the task, not the server
            task.status, task.error = "failed", f"{type(e).__name__}: {e}"
            return task.to_dict()
        task.artifacts, task.status = [{"type": "text", "text": final_response(hist)}], "completed"
        return task.to_dict()

    def _task(self, params: Mapping[str, Any]) -> A2ATask:
        tid = params.get("id")
        if not isinstance(tid, str):
            raise RpcError(INVALID_PARAMS, "task 'id' must be a string")
        task = self.store.get(tid)
        if task is None:
            raise RpcError(TASK_NOT_FOUND, f"task not found: {tid}")
        return task

    def _get(self, params: Mapping[str, Any]) -> dict[str, Any]:
        return self._task(params).to_dict()

    def _cancel(self, params: Mapping[str, Any]) -> dict[str, Any]:
        task = self._task(params)
        if task.status not in ("completed", "failed", "canceled"):
            task.status = "canceled"
        return task.to_dict()


class A2AClientError(RuntimeError):
    pass


class A2AClient(JsonRpcClient):
    def __init__(self, channel: JsonRpcChannel) -> None:
        super().__init__(channel, A2AClientError)

    def _dict(self, method: str, params: Mapping[str, Any]) -> dict[str, Any]:
        res = self.request(method, params)
        if not isinstance(res, Mapping):
            raise A2AClientError(f"{method} returned a non-object result")
        return dict(res)

    def send_task(self, message: str, *, session_id: str | None = None, task_id: str | None = None) -> dict[str, Any]:
        p: dict[str, Any] = {"message": message}
        if session_id is not None:
            p["sessionId"] = session_id
        if task_id is not None:
            p["id"] = task_id
        return self._dict("tasks/send", p)

    def get_task(self, task_id: str) -> dict[str, Any]:
        return self._dict("tasks/get", {"id": task_id})

    def cancel_task(self, task_id: str) -> dict[str, Any]:
        return self._dict("tasks/cancel", {"id": task_id})

    def agent_info(self) -> dict[str, Any]:
        return self._dict("agent/info", {})


def send_to_agent(channel: JsonRpcChannel, message: str, *, session_id: str | None = None) -> str:
    task = A2AClient(channel).send_task(message, session_id=session_id)
    return "\n".join(str(a.get("text", "")) for a in task.get("artifacts") or []
                     if isinstance(a, Mapping) and a.get("type") == "text")


__all__ = ["A2AClient", "A2AClientError", "A2AServer", "A2ATask", "A2A_PROTOCOL_VERSION", "InMemoryJsonRpcChannel",
           "InMemoryTaskStore", "JsonRpcChannel", "JsonRpcClient", "JsonRpcServer", "MCPClientError", "MCPServer",
           "MCP_PROTOCOL_VERSION", "RpcError", "StdioJsonRpcChannel", "final_response", "mcp_client_tools",
           "mcp_list_tools", "pair_channels", "send_to_agent"]
