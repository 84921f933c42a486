"""Agent building blocks: messages and tool calls, tools and the registry, policies, the
think -> act -> observe agent loop and a round-robin multi-agent runtime
(reference: ``saint_llm_agents/{message,tool,policy,lm_policy,agent,runtime}.py``)."""

from __future__ import annotations

from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass, field, replace
from typing import Any, Literal, Protocol


@dataclass(frozen=True)
class ToolCall:
    id: str
    name: str
    arguments: Mapping[str, Any] = field(default_factory=dict)


@dataclass(frozen=True)
class Message:
    role: str
    content: str
    tool_calls: tuple[ToolCall, ...] = ()
    tool_call_id: str | None = None
    name: str | None = None

    def __post_init__(self) -> None:
        if self.role == "tool" and self.tool_call_id is None:
            raise ValueError("tool messages must reference a tool_call_id")
        if self.tool_calls and self.role != "assistant":
            raise ValueError(f"only assistant messages may carry tool_calls; got role={self.role!r}")


@dataclass(frozen=True)
class ToolSpec:
    """Name, description and JSON-Schema parameters (the OpenAI/Anthropic/MCP tool shape)."""

    name: str
    description: str
    parameters: Mapping[str, Any] = field(default_factory=dict)


class Tool(Protocol):
    spec: ToolSpec

    def __call__(self, **kwargs: Any) -> Any: ...


@dataclass(frozen=True)
class FunctionTool:
    spec: ToolSpec
    fn: Callable[..., Any]

    def __call__(self, **kwargs: Any) -> Any:
        return self.fn(**kwargs)


class ToolRegistry:
    def __init__(self) -> None:
        self._tools: dict[str, Tool] = {}

    def register(self, tool: Tool) -> None:
        if tool.spec.name in self._tools:
            raise ValueError(f"tool {tool.spec.name!r} already registered")
        self._tools[tool.spec.name] = tool

    def get(self, name: str) -> Tool:
        if name not in self._tools:
            raise KeyError(f"tool {name!r} not registered")
        return self._tools[name]

    def specs(self) -> tuple[ToolSpec, ...]:
        return tuple(t.spec for t in self._tools.values())

    def execute(self, call: ToolCall) -> Message:
        """Run a call; errors become ``"ERROR: <type>: <text>"`` results the model can read."""
        try:
            res = self.get(call.name)(**dict(call.arguments))
            content = "" if res is None else str(res)
        except Exception as e:  # noqa: BLE001 - a failing tool must not kill the agent loop
            content = f"ERROR: {type(e).__name__}: {e}"
        return Message(role="tool", content=content, tool_call_id=call.id)

    def __len__(self) -> int:
        return len(self._tools)

    def __contains__(self, name: object) -> bool:
        return isinstance(name, str) and name in self._tools


class Policy(Protocol):
    def act(self, messages: Sequence[Message], *, tools: Sequence[ToolSpec] = ()) -> Message: ...


class CallablePolicy:
    def __init__(self, fn: Callable[..., Message]) -> None:
        self._fn = fn

    def act(self, messages: Sequence[Message], *, tools: Sequence[ToolSpec] = ()) -> Message:
        return self._fn(messages, tools=tools)


class MockPolicy:
    """Replays fixed responses; raises ``StopIteration`` when exhausted."""

    def __init__(self, responses: Sequence[Message]) -> None:
        self._responses, self._idx = list(responses), 0

    def act(self, messages: Sequence[Message], *, tools: Sequence[ToolSpec] = ()) -> Message:
        if self._idx >= len(self._responses):
            raise StopIteration("MockPolicy exhausted")
        self._idx += 1
        return self._responses[self._idx - 1]

    @property
    def remaining(self) -> int:
        return len(self._responses) - self._idx


GenerateFn = Callable[[Sequence[Message]], str]


class TextLMPolicy:
    """Text generator + tool-call parsing (``xml`` / ``json`` / ``auto`` / ``none``)."""

    def __init__(self, generate: GenerateFn, *, parse_format: Literal["xml", "json", "auto", "none"] = "auto",
                 strict: bool = False) -> None:
        self._generate, self._fmt, self._strict = generate, parse_format, strict

    def act(self, messages: Sequence[Message], *, tools: Sequence[ToolSpec] = ()) -> Message:
        from saint_llm_b200.agents.parsing import parse_tool_calls

        text = self._generate(messages)
        if not isinstance(text, str):
            raise TypeError(f"generate(history) must return str; got {type(text).__name__}")
        calls = () if self._fmt == "none" else tuple(parse_tool_calls(text, fmt=self._fmt, strict=self._strict))
        return Message(role="assistant", content=text, tool_calls=calls)


class Agent:
    def __init__(self, *, name: str, policy: Policy, system: str = "", tools: ToolRegistry | None = None) -> None:
        self.name, self.policy = name, policy
        self.tools = tools if tools is not None else ToolRegistry()
        self.history: list[Message] = [Message(role="system", content=system)] if system else []

    def step(self, inbox: Sequence[Message] = ()) -> list[Message]:
        self.history.extend(inbox)
        msg = self.policy.act(self.history, tools=self.tools.specs())
        if msg.role != "assistant":
            raise ValueError(f"policy for agent {self.name!r} returned role={msg.role!r}; must be 'assistant'")
        if msg.name is None:
            msg = replace(msg, name=self.name)
        produced = [msg] + [self.tools.execute(c) for c in msg.tool_calls]
        self.history.extend(produced)
        return produced

    def run(self, *, user_message: str, max_steps: int = 8) -> list[Message]:
        if max_steps <= 0:
            raise ValueError(f"max_steps must be positive; got {max_steps}")
        produced = self.step([Message(role="user", content=user_message)])
        for _ in range(max_steps - 1):
            if not produced[0].tool_calls:
                break
            produced = self.step()
        return list(self.history)


@dataclass
class _Seat:
    """One agent at the round table and the messages waiting for it."""

    agent: Agent
    waiting: list[Message] = field(default_factory=list)

    def take(self) -> list[Message]:
        got, self.waiting = self.waiting, []
        return got


class Runtime:
    """Several agents taking turns (reference ``agents/runtime.py``: round-robin, each
    agent's non-empty assistant text goes to the next agent as a user message).

    The table is a ring of seats; ``tick()`` lets the agent at the current seat act on
    everything queued for it, appends what it produced to the shared transcript and
    passes its spoken text (assistant messages with content; tool traffic stays private)
    to the next seat, then moves on."""

    def __init__(self, agents: Sequence[Agent]) -> None:
        seats = [_Seat(a) for a in agents]
        if len(seats) < 2:
            raise ValueError(f"a Runtime is a conversation between agents: pass two or more (got {len(seats)})")
        by_name: dict[str, _Seat] = {}
        for seat in seats:
            if seat.agent.name in by_name:
                raise ValueError(f"two agents share the name {seat.agent.name!r}; names address the inboxes")
            by_name[seat.agent.name] = seat
        self._seats = seats
        self._by_name = by_name
        self._turn = 0
        self._log: list[Message] = []

    @property
    def agents(self) -> tuple[Agent, ...]:
        return tuple(seat.agent for seat in self._seats)

    @property
    def transcript(self) -> list[Message]:
        return list(self._log)

    @property
    def cursor(self) -> int:
        return self._turn % len(self._seats)

    def _seat(self, name: str) -> _Seat:
        try:
            return self._by_name[name]
        except KeyError:
            raise KeyError(f"no agent named {name!r} at this table") from None

    def inbox_for(self, name: str) -> list[Message]:
        return list(self._seat(name).waiting)

    def send(self, *, to: str, content: str, sender: str = "user") -> None:
        """Queue an outside message for agent ``to`` (it is also logged)."""
        msg = Message(role="user", content=content, name=sender)
        self._seat(to).waiting.append(msg)
        self._log.append(msg)

    def tick(self) -> list[Message]:
        n = len(self._seats)
        seat, nxt = self._seats[self._turn % n], self._seats[(self._turn + 1) % n]
        produced = seat.agent.step(seat.take())
        self._log += produced
        spoken = [m.content for m in produced if m.role == "assistant" and m.content]
        nxt.waiting += [Message(role="user", content=text, name=seat.agent.name) for text in spoken]
        self._turn = (self._turn + 1) % n
        return produced

    def run(self, *, max_ticks: int = 20) -> list[Message]:
        """Exactly ``max_ticks`` turns; returns the transcript."""
        if max_ticks < 1:
            raise ValueError(f"max_ticks={max_ticks}: run needs at least one turn")
        for _ in range(max_ticks):
            self.tick()
        return self.transcript


__all__ = ["Agent", "CallablePolicy", "FunctionTool", "GenerateFn", "Message", "MockPolicy", "Policy", "Runtime",
           "TextLMPolicy", "Tool", "ToolCall", "ToolRegistry", "ToolSpec"]
