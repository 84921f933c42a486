"""Code Mode: the model writes a Python snippet against a generated ``tools`` API instead of
emitting tool-call envelopes; an executor runs it with the tools bound
(reference: ``saint_llm_agents/code_mode/*.py``).

Executors: ``InProcessExecutor`` (``exec`` in a fresh scope -- trusted code only) and
``SandboxExecutor``, which runs the snippet in a :class:`FunctionCallSandbox` subprocess and
serves its tool calls over a pipe, so untrusted code never shares the interpreter with the
registry.
"""

from __future__ import annotations

import contextlib
import io
import json
import os
import subprocess
import sys
import textwrap
import traceback
from collections.abc import Sequence
from dataclasses import dataclass, field
from typing import Any, Protocol

from saint_llm_b200.agents.core import Message, Policy, ToolRegistry, ToolSpec


@dataclass(frozen=True)
class ApiStub:
    source: str
    names: tuple[str, ...]


def _param_doc(params: dict) -> str:
    props = (params or {}).get("properties", {})
    if not props:
        return "    No parameters."
    req = set(params.get("required", []))
    lines = ["    Args:"]
    for name, sch in props.items():
        line = f"        {name} ({sch.get('type', 'any')}){' (required)' if name in req else ''}"
        if sch.get("description"):
            line += f": {sch['description']}"
        lines.append(line)
    return "\n".join(lines)


def generate_api_stub(specs: list[ToolSpec], *, namespace: str = "tools") -> ApiStub:
    """Python source declaring ``class <namespace>`` with one documented static method per tool."""
    if not specs:
        return ApiStub(f"class {namespace}:\n    pass\n", ())
    lines = [f"class {namespace}:"]
    for s in specs:
        lines += ["    @staticmethod", f"    def {s.name}(**kwargs):", f'        """{s.description}\n',
                  _param_doc(dict(s.parameters)), '        """', "        ...  # runtime-bound", ""]
    return ApiStub("\n".join(lines), tuple(s.name for s in specs))


@dataclass
class ExecutionResult:
    ok: bool
    stdout: str = ""
    stderr: str = ""
    return_value: Any = None
    error_type: str | None = None
    error_message: str | None = None
    tool_calls: list[dict[str, Any]] = field(default_factory=list)


class Executor(Protocol):
    def execute(self, code: str, *, registry: ToolRegistry) -> ExecutionResult: ...


class _Namespace:
    def __init__(self, registry: ToolRegistry, log: list[dict[str, Any]]) -> None:
        self._r, self._log = registry, log

    def __getattr__(self, name: str) -> Any:
        if name.startswith("_") or name not in self._r:
            raise AttributeError(f"tool {name!r} is not registered")
        tool = self._r.get(name)

        def call(**kw: Any) -> Any:
            self._log.append({"name": name, "arguments": dict(kw)})
            return tool(**kw)

        return call


class InProcessExecutor:
    """NOT a security boundary: for trusted snippets (tests, development)."""

    def execute(self, code: str, *, registry: ToolRegistry) -> ExecutionResult:
        log: list[dict[str, Any]] = []
        scope: dict[str, Any] = {"tools": _Namespace(registry, log), "RESULT": None}
        out, err = io.StringIO(), io.StringIO()
        try:
            with contextlib.redirect_stdout(out), contextlib.redirect_stderr(err):
                exec(code, scope)  # noqa: S102 - the point of this executor
            return ExecutionResult(True, out.getvalue(), err.getvalue(), scope.get("RESULT"), tool_calls=log)
        except Exception as e:  # noqa: BLE001
            return ExecutionResult(False, out.getvalue(), err.getvalue() + traceback.format_exc(), None,
                                   type(e).__name__, str(e), log)


_CHILD = textwrap.dedent('''
    import contextlib, io, json, os, sys, traceback
    rd, wr = os.fdopen(int(sys.argv[1]), "r"), os.fdopen(int(sys.argv[2]), "w")
    class _T:
        def __getattr__(self, name):
            if name.startswith("_"):
                raise AttributeError(name)
            def call(**kw):
                wr.write(json.dumps({"call": name, "arguments": kw}) + "\\n"); wr.flush()
                rep = json.loads(rd.readline())
                if "error" in rep:
                    raise AttributeError(rep["error"]) if rep.get("kind") == "missing" else RuntimeError(rep["error"])
                return rep["result"]
            return call
    code = sys.stdin.read()
    scope = {"tools": _T(), "RESULT": None}
    out, err = io.StringIO(), io.StringIO()
    try:
        with contextlib.redirect_stdout(out), contextlib.redirect_stderr(err):
            exec(code, scope)
        res = {"ok": True, "result": repr(scope.get("RESULT")) if scope.get("RESULT") is not None else None}
    except Exception as e:
        res = {"ok": False, "etype": type(e).__name__, "emsg": str(e), "tb": traceback.format_exc()}
    res.update(stdout=out.getvalue(), stderr=err.getvalue())
    wr.write(json.dumps({"done": res}) + "\\n"); wr.flush()
''')


class SandboxExecutor:
    """Runs the snippet in a resource-limited subprocess; tool calls travel over a pipe pair and
    execute in this process.  ``return_value`` is the ``repr`` of the child's ``RESULT``."""

    def __init__(self, *, timeout_s: float = 30.0, memory_mb: int = 1024) -> None:
        self.timeout_s, self.memory_mb = timeout_s, memory_mb

    def execute(self, code: str, *, registry: ToolRegistry) -> ExecutionResult:
        import resource
        import select
        import time

        c2p_r, c2p_w = os.pipe()
        p2c_r, p2c_w = os.pipe()
        mem = self.memory_mb * 1024 * 1024

        def limits() -> None:
            os.setsid()
            with contextlib.suppress(ValueError, OSError):
                resource.setrlimit(resource.RLIMIT_AS, (mem, mem))
                resource.setrlimit(resource.RLIMIT_CORE, (0, 0))

        proc = subprocess.Popen([sys.executable, "-c", _CHILD, str(p2c_r), str(c2p_w)], stdin=subprocess.PIPE,
                                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL, pass_fds=(p2c_r, c2p_w),
                                preexec_fn=limits)
        os.close(p2c_r)
        os.close(c2p_w)
        log: list[dict[str, Any]] = []
        done: dict[str, Any] | None = None
        deadline = time.monotonic() + self.timeout_s
        with os.fdopen(c2p_r, "r") as rd, os.fdopen(p2c_w, "w") as wr:
            proc.stdin.write(code.encode())
            proc.stdin.close()
            while done is None:
                left = deadline - time.monotonic()
                if left <= 0 or not select.select([rd], [], [], left)[0]:
                    break
                line = rd.readline()
                if not line:
                    break
                msg = json.loads(line)
                if "done" in msg:
                    done = msg["done"]
                    break
                name, kw = msg["call"], msg.get("arguments", {})
                log.append({"name": name, "arguments": kw})
                if name not in registry:
                    rep = {"error": f"tool {name!r} is not registered", "kind": "missing"}
                else:
                    try:
                        rep = {"result": registry.get(name)(**kw)}
                        json.dumps(rep)
                    except Exception as e:  # noqa: BLE001
                        rep = {"error": f"{type(e).__name__}: {e}"}
                wr.write(json.dumps(rep, default=str) + "\n")
                wr.flush()
        if proc.poll() is None:
            with contextlib.suppress(ProcessLookupError):
                os.killpg(proc.pid, 9)
        proc.wait()
        if done is None:
            return ExecutionResult(False, error_type="TimeoutError" if time.monotonic() >= deadline else "ChildExited",
                                   error_message=f"no result within {self.timeout_s}s", tool_calls=log)
        if done["ok"]:
            return ExecutionResult(True, done["stdout"], done["stderr"], done["result"], tool_calls=log)
        return ExecutionResult(False, done["stdout"], done["stderr"] + done.get("tb", ""), None, done["etype"],
                               done["emsg"], log)


DEFAULT_CODE_MODE_PREFIX = ("You are operating in Code Mode. Write a short Python snippet that calls the tools API "
                            "below. Do NOT explain — output only executable Python. Assign your final answer to "
                            "``RESULT``.\n\n")


@dataclass
class CodeModePolicy:
    base_policy: Policy
    registry: ToolRegistry
    executor: Executor | None = None
    api_namespace: str = "tools"
    prompt_prefix: str = DEFAULT_CODE_MODE_PREFIX

    def __post_init__(self) -> None:
        if self.executor is None:
            self.executor = InProcessExecutor()

    def act(self, messages: Sequence[Message], *, tools: Sequence[ToolSpec] = ()) -> Message:
        stub = generate_api_stub(list(self.registry.specs()), namespace=self.api_namespace)
        sys_msg = Message(role="system", content=f"{self.prompt_prefix}```python\n{stub.source}\n```")
        draft = self.base_policy.act([sys_msg, *messages], tools=())
        if draft.role != "assistant":
            raise ValueError(f"Code Mode base policy must return assistant; got {draft.role!r}")
        res = self.executor.execute(draft.content, registry=self.registry)  # type: ignore[union-attr]
        if res.ok:
            text = (f"Code Mode result: {res.return_value!r}" if res.return_value is not None
                    else "Code Mode result: (no RESULT assigned)")
            if res.stdout:
                text += f"\n[stdout]\n{res.stdout}"
        else:
            text = f"Code Mode error: {res.error_type}: {res.error_message}"
            if res.stderr:
                text += f"\n[stderr]\n{res.stderr}"
        return Message(role="assistant", content=text, name="code_mode")


__all__ = ["ApiStub", "CodeModePolicy", "ExecutionResult", "Executor", "InProcessExecutor", "SandboxExecutor",
           "generate_api_stub"]
