"""Process sandboxes for tool / code execution (reference: ``saint_llm_sandbox``).

``FunctionCallSandbox`` runs a subprocess with an address-space cap (``RLIMIT_AS``), no
core dumps, a CPU-time cap, an optional network cut (a new network namespace when the
kernel allows unprivileged ones) and a wall-clock timeout after which the whole process
group is killed.  Container / micro-VM / full-VM backends are declared with the same
interface and raise ``NotImplementedError`` (no such runtime exists on these machines).
"""

from __future__ import annotations

import contextlib
import os
import resource
import signal
import subprocess
import sys
import time
from collections.abc import Mapping
from dataclasses import dataclass, field
from pathlib import Path
from typing import Protocol


@dataclass(frozen=True)
class SandboxResult:
    ok: bool
    exit_code: int
    stdout: str = ""
    stderr: str = ""
    duration_s: float = 0.0
    error: str | None = None
    files: dict[str, bytes] = field(default_factory=dict)


@dataclass(frozen=True)
class SandboxConfig:
    timeout_s: float = 30.0
    memory_mb: int = 1024
    cpu_cores: int = 1
    env: Mapping[str, str] = field(default_factory=dict)
    cwd: str = "/tmp"
    readonly: bool = True
    network: bool = False


class Sandbox(Protocol):
    def run(self, argv: list[str], *, stdin: bytes = b"", config: SandboxConfig | None = None) -> SandboxResult: ...

    def run_python(self, code: str, *, config: SandboxConfig | None = None) -> SandboxResult: ...


def _limits(cfg: SandboxConfig) -> None:  # runs in the child before exec
    os.setsid()
    mem = max(1, cfg.memory_mb) * 1024 * 1024
    for res, val in ((resource.RLIMIT_AS, mem), (resource.RLIMIT_CORE, 0),
                     (resource.RLIMIT_CPU, max(1, int(cfg.timeout_s) + 1))):
        with contextlib.suppress(ValueError, OSError):
            resource.setrlimit(res, (val, val))
    if cfg.cpu_cores > 0 and hasattr(os, "sched_setaffinity"):
        with contextlib.suppress(OSError):
            cpus = sorted(os.sched_getaffinity(0))[: cfg.cpu_cores]
            os.sched_setaffinity(0, cpus)
    if not cfg.network and hasattr(os, "unshare") and hasattr(os, "CLONE_NEWNET"):
        with contextlib.suppress(OSError):  # unprivileged user namespaces may be disabled
            os.unshare(os.CLONE_NEWUSER | os.CLONE_NEWNET)


class FunctionCallSandbox:
    def __init__(self, *, python_exe: str | None = None) -> None:
        self._python = python_exe or sys.executable or "python3"

    def run(self, argv: list[str], *, stdin: bytes = b"", config: SandboxConfig | None = None) -> SandboxResult:
        cfg = config or SandboxConfig()
        env = dict(cfg.env) if cfg.env else dict(os.environ)
        t0 = time.perf_counter()
        try:
            proc = subprocess.Popen(argv, stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                    env=env, cwd=str(Path(cfg.cwd)) if cfg.cwd else None,
                                    preexec_fn=(lambda: _limits(cfg)) if os.name == "posix" else None)
        except (FileNotFoundError, PermissionError) as e:
            return SandboxResult(False, -1, duration_s=time.perf_counter() - t0, error=f"executable not found: {e}")
        try:
            out, err = proc.communicate(stdin, timeout=cfg.timeout_s)
        except subprocess.TimeoutExpired:
            with contextlib.suppress(ProcessLookupError):
                os.killpg(proc.pid, signal.SIGKILL)
            out, err = proc.communicate()
            return SandboxResult(False, -1, out.decode(errors="replace"), err.decode(errors="replace"),
                                 time.perf_counter() - t0, f"timeout after {cfg.timeout_s}s")
        return SandboxResult(proc.returncode == 0, proc.returncode, out.decode(errors="replace"),
                             err.decode(errors="replace"), time.perf_counter() - t0)

    def run_python(self, code: str, *, config: SandboxConfig | None = None) -> SandboxResult:
        return self.run([self._python, "-c", code], config=config)


class _Unavailable:
    name = "unavailable"

    def run(self, argv: list[str], *, stdin: bytes = b"", config: SandboxConfig | None = None) -> SandboxResult:
        raise NotImplementedError(f"{self.name} sandbox is not available; use FunctionCallSandbox")

    def run_python(self, code: str, *, config: SandboxConfig | None = None) -> SandboxResult:
        raise NotImplementedError(f"{self.name} sandbox is not available; use FunctionCallSandbox")


class ContainerSandbox(_Unavailable):
    name = "container"


class MicroVMSandbox(_Unavailable):
    name = "microvm"


class FullVMSandbox(_Unavailable):
    name = "fullvm"


__all__ = ["ContainerSandbox", "FullVMSandbox", "FunctionCallSandbox", "MicroVMSandbox", "Sandbox", "SandboxConfig",
           "SandboxResult"]
