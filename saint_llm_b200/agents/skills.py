"""Skills: directories with a ``SKILL.md`` (front matter ``name``, ``description``, optional
``license`` and ``allowed-tools``, then Markdown instructions) and an optional ``scripts/``
folder (reference: ``saint_llm_agents/skills/*.py``).  Skills can be exposed to an agent as
``use_<name>`` tools returning their instructions, and their scripts as tools run by a
script runner (a sandbox by default)."""

from __future__ import annotations

import json
from collections.abc import Iterable, Iterator, Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Literal, Protocol

from saint_llm_b200.agents.core import FunctionTool, ToolRegistry, ToolSpec

SKILL_FILE_NAME = "SKILL.md"


class SkillLoadError(ValueError):
    pass


@dataclass(frozen=True)
class Skill:
    name: str
    description: str
    instructions: str
    license: str | None = None
    allowed_tools: tuple[str, ...] = ()
    root: Path | None = None

    @property
    def scripts_dir(self) -> Path | None:
        d = self.root / "scripts" if self.root is not None else None
        return d if d is not None and d.is_dir() else None


def _unquote(v: str) -> str:
    return v[1:-1] if len(v) >= 2 and v[0] == v[-1] and v[0] in "\"'" else v


def parse_front_matter(text: str, *, source: str = "<front matter>") -> dict[str, str | list[str]]:
    """The flat subset used by skill front matter: ``key: value`` and ``key:`` + indented ``- items``."""
    out: dict[str, str | list[str]] = {}
    key: str | None = None
    items: list[str] = []

    def flush() -> None:
        nonlocal key, items
        if key is not None and items:
            out[key] = items
        key, items = None, []

    for raw in text.splitlines():
        line = raw.rstrip()
        body = line.lstrip()
        if not body or body.startswith("#"):
            continue
        if body.startswith("- ") and key is not None and len(line) > len(body):
            items.append(_unquote(body[2:].strip()))
            continue
        flush()
        if ":" not in body:
            raise SkillLoadError(f"{source}: expected 'key: value', got {body!r}")
        k, _, v = body.partition(":")
        k, v = k.strip(), v.strip()
        if not k:
            raise SkillLoadError(f"{source}: empty key in {body!r}")
        if v:
            out[k] = _unquote(v)
        else:
            key = k
    flush()
    return out


def load_skill(skill_dir: Path | str) -> Skill:
    skill_dir = Path(skill_dir)
    md = skill_dir / SKILL_FILE_NAME
    if not md.is_file():
        raise SkillLoadError(f"missing {SKILL_FILE_NAME} in {skill_dir}")
    lines = md.read_text(encoding="utf-8").splitlines()
    meta: dict[str, str | list[str]] = {}
    body = "\n".join(lines)
    if lines and lines[0].strip() == "---":
        end = next((i for i in range(1, len(lines)) if lines[i].strip() == "---"), -1)
        if end < 0:
            raise SkillLoadError(f"{md}: unterminated front matter")
        meta = parse_front_matter("\n".join(lines[1:end]), source=str(md))
        body = "\n".join(lines[end + 1:])
    if not meta.get("name"):
        raise SkillLoadError(f"{md}: front matter missing 'name'")
    allowed = meta.get("allowed-tools") or meta.get("allowed_tools")
    allowed_t = tuple(x.strip() for x in allowed.split(",") if x.strip()) if isinstance(allowed, str) else \
        tuple(map(str, allowed or ()))
    lic = meta.get("license")
    return Skill(str(meta["name"]), str(meta.get("description") or ""), body.strip(), str(lic) if lic else None,
                 allowed_t, skill_dir)


def load_skills(root: Path | str) -> tuple[Skill, ...]:
    root = Path(root)
    if not root.is_dir():
        raise SkillLoadError(f"skills root is not a directory: {root}")
    if (root / SKILL_FILE_NAME).is_file():
        return (load_skill(root),)
    return tuple(load_skill(p) for p in sorted(root.iterdir())
                 if p.is_dir() and not p.name.startswith(".") and (p / SKILL_FILE_NAME).is_file())


class SkillRegistry:
    def __init__(self, skills: Iterable[Skill] = ()) -> None:
        self._skills: dict[str, Skill] = {}
        for s in skills:
            self.add(s)

    def add(self, skill: Skill) -> None:
        if skill.name in self._skills:
            raise ValueError(f"skill {skill.name!r} already registered")
        self._skills[skill.name] = skill

    def get(self, name: str) -> Skill:
        if name not in self._skills:
            raise KeyError(f"skill {name!r} not registered")
        return self._skills[name]

    def names(self) -> tuple[str, ...]:
        return tuple(self._skills)

    def __contains__(self, name: object) -> bool:
        return isinstance(name, str) and name in self._skills

    def __len__(self) -> int:
        return len(self._skills)

    def __iter__(self) -> Iterator[Skill]:
        return iter(self._skills.values())

    def catalog(self, *, header: str = "Available skills:") -> str:
        if not self._skills:
            return ""
        return "\n".join([header] + [f"- {s.name}: {s.description or '(no description)'}" for s in self])


def register_skills_as_tools(registry: ToolRegistry, skills: Sequence[Skill] | SkillRegistry, *,
                             tool_name_prefix: str = "use_") -> None:
    for s in skills:
        text = s.instructions
        registry.register(FunctionTool(
            ToolSpec(f"{tool_name_prefix}{s.name}", f"Load instructions for the {s.name!r} skill. "
                     f"Description: {s.description}".strip(), {"type": "object", "properties": {}, "required": []}),
            lambda _t=text, **_: _t))


@dataclass(frozen=True)
class ScriptResult:
    ok: bool
    stdout: str
    stderr: str = ""
    exit_code: int = 0


class ScriptRunner(Protocol):
    def run(self, script_path: Path, args: Sequence[str]) -> ScriptResult: ...


class SandboxScriptRunner:
    """Runs ``python <script> args...`` (``.py``) or the file itself in a resource-limited subprocess."""

    def __init__(self, *, timeout_s: float = 30.0, memory_mb: int = 1024) -> None:
        from saint_llm_b200.sandbox import FunctionCallSandbox, SandboxConfig

        self._sb = FunctionCallSandbox()
        self._cfg = SandboxConfig(timeout_s=timeout_s, memory_mb=memory_mb, cwd="")

    def run(self, script_path: Path, args: Sequence[str]) -> ScriptResult:
        import sys

        argv = ([sys.executable, str(script_path)] if script_path.suffix == ".py" else [str(script_path)]) + list(args)
        r = self._sb.run(argv, config=self._cfg)
        return ScriptResult(r.ok, r.stdout, r.stderr or (r.error or ""), r.exit_code)


def kwargs_to_argv(kwargs: dict[str, Any], *, arg_format: Literal["flags", "json"]) -> list[str]:
    """``flags``: ``--key value`` (``--key`` / ``--no-key`` for booleans); ``json``: one JSON argument."""
    if arg_format == "json":
        return [json.dumps(kwargs)]
    if arg_format != "flags":
        raise ValueError(f"unknown arg_format {arg_format!r}")
    argv: list[str] = []
    for k, v in kwargs.items():
        flag = k.replace("_", "-")
        argv += [f"--{flag}"] if v is True else [f"--no-{flag}"] if v is False else [f"--{flag}", str(v)]
    return argv


def register_skill_scripts(registry: ToolRegistry, skill: Skill, runner: ScriptRunner | None = None, *,
                           arg_format: Literal["flags", "json"] = "flags", tool_name_prefix: str | None = None) -> int:
    if skill.scripts_dir is None:
        return 0
    runner = runner or SandboxScriptRunner()
    prefix = f"{skill.name}_" if tool_name_prefix is None else tool_name_prefix
    n = 0
    for path in sorted(skill.scripts_dir.iterdir()):
        if not path.is_file() or path.name.startswith("."):
            continue

        def call(_p: Path = path, **kw: Any) -> str:
            r = runner.run(_p, kwargs_to_argv(kw, arg_format=arg_format))
            return r.stdout if r.ok else f"ERROR (exit {r.exit_code}): {r.stderr.strip() or r.stdout}"

        how = "--key value flags" if arg_format == "flags" else "a single JSON positional"
        registry.register(FunctionTool(ToolSpec(f"{prefix}{path.stem}",
                                                f"Run the {path.name!r} script from skill {skill.name!r}. "
                                                f"Arguments are forwarded as {how}.",
                                                {"type": "object", "properties": {}, "additionalProperties": True}),
                                       call))
        n += 1
    return n


__all__ = ["SKILL_FILE_NAME", "SandboxScriptRunner", "ScriptResult", "ScriptRunner", "Skill", "SkillLoadError",
           "SkillRegistry", "kwargs_to_argv", "load_skill", "load_skills", "parse_front_matter",
           "register_skill_scripts", "register_skills_as_tools"]
