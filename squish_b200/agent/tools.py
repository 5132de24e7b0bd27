"""Tool registry and built-in tools for the agent loop.

Same shape as the reference's ToolRegistry (squish/agent/tool_registry.py:128-400): tools are
(name, description, JSON-schema parameters, callable); arguments are checked against the schema
(required keys, no unknown keys) with lenient coercion of the strings models often emit for
numbers / booleans / JSON values; a call returns a ToolResult that renders as an OpenAI
``tool`` message. Built-in tools (squish/agent/builtin_tools.py) read, write and list files
under a sandbox root; the shell tool is registered only when explicitly enabled.
"""
from __future__ import annotations

import json
import os
import subprocess
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable


class ToolCallError(Exception):
    pass


@dataclass
class ToolDefinition:
    name: str
    description: str
    parameters: dict
    fn: Callable[..., Any]
    source: str = "builtin"

    def to_openai_schema(self) -> dict:
        return {"type": "function", "function": {"name": self.name, "description": self.description,
                                                 "parameters": self.parameters}}


@dataclass
class ToolResult:
    call_id: str
    name: str
    content: str
    error: str | None = None
    elapsed_ms: float = 0.0

    @property
    def ok(self) -> bool:
        return self.error is None

    def to_message(self) -> dict:
        return {"role": "tool", "tool_call_id": self.call_id, "name": self.name,
                "content": self.content if self.ok else f"error: {self.error}"}


def _coerce(value: Any, typ: str | None) -> Any:
    if typ == "integer":
        if isinstance(value, bool):
            raise ToolCallError("expected an integer, got a boolean")
        if isinstance(value, float) and value.is_integer():
            return int(value)
        if isinstance(value, str):
            try:
                return int(value.strip())
            except ValueError as exc:
                raise ToolCallError(f"expected an integer, got {value!r}") from exc
        if not isinstance(value, int):
            raise ToolCallError(f"expected an integer, got {type(value).__name__}")
        return value
    if typ == "number":
        if isinstance(value, bool):
            raise ToolCallError("expected a number, got a boolean")
        if isinstance(value, str):
            try:
                return float(value.strip())
            except ValueError as exc:
                raise ToolCallError(f"expected a number, got {value!r}") from exc
        if not isinstance(value, (int, float)):
            raise ToolCallError(f"expected a number, got {type(value).__name__}")
        return value
    if typ == "boolean":
        if isinstance(value, str) and value.strip().lower() in ("true", "false"):
            return value.strip().lower() == "true"
        if not isinstance(value, bool):
            raise ToolCallError(f"expected a boolean, got {value!r}")
        return value
    if typ in ("object", "array"):
        if isinstance(value, str):
            try:
                value = json.loads(value)
            except ValueError as exc:
                raise ToolCallError(f"expected JSON {typ}") from exc
        if not isinstance(value, dict if typ == "object" else list):
            raise ToolCallError(f"expected an {typ}")
        return value
    if typ == "string" and not isinstance(value, str):
        return json.dumps(value) if isinstance(value, (dict, list)) else str(value)
    return value


class ToolRegistry:
    def __init__(self) -> None:
        self._tools: dict[str, ToolDefinition] = {}

    def register(self, defn: ToolDefinition) -> None:
        self._tools[defn.name] = defn

    def tool(self, name: str, description: str, parameters: dict):
        def deco(fn):
            self.register(ToolDefinition(name, description, parameters, fn))
            return fn

        return deco

    def unregister(self, name: str) -> None:
        self._tools.pop(name, None)

    def get(self, name: str) -> ToolDefinition | None:
        return self._tools.get(name)

    def names(self) -> list[str]:
        return sorted(self._tools)

    def __contains__(self, name: str) -> bool:
        return name in self._tools

    def __len__(self) -> int:
        return len(self._tools)

    def to_openai_schemas(self) -> list[dict]:
        return [self._tools[n].to_openai_schema() for n in self.names()]

    def validate_call(self, name: str, arguments: dict) -> dict:
        d = self._tools.get(name)
        if d is None:
            raise ToolCallError(f"unknown tool {name!r}")
        if not isinstance(arguments, dict):
            raise ToolCallError("arguments must be a JSON object")
        props = d.parameters.get("properties", {})
        missing = [r for r in d.parameters.get("required", []) if r not in arguments]
        if missing:
            raise ToolCallError(f"missing required argument(s) {missing}")
        unknown = [k for k in arguments if props and k not in props]
        if unknown:
            raise ToolCallError(f"unknown argument(s) {unknown}")
        return {k: _coerce(v, props.get(k, {}).get("type")) for k, v in arguments.items()}

    def call(self, name: str, arguments: dict | str, call_id: str = "") -> ToolResult:
        t0 = time.perf_counter()
        try:
            args = json.loads(arguments) if isinstance(arguments, str) else dict(arguments or {})
            args = self.validate_call(name, args)
            out = self._tools[name].fn(**args)
            content = out if isinstance(out, str) else json.dumps(out)
            return ToolResult(call_id, name, content, None, (time.perf_counter() - t0) * 1e3)
        except Exception as exc:  # noqa: BLE001 - reported to the model as the tool's error
            return ToolResult(call_id, name, "", f"{type(exc).__name__}: {exc}", (time.perf_counter() - t0) * 1e3)


# ------------------------------------------------------------------------------ built-ins
@dataclass
class Sandbox:
    root: Path = field(default_factory=lambda: Path(os.environ.get("SQUISH_AGENT_ROOT", os.getcwd())).resolve())
    max_bytes: int = 1 << 20

    def path(self, p: str) -> Path:
        q = (self.root / p).resolve() if not os.path.isabs(p) else Path(p).resolve()
        if q != self.root and self.root not in q.parents:
            raise PermissionError(f"{p!r} is outside the agent root {self.root}")
        return q


def register_builtin_tools(reg: ToolRegistry, sandbox: Sandbox | None = None, shell: bool | None = None) -> None:
    sb = sandbox or Sandbox()
    shell = (os.environ.get("SQUISH_AGENT_SHELL") == "1") if shell is None else shell

    def read_file(path: str, start_line: int = 1, end_line: int = 200) -> str:
        lines = sb.path(path).read_text(errors="replace").splitlines()
        return "\n".join(lines[max(0, start_line - 1):end_line])

    def write_file(path: str, content: str) -> str:
        if len(content.encode()) > sb.max_bytes:
            raise ValueError("content too large")
        p = sb.path(path)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(content)
        return f"wrote {len(content)} characters to {p.relative_to(sb.root)}"

    def list_dir(path: str = ".") -> str:
        p = sb.path(path)
        return "\n".join(f"{c.name}/" if c.is_dir() else c.name for c in sorted(p.iterdir()))

    reg.register(ToolDefinition("read_file", "Read lines of a text file.", {
        "type": "object", "properties": {"path": {"type": "string"}, "start_line": {"type": "integer"},
                                         "end_line": {"type": "integer"}}, "required": ["path"]}, read_file))
    reg.register(ToolDefinition("write_file", "Write a text file (creates directories).", {
        "type": "object", "properties": {"path": {"type": "string"}, "content": {"type": "string"}},
        "required": ["path", "content"]}, write_file))
    reg.register(ToolDefinition("list_dir", "List a directory.", {
        "type": "object", "properties": {"path": {"type": "string"}}, "required": []}, list_dir))
    if shell:
        def run_shell(command: str, timeout: int = 30) -> str:
            r = subprocess.run(command, shell=True, cwd=sb.root, capture_output=True, text=True,  # noqa: S602
                               timeout=max(1, min(timeout, 300)))
            return (r.stdout + r.stderr)[-20000:] + f"\n[exit {r.returncode}]"

        reg.register(ToolDefinition("run_shell", "Run a shell command in the agent root.", {
            "type": "object", "properties": {"command": {"type": "string"}, "timeout": {"type": "integer"}},
            "required": ["command"]}, run_shell))
