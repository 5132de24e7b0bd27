"""Model Context Protocol client (stdio transport): JSON-RPC 2.0 ``initialize`` ->
``notifications/initialized`` -> ``tools/list`` -> ``tools/call``, one JSON message per line,
as the reference's MCPClient (squish/serving/mcp_client.py); tools found on a server are
registered in a :class:`ToolRegistry` under ``<server>.<tool>``-free plain names.
"""
from __future__ import annotations

import json
import shlex
import subprocess
import threading

from .tools import ToolDefinition, ToolRegistry


class MCPError(RuntimeError):
    pass


class MCPClient:
    PROTOCOL = "2024-11-05"

    def __init__(self, command: str | list[str], timeout: float = 30.0, env: dict | None = None):
        self.argv = shlex.split(command) if isinstance(command, str) else list(command)
        self.timeout = timeout
        self.env = env
        self.proc: subprocess.Popen | None = None
        self._id = 0
        self._lock = threading.Lock()
        self.server_info: dict = {}

    def __enter__(self) -> "MCPClient":
        self.start()
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def start(self) -> None:
        self.proc = subprocess.Popen(self.argv, stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                     stderr=subprocess.DEVNULL, text=True, bufsize=1, env=self.env)
        r = self.request("initialize", {"protocolVersion": self.PROTOCOL, "capabilities": {},
                                        "clientInfo": {"name": "squish-b200", "version": "0.1"}})
        self.server_info = r.get("serverInfo", {})
        self._send({"jsonrpc": "2.0", "method": "notifications/initialized"})

    def close(self) -> None:
        if self.proc is not None:
            try:
                self.proc.stdin.close()
                self.proc.wait(timeout=5)
            except (OSError, subprocess.TimeoutExpired):
                self.proc.kill()
            self.proc = None

    def _send(self, msg: dict) -> None:
        if self.proc is None or self.proc.poll() is not None:
            raise MCPError("MCP server is not running")
        self.proc.stdin.write(json.dumps(msg) + "\n")
        self.proc.stdin.flush()

    def request(self, method: str, params: dict | None = None) -> dict:
        with self._lock:
            self._id += 1
            rid = self._id
            self._send({"jsonrpc": "2.0", "id": rid, "method": method, "params": params or {}})
            result: dict = {}

            def read():
                while True:
                    line = self.proc.stdout.readline()
                    if not line:
                        result["error"] = {"message": "server closed the connection"}
                        return
                    try:
                        m = json.loads(line)
                    except ValueError:
                        continue  # log lines on stdout
                    if m.get("id") == rid:
                        result.update(m)
                        return

            t = threading.Thread(target=read, daemon=True)
            t.start()
            t.join(self.timeout)
            if t.is_alive():
                raise MCPError(f"MCP request {method!r} timed out after {self.timeout}s")
            if "error" in result:
                raise MCPError(f"MCP {method} failed: {result['error'].get('message')}")
            return result.get("result", {})

    def list_tools(self) -> list[dict]:
        return self.request("tools/list").get("tools", [])

    def call_tool(self, name: str, arguments: dict) -> str:
        r = self.request("tools/call", {"name": name, "arguments": arguments})
        text = "\n".join(c.get("text", "") for c in r.get("content", []) if c.get("type") == "text")
        if r.get("isError"):
            raise MCPError(text or "tool reported an error")
        return text


def register_mcp_tools(client: MCPClient, reg: ToolRegistry, source: str) -> list[str]:
    names = []
    for t in client.list_tools():
        name = t["name"]

        def fn(_n=name, **kw):
            return client.call_tool(_n, kw)

        reg.register(ToolDefinition(name, t.get("description", ""), t.get("inputSchema") or
                                    {"type": "object", "properties": {}}, fn, source=source))
        names.append(name)
    return names
