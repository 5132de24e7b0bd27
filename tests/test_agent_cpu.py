"""Agent tooling: registry, built-in tools, MCP stdio client, the tool loop and its routes."""
import asyncio
import json
import os
import sys

import pytest

from squish_b200.agent.loop import run_agent
from squish_b200.agent.mcp import MCPClient, MCPError, register_mcp_tools
from squish_b200.agent.tools import Sandbox, ToolRegistry, register_builtin_tools

ECHO = [sys.executable, os.path.join(os.path.dirname(__file__), "mcp_echo_server.py")]


def test_registry_builtin_tools_and_sandbox(tmp_path):
    reg = ToolRegistry()
    register_builtin_tools(reg, Sandbox(tmp_path), shell=False)
    assert reg.names() == ["list_dir", "read_file", "write_file"] and "run_shell" not in reg
    assert reg.call("write_file", {"path": "d/a.txt", "content": "x\ny\nz"}).ok
    assert reg.call("read_file", '{"path": "d/a.txt", "start_line": "2", "end_line": 2}').content == "y"
    assert reg.call("list_dir", {"path": "d"}).content == "a.txt"
    bad = reg.call("read_file", {"path": "../../etc/passwd"})
    assert not bad.ok and "outside" in bad.error
    assert "missing" in reg.call("write_file", {"path": "b"}).error
    assert "unknown argument" in reg.call("list_dir", {"path": ".", "x": 1}).error
    assert "unknown tool" in reg.call("nope", {}).error
    msg = reg.call("list_dir", {}, call_id="c1").to_message()
    assert msg["role"] == "tool" and msg["tool_call_id"] == "c1"
    sh = ToolRegistry()
    register_builtin_tools(sh, Sandbox(tmp_path), shell=True)
    assert "[exit 0]" in sh.call("run_shell", {"command": "echo hi"}).content


def test_mcp_stdio_client():
    with MCPClient(ECHO, timeout=20) as c:
        assert c.server_info["name"] == "echo"
        assert [t["name"] for t in c.list_tools()] == ["echo"]
        assert c.call_tool("echo", {"text": "a"}) == "echo: a"
        with pytest.raises(MCPError):
            c.call_tool("echo", {"text": "a", "fail": True})
        with pytest.raises(MCPError):
            c.request("bogus/method")
        reg = ToolRegistry()
        assert register_mcp_tools(c, reg, "m1") == ["echo"]
        assert reg.call("echo", {"text": "z"}).content == "echo: z"


def test_agent_loop_runs_tools(tmp_path):
    reg = ToolRegistry()
    register_builtin_tools(reg, Sandbox(tmp_path), shell=False)
    script = ['Writing it now. <tool_call>{"name": "write_file", "arguments": {"path": "n.txt", "content": "42"}}'
              '</tool_call>', '<tool_call>{"name": "read_file", "arguments": {"path": "n.txt"}}</tool_call>',
              "The file says 42."]
    seen = []

    async def gen(msgs, tools):
        seen.append(msgs)
        assert {t["function"]["name"] for t in tools} >= {"read_file", "write_file", "extra"}
        return script[len(seen) - 1]

    async def collect():
        extra = [{"type": "function", "function": {"name": "extra", "parameters": {}}}]
        return [e async for e in run_agent(gen, reg, [{"role": "user", "content": "go"}], extra, max_steps=5)]

    evs = asyncio.run(collect())
    kinds = [e["type"] for e in evs]
    assert kinds == ["text_delta", "tool_call_start", "tool_call_result", "step_complete", "tool_call_start",
                     "tool_call_result", "step_complete", "text_delta", "step_complete", "done"]
    assert (tmp_path / "n.txt").read_text() == "42"
    assert evs[5]["result"] == "42" and evs[-1] == {"type": "done", "total_steps": 3, "total_tool_calls": 2}
    assert seen[2][-1]["role"] == "tool" and seen[2][-1]["content"] == "42"


def test_agent_routes():
    from fastapi.testclient import TestClient

    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.models.config import get_preset
    from squish_b200.models.weights import random_checkpoint
    from squish_b200.serving.async_engine import AsyncEngine
    from squish_b200.serving.server import ServerState, create_app
    from squish_b200.serving.tokenizer import ByteTokenizer

    cfg, q = get_preset("tiny-llama")
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0, device="cpu"), "cpu",
                                    EngineConfig(max_num_seqs=2, max_model_len=512, num_pages=64))
    aeng = AsyncEngine(eng, ByteTokenizer(cfg.vocab_size, cfg.eos_token_id), model_name="tiny").start()
    try:
        with TestClient(create_app(ServerState(aeng, "tiny", arch="llama"))) as c:
            names = {t["function"]["name"] for t in c.get("/v1/agent/tools").json()["tools"]}
            assert {"read_file", "write_file", "list_dir"} <= names
            r = c.post("/v1/agent/mcp", json={"command": " ".join(ECHO), "id": "e"}).json()
            assert r == {"id": "e", "tools": ["echo"]}
            assert "echo" in {t["function"]["name"] for t in c.get("/v1/agent/tools").json()["tools"]}
            assert c.get("/v1/agent/mcp").json()["servers"][0]["id"] == "e"
            assert c.delete("/v1/agent/mcp/e").json()["disconnected"]
            assert c.delete("/v1/agent/mcp/e").status_code == 404
            with c.stream("POST", "/v1/agent/run", json={"messages": [{"role": "user", "content": "hi"}],
                                                         "max_steps": 2, "max_tokens": 8, "temperature": 0}) as s:
                evs = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: {")]
            assert evs[-1]["type"] in ("done", "error")
    finally:
        aeng.stop()
