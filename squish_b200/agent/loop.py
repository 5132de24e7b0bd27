"""The multi-step tool-calling loop behind ``POST /v1/agent/run``.

Event protocol of the reference (squish/server.py:4228-4330): ``text_delta``,
``tool_call_start``, ``tool_call_result`` (result, error, elapsed_ms), ``step_complete``,
``done`` (total_steps, total_tool_calls), ``error``. Each step renders the conversation with the
tool schemas, generates, splits the text into content and tool calls
(serving/tool_calling.py), runs the calls through the registry and appends the results as
``tool`` messages; a step without tool calls ends the run.
"""
from __future__ import annotations

import asyncio
import json
from typing import AsyncIterator, Awaitable, Callable

from ..serving.tool_calling import parse_tool_calls
from .tools import ToolRegistry

Generate = Callable[[list, list], Awaitable[str]]


async def run_agent(generate: Generate, registry: ToolRegistry, messages: list, extra_tools: list | None = None,
                    max_steps: int = 10) -> AsyncIterator[dict]:
    builtin = registry.to_openai_schemas()
    names = {t["function"]["name"] for t in builtin}
    tools = builtin + [t for t in (extra_tools or []) if t.get("function", {}).get("name") not in names]
    current = list(messages)
    calls_total = 0
    step = 0
    try:
        for step in range(1, max_steps + 1):
            text = await generate(current, tools)
            content, calls = parse_tool_calls(text)
            if content:
                yield {"type": "text_delta", "delta": content}
            if not calls:
                yield {"type": "step_complete", "step": step}
                break
            current.append({"role": "assistant", "content": content or None, "tool_calls": calls})
            for c in calls:
                name, args = c["function"]["name"], c["function"]["arguments"]
                try:
                    parsed = json.loads(args) if isinstance(args, str) else args
                except ValueError:
                    parsed = args
                yield {"type": "tool_call_start", "call_id": c["id"], "tool_name": name, "arguments": parsed}
                if name in registry:
                    res = await asyncio.to_thread(registry.call, name, args, c["id"])
                else:  # a caller-supplied schema with no implementation here
                    from .tools import ToolResult

                    res = ToolResult(c["id"], name, "", f"tool {name!r} is not available on this server")
                calls_total += 1
                yield {"type": "tool_call_result", "call_id": c["id"], "tool_name": name, "result": res.content,
                       "error": res.error, "elapsed_ms": round(res.elapsed_ms, 3)}
                current.append(res.to_message())
            yield {"type": "step_complete", "step": step}
        yield {"type": "done", "total_steps": step, "total_tool_calls": calls_total}
    except Exception as exc:  # noqa: BLE001 - the stream ends with an error event
        yield {"type": "error", "message": f"{type(exc).__name__}: {exc}"}
