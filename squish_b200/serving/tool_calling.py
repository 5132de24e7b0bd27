"""Tool-call parsing for OpenAI ``tools`` requests.

Models prompted with the tools block (chat_template.tools_system_block) answer with
``<tool_call>{"name": ..., "arguments": {...}}</tool_call>`` segments, the convention of
the reference's tool layer (squish/serving/tool_calling.py:67-465). Bare JSON objects
with a ``name`` field are accepted too.
"""
from __future__ import annotations

import json
import re
import uuid

_TAG = re.compile(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", re.S)


def _extract_json_objects(text: str) -> list[str]:
    objs, depth, start, in_str, esc = [], 0, -1, False, False
    for i, ch in enumerate(text):
        if in_str:
            if esc:
                esc = False
            elif ch == "\\":
                esc = True
            elif ch == '"':
                in_str = False
            continue
        if ch == '"':
            in_str = True
        elif ch == "{":
            if depth == 0:
                start = i
            depth += 1
        elif ch == "}" and depth:
            depth -= 1
            if depth == 0:
                objs.append(text[start:i + 1])
    return objs


def parse_tool_calls(text: str) -> tuple[str, list[dict]]:
    """Split a completion into (plain content, OpenAI tool_calls list)."""
    raw = _TAG.findall(text)
    content = _TAG.sub("", text).strip()
    if not raw:
        cands = [o for o in _extract_json_objects(text) if '"name"' in o]
        if cands:
            raw = cands
            for c in cands:
                content = content.replace(c, "")
            content = content.strip()
    calls = []
    for r in raw:
        try:
            obj = json.loads(r)
        except json.JSONDecodeError:
            continue
        if not isinstance(obj, dict) or "name" not in obj:
            continue
        args = obj.get("arguments", obj.get("parameters", {}))
        calls.append({"id": f"call_{uuid.uuid4().hex[:24]}", "type": "function",
                      "function": {"name": str(obj["name"]),
                                   "arguments": args if isinstance(args, str) else json.dumps(args)}})
    return content, calls


class ToolCallStreamFilter:
    """Holds back streamed text once a ``<tool_call>`` opens, so calls are emitted whole."""

    def __init__(self):
        self.buf = ""
        self.in_call = False

    def push(self, delta: str) -> str:
        self.buf += delta
        if self.in_call:
            return ""
        idx = self.buf.find("<tool_call>")
        if idx >= 0:
            self.in_call = True
            out, self.buf = self.buf[:idx], self.buf[idx:]
            return out
        # keep a possible partial tag at the end
        keep = 0
        for k in range(1, len("<tool_call>")):
            if self.buf.endswith("<tool_call>"[:k]):
                keep = k
        out = self.buf[:len(self.buf) - keep]
        self.buf = self.buf[len(self.buf) - keep:]
        return out
