"""Chat prompt rendering when the tokenizer brings no template of its own.

ChatML (the Qwen2/Qwen3 format) is the default; Llama-3 headers are used for Llama
models. Tools are announced in the system turn the way Qwen's template does (a
``<tools>`` JSON block and the ``<tool_call>`` reply convention), which the tool-call
parser (tool_calling.py) understands.
"""
from __future__ import annotations

import json


def _content(m) -> str:
    c = m.get("content", "")
    if isinstance(c, list):  # OpenAI content parts
        return "".join(p.get("text", "") for p in c if isinstance(p, dict))
    return c or ""


def tools_system_block(tools) -> str:
    lines = ["# Tools", "", "You may call one or more functions to assist with the user query.", "",
             "You are provided with function signatures within <tools></tools> XML tags:", "<tools>"]
    for t in tools:
        lines.append(json.dumps(t.get("function", t), ensure_ascii=False))
    lines += ["</tools>", "",
              "For each function call, return a json object with function name and arguments within "
              "<tool_call></tool_call> XML tags:",
              "<tool_call>", '{"name": <function-name>, "arguments": <args-json-object>}', "</tool_call>"]
    return "\n".join(lines)


def render_chatml(messages, add_generation_prompt: bool = True, tools=None) -> str:
    out = []
    msgs = list(messages)
    if tools:
        sys_text = tools_system_block(tools)
        if msgs and msgs[0].get("role") == "system":
            msgs[0] = {"role": "system", "content": _content(msgs[0]) + "\n\n" + sys_text}
        else:
            msgs.insert(0, {"role": "system", "content": sys_text})
    for m in msgs:
        role = m.get("role", "user")
        if role == "tool":
            out.append(f"<|im_start|>user\n<tool_response>\n{_content(m)}\n</tool_response><|im_end|>\n")
            continue
        text = _content(m)
        for call in m.get("tool_calls") or []:
            fn = call.get("function", {})
            args = fn.get("arguments", "{}")
            if not isinstance(args, str):
                args = json.dumps(args)
            text += f'\n<tool_call>\n{{"name": "{fn.get("name", "")}", "arguments": {args}}}\n</tool_call>'
        out.append(f"<|im_start|>{role}\n{text}<|im_end|>\n")
    if add_generation_prompt:
        out.append("<|im_start|>assistant\n")
    return "".join(out)


def render_llama3(messages, add_generation_prompt: bool = True, tools=None) -> str:
    out = ["<|begin_of_text|>"]
    for m in messages:
        out.append(f"<|start_header_id|>{m.get('role', 'user')}<|end_header_id|>\n\n{_content(m)}<|eot_id|>")
    if add_generation_prompt:
        out.append("<|start_header_id|>assistant<|end_header_id|>\n\n")
    return "".join(out)


def apply_chat_template(messages, tokenizer, arch: str = "qwen2", tools=None) -> str:
    if tokenizer is not None and hasattr(tokenizer, "tok") and getattr(tokenizer.tok, "chat_template", None):
        kw = {"tools": tools} if tools else {}
        return tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True, **kw)
    if arch == "llama":
        return render_llama3(messages, True, tools)
    return render_chatml(messages, True, tools)
