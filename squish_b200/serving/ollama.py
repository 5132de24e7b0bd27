"""Ollama-compatible routes (``/api/*``), the counterpart of the reference's
squish/serving/ollama_compat.py:51-536: version, tags, show, ps, generate and chat
(NDJSON streaming by default), embeddings/embed, and the model-management verbs, which on
an offline server answer with explicit errors instead of pretending to succeed.
"""
from __future__ import annotations

import json
import time
from datetime import datetime, timezone

from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, StreamingResponse

from ..engine.sampling import SamplingParams
from .chat_template import apply_chat_template
from .tokenizer import IncrementalDetokenizer
from .tool_calling import parse_tool_calls

OLLAMA_VERSION = "0.5.0"


def _now() -> str:
    return datetime.now(timezone.utc).isoformat().replace("+00:00", "Z")


def _params(body: dict, eos) -> tuple[SamplingParams, list[str]]:
    o = body.get("options") or {}
    stops = o.get("stop") or []
    if isinstance(stops, str):
        stops = [stops]
    p = SamplingParams(
        max_tokens=max(1, int(o.get("num_predict", 256) if o.get("num_predict", 256) not in (-1, -2) else 4096)),
        temperature=float(o.get("temperature", 0.8)), top_p=float(o.get("top_p", 0.9) or 0.9),
        top_k=int(o.get("top_k", 40) or 0), min_p=float(o.get("min_p", 0.0) or 0.0),
        repetition_penalty=float(o.get("repeat_penalty", 1.1) or 1.0), seed=o.get("seed"),
        stop_token_ids=[eos] if eos is not None else [])
    return p.validate(), stops


def _details(st) -> dict:
    cfg = st.aeng.engine.cfg
    q = st.aeng.engine.qcfg
    return {"parent_model": "", "format": "squish", "family": cfg.arch, "families": [cfg.arch],
            "parameter_size": f"{cfg.num_params() / 1e9:.1f}B",
            "quantization_level": f"INT{q.weight_bits}_g{q.group_size}" if q.weight_bits < 16 else "BF16"}


def mount_ollama(app: FastAPI, st) -> None:
    def model_size() -> int:
        r = st.aeng.engine.runner
        return int(sum(t.numel() * t.element_size() for t in _tensors(r)))

    @app.get("/api/version")
    async def version():
        return {"version": OLLAMA_VERSION}

    @app.get("/api/tags")
    async def tags():
        return {"models": [{"name": st.model_name, "model": st.model_name, "modified_at": _now(),
                            "size": model_size(), "digest": "", "details": _details(st)}]}

    @app.post("/api/show")
    async def show(request: Request):
        body = await request.json()
        name = body.get("model") or body.get("name")
        if name and name != st.model_name:
            raise HTTPException(status_code=404, detail=f"model '{name}' not found")
        cfg = st.aeng.engine.cfg
        return {"modelfile": f"FROM {st.model_name}", "parameters": "", "template": "{{ .Prompt }}",
                "details": _details(st),
                "model_info": {"general.architecture": cfg.arch, "general.parameter_count": cfg.num_params(),
                               f"{cfg.arch}.context_length": st.aeng.engine.ecfg.max_model_len,
                               f"{cfg.arch}.embedding_length": cfg.hidden_size,
                               f"{cfg.arch}.block_count": cfg.num_layers,
                               f"{cfg.arch}.attention.head_count": cfg.num_heads,
                               f"{cfg.arch}.attention.head_count_kv": cfg.num_kv_heads}}

    @app.get("/api/ps")
    async def ps():
        size = model_size()
        return {"models": [{"name": st.model_name, "model": st.model_name, "size": size, "size_vram": size,
                            "digest": "", "details": _details(st), "expires_at": "0001-01-01T00:00:00Z"}]}

    async def _gen(prompt_ids, params, stops, chat: bool, t_start: float):
        detok = IncrementalDetokenizer(st.tok)
        text, n_out, reason, t_first = "", 0, "stop", None
        async for ev in st.aeng.stream(prompt_ids, params):
            if t_first is None:
                t_first = time.perf_counter()
            n_out += len(ev.token_ids)
            delta = detok.push(ev.token_ids)
            text += delta
            hit = any(s in text for s in stops)
            if hit:
                cut = min(text.find(s) for s in stops if s in text)
                delta = delta[: max(0, len(delta) - (len(text) - cut))]
                text = text[:cut]
            yield delta, False, None, n_out, t_first
            if hit:
                break
            if ev.finished:
                reason = ev.reason if ev.reason in ("length", "repetition") else "stop"
                break
        yield "", True, reason, n_out, t_first

    def _final(prompt_ids, n_out, reason, t_start, t_first, extra):
        now = time.perf_counter()
        t_first = t_first or now
        d = {"model": st.model_name, "created_at": _now(), "done": True, "done_reason": reason,
             "total_duration": int((now - t_start) * 1e9), "load_duration": 0,
             "prompt_eval_count": len(prompt_ids), "prompt_eval_duration": int((t_first - t_start) * 1e9),
             "eval_count": n_out, "eval_duration": int((now - t_first) * 1e9)}
        d.update(extra)
        return d

    @app.post("/api/generate")
    async def generate(request: Request):
        body = await request.json()
        prompt = body.get("prompt", "")
        t_start = time.perf_counter()
        if not prompt:  # an empty prompt loads the model: answer done immediately
            return {"model": st.model_name, "created_at": _now(), "response": "", "done": True,
                    "done_reason": "load"}
        if body.get("raw"):
            text = prompt
        else:
            msgs = ([{"role": "system", "content": body["system"]}] if body.get("system") else []) + \
                   [{"role": "user", "content": prompt}]
            text = apply_chat_template(msgs, st.tok, st.arch)
        prompt_ids = list(body.get("context") or []) + st.tok.encode(text)
        params, stops = _params(body, st.tok.eos_token_id)
        if body.get("format") == "json":
            params.grammar = st.grammar_factory().json()
        elif isinstance(body.get("format"), dict):  # a JSON schema
            params.grammar = st.grammar_factory().schema(body["format"])
        stream = body.get("stream", True)

        async def lines():
            out_ids = []
            async for delta, done, reason, n_out, t_first in _gen(prompt_ids, params, stops, False, t_start):
                if not done:
                    yield json.dumps({"model": st.model_name, "created_at": _now(), "response": delta,
                                      "done": False}) + "\n"
                else:
                    yield json.dumps(_final(prompt_ids, n_out, reason, t_start, t_first,
                                            {"response": "", "context": prompt_ids + out_ids})) + "\n"

        if stream:
            return StreamingResponse(lines(), media_type="application/x-ndjson")
        text_out, final = "", None
        async for delta, done, reason, n_out, t_first in _gen(prompt_ids, params, stops, False, t_start):
            text_out += delta
            if done:
                final = _final(prompt_ids, n_out, reason, t_start, t_first, {"response": text_out})
        return final

    @app.post("/api/chat")
    async def chat(request: Request):
        body = await request.json()
        msgs = body.get("messages") or []
        if not isinstance(msgs, list):
            raise HTTPException(status_code=400, detail="'messages' must be a list")
        tools = body.get("tools") or None
        t_start = time.perf_counter()
        prompt_ids = st.tok.encode(apply_chat_template(msgs, st.tok, st.arch, tools=tools))
        params, stops = _params(body, st.tok.eos_token_id)
        if body.get("format") == "json":
            params.grammar = st.grammar_factory().json()
        elif isinstance(body.get("format"), dict):  # a JSON schema
            params.grammar = st.grammar_factory().schema(body["format"])

        async def lines():
            async for delta, done, reason, n_out, t_first in _gen(prompt_ids, params, stops, True, t_start):
                if not done:
                    yield json.dumps({"model": st.model_name, "created_at": _now(),
                                      "message": {"role": "assistant", "content": delta}, "done": False}) + "\n"
                else:
                    yield json.dumps(_final(prompt_ids, n_out, reason, t_start, t_first,
                                            {"message": {"role": "assistant", "content": ""}})) + "\n"

        if body.get("stream", True):
            return StreamingResponse(lines(), media_type="application/x-ndjson")
        text_out, final = "", None
        async for delta, done, reason, n_out, t_first in _gen(prompt_ids, params, stops, True, t_start):
            text_out += delta
            if done:
                msg = {"role": "assistant", "content": text_out}
                if tools:
                    content, calls = parse_tool_calls(text_out)
                    if calls:
                        msg = {"role": "assistant", "content": content,
                               "tool_calls": [{"function": {"name": c["function"]["name"],
                                                            "arguments": json.loads(c["function"]["arguments"])}}
                                              for c in calls]}
                final = _final(prompt_ids, n_out, reason, t_start, t_first, {"message": msg})
        return final

    @app.post("/api/embeddings")
    async def embeddings_legacy(request: Request):
        from .server import embed_texts

        body = await request.json()
        vecs, _ = await embed_texts(st, [body.get("prompt", "") or " "])
        return {"embedding": vecs[0]}

    @app.post("/api/embed")
    async def embed(request: Request):
        from .server import embed_texts

        body = await request.json()
        inp = body.get("input", "")
        texts = [inp] if isinstance(inp, str) else list(inp)
        vecs, n = await embed_texts(st, texts)
        return {"model": st.model_name, "embeddings": vecs, "prompt_eval_count": n}

    @app.post("/api/pull")
    async def pull(request: Request):
        return JSONResponse({"error": "pull is not available on an offline server; use `squish pull` on a host "
                                      "with network access and point the server at the local directory"},
                            status_code=501)

    @app.post("/api/push")
    async def push(request: Request):
        return JSONResponse({"error": "push is not supported"}, status_code=501)

    @app.post("/api/create")
    async def create(request: Request):
        return JSONResponse({"error": "create is not supported; convert with `squish compress`"}, status_code=501)

    @app.post("/api/copy")
    async def copy(request: Request):
        return JSONResponse({"error": "copy is not supported by a single-model server"}, status_code=501)

    @app.delete("/api/delete")
    async def delete(request: Request):
        return JSONResponse({"error": "the loaded model cannot be deleted while serving"}, status_code=409)

    @app.head("/api/blobs/{digest}")
    async def blob_head(digest: str):
        return JSONResponse({}, status_code=404)


def _tensors(runner):
    import torch

    seen = []
    for v in getattr(runner, "__dict__", {}).values():
        if isinstance(v, torch.Tensor):
            seen.append(v)
    for lw in getattr(runner, "layers", []):
        for v in getattr(lw, "__dict__", {}).values():
            if isinstance(v, torch.Tensor):
                seen.append(v)
            elif hasattr(v, "wq"):
                seen.append(v.wq)
    return seen
