"""HTTP server: OpenAI-compatible ``/v1/*``, Ollama-compatible ``/api/*`` (ollama.py) and the
LocalAI probes, over an :class:`AsyncEngine`.

Route set and response shapes follow the reference server (squish/server.py:3374-4835):
chat/completions (SSE streaming with ``stream_options.include_usage``, tools), completions
(string, token list or batch), embeddings, models, tokenize, health, model/status,
Prometheus metrics, trace, quality. Requests are batched by the engine (continuous
batching), not serialised on one inference thread.
"""
from __future__ import annotations

import asyncio
import dataclasses
import json
import time
import uuid

import numpy as np
from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from ..engine.sampling import SamplingParams
from ..utils import telemetry
from .async_engine import AsyncEngine, GenEvent, QueueFullError
from .chat_template import apply_chat_template
from .tokenizer import IncrementalDetokenizer
from .tool_calling import ToolCallStreamFilter, parse_tool_calls
from .validation import parse_embedding_input, parse_int, parse_max_tokens, parse_temperature, parse_top_p

VERSION = "0.1.0"


class ServerState:
    def __init__(self, aeng: AsyncEngine, model_name: str, api_key: str | None = None, arch: str = "qwen2",
                 governor=None, load_time_s: float = 0.0, response_cache: int = 256,
                 compress_prompt: dict | None = None):
        from .response_cache import ResponseCache

        self.aeng = aeng
        self.cache = ResponseCache(response_cache)
        self._grammar = None
        # {"ratio", "min_tokens", "preserve_tokens"}: extractive compression of long user messages
        self.compress_prompt = compress_prompt
        self.model_name = model_name
        self.api_key = api_key
        self.arch = arch
        self.governor = governor
        self.load_time_s = load_time_s
        self.loaded_at = time.time()
        self.created = int(time.time())

    @property
    def tok(self):
        return self.aeng.tokenizer

    def grammar_factory(self):
        """JSON matcher factory (the vocabulary trie is built on first use)."""
        if self._grammar is None:
            from .grammar import GrammarFactory

            eng = self.aeng.engine
            self._grammar = GrammarFactory(self.tok, eng.cfg.vocab_size, self.tok.eos_token_id)
        return self._grammar

    def format_factory(self, response_format):
        """Something whose ``json()`` gives a fresh grammar for ``response_format`` (JSON object,
        or a JSON schema), or None when the output is unconstrained."""
        from .grammar import grammar_for, wants_json

        try:
            if not wants_json(response_format):
                return None
            grammar_for(self.grammar_factory(), response_format)  # validates the schema once
        except (ValueError, KeyError, TypeError) as exc:
            raise HTTPException(status_code=400, detail=f"response_format: {exc}") from exc
        fac = self.grammar_factory()

        class _Per:
            @staticmethod
            def json():
                return grammar_for(fac, response_format)

        return _Per


def _check_auth(request: Request, st: ServerState) -> None:
    if not st.api_key:
        return
    h = request.headers.get("authorization", "")
    if not h.lower().startswith("bearer ") or h[7:].strip() != st.api_key:
        raise HTTPException(status_code=401, detail="invalid or missing API key")


async def _json(request: Request) -> dict:
    try:
        body = await request.json()
    except (json.JSONDecodeError, ValueError, UnicodeDecodeError) as exc:
        raise HTTPException(status_code=400, detail="request body must be valid JSON") from exc
    if not isinstance(body, dict):
        raise HTTPException(status_code=400, detail="request body must be a JSON object")
    return body


def sampling_from_openai(body: dict, default_max: int, eos_ids: list[int] | None = None) -> SamplingParams:
    stop_ids = list(eos_ids or [])
    return SamplingParams(
        max_tokens=max(1, parse_max_tokens(body.get("max_tokens", body.get("max_completion_tokens")), default_max)),
        temperature=parse_temperature(body.get("temperature")),
        top_p=parse_top_p(body.get("top_p")),
        top_k=parse_int(body.get("top_k"), "top_k", 0),
        min_p=float(body.get("min_p", 0.0) or 0.0),
        repetition_penalty=float(body.get("repetition_penalty", body.get("repeat_penalty", 1.0)) or 1.0),
        seed=body.get("seed"),
        stop_token_ids=stop_ids,
        ignore_eos=bool(body.get("ignore_eos", False)),
    )


def _stop_strings(body: dict) -> list[str]:
    s = body.get("stop")
    if s is None:
        return []
    if isinstance(s, str):
        return [s]
    if isinstance(s, list):
        return [x for x in s if isinstance(x, str) and x]
    raise HTTPException(status_code=400, detail="'stop' must be a string or list of strings")


def _truncate_at_stop(text: str, stops: list[str]) -> tuple[str, bool]:
    cut = min((text.find(s) for s in stops if s in text), default=-1)
    return (text[:cut], True) if cut >= 0 else (text, False)


def _finish_reason(ev_reason: str | None) -> str:
    return ev_reason if ev_reason in ("length", "repetition") else "stop"


def _cache_key(st: ServerState, prompt_ids, params, stops) -> str | None:
    return st.cache.key(prompt_ids, params, repr(stops)) if st.cache.maxsize > 0 and st.cache.eligible(params) \
        else None


async def _run_one(st: ServerState, prompt_ids: list[int], params: SamplingParams, stops: list[str]):
    """Collect one request; returns (text, token ids, finish_reason, prompt_tokens). Greedy
    requests seen before are answered from the response cache."""
    key = _cache_key(st, prompt_ids, params, stops)
    if key is not None and (hit := st.cache.get(key)) is not None:
        text, ids, reason = hit
        return text, list(ids), reason, len(prompt_ids)
    detok = IncrementalDetokenizer(st.tok)
    text, ids, reason, ptoks = "", [], "stop", len(prompt_ids)
    async for ev in st.aeng.stream(prompt_ids, params):
        ids.extend(ev.token_ids)
        text += detok.push(ev.token_ids)
        if stops:
            text, hit = _truncate_at_stop(text, stops)
            if hit:
                reason = "stop"
                break
        if ev.finished:
            reason = "length" if ev.reason == "length" else ("stop" if ev.reason in ("stop", None) else ev.reason)
            break
    if key is not None and reason in ("stop", "length"):
        st.cache.put(key, (text, tuple(ids), reason))
    return text, ids, reason, ptoks


async def _events(st: ServerState, prompt_ids, params, stops):
    """Token events of one request, or one synthetic event replaying a cached greedy answer
    (its text is carried in ``cached_text``)."""
    key = _cache_key(st, prompt_ids, params, stops)
    if key is not None and (hit := st.cache.get(key)) is not None:
        text, ids, reason = hit
        ev = GenEvent(list(ids), True, reason, len(prompt_ids), len(ids))
        ev.cached_text = text
        yield ev
        return
    async for ev in st.aeng.stream(prompt_ids, params):
        yield ev


def create_app(st: ServerState) -> FastAPI:
    app = FastAPI(title="squish-b200", version=VERSION)
    app.state.squish = st

    @app.middleware("http")
    async def shed_on_memory_pressure(request: Request, call_next):
        gov = st.governor
        if gov is not None and gov.critical and request.url.path not in ("/health", "/v1/metrics", "/model/status"):
            return JSONResponse({"error": {"message": "server under memory pressure", "type": "overloaded"}},
                                status_code=503, headers={"Retry-After": "2"})
        return await call_next(request)

    @app.exception_handler(QueueFullError)
    async def _queue_full(request: Request, exc: QueueFullError):
        return JSONResponse({"error": {"message": str(exc), "type": "rate_limit"}}, status_code=429,
                            headers={"Retry-After": "1"})

    def model_card() -> dict:
        return {"id": st.model_name, "object": "model", "created": st.created, "owned_by": "squish"}

    # ------------------------------------------------------------------ models / health
    @app.get("/v1/models")
    async def list_models(request: Request):
        _check_auth(request, st)
        return {"object": "list", "data": [model_card()]}

    @app.get("/v1/models/{model_id:path}")
    async def get_model(model_id: str, request: Request):
        _check_auth(request, st)
        if model_id != st.model_name:
            raise HTTPException(status_code=404, detail=f"model {model_id!r} not found")
        return model_card()

    @app.get("/health")
    async def health():
        a = st.aeng
        gov = st.governor
        wd = a.watchdog
        ok = a.alive and not wd.poll()
        return {"status": "ok" if ok else "degraded", "degraded_reason": None if ok else (wd.reason or "engine stopped"),
                "model": st.model_name, "loaded": True,
                "model_loaded": True, "load_mode": "eager", "load_error": a.last_error, "loader": "squish-b200",
                "load_time_s": round(st.load_time_s, 2), "requests": a.requests_total, "tokens_gen": a.tokens_total,
                "inflight": a.inflight, "avg_tps": round(a.avg_tps, 1), "avg_ttft_s": round(a.avg_ttft, 3),
                "uptime_s": round(time.time() - st.loaded_at, 1),
                "mem_available_gb": None if gov is None else round(gov.available_gb, 2),
                "mem_pressure": None if gov is None else gov.level,
                "engine_heartbeat_age_s": round(time.time() - a.heartbeat, 3)}

    @app.get("/model/status")
    async def model_status():
        return {"load_mode": "eager", "model_loaded": True, "model": st.model_name,
                "load_time_s": round(st.load_time_s, 2), "load_error": None}

    @app.get("/v1/metrics")
    async def metrics():
        a, eng = st.aeng, st.aeng.engine
        bm = eng.blocks
        used = bm.num_pages - bm.num_free()
        stats = eng.stats
        lines = []

        def m(name, typ, help_, val):
            lines.extend([f"# HELP {name} {help_}", f"# TYPE {name} {typ}", f"{name} {val}"])

        m("squish_requests_total", "counter", "Total inference requests served", a.requests_total)
        m("squish_tokens_generated_total", "counter", "Total tokens generated", a.tokens_total)
        m("squish_inflight_requests", "gauge", "Current in-flight requests", a.inflight)
        m("squish_avg_tokens_per_second", "gauge", "Rolling average tokens/sec (last 20 requests)",
          f"{a.avg_tps:.2f}")
        m("squish_avg_ttft_seconds", "gauge", "Rolling average time-to-first-token (last 20 requests)",
          f"{a.avg_ttft:.4f}")
        m("squish_uptime_seconds", "counter", "Server uptime", round(time.time() - st.loaded_at, 1))
        m("squish_model_load_seconds", "gauge", "Time taken to load the model", f"{st.load_time_s:.3f}")
        m("squish_prefix_cache_hits_total", "counter", "Prefix page-cache hits", bm.hits)
        m("squish_prefix_cache_hit_tokens_total", "counter", "Prompt tokens served from shared pages", bm.hit_tokens)
        m("squish_paged_kv_free_blocks", "gauge", "Paged KV cache free pages", bm.num_free())
        m("squish_paged_kv_used_blocks", "gauge", "Paged KV cache used pages", used)
        m("squish_kv_cache_tokens", "gauge", "KV cache token capacity in use", used * bm.page_size)
        m("squish_engine_steps_total", "counter", "Engine iterations", stats.steps)
        m("squish_preemptions_total", "counter", "Requests preempted for KV capacity", stats.preemptions)
        m("squish_errors_total", "counter", "Engine step failures", a.errors_total)
        runner = getattr(eng, "runner", None)  # (a data-parallel router view has none)
        gpu = getattr(getattr(runner, "device", None), "index", None)
        lab = f'gpu="{gpu if gpu is not None else "cpu"}"'
        lines.extend(["# HELP squish_step_seconds Engine step wall time", "# TYPE squish_step_seconds histogram"])
        for b, c in zip(stats.step_buckets, stats.step_counts):
            le = "+Inf" if b == float("inf") else f"{b:g}"
            lines.append(f'squish_step_seconds_bucket{{{lab},le="{le}"}} {c}')
        lines.append(f"squish_step_seconds_sum{{{lab}}} {stats.step_time_sum:.6f}")
        lines.append(f"squish_step_seconds_count{{{lab}}} {stats.step_counts[-1]}")
        comm = getattr(runner, "comm", None)
        if comm is not None:
            m("squish_tp_link_bytes_total", "counter", "Tensor-parallel collective payload bytes received by this rank",
              comm.link_bytes)
        ttfts = sorted(stats.ttfts[-1000:])
        if ttfts:
            m("squish_ttft_p50_seconds", "gauge", "Median TTFT (last 1000)", f"{ttfts[len(ttfts) // 2]:.4f}")
            m("squish_ttft_p99_seconds", "gauge", "p99 TTFT (last 1000)",
              f"{ttfts[min(len(ttfts) - 1, int(0.99 * len(ttfts)))]:.4f}")
        return PlainTextResponse("\n".join(lines) + "\n", media_type="text/plain; version=0.0.4")

    @app.get("/v1/quality")
    async def quality(window: int = 300, model: str = ""):
        """Rolling-window latency / throughput / TTFT percentiles and error rate per model."""
        if window < 1 or window > 86400:
            raise HTTPException(status_code=400, detail="window must be in [1, 86400] seconds")
        out = st.aeng.quality.stats(window, model)
        out["response_cache"] = {"size": st.cache.size, "hits": st.cache.hits, "misses": st.cache.misses}
        out["loops_stopped"] = st.aeng.loops_stopped
        return out

    # ------------------------------------------------------------------ agent
    def agent_registry():
        if getattr(st, "agent", None) is None:
            from ..agent.tools import ToolRegistry, register_builtin_tools

            st.agent = ToolRegistry()
            st.mcp = {}
            register_builtin_tools(st.agent)
        return st.agent

    @app.get("/v1/agent/tools")
    async def agent_tools(request: Request):
        _check_auth(request, st)
        return {"tools": agent_registry().to_openai_schemas()}

    @app.get("/v1/agent/mcp")
    async def agent_mcp_list(request: Request):
        _check_auth(request, st)
        agent_registry()
        return {"servers": [{"id": k, "command": v["command"], "tools": v["tools"]} for k, v in st.mcp.items()]}

    @app.post("/v1/agent/mcp")
    async def agent_mcp_connect(request: Request):
        """Start an MCP server (stdio) and register its tools."""
        from ..agent.mcp import MCPClient, MCPError, register_mcp_tools

        _check_auth(request, st)
        body = await _json(request)
        cmd = body.get("command")
        if not cmd:
            raise HTTPException(status_code=400, detail="Provide 'command' (an MCP server started over stdio)")
        reg = agent_registry()
        sid = body.get("id") or f"mcp{len(st.mcp) + 1}"
        try:
            cl = MCPClient(cmd, timeout=float(body.get("timeout", 30)))
            await asyncio.to_thread(cl.start)
            names = await asyncio.to_thread(register_mcp_tools, cl, reg, sid)
        except (MCPError, OSError, ValueError) as exc:
            raise HTTPException(status_code=502, detail=f"MCP connect failed: {exc}") from exc
        st.mcp[sid] = {"client": cl, "command": cmd, "tools": names}
        return {"id": sid, "tools": names}

    @app.delete("/v1/agent/mcp/{sid}")
    async def agent_mcp_disconnect(sid: str, request: Request):
        _check_auth(request, st)
        agent_registry()
        ent = st.mcp.pop(sid, None)
        if ent is None:
            raise HTTPException(status_code=404, detail=f"no MCP server {sid!r}")
        for n in ent["tools"]:
            st.agent.unregister(n)
        await asyncio.to_thread(ent["client"].close)
        return {"id": sid, "disconnected": True}

    @app.post("/v1/agent/run")
    async def agent_run(request: Request):
        """Multi-step tool-calling loop, streamed as SSE events."""
        from ..agent.loop import run_agent

        _check_auth(request, st)
        body = await _json(request)
        messages = body.get("messages")
        if not isinstance(messages, list) or not messages:
            raise HTTPException(status_code=400, detail="'messages' must be a non-empty list")
        max_steps = max(1, min(parse_int(body.get("max_steps"), "max_steps", 10), 50))
        params = sampling_from_openai(dict(body, max_tokens=body.get("max_tokens", 1024)), 1024,
                                      [st.tok.eos_token_id] if st.tok.eos_token_id is not None else [])

        async def generate(msgs, tools):
            prompt = apply_chat_template(msgs, st.tok, st.arch, tools=tools)
            text, _, _, _ = await _run_one(st, st.tok.encode(prompt), dataclasses.replace(params), [])
            return text

        async def events():
            async for ev in run_agent(generate, agent_registry(), messages, body.get("tools") or [], max_steps):
                yield _sse(ev)
            yield b"data: [DONE]\n\n"

        return StreamingResponse(events(), media_type="text/event-stream")

    @app.post("/v1/route")
    async def route(request: Request):
        """Task category and model-family hint of a prompt (rule-based, no model call)."""
        from .router import get_default_router

        body = await _json(request)
        prompt = body.get("prompt")
        if prompt is None and isinstance(body.get("messages"), list):
            prompt = " ".join(str(m.get("content", "")) for m in body["messages"] if isinstance(m, dict)
                              and m.get("role") == "user")
        if not isinstance(prompt, str):
            raise HTTPException(status_code=400, detail="Provide 'prompt' or 'messages'")
        d = get_default_router().route(prompt)
        return {"category": d.category.value, "confidence": d.confidence, "model_hint": d.model_hint,
                "rule": d.rule, "reasoning": d.reasoning}

    @app.get("/v1/obs-report")
    async def obs_report(threshold_ms: float = 200.0):
        """Latency percentiles per operation and the ones above ``threshold_ms`` with hints."""
        from .obs_report import generate_report

        return generate_report(st.aeng, telemetry.tracer(), threshold_ms)

    @app.get("/v1/startup")
    async def startup():
        """Wall time of each initialisation phase of this process."""
        from ..utils.startup import report

        return report().to_dict()

    @app.get("/v1/trace")
    async def get_trace():
        return telemetry.tracer().to_chrome()

    @app.delete("/v1/trace")
    async def clear_trace():
        telemetry.tracer().clear()
        return {"cleared": True}

    @app.post("/v1/tokenize")
    async def tokenize(request: Request):
        _check_auth(request, st)
        body = await _json(request)
        if "messages" in body:
            text = apply_chat_template(body["messages"], st.tok, st.arch)
        elif "text" in body:
            text = body["text"]
        else:
            raise HTTPException(status_code=400, detail="Provide 'text' or 'messages' in request body")
        ids = st.tok.encode(text)
        return {"token_ids": ids, "token_count": len(ids), "model": st.model_name}

    @app.post("/v1/sessions/save")
    async def save_session(request: Request):
        """Keep a conversation's KV cache: the chat (``messages``, with the assistant's reply as
        the last message) or ``text`` is tokenized as the model saw it, and its cached blocks are
        copied to the host / disk KV tiers now, so a follow-up turn, also after a restart on the
        same disk directory, starts from them."""
        _check_auth(request, st)
        body = await _json(request)
        if "messages" in body:
            # (the template's trailing assistant prompt only touches the last, partial block)
            text = apply_chat_template(body["messages"], st.tok, st.arch)
        elif "text" in body:
            text = body["text"]
        else:
            raise HTTPException(status_code=400, detail="Provide 'text' or 'messages' in request body")
        ids = st.tok.encode(text)
        loop = asyncio.get_running_loop()
        try:
            n = await loop.run_in_executor(None, lambda: st.aeng.call(lambda eng: eng.save_session(ids)))
        except ValueError as exc:
            raise HTTPException(status_code=400, detail=str(exc)) from exc
        return {"blocks_saved": n, "token_count": len(ids), "model": st.model_name}

    @app.post("/v1/detokenize")
    async def detokenize(request: Request):
        _check_auth(request, st)
        body = await _json(request)
        ids = body.get("token_ids") or body.get("tokens")
        if not isinstance(ids, list):
            raise HTTPException(status_code=400, detail="Provide 'token_ids'")
        return {"text": st.tok.decode(ids), "model": st.model_name}

    # ------------------------------------------------------------------ chat completions
    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        _check_auth(request, st)
        body = await _json(request)
        messages = body.get("messages")
        if not isinstance(messages, list) or not messages:
            raise HTTPException(status_code=400, detail="'messages' must be a non-empty list")
        tools = body.get("tools") or None
        if body.get("tool_choice") == "none":
            tools = None
        if st.compress_prompt:
            from ..context.prompt_compressor import compress_messages

            cp = st.compress_prompt
            messages = compress_messages(messages, cp.get("ratio", 0.5), cp.get("min_tokens", 256),
                                         cp.get("preserve_tokens", 0))
        with telemetry.span("chat_template"):
            prompt = apply_chat_template(messages, st.tok, st.arch, tools=tools)
            prompt_ids = st.tok.encode(prompt)
        params = sampling_from_openai(body, 512, [st.tok.eos_token_id] if st.tok.eos_token_id is not None else [])
        stops = _stop_strings(body)
        n = max(1, parse_int(body.get("n"), "n", 1, lo=1))
        rid = f"chatcmpl-{uuid.uuid4().hex[:24]}"
        created = int(time.time())
        include_usage = bool((body.get("stream_options") or {}).get("include_usage"))
        if body.get("stream"):
            if n != 1:
                raise HTTPException(status_code=400, detail="streaming supports n = 1")
            gf = st.format_factory(body.get("response_format"))
            if gf:
                params = dataclasses.replace(params, grammar=gf.json())
            return StreamingResponse(_chat_stream(st, rid, created, prompt_ids, params, stops, tools, include_usage),
                                     media_type="text/event-stream")
        gf = st.format_factory(body.get("response_format"))
        sc = body.get("self_consistency")
        if isinstance(sc, dict):  # sample k chains, answer with the majority's chain
            n = max(2, min(parse_int(sc.get("k"), "self_consistency.k", 5), 32))
            if params.temperature <= 0:
                params = dataclasses.replace(params, temperature=float(sc.get("temperature", 0.7)))
        per = [dataclasses.replace(params, grammar=gf.json() if gf else None,
                                   seed=None if params.seed is None else params.seed + i) for i in range(n)]
        results = await asyncio.gather(*[_run_one(st, prompt_ids, p, stops) for p in per])
        if isinstance(sc, dict):
            from ..reasoning.self_consistency import SelfConsistencyConfig, SelfConsistencyVoter

            vote = SelfConsistencyVoter(SelfConsistencyConfig(k=n, answer_pattern=sc.get("answer_pattern"))).vote(
                [r[0] for r in results])
            ctoks = sum(len(r[1]) for r in results)
            text, _, reason, _ = results[vote.winner_index]
            return {"id": rid, "object": "chat.completion", "created": created, "model": st.model_name,
                    "choices": [{"index": 0, "message": {"role": "assistant", "content": text},
                                 "finish_reason": reason, "logprobs": None}],
                    "self_consistency": {"answer": vote.answer, "votes": vote.votes, "k": n,
                                         "agreement": vote.agreement, "distribution": vote.distribution},
                    "usage": {"prompt_tokens": len(prompt_ids), "completion_tokens": ctoks,
                              "total_tokens": len(prompt_ids) + ctoks}}
        choices, completion_tokens = [], 0
        for i, (text, ids, reason, _) in enumerate(results):
            msg = {"role": "assistant", "content": text}
            if tools:
                content, calls = parse_tool_calls(text)
                if calls:
                    msg = {"role": "assistant", "content": content or None, "tool_calls": calls}
                    reason = "tool_calls"
            choices.append({"index": i, "message": msg, "finish_reason": reason, "logprobs": None})
            completion_tokens += len(ids)
        return {"id": rid, "object": "chat.completion", "created": created, "model": st.model_name,
                "choices": choices,
                "usage": {"prompt_tokens": len(prompt_ids), "completion_tokens": completion_tokens,
                          "total_tokens": len(prompt_ids) + completion_tokens}}

    # ------------------------------------------------------------------ completions
    @app.post("/v1/completions")
    async def completions(request: Request):
        _check_auth(request, st)
        body = await _json(request)
        prompt = body.get("prompt")
        if isinstance(prompt, str):
            prompts = [st.tok.encode(prompt)]
        elif isinstance(prompt, list) and prompt and all(isinstance(t, int) for t in prompt):
            prompts = [prompt]
        elif isinstance(prompt, list) and prompt and all(isinstance(p, str) for p in prompt):
            prompts = [st.tok.encode(p) for p in prompt]
        elif isinstance(prompt, list) and prompt and all(isinstance(p, list) for p in prompt):
            prompts = [list(map(int, p)) for p in prompt]
        else:
            raise HTTPException(status_code=400, detail="'prompt' must be a string, token list, or a list of those")
        params = sampling_from_openai(body, 256, [st.tok.eos_token_id] if st.tok.eos_token_id is not None else [])
        stops = _stop_strings(body)
        rid = f"cmpl-{uuid.uuid4().hex[:24]}"
        created = int(time.time())
        if body.get("stream"):
            if len(prompts) != 1:
                raise HTTPException(status_code=400, detail="streaming supports a single prompt")
            gf = st.format_factory(body.get("response_format"))
            if gf:
                params = dataclasses.replace(params, grammar=gf.json())
            return StreamingResponse(_completion_stream(st, rid, created, prompts[0], params, stops),
                                     media_type="text/event-stream")
        gf = st.format_factory(body.get("response_format"))
        results = await asyncio.gather(*[_run_one(st, p, dataclasses.replace(params, grammar=gf.json()) if gf
                                                  else params, stops) for p in prompts])
        echo = bool(body.get("echo"))
        choices, ptoks, ctoks = [], 0, 0
        for i, ((text, ids, reason, pt), p) in enumerate(zip(results, prompts)):
            if echo:
                text = st.tok.decode(p) + text
            choices.append({"index": i, "text": text, "finish_reason": reason, "logprobs": None})
            ptoks += pt
            ctoks += len(ids)
        return {"id": rid, "object": "text_completion", "created": created, "model": st.model_name,
                "choices": choices, "usage": {"prompt_tokens": ptoks, "completion_tokens": ctoks,
                                              "total_tokens": ptoks + ctoks}}

    # ------------------------------------------------------------------ embeddings
    @app.post("/v1/embeddings")
    async def embeddings(request: Request):
        _check_auth(request, st)
        body = await _json(request)
        inputs = parse_embedding_input(body.get("input"))
        vecs, total = await embed_texts(st, inputs)
        return {"object": "list", "model": st.model_name,
                "data": [{"object": "embedding", "index": i, "embedding": v} for i, v in enumerate(vecs)],
                "usage": {"prompt_tokens": total, "total_tokens": total}}

    # ------------------------------------------------------------------ LocalAI probes
    @app.get("/")
    async def root():
        return {"status": "ok", "name": "squish-b200", "version": VERSION}

    @app.get("/chat")
    async def chat_ui():
        """Browser chat page (streams from /v1/chat/completions)."""
        from pathlib import Path

        from fastapi.responses import HTMLResponse

        return HTMLResponse((Path(__file__).parent / "static" / "chat.html").read_text())

    @app.get("/v1/version")
    async def version():
        return {"version": VERSION}

    @app.get("/readyz")
    async def readyz():
        return {"status": "ready" if st.aeng.alive else "starting"}

    from .ollama import mount_ollama

    mount_ollama(app, st)
    return app


async def embed_texts(st: ServerState, texts: list[str]) -> tuple[list[list[float]], int]:
    """Last-token hidden state (after the final RMSNorm), L2-normalised, per input."""
    out, total = [], 0
    for t in texts:
        ids = st.tok.encode(t) or [st.tok.eos_token_id or 0]
        total += len(ids)
        params = SamplingParams(max_tokens=1, temperature=0.0, ignore_eos=True, return_hidden=True)
        rid, sink = st.aeng.submit(ids, params, asyncio.get_running_loop())
        ev = None
        while True:
            ev = await sink.aq.get()
            if ev.finished:
                break
        h = st.aeng.engine.hidden_states.pop(rid, None)
        if h is None:
            raise HTTPException(status_code=500, detail="embedding unavailable")
        v = np.asarray(h, dtype=np.float32)
        v = v / (np.linalg.norm(v) + 1e-12)
        out.append(v.tolist())
    return out, total


def _sse(obj) -> bytes:
    return f"data: {json.dumps(obj)}\n\n".encode()


async def _chat_stream(st, rid, created, prompt_ids, params, stops, tools, include_usage):
    base = {"id": rid, "object": "chat.completion.chunk", "created": created, "model": st.model_name}
    yield _sse({**base, "choices": [{"index": 0, "delta": {"role": "assistant", "content": ""},
                                     "finish_reason": None}]})
    detok = IncrementalDetokenizer(st.tok)
    filt = ToolCallStreamFilter() if tools else None
    text_all, n_out, reason, ids = "", 0, "stop", []
    key = _cache_key(st, prompt_ids, params, stops)
    async for ev in _events(st, prompt_ids, params, stops):
        n_out += len(ev.token_ids)
        ids.extend(ev.token_ids)
        delta = getattr(ev, "cached_text", None)
        if delta is None:
            delta = detok.push(ev.token_ids)
        text_all += delta
        hit = False
        if stops:
            cut, hit = _truncate_at_stop(text_all, stops)
            if hit:
                delta = delta[: max(0, len(delta) - (len(text_all) - len(cut)))]
                text_all = cut
        if filt is not None:
            delta = filt.push(delta)
        if delta:
            yield _sse({**base, "choices": [{"index": 0, "delta": {"content": delta}, "finish_reason": None}]})
        if hit:
            reason = "stop"
            break
        if ev.finished:
            reason = _finish_reason(ev.reason)
            break
    if key is not None and reason in ("stop", "length") and not hasattr(ev, "cached_text"):
        st.cache.put(key, (text_all, tuple(ids), reason))
    if tools:
        _, calls = parse_tool_calls(text_all)
        if calls:
            reason = "tool_calls"
            yield _sse({**base, "choices": [{"index": 0, "delta": {"tool_calls": [dict(c, index=i) for i, c in
                                                                                  enumerate(calls)]},
                                             "finish_reason": None}]})
    yield _sse({**base, "choices": [{"index": 0, "delta": {}, "finish_reason": reason}]})
    if include_usage:
        yield _sse({**base, "choices": [], "usage": {"prompt_tokens": len(prompt_ids), "completion_tokens": n_out,
                                                     "total_tokens": len(prompt_ids) + n_out}})
    yield b"data: [DONE]\n\n"


async def _completion_stream(st, rid, created, prompt_ids, params, stops):
    base = {"id": rid, "object": "text_completion", "created": created, "model": st.model_name}
    detok = IncrementalDetokenizer(st.tok)
    text_all = ""
    async for ev in _events(st, prompt_ids, params, stops):
        delta = getattr(ev, "cached_text", None)
        if delta is None:
            delta = detok.push(ev.token_ids)
        text_all += delta
        hit = False
        if stops:
            cut, hit = _truncate_at_stop(text_all, stops)
            if hit:
                delta = delta[: max(0, len(delta) - (len(text_all) - len(cut)))]
        reason = None
        if hit:
            reason = "stop"
        elif ev.finished:
            reason = _finish_reason(ev.reason)
        yield _sse({**base, "choices": [{"index": 0, "text": delta, "finish_reason": reason, "logprobs": None}]})
        if reason:
            break
    yield b"data: [DONE]\n\n"
