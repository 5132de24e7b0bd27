"""HTTP surface (OpenAI, Ollama, LocalAI, metrics) over the CPU oracle engine."""
import json

import pytest
from fastapi.testclient import TestClient

from squish_b200.engine.engine import EngineConfig, LLMEngine
from squish_b200.models.config import get_preset
from squish_b200.models.weights import random_checkpoint
from squish_b200.serving.async_engine import AsyncEngine
from squish_b200.serving.memory_governor import CRITICAL, MemoryGovernor
from squish_b200.serving.server import ServerState, create_app
from squish_b200.serving.tokenizer import ByteTokenizer
from squish_b200.serving.tool_calling import parse_tool_calls


@pytest.fixture(scope="module")
def client():
    cfg, q = get_preset("tiny-llama")
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0, device="cpu"), "cpu",
                                    EngineConfig(max_num_seqs=8, max_model_len=512, num_pages=256))
    aeng = AsyncEngine(eng, ByteTokenizer(cfg.vocab_size, cfg.eos_token_id), model_name="tiny").start()
    st = ServerState(aeng, "tiny", api_key=None, arch="llama")
    with TestClient(create_app(st)) as c:
        yield c
    aeng.stop()


def test_models_health_metrics(client):
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    h = client.get("/health").json()
    assert h["status"] == "ok" and h["model_loaded"]
    m = client.get("/v1/metrics").text
    assert "squish_requests_total" in m and "squish_paged_kv_free_blocks" in m
    assert 'squish_step_seconds_bucket{gpu="cpu",le="+Inf"}' in m and "squish_step_seconds_sum" in m
    assert client.get("/readyz").json()["status"] == "ready"


def test_chat_completion_nonstream(client):
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 5,
                                                  "temperature": 0, "ignore_eos": True})
    assert r.status_code == 200, r.text
    d = r.json()
    assert d["object"] == "chat.completion"
    assert d["usage"]["completion_tokens"] == 5
    assert d["choices"][0]["finish_reason"] == "length"


def test_chat_completion_stream_with_usage(client):
    with client.stream("POST", "/v1/chat/completions",
                       json={"messages": [{"role": "user", "content": "hello"}], "max_tokens": 4, "stream": True,
                             "temperature": 0, "ignore_eos": True, "stream_options": {"include_usage": True}}) as r:
        lines = [l for l in r.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(l[6:]) for l in lines[:-1]]
    assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
    assert chunks[-1]["usage"]["completion_tokens"] == 4
    assert any(c["choices"] and c["choices"][0]["finish_reason"] == "length" for c in chunks)


def test_completions_tokens_and_batch(client):
    r = client.post("/v1/completions", json={"prompt": ["a", "bb"], "max_tokens": 3, "temperature": 0,
                                             "ignore_eos": True})
    d = r.json()
    assert len(d["choices"]) == 2 and d["usage"]["completion_tokens"] == 6
    r = client.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 2, "temperature": 0,
                                             "ignore_eos": True})
    assert r.json()["usage"]["prompt_tokens"] == 3


def test_validation_errors(client):
    assert client.post("/v1/chat/completions", json={"messages": []}).status_code == 400
    assert client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                      "temperature": 5}).status_code == 400
    assert client.post("/v1/completions", content="not json").status_code == 400


def test_tokenize_and_embeddings(client):
    t = client.post("/v1/tokenize", json={"text": "abc"}).json()
    assert t["token_count"] == 3
    e = client.post("/v1/embeddings", json={"input": ["abc", "de"]}).json()
    assert len(e["data"]) == 2 and len(e["data"][0]["embedding"]) == 256
    v = e["data"][0]["embedding"]
    assert abs(sum(x * x for x in v) - 1.0) < 1e-3


def test_ollama_routes(client):
    assert "version" in client.get("/api/version").json()
    assert client.get("/api/tags").json()["models"][0]["name"] == "tiny"
    r = client.post("/api/generate", json={"model": "tiny", "prompt": "hey", "stream": False,
                                           "options": {"num_predict": 3, "temperature": 0}})
    d = r.json()
    assert d["done"] and d["eval_count"] >= 1
    with client.stream("POST", "/api/chat", json={"model": "tiny", "messages": [{"role": "user", "content": "yo"}],
                                                  "options": {"num_predict": 3, "temperature": 0}}) as r:
        rows = [json.loads(l) for l in r.iter_lines() if l]
    assert rows[-1]["done"] and rows[-1]["eval_count"] >= 1
    assert client.post("/api/pull", json={"name": "x"}).status_code == 501
    assert client.post("/api/show", json={"model": "tiny"}).json()["details"]["family"] == "llama"


def test_tool_call_parsing():
    content, calls = parse_tool_calls('ok <tool_call>{"name": "get_weather", "arguments": {"city": "Oslo"}}'
                                      '</tool_call>')
    assert content == "ok" and calls[0]["function"]["name"] == "get_weather"
    assert json.loads(calls[0]["function"]["arguments"]) == {"city": "Oslo"}


def test_memory_governor_levels():
    state = {"free": 50.0}
    gov = MemoryGovernor(mem_probe=lambda: (state["free"], 100.0), kv_usage=lambda: 0.1)
    seen = []
    gov.on_change(lambda a, b: seen.append(b))
    assert gov.evaluate() == 0
    state["free"] = 1.0
    assert gov.evaluate() == CRITICAL and gov.critical
    assert seen == [CRITICAL]


def test_response_cache_quality_and_chat_page(client):
    body = {"messages": [{"role": "user", "content": "cache me"}], "max_tokens": 6, "temperature": 0,
            "ignore_eos": True}
    q0 = client.get("/v1/quality").json()["response_cache"]
    a = client.post("/v1/chat/completions", json=body).json()
    b = client.post("/v1/chat/completions", json=body).json()
    assert a["choices"][0]["message"] == b["choices"][0]["message"]
    assert a["usage"] == b["usage"]
    q = client.get("/v1/quality?window=600").json()
    assert q["response_cache"]["hits"] == q0["hits"] + 1
    # the streamed form of the same request replays the cached answer
    with client.stream("POST", "/v1/chat/completions", json=dict(body, stream=True)) as r:
        chunks = [json.loads(l[6:]) for l in r.iter_lines() if l.startswith("data: {")]
    text = "".join(c["choices"][0]["delta"].get("content", "") for c in chunks if c["choices"])
    assert text == a["choices"][0]["message"]["content"]
    # sampled requests are never cached
    client.post("/v1/chat/completions", json=dict(body, temperature=0.8, seed=1))
    assert client.get("/v1/quality").json()["response_cache"]["hits"] == q0["hits"] + 2
    m = q["models"][0]
    assert m["model_id"] == "tiny" and m["n_requests"] >= 1 and m["error_rate"] == 0.0
    assert m["latency_p50_ms"] > 0 and m["ttft_p50_ms"] is not None
    assert client.get("/v1/quality?window=0").status_code == 400
    page = client.get("/chat")
    assert page.status_code == 200 and "/v1/chat/completions" in page.text


def test_loop_detector():
    import numpy as np

    from squish_b200.serving.loop_guard import LoopGuard, detect_loop

    rng = np.random.default_rng(0)
    assert not detect_loop(rng.integers(0, 30000, 400).tolist())
    assert detect_loop(rng.integers(0, 100, 50).tolist() + [5, 6, 7] * 4)          # short unit, 4 reps
    assert not detect_loop(rng.integers(0, 100, 50).tolist() + [5, 6, 7] * 3)      # 3 reps: not yet
    block = rng.integers(0, 30000, 40).tolist()
    assert detect_loop(rng.integers(0, 100, 20).tolist() + block * 2)               # a sentence twice
    noisy = block * 3
    noisy[70] = 1                                                                    # one drifting token
    assert detect_loop(noisy)
    g = LoopGuard()
    fired = [g.feed([9, 8]) for _ in range(20)]
    assert fired.index(True) == 7  # first check after 16 tokens


class _LoopingEngine:
    """Engine stand-in whose only request emits the same two tokens forever."""

    def __init__(self):
        from squish_b200.engine.request import RequestOutput

        self.RO = RequestOutput
        self.requests, self.live, self.aborted = {}, set(), []

    def add_request(self, prompt, params, rid):
        self.requests[rid] = params
        self.live.add(rid)

    def has_unfinished(self):
        return bool(self.live)

    def abort(self, rid):
        self.aborted.append(rid)
        self.live.discard(rid)

    def step(self):
        return [self.RO(r, [11, 12], False, None, 3, 0) for r in list(self.live)]


def test_async_engine_stops_a_loop_with_repetition():
    from squish_b200.engine.sampling import SamplingParams

    eng = _LoopingEngine()
    aeng = AsyncEngine(eng, ByteTokenizer(300, 2), model_name="fake").start()
    try:
        ev = aeng.generate([1, 2, 3], SamplingParams(max_tokens=10_000), timeout=30)
    finally:
        aeng.stop()
    assert ev.reason == "repetition" and ev.finished
    assert 16 <= len(ev.token_ids) <= 64
    assert eng.aborted and aeng.loops_stopped == 1
    # ignore_eos requests (benchmarks) run to max_tokens even when they loop
    eng2 = _LoopingEngine()
    aeng2 = AsyncEngine(eng2, ByteTokenizer(300, 2), model_name="fake").start()
    try:
        rid, sink = aeng2.submit([1, 2, 3], SamplingParams(max_tokens=100, ignore_eos=True))
        got = []
        import time as _t

        t0 = _t.time()
        while len(got) < 100 and _t.time() - t0 < 20:
            try:
                ev = sink.q.get(timeout=1)
            except Exception:  # noqa: BLE001
                continue
            got += ev.token_ids
            assert ev.reason != "repetition"
        aeng2.abort(rid)
    finally:
        aeng2.stop()
    assert len(got) >= 100 and aeng2.loops_stopped == 0


def test_obs_report(client):
    client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 3, "temperature": 0.5, "seed": 3})
    r = client.get("/v1/obs-report?threshold_ms=0").json()
    assert r["status"] == "degraded" and "engine.step" in r["profile"]
    assert r["profile"]["engine.step"]["n_samples"] >= 1
    ops = {b["op"] for b in r["bottlenecks"]}
    assert "engine.step" in ops and all(b["hint"] for b in r["bottlenecks"] if b["op"] in ("engine.step", "ttft_ms"))
    assert client.get("/v1/obs-report?threshold_ms=1e9").json()["status"] == "ok"


def test_prompt_router_and_backend_router(client, monkeypatch):
    import re

    from squish_b200.serving.backend_router import BackendConfig, BackendRouter
    from squish_b200.serving.router import PromptRouter, RouterCategory, RouterConfig, RouterRule

    r = PromptRouter()
    assert r.route("```python\nprint(1)\n```").category == RouterCategory.CODE
    assert r.route("Solve the equation 3x + 2 = 11").category == RouterCategory.MATH
    assert r.route("Write a poem about the sea").category == RouterCategory.CREATIVE
    assert r.route("Who painted the Mona Lisa?").category == RouterCategory.FACTUAL
    d = r.route("hey there, nice to meet you")
    assert d.category == RouterCategory.CONVERSATION and d.confidence == 0.5
    assert r.route("   ").category == RouterCategory.UNKNOWN
    custom = PromptRouter(RouterConfig(rules=[RouterRule("sql", RouterCategory.CODE, re.compile("select .* from",
                                                                                              re.I), 99, "sql-model")]))
    assert custom.route("SELECT a FROM t").model_hint == "sql-model"
    j = client.post("/v1/route", json={"messages": [{"role": "user", "content": "debug this rust function"}]}).json()
    assert j["category"] == "code" and j["confidence"] == 1.0
    monkeypatch.setenv("SQUISH_BACKEND", "ollama")
    monkeypatch.delenv("SQUISH_BACKEND_URL", raising=False)
    br = BackendRouter(BackendConfig())
    assert br.proxy_url("v1/chat/completions") == "http://127.0.0.1:11434/v1/chat/completions"
    monkeypatch.setenv("SQUISH_BACKEND_URL", "http://127.0.0.1:9/")
    assert BackendRouter(BackendConfig()).health_check(timeout=0.2) is False  # nothing listens on port 9
    with pytest.raises(ValueError):
        BackendConfig(backend="nope")


def test_session_save_route(tmp_path):
    """POST /v1/sessions/save runs on the engine thread: without a KV tier it is refused, with a
    disk tier the conversation's full blocks land on disk."""
    from squish_b200.serving.async_engine import AsyncEngine
    from squish_b200.serving.server import ServerState, create_app

    cfg, q = get_preset("tiny-llama")
    for tier, want in ((False, 400), (True, 200)):
        kw = {"kv_disk_dir": str(tmp_path / "kv"), "kv_host_bytes": 1 << 20} if tier else {}
        eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0, device="cpu"), "cpu",
                                        EngineConfig(max_num_seqs=4, max_model_len=512, num_pages=64, **kw))
        aeng = AsyncEngine(eng, ByteTokenizer(cfg.vocab_size, cfg.eos_token_id), model_name="tiny").start()
        with TestClient(create_app(ServerState(aeng, "tiny", api_key=None, arch="llama"))) as c:
            text = "a conversation long enough to fill a few sixteen-token KV pages " * 2
            c.post("/v1/completions", json={"prompt": text, "max_tokens": 2, "temperature": 0})
            r = c.post("/v1/sessions/save", json={"text": text})
            assert r.status_code == want, r.text
            if tier:
                assert r.json()["blocks_saved"] >= 4 and list((tmp_path / "kv").glob("*.npz"))
        aeng.stop()


def test_engine_thread_call_returns_and_raises():
    """AsyncEngine.call runs a function on the engine thread between steps and hands back its
    result or its exception."""
    cfg, q = get_preset("tiny-llama")
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0, device="cpu"), "cpu",
                                    EngineConfig(max_num_seqs=2, max_model_len=256, num_pages=32))
    aeng = AsyncEngine(eng, ByteTokenizer(cfg.vocab_size, cfg.eos_token_id), model_name="tiny").start()
    try:
        import threading

        assert aeng.call(lambda e: (e is eng, threading.current_thread() is not threading.main_thread())) == (True, True)
        with pytest.raises(ValueError, match="KV tier"):
            aeng.call(lambda e: e.save_session(list(range(64))))
    finally:
        aeng.stop()
