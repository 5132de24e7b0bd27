"""Serving flags on CPU ranks: speculative decoding through the HTTP API (prompt lookup,
draft model, Jacobi must reproduce plain greedy output), the data-parallel request router,
the tensor-parallel serving loop over gloo ranks, page size, and JSON logging.

The reference serves with prompt lookup on by default (squish/server.py:5194, dispatch
:1992-2016) and takes ``--draft-model`` (:4892), ``--jacobi`` (:5241) and ``--log-level``
(:5009); greedy-lossless speculation is its contract (tests/test_prompt_lookup_batched.py).
"""
import io
import json
import logging
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from fastapi.testclient import TestClient

from squish_b200.api import load_engine
from squish_b200.cli import _ecfg, _parallel, _spec, build_parser
from squish_b200.engine.sampling import SamplingParams
from squish_b200.serving.async_engine import AsyncEngine
from squish_b200.serving.multi import DPRouter
from squish_b200.serving.server import ServerState, create_app
from squish_b200.serving.tokenizer import ByteTokenizer

BASE = ["serve", "tiny-llama", "--device", "cpu", "--max-num-seqs", "4", "--max-model-len", "512",
        "--no-cuda-graphs"]


def _args(*extra):
    return build_parser().parse_args(BASE + list(extra))


def test_flags_build_the_engine_config():
    assert _spec(_args()).method == "prompt_lookup"  # on by default, as in the reference
    assert _spec(_args("--no-prompt-lookup")) is None
    sc = _spec(_args("--medusa-heads", "heads.safetensors", "--medusa-top-k", "3"))
    assert (sc.method, sc.medusa_heads, sc.medusa_top_k) == ("medusa", "heads.safetensors", 3)
    sc = _spec(_args("--eagle-head", "eagle_dir", "--medusa-heads", "x"))
    assert (sc.method, sc.eagle_head) == ("eagle", "eagle_dir")
    sc = _spec(_args("--redrafter-head", "rd.safetensors", "--eagle-head", "e"))
    assert (sc.method, sc.redrafter_head) == ("redrafter", "rd.safetensors")
    s = _spec(_args("--prompt-lookup-n", "4", "--prompt-lookup-k", "6"))
    assert (s.ngram_max, s.k) == (4, 6)
    assert _spec(_args("--jacobi", "--draft-depth", "3")).method == "jacobi"
    d = _spec(_args("--draft-model", "tiny-llama", "--draft-depth", "2", "--jacobi"))
    assert (d.method, d.draft_model, d.k) == ("draft", "tiny-llama", 2)
    assert _parallel(_args("--gpus", "8", "--tp", "2")) == (2, 4)
    assert _parallel(_args("--ep", "4")) == (4, 1)
    assert _parallel(_args("--dp", "2")) == (1, 2)
    with pytest.raises(SystemExit):
        _parallel(_args("--gpus", "6", "--tp", "4"))
    e = _ecfg(_args("--tp", "2", "--tp-mode", "nccl"))
    assert (e.tp, e.tp_mode) == (2, "nccl")
    e = _ecfg(_args("--kv-sink-tokens", "4", "--kv-window-tokens", "256", "--prompt-logit-cache", "0"))
    assert (e.kv_sink_tokens, e.kv_window_tokens, e.prompt_logit_cache) == (4, 256, 0)
    assert _ecfg(_args()).prompt_logit_cache > 0
    assert _ecfg(_args("--pp", "2")).pp == 2
    assert _ecfg(_args("--offload-layers", "3")).offload_layers == 3
    e = _ecfg(_args("--kv-h2o-budget", "512", "--kv-h2o-interval", "8", "--kv-h2o-decay", "0.9"))
    assert (e.kv_h2o_budget, e.kv_h2o_interval, e.kv_h2o_decay) == (512, 8, 0.9)
    assert _ecfg(_args("--kv-budget-adaptive")).kv_budget_adaptive


def _client(*extra):
    a = _args(*extra)
    ld = load_engine("tiny-llama", "cpu", seed=0, ecfg=_ecfg(a), page_size=a.page_size)
    tok = ByteTokenizer(ld.engine.cfg.vocab_size, ld.engine.cfg.eos_token_id)
    aeng = AsyncEngine(ld.engine, tok, model_name="tiny").start()
    return aeng, TestClient(create_app(ServerState(aeng, "tiny", api_key=None, arch="llama")))


def _greedy(client, text, n=24):
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": text, "max_tokens": n, "temperature": 0})
    assert r.status_code == 200, r.text
    return r.json()["choices"][0]["text"]


# a prompt that repeats itself, so n-gram drafts exist and get verified
PROMPT = "the cat sat on the mat. the cat sat on the mat. the cat sat on the"


@pytest.mark.parametrize("flags", [["--no-prompt-lookup"], [], ["--prompt-lookup-k", "6", "--spec-branches", "2"],
                                   ["--jacobi"], ["--draft-model", "tiny-llama", "--draft-depth", "3"]])
def test_speculative_serving_is_greedy_lossless(flags):
    base_eng, base = _client("--no-prompt-lookup")
    want = _greedy(base, PROMPT)
    base_eng.stop()
    aeng, c = _client(*flags)
    try:
        got = _greedy(c, PROMPT)
        assert got == want
        if flags and flags[0] in ("--jacobi", "--draft-model") or flags == []:
            assert aeng.engine.proposer is not None
    finally:
        aeng.stop()


def test_page_size_flag_reaches_the_kv_pool():
    aeng, c = _client("--page-size", "32", "--no-prompt-lookup")
    try:
        assert aeng.engine.qcfg.page_size == 32 and aeng.engine.blocks.page_size == 32
        assert _greedy(c, "hello there", 8)
    finally:
        aeng.stop()


def test_dp_router_spreads_requests_and_serves_http():
    reps = []
    for _ in range(2):
        a = _args("--no-prompt-lookup")
        ld = load_engine("tiny-llama", "cpu", seed=0, ecfg=_ecfg(a))
        tok = ByteTokenizer(ld.engine.cfg.vocab_size, ld.engine.cfg.eos_token_id)
        reps.append(AsyncEngine(ld.engine, tok, model_name="tiny"))
    router = DPRouter(reps).start()
    try:
        c = TestClient(create_app(ServerState(router, "tiny", api_key=None, arch="llama")))
        outs = [_greedy(c, f"request {i}", 6) for i in range(4)]
        assert len(set(outs)) >= 1
        assert all(r.requests_total >= 1 for r in reps)  # both replicas served
        # same weights on both replicas: the same prompt gives the same greedy text on either
        assert _greedy(c, "same prompt", 10) == _greedy(c, "same prompt", 10)
        m = c.get("/v1/metrics").text
        assert "squish_requests_total" in m and "squish_paged_kv_free_blocks" in m
        ev = router.generate([5, 6, 7], SamplingParams(max_tokens=4, ignore_eos=True))
        assert ev.finished and len(ev.token_ids) == 4
        e = c.post("/v1/embeddings", json={"model": "tiny", "input": ["a", "bb"]})
        assert e.status_code == 200 and len(e.json()["data"]) == 2
    finally:
        router.stop()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_engine(ecfg):
    """tiny-llama with an FFN width whose halves stay aligned to the quantization groups."""
    import dataclasses

    from squish_b200.engine.engine import LLMEngine
    from squish_b200.models.config import get_preset
    from squish_b200.models.weights import random_checkpoint

    cfg, q = get_preset("tiny-llama")
    cfg = dataclasses.replace(cfg, tie_embeddings=False, intermediate_size=512)
    ecfg.num_pages = 128
    return LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0), "cpu", ecfg)


def _tp_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from squish_b200.serving.multi import TPAsyncEngine, TPControl, follow

        a = _args("--tp", str(world), "--no-prompt-lookup", "--max-num-batched-tokens", "64")
        eng = _tp_engine(_ecfg(a))
        ctrl = TPControl()
        if rank == 0:
            tok = ByteTokenizer(eng.cfg.vocab_size, eng.cfg.eos_token_id)
            aeng = TPAsyncEngine(eng, ctrl, tok, model_name="tiny").start()
            import concurrent.futures as cf

            prompts = [[3, 4, 5, 6], [9] * 30, list(range(40, 70))]
            with cf.ThreadPoolExecutor(3) as ex:
                evs = list(ex.map(lambda p: aeng.generate(p, SamplingParams(max_tokens=7, ignore_eos=True),
                                                          timeout=120), prompts))
            aeng.stop()
            q.put((rank, [e.token_ids for e in evs]))
        else:
            q.put((rank, follow(eng, ctrl)))
    finally:
        dist.destroy_process_group()


def test_tp_serving_ranks_follow_rank_zero():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[1] > 0  # the follower ran steps
    # the single-process engine gives the same greedy tokens
    a = _args("--no-prompt-lookup", "--max-num-batched-tokens", "64")
    eng = _tp_engine(_ecfg(a))
    prompts = [[3, 4, 5, 6], [9] * 30, list(range(40, 70))]
    want = [o for o in eng.generate(prompts, SamplingParams(max_tokens=7, ignore_eos=True))]
    assert res[0] == want


def test_json_logging_lines():
    from squish_b200.utils.logconfig import configure_logging, get_logger

    buf = io.StringIO()
    configure_logging("info", json_format=True, stream=buf)
    get_logger("serving.test").info("loaded %s", "tiny", extra={"load_s": 1.5})
    get_logger("serving.test").debug("hidden")
    configure_logging("info", json_format=True, stream=buf)  # reconfiguring does not duplicate lines
    get_logger("x").warning("again")
    lines = [json.loads(x) for x in buf.getvalue().splitlines()]
    assert len(lines) == 2
    assert lines[0]["message"] == "loaded tiny" and lines[0]["level"] == "INFO" and lines[0]["load_s"] == 1.5
    assert lines[0]["logger"] == "squish_b200.serving.test"
    assert lines[1]["logger"] == "squish_b200.x"
    configure_logging("warning")
    assert logging.getLogger("squish_b200").level == logging.WARNING
