"""Engine + scheduler on the CPU oracle runner (tiny Llama config, INT4 g32 weights, INT4 g32 KV)."""
import numpy as np
import pytest
import torch

from squish_b200.engine.engine import EngineConfig, LLMEngine
from squish_b200.engine.sampling import SamplingParams
from squish_b200.models.config import get_preset
from squish_b200.models.reference import ReferenceModel
from squish_b200.models.weights import random_checkpoint


@pytest.fixture(scope="module")
def tiny():
    cfg, q = get_preset("tiny-llama")
    ck = random_checkpoint(cfg, q, seed=0, device="cpu")
    return ck


def _prompt(seed, n, vocab=32000):
    g = np.random.default_rng(seed)
    return g.integers(0, vocab, n).tolist()


def test_engine_greedy_matches_dense_oracle(tiny):
    ref = ReferenceModel(tiny)
    prompts = [_prompt(1, 32), _prompt(2, 19), _prompt(3, 45)]
    want = [ref.greedy(p, 12)[0] for p in prompts]
    eng = LLMEngine.from_checkpoint(tiny, "cpu", EngineConfig(max_num_seqs=4, max_num_batched_tokens=24,
                                                              max_model_len=256, num_pages=64))
    got = eng.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True))
    assert got == want
    assert eng.stats.generated_tokens == 36


def test_prefix_reuse_shares_pages_and_keeps_tokens(tiny):
    shared = _prompt(7, 48)
    p1 = shared + _prompt(8, 10)
    p2 = shared + _prompt(9, 7)
    ref = ReferenceModel(tiny)
    want2 = ref.greedy(p2, 6)[0]
    eng = LLMEngine.from_checkpoint(tiny, "cpu", EngineConfig(max_num_seqs=2, max_num_batched_tokens=64,
                                                              max_model_len=256, num_pages=64))
    eng.generate([p1], SamplingParams(max_tokens=6, ignore_eos=True))
    rid = eng.add_request(p2, SamplingParams(max_tokens=6, ignore_eos=True))
    while eng.has_unfinished():
        eng.step()
    r = eng.requests[rid]
    assert r.prefix_hit_tokens == 48  # three full 16-token pages reused
    assert r.output == want2


def test_preemption_recomputes_and_finishes(tiny):
    prompts = [_prompt(20 + i, 30) for i in range(4)]
    ref = ReferenceModel(tiny)
    want = [ref.greedy(p, 20)[0] for p in prompts]
    # 10 pages of 16 tokens cannot hold 4 x 50 tokens at once -> preemption
    eng = LLMEngine.from_checkpoint(tiny, "cpu", EngineConfig(max_num_seqs=4, max_num_batched_tokens=128,
                                                              max_model_len=128, num_pages=10,
                                                              enable_prefix_caching=False))
    got = eng.generate(prompts, SamplingParams(max_tokens=20, ignore_eos=True))
    assert eng.stats.preemptions > 0
    assert got == want


def test_sampling_params_and_stop(tiny):
    eng = LLMEngine.from_checkpoint(tiny, "cpu", EngineConfig(max_num_seqs=2, max_model_len=128, num_pages=32))
    out = eng.generate([_prompt(30, 10)], SamplingParams(max_tokens=5, temperature=0.8, top_k=20, top_p=0.9,
                                                         seed=1))
    assert len(out[0]) == 5
    first = eng.generate([_prompt(31, 10)], SamplingParams(max_tokens=8, ignore_eos=True))[0]
    tok = first[2]
    stop = eng.generate([_prompt(31, 10)], SamplingParams(max_tokens=8, stop_token_ids=[tok]))[0]
    assert stop == first[: first.index(tok) + 1]
    with pytest.raises(ValueError):
        SamplingParams(top_p=0.0).validate()


def test_repeat_prompt_first_token_without_forward(tiny):
    """A repeated prompt gets its first token from the prompt-logit cache (no step runs for
    it), and the rest of the output is the same as the first time (greedy and sampled)."""
    p = _prompt(31, 37)
    eng = LLMEngine.from_checkpoint(tiny, "cpu", EngineConfig(max_num_seqs=4, max_num_batched_tokens=64,
                                                              max_model_len=256, num_pages=64))
    for params in (SamplingParams(max_tokens=8, ignore_eos=True),
                   SamplingParams(max_tokens=8, ignore_eos=True, temperature=0.8, top_k=50, repetition_penalty=1.2)):
        rid1 = eng.add_request(p, params)
        while eng.has_unfinished():
            eng.step()
        first = eng.requests[rid1].output
        n0, steps0 = eng.stats.instant_first_tokens, eng.stats.steps
        rid2 = eng.add_request(p, params, rid=rid1 + "-again")
        assert eng.stats.instant_first_tokens == n0 + 1
        r2 = eng.requests[rid2]
        assert len(r2.output) == 1 and r2.first_token_time is not None  # before any step
        outs = eng.step()
        assert outs[0].rid == rid2 and outs[0].new_tokens == r2.output[:1]
        while eng.has_unfinished():
            eng.step()
        if params.temperature == 0:
            assert r2.output == first
        assert len(r2.output) == 8 and eng.stats.steps > steps0
    # a one-token request finishes at add time, and the engine reports it on the next step
    rid3 = eng.add_request(p, SamplingParams(max_tokens=1, ignore_eos=True))
    r3 = eng.requests[rid3]
    assert r3.finish_reason == "length" and eng.has_unfinished()
    assert [o.rid for o in eng.step()] == [rid3] and not eng.has_unfinished()


def window_rule(sink_tokens, window, ps=16):
    """Keys the engine's page-granular sink + window eviction leaves visible to query q: after the
    step that made num_computed = q, pages [ceil(sink / ps), (q - window) // ps) are gone."""
    sink = -(-sink_tokens // ps)

    def visible(q, k):
        page = k // ps
        return (page < sink) | (page >= torch.div(q - window, ps, rounding_mode="floor"))
    return visible


def test_sink_and_window_eviction_matches_windowed_oracle(tiny):
    p = _prompt(33, 40)
    eng = LLMEngine.from_checkpoint(tiny, "cpu", EngineConfig(max_num_seqs=2, max_num_batched_tokens=64,
                                                              max_model_len=256, num_pages=64, kv_sink_tokens=4,
                                                              kv_window_tokens=32))
    got = eng.generate([p], SamplingParams(max_tokens=70, ignore_eos=True))[0]
    # the last step computes position 108 (109 tokens): pages [1, (109 - 32) // 16 = 4) were given
    # back; page 0 holds the sinks
    assert eng.stats.evicted_pages == 3
    ref = ReferenceModel(tiny)
    ref.kv_visible = window_rule(4, 32)
    assert got == ref.greedy(p, 70)[0]
    # logits of the last step: equal to the windowed oracle's, and not to full attention's
    seq = p + got[:-1]
    win = ref.forward(seq, ref.new_cache(), 0)[-1]
    full_ref = ReferenceModel(tiny)
    full = full_ref.forward(seq, full_ref.new_cache(), 0)[-1]
    last = eng.runner.last_logits[0]
    assert torch.allclose(last, win, atol=1e-4, rtol=1e-4)
    assert (last - full).abs().max() > 100 * (last - win).abs().max()


def test_hadamard_rotated_kv_keeps_the_model_and_cuts_kv_error(tiny):
    """Rotating q/k/v by a randomized Hadamard transform before the KV codec leaves the model
    unchanged up to quantization (scores and outputs are rotation invariant) and, for INT4 KV
    with outlier channels, lowers the cache's reconstruction error."""
    import dataclasses

    from squish_b200.ops.kernels import sylvester

    d = tiny.config.head_dim
    H = sylvester(d).float()
    assert torch.allclose(H @ H, torch.eye(d), atol=1e-6)
    ck_rot = dataclasses.replace(tiny, quant=dataclasses.replace(tiny.quant, kv_dtype="bf16", kv_hadamard=True))
    ck_bf = dataclasses.replace(tiny, quant=dataclasses.replace(tiny.quant, kv_dtype="bf16"))
    p = _prompt(34, 30)
    a, b = ReferenceModel(ck_rot), ReferenceModel(ck_bf)
    la, lb = a.forward(p, a.new_cache(), 0), b.forward(p, b.new_cache(), 0)
    assert torch.nn.functional.cosine_similarity(la[-1], lb[-1], dim=0) > 0.9999
    # INT4 reconstruction error on keys with outlier channels, with and without rotation
    g = torch.Generator().manual_seed(0)
    k = torch.randn(256, 1, d, generator=g)
    k[..., 3] *= 20.0
    k[..., d - 7] *= 12.0
    m_rot = ReferenceModel(dataclasses.replace(tiny, quant=dataclasses.replace(tiny.quant, kv_hadamard=True)))
    m_plain = ReferenceModel(tiny)
    _, kr, _ = m_rot.rotate_kv(k, k, k)
    err_rot = (m_rot._kv_roundtrip(kr, m_rot.fk) - kr).pow(2).mean()
    err_plain = (m_plain._kv_roundtrip(k, m_plain.fk) - k).pow(2).mean()
    assert err_rot < 0.5 * err_plain
    # the engine on the CPU runner with rotated INT4 KV matches the rotated oracle exactly
    ck4 = dataclasses.replace(tiny, quant=dataclasses.replace(tiny.quant, kv_hadamard=True))
    eng = LLMEngine.from_checkpoint(ck4, "cpu", EngineConfig(max_num_seqs=2, max_num_batched_tokens=64,
                                                             max_model_len=256, num_pages=32))
    assert eng.generate([p], SamplingParams(max_tokens=10, ignore_eos=True))[0] == ReferenceModel(ck4).greedy(p, 10)[0]


def eviction_log_rule(r, ps=16):
    """Keys visible to query position q given a request's eviction record: page b is gone for
    every query at or after the num_computed at which it was evicted."""
    gone = torch.full(((len(r.prompt) + len(r.output)) // ps + 2,), 1 << 30, dtype=torch.int64)
    for b, at in r.evicted_at.items():
        gone[b] = at

    def visible(q, k):
        return q < gone[torch.div(k, ps, rounding_mode="floor")]
    return visible


@pytest.mark.parametrize("decay", [1.0, 0.5])
def test_heavy_hitter_eviction_keeps_budget_and_matches_oracle(tiny, decay):
    """H2O-style eviction: the engine scores pages by accumulated (decay 1) or recency-weighted
    (decay < 1) attention mass, keeps the sequence within its token budget (sinks and the
    recent window always kept), and every token equals the oracle's with exactly the pages the
    engine dropped hidden from the queries that came after each drop."""
    p = _prompt(35, 40)
    eng = LLMEngine.from_checkpoint(tiny, "cpu", EngineConfig(max_num_seqs=2, max_num_batched_tokens=64,
                                                              max_model_len=256, num_pages=64, kv_sink_tokens=16,
                                                              kv_window_tokens=32, kv_h2o_budget=80,
                                                              kv_h2o_interval=2, kv_h2o_decay=decay))
    rid = eng.add_request(p, SamplingParams(max_tokens=90, ignore_eos=True))
    kept_max = 0
    while eng.has_unfinished():
        eng.step()
        r = eng.requests[rid]
        if r.status.name == "RUNNING":
            kept_max = max(kept_max, r.num_computed - r.evicted_tokens)
    r = eng.requests[rid]
    assert eng.stats.evicted_pages >= 3 and kept_max <= 80 + 16
    assert 0 not in r.evicted_at  # the sink page stays
    assert all(b < (at - 32) // 16 for b, at in r.evicted_at.items())  # never inside the window
    ref = ReferenceModel(tiny)
    ref.kv_visible = eviction_log_rule(r)
    assert r.output == ref.greedy(p, 90)[0]


def test_layer_slice_renumbers_layers_and_shares_tensors(tiny):
    from squish_b200.models.decoder import layer_slice

    part = layer_slice(tiny, 1, 3)
    assert part.config.num_layers == 2 and part.quant is tiny.quant
    assert "model.layers.0.self_attn.q_proj.weight" in part.tensors and "model.layers.2.mlp.up_proj.weight" not in part
    assert part.tensors["model.layers.1.mlp.down_proj.weight"] is tiny.tensors["model.layers.2.mlp.down_proj.weight"]
    assert part.tensors["model.embed_tokens.weight"] is tiny.tensors["model.embed_tokens.weight"]
    n_layer = sum(k.startswith("model.layers.") for k in tiny.tensors) // tiny.config.num_layers
    assert sum(k.startswith("model.layers.") for k in part.tensors) == 2 * n_layer


def test_kv_budget_broker_shares():
    from squish_b200.kv.budget import KVBudgetBroker

    b = KVBudgetBroker(0)
    assert b.register("a", 500) == 500 and b.register("b", 300) == 300  # unconstrained
    b.set_total(1000)
    assert (b.allocated("a"), b.allocated("b")) == (500, 300)  # fits
    b.register("c", 400)
    al = b.snapshot()["allocated"]
    assert sum(al.values()) == 1000 and al["a"] > al["c"] > al["b"]  # proportional
    assert abs(al["a"] - 1000 * 500 / 1200) <= 1
    b.set_total(2)
    assert all(v >= 1 for v in b.snapshot()["allocated"].values())
    b.unregister("c")
    b.set_total(0)
    assert b.snapshot()["allocated"] == {"a": 500, "b": 300}


def test_adaptive_heavy_hitter_budgets_share_the_pool(tiny):
    """With budgets arbitrated against a small page pool, two long sequences each keep a
    proportional share (below kv_h2o_budget), and each output still equals the oracle's under
    its own eviction record."""
    prompts = [_prompt(40, 30), _prompt(41, 30)]
    eng = LLMEngine.from_checkpoint(tiny, "cpu", EngineConfig(max_num_seqs=2, max_num_batched_tokens=64,
                                                              max_model_len=256, num_pages=14, kv_sink_tokens=16,
                                                              kv_window_tokens=32, kv_h2o_budget=160,
                                                              kv_h2o_interval=1, kv_budget_adaptive=True))
    rids = [eng.add_request(p, SamplingParams(max_tokens=120, ignore_eos=True)) for p in prompts]
    shares = set()
    while eng.has_unfinished():
        eng.step()
        for rid in rids:
            r = eng.requests[rid]
            if r.status.name == "RUNNING":
                shares.add(eng.h2o_budget(r))
    assert min(shares) < 160  # the pool (14 pages = 224 tokens) cannot hold two 160-token budgets
    assert eng.stats.evicted_pages > 0
    ref = ReferenceModel(tiny)
    for p, rid in zip(prompts, rids):
        r = eng.requests[rid]
        ref.kv_visible = eviction_log_rule(r)
        assert r.output == ref.greedy(p, 120)[0]
