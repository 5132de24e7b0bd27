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
