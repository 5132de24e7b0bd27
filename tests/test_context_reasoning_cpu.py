"""Extractive prompt compression and self-consistency voting."""
import pytest

from squish_b200.context.prompt_compressor import compress, compress_messages, sentences
from squish_b200.reasoning.self_consistency import SelfConsistencyConfig, SelfConsistencyVoter

DOC = ("The B200 has 148 streaming multiprocessors. Lunch was a sandwich. "
       "Each multiprocessor has tensor memory for accumulators. It rained. "
       "Tensor memory holds 256 KB per multiprocessor. The cat slept. ")


def test_compress_keeps_informative_sentences_in_order():
    out = compress(DOC, ratio=0.5)
    kept = sentences(out)
    assert len(kept) == 3 and all(k in sentences(DOC) for k in kept)
    assert [sentences(DOC).index(k) for k in kept] == sorted(sentences(DOC).index(k) for k in kept)
    assert "multiprocessor" in out and "cat" not in out
    q = compress(DOC, ratio=1 / 6, question="What did I eat for lunch?")
    assert q == "Lunch was a sandwich."
    assert compress("one sentence only.", 0.3) == "one sentence only."
    assert compress(DOC, 0.5, min_tokens=10_000) == DOC
    pre = compress("SYSTEM PROMPT HERE " + DOC, 0.5, preserve_tokens=3)
    assert pre.startswith("SYSTEM PROMPT HERE ")
    with pytest.raises(ValueError):
        compress(DOC, 0.0)
    msgs = compress_messages([{"role": "system", "content": DOC}, {"role": "user", "content": DOC}], 0.5, 5)
    assert msgs[0]["content"] == DOC and len(sentences(msgs[1]["content"])) == 3


def test_self_consistency_vote():
    v = SelfConsistencyVoter()
    chains = ["2+2... so the answer is 4.", "I think\n= 4", "The answer is 5", "so: answer: 4"]
    r = v.vote(chains)
    assert r.answer == "4" and r.votes == 3 and r.total == 4 and r.agreement == 0.75 and r.winner_index == 0
    v2 = SelfConsistencyVoter(SelfConsistencyConfig(answer_pattern=r"FINAL\((\w+)\)"))
    assert v2.vote(["x FINAL(b)", "FINAL(a)", "y FINAL(a)"]).answer == "a"
    assert v.vote(["a", "b"]).answer == "a"  # tie: first seen
    with pytest.raises(ValueError):
        v.vote([])


def test_self_consistency_over_http():
    from fastapi.testclient import TestClient

    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.models.config import get_preset
    from squish_b200.models.weights import random_checkpoint
    from squish_b200.serving.async_engine import AsyncEngine
    from squish_b200.serving.server import ServerState, create_app
    from squish_b200.serving.tokenizer import ByteTokenizer

    cfg, q = get_preset("tiny-llama")
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0, device="cpu"), "cpu",
                                    EngineConfig(max_num_seqs=8, max_model_len=512, num_pages=128))
    aeng = AsyncEngine(eng, ByteTokenizer(cfg.vocab_size, cfg.eos_token_id), model_name="tiny").start()
    try:
        st = ServerState(aeng, "tiny", arch="llama", compress_prompt={"ratio": 0.5, "min_tokens": 5})
        with TestClient(create_app(st)) as c:
            r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": DOC}], "max_tokens": 6,
                                                     "seed": 3, "self_consistency": {"k": 3}}).json()
            sc = r["self_consistency"]
            assert sc["k"] == 3 and 1 <= sc["votes"] <= 3 and len(r["choices"]) == 1
            assert r["usage"]["completion_tokens"] <= 18
    finally:
        aeng.stop()
