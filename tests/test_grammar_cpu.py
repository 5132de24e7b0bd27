"""JSON-constrained decoding: the C++ matcher, its token masks, and the HTTP surface."""
import json
import random

import numpy as np
import pytest
import torch

from squish_b200._ext import native
from squish_b200.serving.grammar import GrammarFactory, _byte_level_decoder, token_bytes
from squish_b200.serving.tokenizer import ByteTokenizer


def _feed(g, text: str, off: int = 3) -> bool:
    for b in text.encode():
        m = g.allowed_mask()
        t = b + off
        if not (m[t >> 5] >> (t & 31)) & 1:
            return False
        assert g.advance(t)
    return True


def _rand_json(rng, depth=0):
    k = rng.randrange(7 if depth < 3 else 4)
    if k == 0:
        return rng.choice([True, False, None])
    if k == 1:
        return rng.randint(-10 ** 6, 10 ** 6)
    if k == 2:
        return rng.uniform(-1e6, 1e6)
    if k == 3:
        return "".join(rng.choice('ab"\\\n\t é✓') for _ in range(rng.randrange(6)))
    if k in (4, 5):
        return {f"k{i}": _rand_json(rng, depth + 1) for i in range(rng.randrange(4))}
    return [_rand_json(rng, depth + 1) for _ in range(rng.randrange(4))]


def test_matcher_accepts_valid_json_objects():
    f = GrammarFactory(ByteTokenizer(300, 2), 300, 2)
    rng = random.Random(0)
    for i in range(300):
        doc = {"root": _rand_json(rng)}
        text = json.dumps(doc, ensure_ascii=bool(i % 2), indent=None if i % 3 else 1)
        g = f.json()
        assert _feed(g, text), text
        assert g.is_complete() and g.is_terminated()
        m = g.allowed_mask()
        assert (m[0] >> 2) & 1  # EOS
        assert not any((m[(b + 3) >> 5] >> ((b + 3) & 31)) & 1 for b in b"{}[],:\"x1")


@pytest.mark.parametrize("bad", ['[1]', '{"a" 1}', '{"a":01}', '{"a":tru}', '{,}', '{"a":1,}', '{"a":"\x01"}',
                                 '{"a":"\\q"}', '{"a":1.}', '{"a":-}', '{"a":1e}', '{"a":[1 2]}', '{"a":1}}'])
def test_matcher_rejects_invalid_json(bad):
    g = GrammarFactory(ByteTokenizer(300, 2), 300, 2).json()
    ok = _feed(g, bad)
    assert not (ok and g.is_complete()), bad


def test_masks_agree_with_stepwise_advance_on_multibyte_vocab():
    """The trie walk (and the plain-string shortcut) allows exactly the tokens advance() accepts."""
    rng = random.Random(1)
    alphabet = ['{', '}', '[', ']', '"', ':', ',', ' ', '\n', 'a', 'b', 'true', 'fals', 'e', 'null', '0', '1', '-',
                '.', 'e5', '\\', 'n', 'u', '00e9', '": ', '", "', '{"', '"}', ' {', '": {"', '1.5', 'x y', '✓']
    vocab = [b""] * 3 + [s.encode() for s in alphabet] + [bytes([rng.randrange(32, 127)]) + b"ab" for _ in range(40)]
    idx = native().grammar.VocabIndex(vocab, 2)
    for trial in range(30):
        hist = []
        g = native().grammar.JsonMatcher(idx, True)
        for step in range(40):
            m = g.allowed_mask().numpy().view(np.uint32)
            allowed = [t for t in range(len(vocab)) if (m[t >> 5] >> (t & 31)) & 1]
            for t in range(3, len(vocab)):
                probe = native().grammar.JsonMatcher(idx, True)
                for h in hist:
                    assert probe.advance(h)
                assert probe.advance(t) == (t in allowed), (vocab[t], [vocab[h] for h in hist])
            choices = [t for t in allowed if t != 2]
            if not choices:
                break
            t = rng.choice(choices)
            hist.append(t)
            assert g.advance(t)


def test_byte_level_bpe_table_is_a_bijection():
    d = _byte_level_decoder()
    assert len(d) == 256 and sorted(d.values()) == list(range(256))
    assert d["Ġ"] == 32 and d["Ċ"] == 10 and d["A"] == 65


def test_response_format_over_http():
    from fastapi.testclient import TestClient

    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.models.config import get_preset
    from squish_b200.models.weights import random_checkpoint
    from squish_b200.serving.async_engine import AsyncEngine
    from squish_b200.serving.server import ServerState, create_app

    cfg, q = get_preset("tiny-llama")
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0, device="cpu"), "cpu",
                                    EngineConfig(max_num_seqs=4, max_model_len=512, num_pages=128))
    aeng = AsyncEngine(eng, ByteTokenizer(cfg.vocab_size, cfg.eos_token_id), model_name="tiny").start()
    try:
        with TestClient(create_app(ServerState(aeng, "tiny", arch="llama"))) as c:
            for seed in range(3):
                r = c.post("/v1/chat/completions", json={
                    "messages": [{"role": "user", "content": "json please"}], "max_tokens": 60, "temperature": 1.0,
                    "seed": seed, "response_format": {"type": "json_object"}}).json()
                text = r["choices"][0]["message"]["content"]
                assert text.lstrip().startswith("{"), text
                if r["choices"][0]["finish_reason"] == "stop":
                    assert isinstance(json.loads(text), dict)
            bad = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                       "response_format": {"type": "yaml"}})
            assert bad.status_code == 400
            o = c.post("/api/generate", json={"model": "tiny", "prompt": "x", "format": "json", "stream": False,
                                              "options": {"num_predict": 40, "seed": 1}}).json()
            assert o["response"].lstrip().startswith("{")
    finally:
        aeng.stop()


SCHEMA = {"type": "object", "$defs": {"tag": {"enum": ["a", "bb", 3, True]}},
          "properties": {"name": {"type": "string"}, "age": {"type": "integer"},
                         "tags": {"type": "array", "items": {"$ref": "#/$defs/tag"}}, "ok": {"type": "boolean"},
                         "pos": {"type": "object", "properties": {"x": {"type": "number"}}, "required": ["x"]},
                         "any": {}},
          "required": ["name", "age"]}


@pytest.mark.parametrize("text,want", [
    ('{"name": "x", "age": 3}', True),
    ('{"age": 3, "name": "x", "tags": ["a", 3, "bb", true]}', True),
    ('{"name":"x","age":-0,"ok":false,"pos":{"x":1.5e3},"any":[{"q":null}]}', True),
    ('{"name": "x"}', False), ('{"name": 1, "age": 2}', False), ('{"age": 1.5, "name": "x"}', False),
    ('{"nam": "x", "age": 1}', False), ('{"name": "x", "age": 1, "zzz": 1}', False),
    ('{"name": "x", "age": 1, "tags": ["c"]}', False), ('{"name": "x", "name": "y", "age": 1}', False),
    ('{"name": "x", "age": 1, "pos": {}}', False), ('{"name": "x", "age": 1, "tags": [33]}', False),
])
def test_schema_matcher(text, want):
    g = GrammarFactory(ByteTokenizer(300, 2), 300, 2).schema(SCHEMA)
    ok = _feed(g, text) and g.is_complete()
    assert ok == want, text
    if want:
        assert json.loads(text)


def test_schema_masks_agree_with_stepwise_advance():
    from squish_b200.serving.grammar import compile_schema

    rng = random.Random(2)
    alphabet = ['{', '}', '[', ']', '"', ':', ',', ' ', 'name', 'age', '"name"', '"age": ', '": "', 'a', 'bb', '3',
                '1', '.', '5', 'true', 'false', 'null', '"tags": [', '"a"', '"bb"', 'x', '"ok":', '"pos": {"x": ']
    vocab = [b""] * 3 + [t.encode() for t in alphabet]
    idx = native().grammar.VocabIndex(vocab, 2)
    sc = compile_schema(SCHEMA)
    for trial in range(25):
        hist = []
        g = native().grammar.SchemaMatcher(idx, sc)
        for step in range(30):
            m = g.allowed_mask().numpy().view(np.uint32)
            allowed = {t for t in range(len(vocab)) if (m[t >> 5] >> (t & 31)) & 1}
            for t in range(3, len(vocab)):
                probe = native().grammar.SchemaMatcher(idx, sc)
                for h in hist:
                    assert probe.advance(h)
                assert probe.advance(t) == (t in allowed)
            choices = sorted(allowed - {2})
            if not choices:
                break
            t = rng.choice(choices)
            hist.append(t)
            assert g.advance(t)


def test_json_schema_over_http():
    from fastapi.testclient import TestClient

    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.models.config import get_preset
    from squish_b200.models.weights import random_checkpoint
    from squish_b200.serving.async_engine import AsyncEngine
    from squish_b200.serving.server import ServerState, create_app

    cfg, q = get_preset("tiny-llama")
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0, device="cpu"), "cpu",
                                    EngineConfig(max_num_seqs=4, max_model_len=512, num_pages=128))
    aeng = AsyncEngine(eng, ByteTokenizer(cfg.vocab_size, cfg.eos_token_id), model_name="tiny").start()
    schema = {"type": "object", "properties": {"v": {"enum": ["yes", "no"]}, "n": {"type": "integer"}},
              "required": ["v", "n"]}
    try:
        with TestClient(create_app(ServerState(aeng, "tiny", arch="llama"))) as c:
            done = 0
            for seed in range(4):
                r = c.post("/v1/chat/completions", json={
                    "messages": [{"role": "user", "content": "answer"}], "max_tokens": 80, "temperature": 1.0,
                    "seed": seed, "response_format": {"type": "json_schema",
                                                      "json_schema": {"name": "a", "schema": schema}}}).json()
                text = r["choices"][0]["message"]["content"]
                assert text.lstrip().startswith("{")
                if r["choices"][0]["finish_reason"] == "stop":
                    d = json.loads(text)
                    assert set(d) == {"v", "n"} and d["v"] in ("yes", "no") and isinstance(d["n"], int)
                    done += 1
            bad = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                       "response_format": {"type": "json_schema", "json_schema": {
                                                           "schema": {"$ref": "http://x/y"}}}})
            assert bad.status_code == 400
    finally:
        aeng.stop()


UNION = {"type": "object", "properties": {
    "n": {"type": ["string", "null"]},
    "v": {"anyOf": [{"type": "integer"}, {"type": "array", "items": {"type": "boolean"}}]},
    "o": {"oneOf": [{"type": "object", "properties": {"a": {"type": "integer"}}, "required": ["a"]},
                    {"type": "object", "properties": {"b": {"type": "string"}}}]},
    "x": {"type": ["integer", "number"]}}, "required": ["n"]}


@pytest.mark.parametrize("text,want", [
    ('{"n": null}', True), ('{"n": "s"}', True), ('{"n": 3}', False), ('{"n": null, "v": 7}', True),
    ('{"n": null, "v": [true, false]}', True), ('{"n": null, "v": "s"}', False), ('{"n":null,"v":[1]}', False),
    ('{"n": null, "o": {"zz": 1}}', True),  # two object alternatives share '{': relaxed to any object
    ('{"n": null, "x": 1.5}', True), ('{"n": null, "x": "q"}', False),
])
def test_schema_unions(text, want):
    g = GrammarFactory(ByteTokenizer(300, 2), 300, 2).schema(UNION)
    assert (_feed(g, text) and g.is_complete()) == want, text


def test_union_masks_agree_with_stepwise_advance():
    from squish_b200.serving.grammar import compile_schema

    rng = random.Random(5)
    alphabet = ['{', '}', '[', ']', '"', ':', ',', ' ', '"n": ', '"v": ', '"x": ', 'null', 'nul', 'l', 'true', '7',
                '1.5', '-', '"s"', 'tr', 'ue', '"o": {', '"zz"']
    vocab = [b""] * 3 + [t.encode() for t in alphabet]
    idx = native().grammar.VocabIndex(vocab, 2)
    sc = compile_schema(UNION)
    for trial in range(20):
        hist = []
        g = native().grammar.SchemaMatcher(idx, sc)
        for step in range(25):
            m = g.allowed_mask().numpy().view(np.uint32)
            allowed = {t for t in range(len(vocab)) if (m[t >> 5] >> (t & 31)) & 1}
            for t in range(3, len(vocab)):
                probe = native().grammar.SchemaMatcher(idx, sc)
                for h in hist:
                    assert probe.advance(h)
                assert probe.advance(t) == (t in allowed)
            choices = sorted(allowed - {2})
            if not choices:
                break
            t = rng.choice(choices)
            hist.append(t)
            assert g.advance(t)
