"""Structured output: JSON-constrained decoding for ``response_format`` (OpenAI) and
``format: "json"`` (Ollama).

The token masks come from the C++ matcher in ``csrc/grammar.cpp`` (a JSON pushdown automaton
walked over a trie of the vocabulary's byte strings); the engine uploads the mask with the
step's metadata and the fused sampler applies it (``csrc/sampler.cu``). The reference does the
same job with xgrammar bitmasks (squish/grammar/grammar_engine.py:220-254).

Token byte strings: byte-level BPE vocabularies (GPT-2 / Qwen / Llama-3 style) map every byte
to a printable code point; the inverse of that map recovers the bytes. SentencePiece
vocabularies write a space as U+2581 and raw bytes as ``<0xNN>``. Special tokens have no bytes
and are never allowed inside JSON (EOS is allowed once the document is complete).
"""
from __future__ import annotations

import json

import numpy as np

from .._ext import native


def _byte_level_decoder() -> dict[str, int]:
    """Inverse of the byte-level BPE byte -> printable-character table: bytes that are printable
    Latin-1 stand for themselves, the other 68 map to U+0100.. in byte order."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    table = {}
    extra = 0
    for b in range(256):
        if b in keep:
            table[chr(b)] = b
        else:
            table[chr(256 + extra)] = b
            extra += 1
    return table


def token_bytes(tokenizer, vocab_size: int) -> list[bytes]:
    """Byte string of every token id below ``vocab_size`` (b"" for special / unknown ids)."""
    out = [b""] * vocab_size
    if getattr(tokenizer, "name_or_path", "") == "byte" or hasattr(tokenizer, "OFFSET"):
        off = tokenizer.OFFSET
        for b in range(256):
            if off + b < vocab_size:
                out[off + b] = bytes([b])
        return out
    hf = getattr(tokenizer, "tok", tokenizer)
    n = min(vocab_size, len(hf))
    pieces = hf.convert_ids_to_tokens(list(range(n)))
    special = set(getattr(hf, "all_special_ids", []) or [])
    dec = _byte_level_decoder()
    byte_level = sum(1 for p in pieces[:5000] if p and ("Ġ" in p or "Ċ" in p)) > 10
    for i, p in enumerate(pieces):
        if p is None or i in special:
            continue
        if byte_level:
            try:
                out[i] = bytes(dec[ch] for ch in p)
            except KeyError:  # added tokens written as plain text
                out[i] = p.encode("utf-8")
        elif p.startswith("<0x") and p.endswith(">") and len(p) == 6:
            out[i] = bytes([int(p[3:5], 16)])
        else:
            out[i] = p.replace("▁", " ").encode("utf-8")
    return out


class JsonGrammar:
    """Per-request grammar state with the engine's interface: ``allowed_mask()`` (uint32 words,
    bit set = allowed), ``advance(token)``, ``is_terminated()``."""

    def __init__(self, index, top_object: bool = True):
        self.m = native().grammar.JsonMatcher(index, top_object)

    def allowed_mask(self) -> np.ndarray:
        return self.m.allowed_mask().numpy().view(np.uint32)

    def advance(self, tok: int) -> bool:
        return self.m.advance(int(tok))

    def is_complete(self) -> bool:
        return self.m.is_complete()

    def is_terminated(self) -> bool:
        return self.m.is_terminated()


K_ANY, K_OBJECT, K_ARRAY, K_STRING, K_INTEGER, K_NUMBER, K_BOOLEAN, K_NULL, K_ENUM, K_UNION = range(10)


def compile_schema(schema: dict):
    """JSON schema -> ``_C.grammar.Schema`` node table. Supported: ``type`` object (``properties``,
    ``required``; only listed properties may appear, each once), array (``items``), string,
    integer, number, boolean, null; ``enum`` / ``const`` (literal values); local ``$ref``
    (``#/$defs/..``, ``#/definitions/..``); unions -- ``anyOf`` / ``oneOf`` and type lists such
    as ``["string", "null"]`` -- choose the alternative by the value's first byte (alternatives
    that share it, e.g. two objects, relax to any JSON value). An object without ``properties``
    accepts any object."""
    kinds, props, required, items, lits = [], [], [], [], []
    memo: dict[int, int] = {}  # id(schema dict) -> node; dicts made here are kept alive in `made`
    made: list = []

    def resolve(node):
        seen = 0
        while isinstance(node, dict) and "$ref" in node:
            ref = node["$ref"]
            if not ref.startswith("#/"):
                raise ValueError(f"only local $ref is supported, got {ref!r}")
            cur = schema
            for part in ref[2:].split("/"):
                cur = cur[part]
            node = cur
            seen += 1
            if seen > 64:
                raise ValueError("$ref cycle")
        return node

    def add(node) -> int:
        node = resolve(node) if isinstance(node, dict) else {}
        key = id(node)
        if key in memo:
            return memo[key]
        i = len(kinds)
        memo[key] = i
        kinds.append(K_ANY)
        props.append([])
        required.append(0)
        items.append(-1)
        lits.append([])
        if "const" in node or "enum" in node:
            vals = [node["const"]] if "const" in node else list(node["enum"])
            if len(vals) > 64:
                raise ValueError("at most 64 enum values")
            kinds[i] = K_ENUM
            lits[i] = [json.dumps(v, separators=(",", ":"), ensure_ascii=False).encode() for v in vals]
            return i
        t = node.get("type")
        alts = node.get("anyOf") or node.get("oneOf")
        if isinstance(t, list) or isinstance(alts, list):
            if isinstance(t, list):
                alts = [dict(node, type=x) for x in t]
                for a in alts:
                    a.pop("anyOf", None)
                    a.pop("oneOf", None)
            if len(alts) > 64:
                raise ValueError("at most 64 union alternatives")
            kinds[i] = K_UNION
            made.extend(alts)
            for a in alts:
                props[i].append((b"", add(a)))
            return i
        if t == "object" and isinstance(node.get("properties"), dict) and node["properties"]:
            names = list(node["properties"])
            if len(names) > 64:
                raise ValueError("at most 64 properties per object")
            kinds[i] = K_OBJECT
            req = set(node.get("required", []))
            required[i] = sum(1 << j for j, nm in enumerate(names) if nm in req)
            props[i] = [(nm.encode(), add(node["properties"][nm])) for nm in names]
        elif t == "array":
            kinds[i] = K_ARRAY
            if isinstance(node.get("items"), dict):
                items[i] = add(node["items"])
        elif t in ("string", "integer", "number", "boolean", "null"):
            kinds[i] = {"string": K_STRING, "integer": K_INTEGER, "number": K_NUMBER, "boolean": K_BOOLEAN,
                        "null": K_NULL}[t]
        return i

    root = add(schema)
    return native().grammar.Schema(kinds, props, required, items, lits, root)


class SchemaGrammar(JsonGrammar):
    """JSON constrained by a compiled schema (same interface as :class:`JsonGrammar`)."""

    def __init__(self, index, schema):  # noqa: super().__init__ is replaced, not extended
        self.m = native().grammar.SchemaMatcher(index, schema)


class GrammarFactory:
    """Builds the vocabulary index once per tokenizer and hands out fresh matchers."""

    def __init__(self, tokenizer, vocab_size: int, eos_token_id: int | None):
        self.index = native().grammar.VocabIndex(token_bytes(tokenizer, vocab_size),
                                                 -1 if eos_token_id is None else int(eos_token_id))

    def json(self, top_object: bool = True) -> JsonGrammar:
        return JsonGrammar(self.index, top_object)

    def schema(self, schema: dict) -> SchemaGrammar:
        return SchemaGrammar(self.index, compile_schema(schema))


def grammar_for(factory: "GrammarFactory", response_format):
    """A fresh grammar for an OpenAI ``response_format`` (None: unconstrained)."""
    if not wants_json(response_format):
        return None
    js = response_format.get("json_schema") if response_format.get("type") == "json_schema" else None
    sch = js.get("schema") if isinstance(js, dict) else None
    return factory.schema(sch) if isinstance(sch, dict) and sch else factory.json()


def wants_json(response_format) -> bool | None:
    """OpenAI ``response_format`` -> True (a JSON object), None (unconstrained)."""
    if not isinstance(response_format, dict):
        return None
    t = response_format.get("type")
    if t in ("json_object", "json_schema"):
        return True
    if t in (None, "text"):
        return None
    raise ValueError(f"unsupported response_format type {t!r}")
