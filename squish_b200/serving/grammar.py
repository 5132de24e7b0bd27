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


class GrammarFactory:
    """Builds the vocabulary index once per tokenizer and hands out fresh matchers."""

    def __init__(self, tokenizer, vocab_size: int, eos_token_id: int | None):
        self.index = native().grammar.VocabIndex(token_bytes(tokenizer, vocab_size),
                                                 -1 if eos_token_id is None else int(eos_token_id))

    def json(self, top_object: bool = True) -> JsonGrammar:
        return JsonGrammar(self.index, top_object)


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
