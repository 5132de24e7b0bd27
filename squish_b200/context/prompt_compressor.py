"""Extractive prompt compression: keep the most informative sentences of long inputs.

The reference's compressor (squish/context/prompt_compressor.py:45-180) ranks sentences by the
sum of their terms' TF-IDF weights (TF = count / sentence length, IDF = log((1 + N) / (1 + df))
+ 1 over the N sentences), keeps the top ceil(ratio * N) in their original order, and can
protect a leading span of words (a fixed system prompt, so prefix caching still hits). Here the
same ranking, plus an optional question whose terms double the weight of sentences that
mention them. The server applies it to long user messages (``--compress-prompt``).
"""
from __future__ import annotations

import math
import re
from collections import Counter

_SENT = re.compile(r"(?<=[.!?])\s+|\n{2,}")
_WORD = re.compile(r"[a-z0-9]+")


def sentences(text: str) -> list[str]:
    return [s.strip() for s in _SENT.split(text) if s and s.strip()]


def compress(text: str, ratio: float = 0.5, question: str = "", min_tokens: int = 0,
             preserve_tokens: int = 0) -> str:
    if not 0.0 < ratio <= 1.0:
        raise ValueError("ratio must be in (0, 1]")
    words = text.split()
    if len(words) < min_tokens:
        return text
    prefix, body = "", text
    if preserve_tokens > 0:
        if len(words) <= preserve_tokens:
            return text
        prefix, body = " ".join(words[:preserve_tokens]), " ".join(words[preserve_tokens:])
    sents = sentences(body)
    n = len(sents)
    keep = max(1, math.ceil(ratio * n))
    if n < 2 or keep >= n:
        return text
    toks = [_WORD.findall(s.lower()) for s in sents]
    df = Counter(t for ts in toks for t in set(ts))
    q = set(_WORD.findall(question.lower()))
    scores = []
    for ts in toks:
        if not ts:
            scores.append(0.0)
            continue
        tf = Counter(ts)
        sc = sum((c / len(ts)) * (math.log((1 + n) / (1 + df[t])) + 1.0) for t, c in tf.items())
        if q and q & set(ts):
            sc *= 2.0
        scores.append(sc)
    top = sorted(sorted(range(n), key=lambda i: -scores[i])[:keep])
    out = " ".join(sents[i] for i in top)
    return f"{prefix} {out}" if prefix else out


def compress_messages(messages: list[dict], ratio: float, min_tokens: int, preserve_tokens: int = 0) -> list[dict]:
    """Compress the text of long user messages (the last user message's trailing question is
    used to favour relevant sentences); other messages pass through."""
    last_user = next((m for m in reversed(messages) if m.get("role") == "user"), None)
    question = ""
    if last_user is not None and isinstance(last_user.get("content"), str):
        ss = sentences(last_user["content"])
        question = ss[-1] if ss else ""
    out = []
    for m in messages:
        c = m.get("content")
        if m.get("role") == "user" and isinstance(c, str) and len(c.split()) >= min_tokens:
            m = dict(m, content=compress(c, ratio, question, min_tokens, preserve_tokens))
        out.append(m)
    return out
