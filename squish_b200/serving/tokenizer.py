"""Tokenizers for the serving layer.

A model directory with HF tokenizer files is loaded through ``transformers`` (offline).
Random-initialised models have no vocabulary; they get :class:`ByteTokenizer`, which maps
UTF-8 bytes to ids 3..258 (0 = pad, 1 = bos, 2 = eos) and renders ids outside that range
as ``<N>``, so every id a model can emit has a printable form.
"""
from __future__ import annotations

import os


class ByteTokenizer:
    pad_token_id = 0
    bos_token_id = 1
    OFFSET = 3

    def __init__(self, vocab_size: int = 259, eos_token_id: int = 2):
        self.vocab_size = max(vocab_size, 259)
        self.eos_token_id = eos_token_id
        self.name_or_path = "byte"

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        ids = [b + self.OFFSET for b in text.encode("utf-8")]
        return ([self.bos_token_id] + ids) if add_special_tokens else ids

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        out = bytearray()
        parts: list[str] = []
        for t in ids:
            t = int(t)
            if self.OFFSET <= t < self.OFFSET + 256:
                out.append(t - self.OFFSET)
                continue
            if out:
                parts.append(out.decode("utf-8", errors="replace"))
                out = bytearray()
            if t in (self.pad_token_id, self.bos_token_id, self.eos_token_id) and skip_special_tokens:
                continue
            parts.append(f"<{t}>")
        if out:
            parts.append(out.decode("utf-8", errors="replace"))
        return "".join(parts)

    def apply_chat_template(self, messages, tokenize=False, add_generation_prompt=True, **kw):
        from .chat_template import render_chatml

        text = render_chatml(messages, add_generation_prompt=add_generation_prompt, tools=kw.get("tools"))
        return self.encode(text) if tokenize else text


class HFTokenizer:
    """Thin adapter over a transformers tokenizer (same method names as ByteTokenizer)."""

    def __init__(self, tok):
        self.tok = tok
        self.eos_token_id = tok.eos_token_id
        self.bos_token_id = tok.bos_token_id
        self.pad_token_id = tok.pad_token_id if tok.pad_token_id is not None else (tok.eos_token_id or 0)
        self.vocab_size = len(tok)
        self.name_or_path = getattr(tok, "name_or_path", "hf")

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        return list(self.tok.encode(text, add_special_tokens=add_special_tokens))

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=skip_special_tokens)

    def apply_chat_template(self, messages, tokenize=False, add_generation_prompt=True, **kw):
        if getattr(self.tok, "chat_template", None):
            return self.tok.apply_chat_template(messages, tokenize=tokenize, add_generation_prompt=add_generation_prompt,
                                                **kw)
        from .chat_template import render_chatml

        text = render_chatml(messages, add_generation_prompt=add_generation_prompt, tools=kw.get("tools"))
        return self.encode(text) if tokenize else text


def load_tokenizer(model_dir: str | None, vocab_size: int = 259, eos_token_id: int = 2):
    if model_dir and os.path.isdir(model_dir) and any(
            os.path.exists(os.path.join(model_dir, f)) for f in ("tokenizer.json", "tokenizer.model",
                                                                 "tokenizer_config.json")):
        try:
            from transformers import AutoTokenizer

            return HFTokenizer(AutoTokenizer.from_pretrained(model_dir, local_files_only=True))
        except Exception:  # noqa: BLE001 - unreadable tokenizer files fall back to bytes
            pass
    return ByteTokenizer(vocab_size, eos_token_id)


class IncrementalDetokenizer:
    """Streams text for a growing token list: emits only newly completed characters.

    Each push decodes a short window, not the whole list: the text of ids[prefix:read] (already
    emitted) and of ids[prefix:] (with the new ids); the difference is the new text. Decoding the
    window from a token that was already emitted keeps tokenizers that render a token
    differently at the start of a string (SentencePiece's leading-space marker) consistent. A
    trailing replacement character (an incomplete UTF-8 sequence) is held back until the next
    token completes it. Cost per push is O(window), not O(generated length).
    """

    def __init__(self, tokenizer):
        self.tok = tokenizer
        self.ids: list[int] = []
        self.text = ""
        self._prefix = 0  # window start (ids before it are emitted and settled)
        self._read = 0    # ids before it are emitted

    def push(self, token_ids) -> str:
        self.ids.extend(int(t) for t in token_ids)
        if len(self.ids) == self._read:
            return ""
        prev = self.tok.decode(self.ids[self._prefix:self._read]) if self._read > self._prefix else ""
        cur = self.tok.decode(self.ids[self._prefix:])
        if len(cur) <= len(prev) or cur.endswith("\ufffd"):
            return ""
        delta = cur[len(prev):] if cur.startswith(prev) else cur[len(prev):]
        self._prefix, self._read = self._read, len(self.ids)
        self.text += delta
        return delta
