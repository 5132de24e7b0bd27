"""Per-request sampling parameters (OpenAI / Ollama request fields map onto these)."""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class SamplingParams:
    max_tokens: int = 256
    temperature: float = 0.0          # <= 0: greedy
    top_p: float = 1.0
    top_k: int = 0
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    seed: int | None = None
    stop_token_ids: list[int] = field(default_factory=list)
    ignore_eos: bool = False
    min_tokens: int = 0
    logprobs: bool = False
    # grammar-constrained decoding: an object with allowed_mask()->np.uint32[ceil(V/32)] and advance(tok)
    grammar: object | None = None
    # keep the final-norm hidden state of the last prompt token (embeddings)
    return_hidden: bool = False

    def validate(self) -> "SamplingParams":
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not (0.0 < self.top_p <= 1.0):
            raise ValueError("top_p must be in (0, 1]")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0")
        if not (0.0 <= self.min_p < 1.0):
            raise ValueError("min_p must be in [0, 1)")
        if self.repetition_penalty <= 0:
            raise ValueError("repetition_penalty must be > 0")
        return self
