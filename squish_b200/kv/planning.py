"""KV storage mode selection and closed-form memory planning.

The reference picks the KV mode from the planned context (``recommended_kv_mode`` /
``recommended_kv_mode_3tier``: <= 8K tokens INT8, 8K-16K INT4, > 16K INT2,
squish/kv/kv_cache.py:549-610) and answers "how much memory at context X" / "how long a
context fits in B bytes" in closed form (``estimate_kv_memory`` / ``estimate_max_context``,
kv_cache.py:747-838). Here the estimate counts this package's paged layout exactly (codes +
fp16 scales per token row, whole pages, every layer and KV head), so it equals the pool the
engine allocates for that many tokens (see ``kv/paged.py::bytes_per_page``).
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass

from ..models.config import ModelConfig, QuantConfig
from .paged import bytes_per_page

INT8_MAX_CONTEXT = 8192     # <= this: INT8 keys and values
INT4_MAX_CONTEXT = 16384    # <= this: INT4; longer contexts: INT2
MODES = ("bf16", "int8", "int4", "int2", "k8v4")


def recommended_kv_mode(context_tokens: int, short_mode: str = "int8", long_mode: str = "int2",
                        threshold: int = INT8_MAX_CONTEXT, medium_mode: str | None = None,
                        medium_threshold: int | None = None) -> str:
    if context_tokens < 0:
        raise ValueError(f"context_tokens must be >= 0, got {context_tokens}")
    if (medium_mode is None) != (medium_threshold is None):
        raise ValueError("medium_mode and medium_threshold must both be set or both be None")
    if medium_mode is not None:
        if medium_threshold > threshold:
            raise ValueError("medium_threshold must not exceed threshold")
        if context_tokens > threshold:
            return long_mode
        return medium_mode if context_tokens > medium_threshold else short_mode
    return long_mode if context_tokens > threshold else short_mode


def recommended_kv_mode_3tier(context_tokens: int, short_threshold: int = INT8_MAX_CONTEXT,
                              long_threshold: int = INT4_MAX_CONTEXT) -> str:
    return recommended_kv_mode(context_tokens, "int8", "int2", long_threshold, "int4", short_threshold)


@dataclass(frozen=True)
class KVMemoryEstimate:
    mode: str
    context_tokens: int
    sequences: int
    pages: int
    bytes_per_page: int
    total_bytes: int

    page_size: int = 16

    @property
    def bytes_per_token(self) -> float:
        """Per token of one sequence, all layers and KV heads."""
        return self.bytes_per_page / self.page_size


def estimate_kv_memory(cfg: ModelConfig, context_tokens: int, mode: str, sequences: int = 1,
                       q: QuantConfig | None = None) -> KVMemoryEstimate:
    """Device bytes of the paged KV cache holding ``sequences`` sequences of ``context_tokens``."""
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
    if context_tokens < 0 or sequences < 1:
        raise ValueError("context_tokens must be >= 0 and sequences >= 1")
    q = dataclasses.replace(q or QuantConfig(), kv_dtype=mode)
    bpp = bytes_per_page(cfg, q)
    pages = sequences * -(-context_tokens // q.page_size)
    return KVMemoryEstimate(mode, context_tokens, sequences, pages, bpp, pages * bpp, q.page_size)


def estimate_max_context(cfg: ModelConfig, budget_bytes: int, mode: str, sequences: int = 1,
                         q: QuantConfig | None = None) -> int:
    """Longest context (tokens, whole pages) whose cache for ``sequences`` sequences fits the budget."""
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
    q = dataclasses.replace(q or QuantConfig(), kv_dtype=mode)
    bpp = bytes_per_page(cfg, q)
    pages_per_seq = max(0, budget_bytes) // bpp // max(1, sequences)
    return pages_per_seq * q.page_size


def auto_kv_mode(max_model_len: int) -> str:
    """``--kv-dtype auto``: the 3-tier choice for the longest context the engine admits."""
    return recommended_kv_mode_3tier(max_model_len)
