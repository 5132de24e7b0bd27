"""Per-request repetition-loop guard of the decode loop.

The reference stops a request whose output has fallen into a verbatim loop (short n-gram
run-ons, or whole sentences repeated) with finish reason "repetition"
(squish/serving/loop_guard.py, wired at squish/server.py:2481-2490). Here the detector runs
on the generated token ids in C++ (``_C.host.detect_token_loop``) every ``check_every``
tokens over a trailing window, on the engine thread.
"""
from __future__ import annotations

from .._ext import native

WINDOW = 400        # trailing tokens inspected
CHECK_EVERY = 16    # tokens between checks
MIN_PERIOD = 2      # shortest repeating unit (tokens)
MAX_PERIOD = 96     # longest (about a paragraph)
SHORT_REPS = 4      # repetitions needed for short units
BLOCK_PERIOD = 32   # units at least this long count as blocks
BLOCK_REPS = 2      # ... and need only two repetitions
MATCH_RATIO = 0.95  # fraction of the span that must match one period earlier


def detect_loop(tokens: list[int]) -> bool:
    return native().host.detect_token_loop(list(tokens), MIN_PERIOD, MAX_PERIOD, SHORT_REPS, BLOCK_PERIOD,
                                           BLOCK_REPS, MATCH_RATIO)


class LoopGuard:
    __slots__ = ("buf", "n")

    def __init__(self) -> None:
        self.buf: list[int] = []
        self.n = 0

    def feed(self, token_ids) -> bool:
        """Add newly generated ids; True when the trailing window is a loop."""
        if not token_ids:
            return False
        before = self.n
        self.buf.extend(token_ids)
        self.n += len(token_ids)
        if len(self.buf) > WINDOW:
            del self.buf[: len(self.buf) - WINDOW]
        if self.n // CHECK_EVERY == before // CHECK_EVERY:
            return False
        return detect_loop(self.buf)
