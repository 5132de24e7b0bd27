"""Span tracer (enable with SQUISH_TRACE=1 or tracer().enable()).

``span(name)`` is a context manager (and ``traced`` a decorator) that records wall-clock
intervals with parent tracking through a ContextVar, exported as Chrome trace JSON
(chrome://tracing, Perfetto) at ``GET /v1/trace`` — the counterpart of the reference's
squish/telemetry.py:446-555. CUDA work is timed separately with events (bench.py) and
NVTX ranges (``nvtx`` below) so device timelines line up in profilers.
"""
from __future__ import annotations

import contextvars
import functools
import os
import threading
import time
from contextlib import contextmanager

_parent: contextvars.ContextVar[int | None] = contextvars.ContextVar("squish_span_parent", default=None)


class Tracer:
    def __init__(self, capacity: int = 100_000):
        self.enabled = os.environ.get("SQUISH_TRACE", "0") not in ("", "0", "false")
        self.capacity = capacity
        self.events: list[dict] = []
        self._lock = threading.Lock()
        self._ids = 0
        self.t0 = time.perf_counter()

    def enable(self, on: bool = True) -> None:
        self.enabled = on

    def clear(self) -> None:
        with self._lock:
            self.events.clear()

    def record(self, name: str, start: float, end: float, parent: int | None, args: dict | None = None) -> int:
        with self._lock:
            self._ids += 1
            sid = self._ids
            if len(self.events) < self.capacity:
                self.events.append({"name": name, "id": sid, "parent": parent, "start": start, "end": end,
                                    "tid": threading.get_ident(), "args": args or {}})
        return sid

    def to_chrome(self) -> dict:
        with self._lock:
            evs = list(self.events)
        out = []
        for e in evs:
            out.append({"name": e["name"], "ph": "X", "ts": (e["start"] - self.t0) * 1e6,
                        "dur": (e["end"] - e["start"]) * 1e6, "pid": os.getpid(), "tid": e["tid"] % 100000,
                        "args": dict(e["args"], span_id=e["id"], parent=e["parent"])})
        return {"traceEvents": out, "displayTimeUnit": "ms"}

    def summary(self) -> dict:
        agg: dict[str, list[float]] = {}
        with self._lock:
            for e in self.events:
                agg.setdefault(e["name"], []).append((e["end"] - e["start"]) * 1e3)
        return {k: {"count": len(v), "total_ms": sum(v), "mean_ms": sum(v) / len(v)} for k, v in agg.items()}


_TRACER = Tracer()


def tracer() -> Tracer:
    return _TRACER


@contextmanager
def span(name: str, **args):
    t = _TRACER
    if not t.enabled:
        yield
        return
    parent = _parent.get()
    start = time.perf_counter()
    token = _parent.set(-1)
    try:
        yield
    finally:
        _parent.reset(token)
        t.record(name, start, time.perf_counter(), parent, args)


def traced(name: str | None = None):
    def deco(fn):
        label = name or fn.__qualname__

        @functools.wraps(fn)
        def wrapper(*a, **kw):
            with span(label):
                return fn(*a, **kw)

        return wrapper

    return deco


@contextmanager
def nvtx(name: str):
    """An NVTX range around device work (no-op without CUDA)."""
    try:
        import torch

        if torch.cuda.is_available():
            torch.cuda.nvtx.range_push(name)
            try:
                yield
            finally:
                torch.cuda.nvtx.range_pop()
            return
    except ImportError:
        pass
    yield
