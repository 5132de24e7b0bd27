"""Startup phase timing (``GET /v1/startup``; printed when ``SQUISH_TRACE_STARTUP=1``).

The reference's StartupTimer / StartupReport (squish/serving/startup_profiler.py) time the
server's initialisation phases so slow starts can be diagnosed. The phases here are this
server's: imports, config, checkpoint read, weight upload and layout, KV pool, CUDA-graph
capture, tokenizer, HTTP start.
"""
from __future__ import annotations

import importlib
import os
import sys
import threading
import time
from enum import Enum


class StartupPhase(str, Enum):
    IMPORTS = "imports"
    CONFIG = "config"
    CHECKPOINT_READ = "checkpoint_read"
    WEIGHT_UPLOAD = "weight_upload"
    KV_CACHE_INIT = "kv_cache_init"
    CUDA_GRAPHS = "cuda_graph_capture"
    TOKENIZER = "tokenizer"
    SERVER_START = "server_start"
    OTHER = "other"


class StartupReport:
    def __init__(self) -> None:
        self.t0 = time.perf_counter()
        self.entries: list[dict] = []
        self._lock = threading.Lock()

    def add(self, phase: str, label: str, start: float, end: float) -> None:
        with self._lock:
            self.entries.append({"phase": str(getattr(phase, "value", phase)), "label": label,
                                 "start_ms": round((start - self.t0) * 1e3, 3),
                                 "elapsed_ms": round((end - start) * 1e3, 3)})

    def total_ms(self) -> float:
        return sum(e["elapsed_ms"] for e in self.entries)

    def slowest(self, n: int = 5) -> list[dict]:
        return sorted(self.entries, key=lambda e: -e["elapsed_ms"])[:n]

    def to_dict(self) -> dict:
        return {"total_ms": round(self.total_ms(), 3), "phases": list(self.entries), "slowest": self.slowest()}

    def clear(self) -> None:
        with self._lock:
            self.entries.clear()
            self.t0 = time.perf_counter()


_REPORT = StartupReport()


def report() -> StartupReport:
    return _REPORT


class StartupTimer:
    """``with StartupTimer(StartupPhase.WEIGHT_UPLOAD, "layers"):`` records one phase."""

    def __init__(self, phase, label: str = "", rep: StartupReport | None = None) -> None:
        self.phase, self.label, self.rep = phase, label, rep or _REPORT

    def __enter__(self) -> "StartupTimer":
        self.start = time.perf_counter()
        return self

    def __exit__(self, *exc) -> None:
        end = time.perf_counter()
        self.rep.add(self.phase, self.label, self.start, end)
        if os.environ.get("SQUISH_TRACE_STARTUP") == "1":
            print(f"[startup] {getattr(self.phase, 'value', self.phase)} {self.label} "
                  f"{(end - self.start) * 1e3:.1f} ms", file=sys.stderr)


def measure_import_ms(module: str) -> float:
    """Wall time of a fresh import of ``module`` (removed from sys.modules first)."""
    sys.modules.pop(module, None)
    t = time.perf_counter()
    importlib.import_module(module)
    return (time.perf_counter() - t) * 1e3
