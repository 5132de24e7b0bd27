"""Memory governor: maps device memory and KV-page occupancy to a pressure level.

The reference polls macOS memory pressure and sheds requests with HTTP 503 at CRITICAL
(squish/serving/memory_governor.py:1-76,183-330; squish/server.py:355-490). Here the
signals are the GPU's free memory (cudaMemGetInfo through torch) and the paged KV pool's
occupancy; callbacks fire on level changes and the HTTP layer sheds new work at CRITICAL.
Probes are injectable so the policy is testable without a GPU.
"""
from __future__ import annotations

import threading
import time
from typing import Callable

NORMAL, WARN, CRITICAL = 0, 1, 2
LEVEL_NAMES = {NORMAL: "normal", WARN: "warn", CRITICAL: "critical"}


def cuda_mem_probe(device=None) -> Callable[[], tuple[float, float]]:
    def probe():
        import torch

        free, total = torch.cuda.mem_get_info(device)
        return free / 2**30, total / 2**30

    return probe


class MemoryGovernor:
    def __init__(self, mem_probe: Callable[[], tuple[float, float]] | None = None,
                 kv_usage: Callable[[], float] | None = None, warn_free_frac: float = 0.05,
                 crit_free_frac: float = 0.02, warn_kv: float = 0.90, crit_kv: float = 0.98, interval_s: float = 1.0):
        self.mem_probe = mem_probe
        self.kv_usage = kv_usage
        self.warn_free_frac, self.crit_free_frac = warn_free_frac, crit_free_frac
        self.warn_kv, self.crit_kv = warn_kv, crit_kv
        self.interval_s = interval_s
        self.level = NORMAL
        self.available_gb = float("nan")
        self._callbacks: list[Callable[[int, int], None]] = []
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    def on_change(self, cb: Callable[[int, int], None]) -> None:
        self._callbacks.append(cb)

    @property
    def critical(self) -> bool:
        return self.level >= CRITICAL

    def evaluate(self) -> int:
        lvl = NORMAL
        if self.mem_probe is not None:
            free, total = self.mem_probe()
            self.available_gb = free
            frac = free / total if total else 1.0
            if frac < self.crit_free_frac:
                lvl = CRITICAL
            elif frac < self.warn_free_frac:
                lvl = max(lvl, WARN)
        if self.kv_usage is not None:
            u = self.kv_usage()
            if u >= self.crit_kv:
                lvl = max(lvl, CRITICAL)
            elif u >= self.warn_kv:
                lvl = max(lvl, WARN)
        if lvl != self.level:
            old, self.level = self.level, lvl
            for cb in list(self._callbacks):
                cb(old, lvl)
        return lvl

    def start(self) -> "MemoryGovernor":
        def loop():
            while not self._stop.wait(self.interval_s):
                try:
                    self.evaluate()
                except Exception:  # noqa: BLE001 - a failing probe must not kill the server
                    pass

        self.evaluate()
        self._thread = threading.Thread(target=loop, name="squish-memgov", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
