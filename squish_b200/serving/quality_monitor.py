"""Rolling-window serving quality statistics (``GET /v1/quality``).

Same record and report fields as the reference's QualityMonitor
(squish/serving/quality_monitor.py:68-300): per finished request its latency, time to first
token, token count, throughput and success; per model over the last ``window`` seconds the
request and error counts, latency p50/p95/p99/mean, tokens/s p50/mean and TTFT p50/p95.
Percentiles interpolate linearly between order statistics (numpy's default).
"""
from __future__ import annotations

import collections
import datetime
import math
import threading
import time
from dataclasses import asdict, dataclass


def percentile(sorted_vals: list[float], p: float) -> float:
    if not sorted_vals:
        return 0.0
    i = (p / 100.0) * (len(sorted_vals) - 1)
    lo, hi = int(math.floor(i)), int(math.ceil(i))
    return sorted_vals[lo] + (sorted_vals[hi] - sorted_vals[lo]) * (i - lo)


@dataclass(frozen=True)
class RequestMetric:
    timestamp: float
    model_id: str
    latency_ms: float
    ttft_ms: float | None
    tokens_generated: int
    tokens_per_sec: float
    success: bool
    error_type: str | None = None


class QualityMonitor:
    def __init__(self, max_window_seconds: int = 3600, max_records: int = 100_000):
        self.max_window = max_window_seconds
        self._dq: collections.deque = collections.deque(maxlen=max_records)
        self._lock = threading.Lock()

    def record(self, m: RequestMetric) -> None:
        with self._lock:
            self._dq.append(m)
            cutoff = m.timestamp - self.max_window
            while self._dq and self._dq[0].timestamp < cutoff:
                self._dq.popleft()

    def record_request(self, model_id: str, latency_s: float, ttft_s: float | None, tokens: int,
                       success: bool = True, error_type: str | None = None) -> None:
        tps = tokens / latency_s if latency_s > 0 else 0.0
        self.record(RequestMetric(time.monotonic(), model_id, latency_s * 1e3,
                                  None if ttft_s is None else ttft_s * 1e3, tokens, tps, success, error_type))

    def stats(self, window_seconds: int = 300, model_id: str = "") -> dict:
        now = time.monotonic()
        with self._lock:
            recs = [m for m in self._dq if m.timestamp >= now - window_seconds and (not model_id or m.model_id == model_id)]
        models = {}
        for mid in sorted({m.model_id for m in recs}):
            rs = [m for m in recs if m.model_id == mid]
            ok = [m for m in rs if m.success]
            lat = sorted(m.latency_ms for m in ok)
            tps = sorted(m.tokens_per_sec for m in ok)
            ttft = sorted(m.ttft_ms for m in ok if m.ttft_ms is not None)
            n_err = len(rs) - len(ok)
            models[mid] = {
                "model_id": mid, "window_seconds": window_seconds, "n_requests": len(rs), "n_errors": n_err,
                "error_rate": n_err / max(1, len(rs)),
                "latency_p50_ms": percentile(lat, 50), "latency_p95_ms": percentile(lat, 95),
                "latency_p99_ms": percentile(lat, 99), "latency_mean_ms": sum(lat) / len(lat) if lat else 0.0,
                "tokens_per_sec_p50": percentile(tps, 50), "tokens_per_sec_mean": sum(tps) / len(tps) if tps else 0.0,
                "ttft_p50_ms": percentile(ttft, 50) if ttft else None,
                "ttft_p95_ms": percentile(ttft, 95) if ttft else None,
            }
        return {"window_seconds": window_seconds, "total_requests": len(recs),
                "generated_at": datetime.datetime.now(datetime.timezone.utc).isoformat(),
                "models": list(models.values())}

    def records(self) -> list[dict]:
        with self._lock:
            return [asdict(m) for m in self._dq]

    def clear(self) -> None:
        with self._lock:
            self._dq.clear()
