"""Bottleneck report (``GET /v1/obs-report``).

As the reference's obs_report (squish/serving/obs_report.py:47-161): per-operation latency
percentiles, the operations whose p99 crosses a threshold with a remediation hint for each,
an overall "ok" / "degraded" status, and the slowest recent trace spans. The operations here
are this server's: traced spans (``SQUISH_TRACE=1``), engine steps (timed on the engine
thread), request latency and time to first token (quality monitor). Hints name this
server's flags.
"""
from __future__ import annotations

from .quality_monitor import percentile

HINTS = {
    "engine.step": "slow engine steps: lower --max-num-batched-tokens (smaller prefill chunks per step) or "
                   "--max-num-seqs; keep CUDA graphs on (no --no-cuda-graphs)",
    "ttft_ms": "high time to first token: lower --max-num-batched-tokens so prefills interleave with decodes, "
               "enable prefix caching (drop --no-prefix-caching) and grid-align chunks (--chunk-align)",
    "latency_ms": "long requests: check queue depth (/v1/metrics) and --max-num-seqs; INT4 KV "
                  "(--kv-dtype int4) fits more sequences per GPU",
    "chat_template": "slow prompt rendering/tokenisation: large message histories; cache system prompts",
}


def hint_for(op: str) -> str:
    if op in HINTS:
        return HINTS[op]
    return next((h for k, h in HINTS.items() if op.startswith(k)), "")


def _stats(vals: list[float]) -> dict:
    v = sorted(vals)
    return {"n_samples": len(v), "mean_ms": round(sum(v) / len(v), 3) if v else 0.0,
            "p50_ms": round(percentile(v, 50), 3), "p95_ms": round(percentile(v, 95), 3),
            "p99_ms": round(percentile(v, 99), 3)}


def latency_profile(aeng, tracer=None) -> dict[str, dict]:
    ops: dict[str, list[float]] = {}
    if tracer is not None:
        with tracer._lock:
            evs = list(tracer.events)
        for e in evs:
            ops.setdefault(e["name"], []).append((e["end"] - e["start"]) * 1e3)
    steps = list(getattr(aeng, "step_ms", []))
    if steps:
        ops["engine.step"] = steps
    recs = aeng.quality.records() if hasattr(aeng, "quality") else []
    ok = [r for r in recs if r["success"]]
    if ok:
        ops["latency_ms"] = [r["latency_ms"] for r in ok]
        tt = [r["ttft_ms"] for r in ok if r["ttft_ms"] is not None]
        if tt:
            ops["ttft_ms"] = tt
    return {k: _stats(v) for k, v in ops.items()}


def detect_bottlenecks(profile: dict[str, dict], threshold_ms: float = 200.0) -> list[dict]:
    out = [{"op": op, "p99_ms": s["p99_ms"], "mean_ms": s["mean_ms"], "n_samples": s["n_samples"],
            "hint": hint_for(op)} for op, s in profile.items() if s["p99_ms"] >= threshold_ms]
    return sorted(out, key=lambda b: -b["p99_ms"])


def generate_report(aeng, tracer=None, threshold_ms: float = 200.0) -> dict:
    prof = latency_profile(aeng, tracer)
    b = detect_bottlenecks(prof, threshold_ms)
    spans = []
    if tracer is not None:
        with tracer._lock:
            evs = list(tracer.events)
        spans = [{"name": e["name"], "duration_ms": round((e["end"] - e["start"]) * 1e3, 3)}
                 for e in sorted(evs, key=lambda e: e["start"] - e["end"])[:10]]
    return {"status": "degraded" if b else "ok", "threshold_ms": threshold_ms, "bottlenecks": b,
            "profile": prof, "recent_spans": spans, "profiler_ops": sorted(prof)}
