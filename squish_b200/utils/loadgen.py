"""Closed-loop serving load generator over an engine (``squish bench``).

Keeps ``concurrency`` requests in flight: prompts of random token ids with lengths uniform
in [prompt_min, prompt_max], ``max_tokens`` outputs each (EOS ignored), a new request
submitted as soon as one finishes, until ``num_requests`` have completed. Reports output
tokens/s over the wall clock, TTFT p50/p99 and mean time per output token. The same
shape as the reference's serving benchmark (benchmarks/perf/serving_baseline.py).
"""
from __future__ import annotations

import time

import numpy as np

from ..engine.sampling import SamplingParams


def _pct(xs, q):
    return float(np.percentile(np.asarray(xs), q)) if len(xs) else float("nan")


def run_load(engine, num_requests: int = 64, concurrency: int = 8, prompt_min: int = 128, prompt_max: int = 2048,
             max_tokens: int = 256, seed: int = 0, sync=None) -> dict:
    rng = np.random.default_rng(seed)
    vocab = engine.cfg.vocab_size
    submitted = 0
    t_submit: dict[str, float] = {}
    ttft: list[float] = []
    first_seen: set[str] = set()
    done = 0
    out_tokens = 0

    def submit():
        nonlocal submitted
        n = int(rng.integers(prompt_min, prompt_max + 1))
        rid = engine.add_request(rng.integers(0, vocab, n).tolist(), SamplingParams(max_tokens=max_tokens,
                                                                                    ignore_eos=True))
        t_submit[rid] = time.perf_counter()
        submitted += 1

    t0 = time.perf_counter()
    while submitted < min(concurrency, num_requests):
        submit()
    while done < num_requests:
        outs = engine.step()
        now = time.perf_counter()
        for o in outs:
            if o.rid not in t_submit:
                continue
            if o.new_tokens and o.rid not in first_seen:
                first_seen.add(o.rid)
                ttft.append((now - t_submit[o.rid]) * 1000)
            out_tokens += len(o.new_tokens)
            if o.finished:
                done += 1
                if submitted < num_requests:
                    submit()
        if not outs and not engine.has_unfinished():
            break
    if sync is not None:
        sync()
    wall = time.perf_counter() - t0
    return {"requests": done, "concurrency": concurrency, "output_tokens": out_tokens, "wall_s": round(wall, 3),
            "output_tok_s": out_tokens / wall if wall > 0 else 0.0, "ttft_ms_p50": _pct(ttft, 50),
            "ttft_ms_p99": _pct(ttft, 99),
            "tpot_ms": (wall * 1000 * concurrency / out_tokens) if out_tokens else float("nan")}
