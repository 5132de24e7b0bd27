#!/usr/bin/env python
"""Serving sweep on one GPU: output tok/s and TTFT p50/p99 over a concurrency sweep.

    python bench/serving_sweep.py [--model qwen2.5-7b] [--concurrency 1 8 32 64]
                                  [--requests 256] [--shared-prefix 0.5 --prefix-len 1024]

Closed loop through ``LLMEngine.step()``: ``--requests`` requests with random-token prompts
of lengths U[prompt_min, prompt_max] and ``--output-len`` tokens each; with
``--shared-prefix p`` a fraction p of the requests start with one common random prefix of
``--prefix-len`` tokens (exercises prefix page sharing). Reports wall-clock tok/s with the
device synchronised, TTFT p50/p99, the device-time share, and the prefix-hit tokens.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from squish_b200.engine.engine import EngineConfig, LLMEngine  # noqa: E402
from squish_b200.engine.sampling import SamplingParams  # noqa: E402


def sweep_point(eng, conc, n_req, pmin, pmax, out_len, shared, prefix_len, seed):
    rng = np.random.default_rng(seed)
    vocab = eng.cfg.vocab_size
    prefix = rng.integers(0, vocab, prefix_len).tolist()
    sub, done, toks = 0, 0, 0
    t_sub, ttft, seen = {}, [], set()
    eng.runner.timing = True
    eng.runner._events = []
    hit0 = eng.stats.prefix_hit_tokens

    def submit():
        nonlocal sub
        n = int(rng.integers(pmin, pmax + 1))
        p = rng.integers(0, vocab, n).tolist()
        if shared and rng.random() < shared:
            p = prefix + p[: max(1, n - prefix_len)]
        rid = eng.add_request(p, SamplingParams(max_tokens=out_len, ignore_eos=True))
        t_sub[rid] = time.perf_counter()
        sub += 1

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    while sub < min(conc, n_req):
        submit()
    while done < n_req:
        outs = eng.step()
        now = time.perf_counter()
        for o in outs:
            if o.new_tokens and o.rid not in seen:
                seen.add(o.rid)
                ttft.append((now - t_sub[o.rid]) * 1000)
            toks += len(o.new_tokens)
            if o.finished:
                done += 1
                if sub < n_req:
                    submit()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    dev_ms = eng.runner.device_time_ms()
    eng.runner.timing = False
    return {"concurrency": conc, "requests": n_req, "output_tokens": toks, "tok_s": round(toks / wall, 1),
            "device_tok_s": round(toks / (dev_ms / 1000), 1), "ttft_ms_p50": round(float(np.percentile(ttft, 50)), 1),
            "ttft_ms_p99": round(float(np.percentile(ttft, 99)), 1), "wall_s": round(wall, 2),
            "prefix_hit_tokens": eng.stats.prefix_hit_tokens - hit0}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--concurrency", type=int, nargs="+", default=[1, 8, 32, 64])
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--prompt-min", type=int, default=128)
    ap.add_argument("--prompt-max", type=int, default=2048)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--shared-prefix", type=float, default=0.0)
    ap.add_argument("--prefix-len", type=int, default=1024)
    ap.add_argument("--max-batched-tokens", type=int, default=2048)
    a = ap.parse_args()
    maxc = max(a.concurrency)
    eng = LLMEngine.from_preset(a.model, device="cuda", seed=0, ecfg=EngineConfig(
        max_num_seqs=maxc, max_num_batched_tokens=a.max_batched_tokens,
        max_model_len=a.prompt_max + a.prefix_len + a.output_len + 32))
    for c in a.concurrency:
        n = max(a.requests if c > 1 else min(a.requests, 8), c)
        r = sweep_point(eng, c, n, a.prompt_min, a.prompt_max, a.output_len, a.shared_prefix, a.prefix_len, c)
        print(json.dumps({"model": a.model, **r}), flush=True)


if __name__ == "__main__":
    main()
