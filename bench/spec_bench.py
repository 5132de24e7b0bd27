#!/usr/bin/env python
"""Speculative decoding benchmark: Qwen2.5-7B-shaped INT4 target, INT4 KV.

    python bench/spec_bench.py [--method draft|prompt_lookup|jacobi] [--batch 1 4 16]
                               [--temps 0 0.7] [--force 0 1 2 3 4]

Draft model (method "draft"): Qwen2.5-0.5B-shaped INT4 g64, random init, k = 4 tokens per
round. Prompt lookup builds trees of up to 16 nodes (4 branches x 4 tokens). Prompts are 512
random token ids, 256 output tokens per request (EOS ignored). Random models agree on
almost nothing, so tokens/s is reported both at the measured acceptance and with the
engine told to accept exactly f drafts per round (``force_accept``, f = 0..k: the
verification and proposal work is unchanged, only the accept decision is overridden),
plus a no-speculation baseline at the same batch. Throughput is end to end through
``LLMEngine.generate`` (wall clock with the device synchronised), one JSON line per case.
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
from squish_b200.engine.speculative import SpecConfig  # noqa: E402
from squish_b200.models.config import get_preset  # noqa: E402
from squish_b200.models.weights import random_checkpoint  # noqa: E402


def run(eng, prompts, temp, out_len):
    sp = SamplingParams(max_tokens=out_len, ignore_eos=True, temperature=temp)
    eng.generate([p[:16] for p in prompts], SamplingParams(max_tokens=4, ignore_eos=True, temperature=temp))  # warm
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    outs = eng.generate(prompts, sp)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    return sum(len(o) for o in outs) / dt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--target", default="qwen2.5-7b")
    ap.add_argument("--draft", default="qwen2.5-0.5b")
    ap.add_argument("--method", default="draft")
    ap.add_argument("--batch", type=int, nargs="+", default=[1, 4, 16])
    ap.add_argument("--temps", type=float, nargs="+", default=[0.0, 0.7])
    ap.add_argument("--force", type=int, nargs="*", default=[0, 1, 2, 3, 4])
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--output-len", type=int, default=256)
    a = ap.parse_args()
    cfg, q = get_preset(a.target)
    dev = torch.device("cuda")
    rng = np.random.default_rng(0)
    maxb = max(a.batch)
    prompts = [rng.integers(0, cfg.vocab_size, a.prompt_len).tolist() for _ in range(maxb)]

    def engine(spec):
        e = EngineConfig(max_num_seqs=maxb, max_num_batched_tokens=2048, max_model_len=a.prompt_len + a.output_len + 64,
                         num_pages=maxb * ((a.prompt_len + a.output_len + 64) // 16 + 4) + 64, spec=spec)
        # the runner takes ownership of the checkpoint's tensors, so every engine gets a fresh one
        return LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0, device=dev), dev, e)

    base = engine(None)
    for b in a.batch:
        for t in a.temps:
            print(json.dumps({"case": "no-spec", "batch": b, "temperature": t,
                              "tok_s": round(run(base, prompts[:b], t, a.output_len), 1)}), flush=True)
    del base
    torch.cuda.empty_cache()
    branches = 4 if a.method == "prompt_lookup" else 1
    sc = SpecConfig(a.method, k=a.k, branches=branches, max_nodes=16, draft_model=a.draft if a.method == "draft"
                    else None, adaptive=False)
    eng = engine(sc)
    for b in a.batch:
        for t in a.temps:
            eng.spec_stats = dict.fromkeys(eng.spec_stats, 0)
            v = run(eng, prompts[:b], t, a.output_len)
            s = eng.spec_stats
            print(json.dumps({"case": f"{a.method} measured", "batch": b, "temperature": t, "tok_s": round(v, 1),
                              "accept_rate": round(s["accepted"] / max(1, s["drafted"]), 3),
                              "tokens_per_verify": round(s["emitted"] / max(1, s["verifies"]), 2)}), flush=True)
        for f in a.force:
            eng.ecfg.spec.force_accept = f
            v = run(eng, prompts[:b], 0.0, a.output_len)
            print(json.dumps({"case": f"{a.method} forced", "batch": b, "accepted_per_round": f,
                              "tok_s": round(v, 1)}), flush=True)
        eng.ecfg.spec.force_accept = None


if __name__ == "__main__":
    main()
