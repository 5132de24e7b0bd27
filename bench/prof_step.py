#!/usr/bin/env python
"""One engine step of the Qwen2.5-7B-shaped INT4 model under a profiler window.

    python bench/prof_step.py [--batch 64] [--ctx 1000] [--mode decode|prefill]

Sets up ``--batch`` running requests with ``--ctx``-token prompts (prefilled outside the
window), warms the decode CUDA graph, then brackets ``--steps`` steps with
cudaProfilerStart/Stop, so ``ncu --profile-from-start off`` sees only those steps:
decode mode = pure decode steps (graph replays); prefill mode = one new request with a
``--ctx``-token prompt arrives, so the step is a prefill chunk mixed with the decodes.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from squish_b200.engine.engine import EngineConfig, LLMEngine  # noqa: E402
from squish_b200.engine.sampling import SamplingParams  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1000)
    ap.add_argument("--mode", default="decode", choices=["decode", "prefill"])
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--no-graphs", action="store_true")
    a = ap.parse_args()
    eng = LLMEngine.from_preset(a.model, device="cuda", seed=0, ecfg=EngineConfig(
        max_num_seqs=a.batch + 1, max_num_batched_tokens=2048, max_model_len=a.ctx + 512,
        cuda_graphs=not a.no_graphs))
    rng = np.random.default_rng(0)
    for _ in range(a.batch):
        eng.add_request(rng.integers(0, eng.cfg.vocab_size, a.ctx).tolist(),
                        SamplingParams(max_tokens=400, ignore_eos=True))
    while any(r.in_prefill for r in eng.scheduler.running) or eng.scheduler.waiting:
        eng.step()
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    if a.mode == "prefill":
        eng.add_request(rng.integers(0, eng.cfg.vocab_size, a.ctx).tolist(), SamplingParams(max_tokens=4))
    torch.cuda.profiler.start()
    for _ in range(a.steps):
        eng.step()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print("ok", eng.stats.graph_steps, eng.stats.mixed_steps)


if __name__ == "__main__":
    main()
