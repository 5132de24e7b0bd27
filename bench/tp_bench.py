#!/usr/bin/env python
"""Tensor-parallel decode benchmark (run under torchrun, one process per GPU).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench/tp_bench.py \
        [--model llama-3-70b] [--batch 16] [--ctx 2048] [--mode nvlink|nccl] [--steps 20]

Sets up ``--batch`` requests with ``--ctx``-token random prompts (k8v4 KV for the 70B
preset), then times ``--steps`` pure decode steps (CUDA-graph replays) with CUDA events on
each rank; reports the max over ranks of the mean step time and the resulting output
tokens/s. Both collective modes run the same sharded model, so their difference is the
cost of the row-parallel all-reduces (fused over NVLink vs NCCL).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from squish_b200.engine.engine import EngineConfig, LLMEngine  # noqa: E402
from squish_b200.engine.sampling import SamplingParams  # noqa: E402
from squish_b200.models.config import get_preset  # noqa: E402
from squish_b200.models.weights import random_checkpoint  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-70b")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--mode", default="nvlink")
    ap.add_argument("--steps", type=int, default=20)
    a = ap.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg, q = get_preset(a.model)
    ck = random_checkpoint(cfg, q, seed=0, device=dev)
    ecfg = EngineConfig(max_num_seqs=a.batch, max_num_batched_tokens=2048, max_model_len=a.ctx + a.steps + 64,
                        tp=world, tp_mode=a.mode, gpu_memory_utilization=0.8)
    eng = LLMEngine.from_checkpoint(ck, dev, ecfg)
    del ck
    rng = np.random.default_rng(0)
    for _ in range(a.batch):
        eng.add_request(rng.integers(0, cfg.vocab_size, a.ctx).tolist(),
                        SamplingParams(max_tokens=a.steps + 8, ignore_eos=True))
    while any(r.in_prefill for r in eng.scheduler.running) or eng.scheduler.waiting:
        eng.step()
    for _ in range(3):
        eng.step()
    eng.runner.timing = True
    eng.runner._events = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    tok0 = eng.stats.generated_tokens
    for _ in range(a.steps):
        eng.step()
    torch.cuda.synchronize()
    ms = eng.runner.device_time_ms() / a.steps
    toks = eng.stats.generated_tokens - tok0
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if hasattr(eng, "comm"):
            eng.comm.check()
    if rank == 0:
        print(json.dumps({"model": a.model, "tp": world, "mode": a.mode, "batch": a.batch, "ctx": a.ctx,
                          "ms_per_step": round(float(t.item()), 3),
                          "tok_s": round(toks / a.steps / float(t.item()) * 1000, 1),
                          "graph_steps": eng.stats.graph_steps}), flush=True)
    eng.graphs = None
    if hasattr(eng, "comm"):
        eng.comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
