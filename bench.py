#!/usr/bin/env python
"""Serving benchmark: output tokens/s and p50/p99 TTFT, Qwen2.5-7B-shaped INT4 model with an
INT4 KV cache, N GPUs of one node (data-parallel replicas, one process per GPU).

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

Workload (per GPU, weak scaling): a closed loop that keeps ``--concurrency`` requests in
flight; prompts are random token ids with lengths uniform in [128, 2048], each request
generates 256 tokens (EOS ignored). Weights are random N(0, 0.02) of the Qwen2.5-7B
architecture quantized INT4 asymmetric group-64 with bf16 scales; KV is INT4 in 16-token
pages. The loop is ramped to steady state (the first wave of requests gets staggered
output lengths), then W untimed steps, then K timed steps. A step is one engine
iteration (one batched forward over every running request: decodes + prefill chunks).

Reported (rank 0, one JSON line):
  value        output tokens/s over all GPUs, device-timed: sum over ranks of tokens
               generated in the K steps / max over ranks of the summed CUDA-event time
               of the steps (metadata H2D .. sampled-token D2H on the stream);
  e2e.value    the same tokens / max over ranks of the wall-clock time of the K calls to
               the public API LLMEngine.step() (host scheduling, pinned H2D of the step's
               inputs, D2H of the sampled tokens included);
  ttft_ms      p50 / p99 over requests whose first token came in the timed window.
The reference arm runs the unmodified reference package from baseline/_ref through its
public torch backend (squish.backend.BE.stream_generate: HF transformers generate with
a KV cache, fp16 weights: the reference's INT4 torch loader dequantizes to fp16 before
loading, so fp16 is what its CUDA path computes with).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "output tok/s + p50/p99 TTFT, Qwen2.5-7B-shape INT4 w/ INT4 KV, 1/2/4/8 B200"
PUBLISHED_VALUE = None  # the reference publishes no B200 number for this metric


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--concurrency", type=int, default=64)
    ap.add_argument("--prompt-min", type=int, default=128)
    ap.add_argument("--prompt-max", type=int, default=2048)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--max-batched-tokens", type=int, default=2048)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--prefill-weight-cache", type=int, default=1,
                    help="1: keep bf16 expansions of the layer weights resident for prefill GEMMs")
    ap.add_argument("--clocks", default="1", help="sample nvidia-smi clocks during the timed region")
    return ap.parse_args()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, enabled: bool = True):
        self.gpu = gpu_index
        self.enabled = enabled
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        if not self.enabled:
            return
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- distributed helpers
def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"WORLD_SIZE={world} but --gpus={args.gpus}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    return world, rank, local


def reduce(vals: list[float], op: str, world: int) -> list[float]:
    if world == 1:
        return vals
    import torch
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return t.tolist()


def gather_list(vals: list[float], world: int) -> list[float]:
    if world == 1:
        return vals
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, vals)
    return [v for part in out for v in part]


def barrier(world: int):
    import torch

    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def pct(xs, q):
    if not xs:
        return None
    xs = sorted(xs)
    k = min(len(xs) - 1, max(0, int(round(q / 100 * (len(xs) - 1)))))
    return xs[k]


# ----------------------------------------------------------------------------- our arm
def run_ours(args, world, rank, local):
    import numpy as np
    import torch

    sys.path.insert(0, HERE)
    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.engine.sampling import SamplingParams
    from squish_b200.ops.kernels import LAUNCHES

    dev = torch.device("cuda", local)
    ecfg = EngineConfig(max_num_seqs=args.concurrency, max_num_batched_tokens=args.max_batched_tokens,
                        max_model_len=args.prompt_max + args.output_len + 16, cuda_graphs=not args.no_graphs,
                        enable_prefix_caching=True, gpu_memory_utilization=0.85,
                        prefill_weight_cache=bool(args.prefill_weight_cache))
    t0 = time.time()
    eng = LLMEngine.from_preset(args.model, device=dev, seed=args.seed, ecfg=ecfg)  # same weights on every rank
    load_s = time.time() - t0
    cache_gb = getattr(eng.runner, "prefill_cache_bytes", 0) / 1e9
    rng = np.random.default_rng(1000 + args.seed + rank)
    vocab = eng.cfg.vocab_size

    def new_request(out_len):
        n = int(rng.integers(args.prompt_min, args.prompt_max + 1))
        prompt = rng.integers(0, vocab, n).tolist()
        return eng.add_request(prompt, SamplingParams(max_tokens=out_len, ignore_eos=True))

    # ramp: first wave with staggered output lengths (steady-state age distribution)
    for _ in range(args.concurrency):
        new_request(int(rng.integers(1, args.output_len + 1)))
    guard = 0
    while (eng.scheduler.waiting or any(r.in_prefill for r in eng.scheduler.running)) and guard < 10000:
        eng.step()
        guard += 1

    def top_up():
        while len(eng.scheduler.running) + len(eng.scheduler.waiting) < args.concurrency:
            new_request(args.output_len)

    for _ in range(args.warmup):
        top_up()
        eng.step()
    # timed region
    runner = eng.runner
    runner.timing = True
    runner._events = []
    tok0 = eng.stats.generated_tokens
    ttft0 = len(eng.stats.ttfts)
    h2d0, d2h0 = eng.stats.h2d_bytes, eng.stats.d2h_bytes
    steps0 = eng.stats.steps
    launches0 = LAUNCHES[0]
    g0, mx0, sched0 = eng.stats.graph_steps, eng.stats.mixed_steps, eng.stats.scheduled_tokens
    clocks = ClockSampler(local, args.clocks != "0")
    barrier(world)
    clocks.start()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        top_up()
        eng.step()
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    barrier(world)
    clk = clocks.stop()
    dev_ms = runner.device_time_ms()
    runner.timing = False
    tokens = eng.stats.generated_tokens - tok0
    ttfts = [t * 1000 for t in eng.stats.ttfts[ttft0:]]
    launches = LAUNCHES[0] - launches0
    h2d = (eng.stats.h2d_bytes - h2d0) / max(1, eng.stats.steps - steps0)
    d2h = (eng.stats.d2h_bytes - d2h0) / max(1, eng.stats.steps - steps0)
    tot_tokens, tot_launch = reduce([tokens, launches], "sum", world)
    max_dev_ms, max_wall = reduce([dev_ms, wall], "max", world)
    all_ttft = gather_list(ttfts, world)
    res = {
        "metric": METRIC,
        "value": tot_tokens / (max_dev_ms / 1000.0),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": max_dev_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 activations, INT4 weights (bf16 scales), INT4 KV",
        "data": "synthetic: random-init N(0,0.02) weights, random token-id prompts",
        "config": {
            "model": "Qwen2.5-7B-shape (28L, h3584, 28q/4kv heads, d128, ffn 18944, vocab 152064), INT4 g64",
            "global_batch": args.concurrency * world,
            "seq_len": f"prompt U[{args.prompt_min},{args.prompt_max}] + {args.output_len} out",
            "parallelism": f"dp{world}",
            "concurrency_per_gpu": args.concurrency,
            "max_batched_tokens": args.max_batched_tokens,
            "kv": "int4 g32, 16-token pages",
            "l2": "no flush: weights (~4.4 GB) and KV exceed the 126 MB L2 every step",
            "cuda_graphs": not args.no_graphs,
            "prefill_weight_cache_gb": round(cache_gb, 2),
            "weights": "INT4 codes read by decode GEMMs; prefill GEMMs (>= 384 rows) read resident bf16 "
                       "expansions of the same codes when prefill_weight_cache_gb > 0",
        },
        "ttft_ms": {"p50": pct(all_ttft, 50), "p99": pct(all_ttft, 99), "n": len(all_ttft)},
        "e2e": {"value": tot_tokens / max_wall, "unit": "tokens/s", "h2d_bytes_per_step": round(h2d),
                "d2h_bytes_per_step": round(d2h), "api": "LLMEngine.step()"},
        "gpu_launches": int(tot_launch),
        "clocks": clk,
        "load_s": round(load_s, 1),
        "steps_detail": {"graph_decode": eng.stats.graph_steps - g0, "with_prefill": eng.stats.mixed_steps - mx0,
                         "tokens_per_step": (eng.stats.scheduled_tokens - sched0) / args.steps},
        "impl": "ours",
    }
    return res


# ----------------------------------------------------------------------------- reference arm
def run_reference(args, world, rank, local):
    ref_root = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "squish")):
        return {"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}
    sys.path.insert(0, ref_root)
    import numpy as np
    import torch

    try:
        from squish.backend import BE  # the reference's public compute backend
    except Exception as exc:  # noqa: BLE001
        return {"impl": "reference", "unavailable": f"reference import failed: {exc!r}"[:200]}
    if getattr(BE, "device", "cpu") != "cuda":
        return {"impl": "reference", "unavailable": "reference backend did not select CUDA"}
    from transformers import AutoModelForCausalLM, Qwen2Config

    # Qwen2.5-7B architecture, random N(0, 0.02) weights, fp16: what the reference's CUDA
    # loader serves (its INT4 npy-dir path dequantizes to fp16 before HF load_state_dict).
    cfg = Qwen2Config(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                      num_attention_heads=28, num_key_value_heads=4, max_position_embeddings=32768,
                      rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=False, torch_dtype="float16")
    torch.manual_seed(args.seed)
    with torch.device("cuda"):
        model = AutoModelForCausalLM.from_config(cfg, torch_dtype=torch.float16)
    model.eval()
    model.generation_config.eos_token_id = None  # fixed-length outputs, as in our arm
    model.generation_config.pad_token_id = 0

    class TokenIdTokenizer:
        """Prompts are random token ids: encode parses them, decode prints them."""

        eos_token_id = None
        pad_token_id = 0

        def __call__(self, text, return_tensors="pt"):
            ids = torch.tensor([[int(t) for t in text.split()]], dtype=torch.long)

            class Enc(dict):
                def to(self, d):
                    return Enc({k: v.to(d) for k, v in self.items()})

            return Enc(input_ids=ids, attention_mask=torch.ones_like(ids))

        def decode(self, ids, skip_special_tokens=True, **kw):
            return " ".join(str(int(i)) for i in ids)

    tok = TokenIdTokenizer()
    rng = np.random.default_rng(1000 + args.seed + rank)
    # one "step" = one generated token of the current request (the reference serves one
    # stream at a time on this path); requests run back to back.
    ttfts, produced, times = [], 0, []

    def one_request(max_tokens, budget):
        nonlocal produced
        n = int(rng.integers(args.prompt_min, args.prompt_max + 1))
        prompt = " ".join(str(int(t)) for t in rng.integers(0, cfg.vocab_size, n))
        t_start = time.perf_counter()
        first = True
        count = 0
        for text, fin in BE.stream_generate(model, tok, prompt, max_tokens=max_tokens, temperature=0.0):
            if fin is not None:
                break
            if first:
                ttfts.append((time.perf_counter() - t_start) * 1000)
                first = False
            count += 1
            if count >= budget:
                break
        return count

    one_request(8, args.warmup)  # warm-up
    barrier(world)
    w0 = time.perf_counter()
    done = 0
    while done < args.steps:
        done += one_request(args.output_len, args.steps - done)
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    barrier(world)
    tot, = reduce([done], "sum", world)
    mx, = reduce([wall], "max", world)
    all_ttft = gather_list(ttfts, world)
    return {"metric": METRIC, "value": tot / mx, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": mx * 1000 / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic: random-init weights, random token-id prompts",
            "config": {"model": "Qwen2.5-7B-shape (HF Qwen2ForCausalLM, fp16)", "global_batch": world,
                       "seq_len": f"prompt U[{args.prompt_min},{args.prompt_max}] + {args.output_len} out",
                       "parallelism": f"dp{world}", "path": "squish.backend.BE.stream_generate (HF generate)"},
            "ttft_ms": {"p50": pct(all_ttft, 50), "p99": pct(all_ttft, 99), "n": len(all_ttft)},
            "timing": "wall clock around the K streamed tokens (the reference path synchronises every token)",
            "impl": "reference"}


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            res = run_reference(args, world, rank, local)
        else:
            res = run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.barrier()
                dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)
    if args.impl == "reference":
        # the reference's HF streamer leaves its generation thread running when a request is
        # cut at the step budget; end the process without waiting for it
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)


if __name__ == "__main__":
    main()
