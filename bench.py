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
  ttft_ms      p50 / p99 over all 256 requests of the full workload (256 requests at the
               concurrency, run through LLMEngine after the timed window; "workload" has
               its wall-clock output tok/s); window_ttft_ms covers the requests whose first
               token came inside the timed window.
The reference arm runs the unmodified reference package from baseline/_ref through its
concurrent CUDA serving path: squish.serving.scheduler.NestedWaitScheduler (the reference
server's --batch-scheduler default) fed through submit_sync with the same concurrency,
prompt distribution and output length; see run_reference.
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
MODEL_DESC = "Qwen2.5-7B-shape (28L, h3584, 28q/4kv heads, d128, ffn 18944, vocab 152064)"
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
    ap.add_argument("--host-profile", action="store_true",
                    help="profile the host side of the timed steps (cProfile, top functions on stderr)")
    ap.add_argument("--ref-budget-s", type=float, default=150.0,
                    help="reference arm: time budget of the timed window (at least 3 steps)")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--prefill-weight-cache", type=int, default=1,
                    help="1: keep bf16 expansions of the layer weights resident for prefill GEMMs")
    ap.add_argument("--clocks", default="1", help="sample nvidia-smi clocks during the timed region")
    ap.add_argument("--workload-requests", type=int, default=256,
                    help="after the timed window, run this many requests at the concurrency (0: skip)")
    ap.add_argument("--sweep", type=lambda v: [int(x) for x in v.split(",") if x], default=[],
                    help="comma-separated concurrencies for a full-workload sweep (e.g. 1,8,32,64)")
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


# ----------------------------------------------------------------------------- workload
PHI = 0.6180339887498949


def prompt_lengths(n: int, lo: int, hi: int, offset: int = 0) -> list[int]:
    """Prompt lengths uniform in [lo, hi] as a golden-ratio low-discrepancy sequence: any run
    of consecutive requests covers the range evenly, so a short timed window sees the same
    mean prefill load as a long one (i.i.d. draws of five requests vary by +-20 %)."""
    span = hi - lo + 1
    return [lo + int(((0.5 + (offset + j) * PHI) % 1.0) * span) for j in range(n)]


def prompt_ids(rng, n: int, vocab: int) -> list[int]:
    return rng.integers(0, vocab, n).tolist()


# ----------------------------------------------------------------------------- our arm
def run_workload(eng, n_req: int, conc: int, args, seed: int) -> dict:
    """The serving workload of the benchmark's config: ``n_req`` requests, ``conc`` in flight
    (a new one is submitted when one finishes), through LLMEngine.step(). TTFT is measured
    from submission to the step that returns the request's first token."""
    import numpy as np
    import torch

    from squish_b200.engine.sampling import SamplingParams

    rng = np.random.default_rng(seed)
    lens = prompt_lengths(n_req, args.prompt_min, args.prompt_max, offset=7919)
    vocab = eng.cfg.vocab_size
    t_sub, ttft, seen = {}, [], set()
    sub = done = toks = 0

    def submit():
        nonlocal sub
        rid = eng.add_request(prompt_ids(rng, lens[sub], vocab), SamplingParams(max_tokens=args.output_len,
                                                                              ignore_eos=True))
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
            if o.rid not in t_sub:
                continue
            if o.new_tokens and o.rid not in seen:
                seen.add(o.rid)
                ttft.append((now - t_sub[o.rid]) * 1000)
            toks += len(o.new_tokens)
            if o.finished:
                done += 1
                if sub < n_req:
                    submit()
        if not outs and not eng.has_unfinished():
            break
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    return {"requests": done, "concurrency": conc, "output_tokens": toks, "wall_s": round(wall, 2),
            "output_tok_s": round(toks / wall, 1), "ttft_ms": {"p50": pct(ttft, 50), "p99": pct(ttft, 99),
                                                              "n": len(ttft)}, "ttft_list": ttft}


def repeat_prompt_ttft(eng, args, rng, n: int = 20, length: int = 1024) -> dict:
    """TTFT of a prompt that was served before (the same token ids), through add_request() +
    step() on an idle engine: the first token comes from the prompt-logit cache. Compared with
    the TTFT of the same prompt when it is new (a full prefill)."""
    import torch

    from squish_b200.engine.sampling import SamplingParams

    def ttft(prompt):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        rid = eng.add_request(prompt, SamplingParams(max_tokens=4, ignore_eos=True))
        t = None
        while eng.has_unfinished():
            for o in eng.step():
                if o.rid == rid and o.new_tokens and t is None:
                    t = (time.perf_counter() - t0) * 1000
        return t

    cold = [ttft(prompt_ids(rng, length, eng.cfg.vocab_size)) for _ in range(5)]
    p = prompt_ids(rng, length, eng.cfg.vocab_size)
    ttft(p)
    warm = [ttft(p) for _ in range(n)]
    return {"prompt_tokens": length, "repeat_p50": pct(warm, 50), "repeat_p99": pct(warm, 99),
            "new_prompt_p50": pct(cold, 50), "n": n,
            "path": "LLMEngine.add_request + step on an idle engine; repeat = prompt-logit cache hit"}


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
    C = args.concurrency
    lens = iter(prompt_lengths(1 << 20, args.prompt_min, args.prompt_max, offset=rank * 104729))

    def new_request(out_len, n=None):
        n = next(lens) if n is None else n
        return eng.add_request(prompt_ids(rng, n, vocab), SamplingParams(max_tokens=out_len, ignore_eos=True))

    # Ramp to the steady state of a closed loop: the first wave's output lengths are chosen
    # so that its requests finish one every output_len / C steps after their (FCFS, chunked)
    # prefill, as they do once the loop has run for a full request lifetime.
    first = [next(lens) for _ in range(C)]
    done_prefill = np.ceil(np.cumsum(first) / args.max_batched_tokens).astype(int)
    ramp = int(done_prefill[-1]) + 1
    for i, n in enumerate(first):
        finish = ramp + int(round((i + 1) * args.output_len / C))
        new_request(max(1, finish - int(done_prefill[i])), n)
    guard = 0
    while (eng.scheduler.waiting or any(r.in_prefill for r in eng.scheduler.running)) and guard < 10000:
        eng.step()
        guard += 1

    def top_up():
        while len(eng.scheduler.running) + len(eng.scheduler.waiting) < C:
            new_request(args.output_len)

    for _ in range(args.warmup):
        top_up()
        eng.step()
    eng.warmup_graphs()  # every decode graph of the steady state captured before timing
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
    host0, wait0 = dict(eng.stats.host_s), runner.sync_wait_s
    clocks = ClockSampler(local, args.clocks != "0")
    barrier(world)
    clocks.start()
    prof = None
    if args.host_profile:
        import cProfile

        prof = cProfile.Profile()
    w0 = time.perf_counter()
    if prof is not None:
        prof.enable()
    for _ in range(args.steps):
        top_up()
        eng.step()
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    if prof is not None:
        import pstats

        prof.disable()
        pstats.Stats(prof, stream=sys.stderr).sort_stats("tottime").print_stats(30)
    barrier(world)
    clk = clocks.stop()
    dev_ms = runner.device_time_ms()
    runner.timing = False
    tokens = eng.stats.generated_tokens - tok0
    ttfts = [t * 1000 for t in eng.stats.ttfts[ttft0:]]
    launches = LAUNCHES[0] - launches0
    h2d = (eng.stats.h2d_bytes - h2d0) / max(1, eng.stats.steps - steps0)
    d2h = (eng.stats.d2h_bytes - d2h0) / max(1, eng.stats.steps - steps0)
    sched_tok = (eng.stats.scheduled_tokens - sched0) / args.steps
    host = {k: round((v - host0[k]) * 1000 / args.steps, 3) for k, v in eng.stats.host_s.items()}
    host["device_wait"] = round((runner.sync_wait_s - wait0) * 1000 / args.steps, 3)
    detail = {"graph_decode": eng.stats.graph_steps - g0, "with_prefill": eng.stats.mixed_steps - mx0,
              "tokens_per_step": sched_tok, "prefill_tokens_per_step": sched_tok - tokens / args.steps,
              "host_ms_per_step": host, "wall_ms_per_step": round(wall * 1000 / args.steps, 3)}
    tot_tokens, tot_launch = reduce([tokens, launches], "sum", world)
    max_dev_ms, max_wall = reduce([dev_ms, wall], "max", world)
    all_ttft = gather_list(ttfts, world)

    # the full workload (every rank runs its own; TTFT over all requests of all ranks)
    for r in list(eng.scheduler.running) + list(eng.scheduler.waiting):
        eng.abort(r.rid)
    while eng.has_unfinished():
        eng.step()
    workload = None
    if args.workload_requests > 0:
        wl = run_workload(eng, args.workload_requests, C, args, seed=2000 + args.seed + rank)
        wl_tok, = reduce([wl["output_tokens"]], "sum", world)
        wl_wall, = reduce([wl["wall_s"]], "max", world)
        wl_ttft = gather_list(wl["ttft_list"], world)
        workload = {"requests_per_gpu": wl["requests"], "concurrency_per_gpu": C,
                    "output_tok_s": round(wl_tok / wl_wall, 1), "wall_s": wl_wall,
                    "ttft_ms": {"p50": pct(wl_ttft, 50), "p99": pct(wl_ttft, 99), "n": len(wl_ttft)},
                    "timing": "wall clock around the whole workload, device synchronised at both ends"}
    repeat = repeat_prompt_ttft(eng, args, rng)
    sweep = []
    for c in args.sweep:
        r = run_workload(eng, max(c, args.workload_requests), c, args, seed=3000 + c)
        r.pop("ttft_list")
        sweep.append(r)

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
            "model": MODEL_DESC,
            "global_batch": C * world,
            "seq_len": f"prompt U[{args.prompt_min},{args.prompt_max}] + {args.output_len} out",
            "parallelism": f"dp{world}",
            "concurrency_per_gpu": C,
            "max_batched_tokens": args.max_batched_tokens,
            "weights": "INT4 asymmetric g64 (bf16 scales): codes read by decode GEMMs; prefill GEMMs (>= 384 rows) "
                       "read resident bf16 expansions of the same codes when prefill_weight_cache_gb > 0",
            "kv": "int4 g32, 16-token pages",
            "l2": "no flush: weights (~4.4 GB) and KV exceed the 126 MB L2 every step",
            "cuda_graphs": not args.no_graphs,
            "prefill_weight_cache_gb": round(cache_gb, 2),
            "prompt_lengths": "golden-ratio low-discrepancy sequence over the range (uniform, even in short windows)",
        },
        "ttft_ms": ({**workload["ttft_ms"], "source": "every request of the workload run"}
                    if workload else
                    {"p50": pct(all_ttft, 50), "p99": pct(all_ttft, 99), "n": len(all_ttft),
                     "source": "requests whose first token came in the timed window"}),
        "window_ttft_ms": {"p50": pct(all_ttft, 50), "p99": pct(all_ttft, 99), "n": len(all_ttft)},
        "e2e": {"value": tot_tokens / max_wall, "unit": "tokens/s", "h2d_bytes_per_step": round(h2d),
                "d2h_bytes_per_step": round(d2h), "api": "LLMEngine.step()"},
        "gpu_launches": int(tot_launch),
        "clocks": clk,
        "load_s": round(load_s, 1),
        "steps_detail": detail,
        "workload": workload,
        "repeat_prompt_ttft_ms": repeat,
        "impl": "ours",
    }
    if sweep:
        res["sweep"] = sweep
    return res


# ----------------------------------------------------------------------------- reference arm
def host_memory_available() -> int:
    """Bytes this process may still allocate on the host: the smaller of the free memory
    the OS reports and the container's cgroup limit minus its current usage."""
    avail = None
    try:
        import psutil

        avail = int(psutil.virtual_memory().available)
    except Exception:  # noqa: BLE001
        pass
    for lim_f, cur_f in (("/sys/fs/cgroup/memory.max", "/sys/fs/cgroup/memory.current"),
                         ("/sys/fs/cgroup/memory/memory.limit_in_bytes", "/sys/fs/cgroup/memory/memory.usage_in_bytes")):
        try:
            lim = open(lim_f).read().strip()
            cur = int(open(cur_f).read().strip())
        except (OSError, ValueError):
            continue
        if lim.isdigit() and int(lim) < (1 << 60):
            left = int(lim) - cur
            avail = left if avail is None else min(avail, left)
        break
    return avail if avail is not None else 0


def keep_host_pages() -> bool:
    """Have glibc keep freed host memory for reuse: every step of the stock path copies tens of
    GB of fp32 logits into a freshly allocated host array; served by mmap, each step pays the
    page faults of the whole array again (measured: ~45 s of a ~48 s step). One arena, no
    mmap for large blocks and no trimming make the next step reuse the pages of the previous
    one. Allocator policy of this process only: the reference's code is unchanged."""
    try:
        import ctypes

        libc = ctypes.CDLL("libc.so.6")
        M_TRIM_THRESHOLD, M_MMAP_MAX, M_ARENA_MAX = -1, -4, -8
        ok = libc.mallopt(M_ARENA_MAX, 1) and libc.mallopt(M_MMAP_MAX, 0)
        ok = ok and libc.mallopt(M_TRIM_THRESHOLD, 1 << 30) and libc.mallopt(M_TRIM_THRESHOLD, 2**31 - 1)
        return bool(ok)
    except (OSError, AttributeError):
        return False


def run_reference(args, world, rank, local):
    """The reference's own concurrent CUDA serving path, unmodified, from baseline/_ref.

    squish.serving.scheduler.NestedWaitScheduler (the reference server's default
    ``--batch-scheduler`` algorithm, squish/server.py:5855-5872) with ``max_batch_size`` =
    the concurrency, fed through its public ``submit_sync`` iterator from one thread per
    request. On Linux its worker runs ``_generate_batch_torch`` (squish/serving/scheduler.py:
    724-800): every step forwards the whole padded batch through the HF model (no KV cache
    is reused between steps), copies the fp32 logits of every position to the host and
    samples each request's next token with numpy. The model is the HF Qwen2 architecture at
    the Qwen2.5-7B shape with random fp16 weights: the reference's INT4 torch loader
    dequantizes to fp16 before load_state_dict, so fp16 is what its CUDA path computes with.

    A step is one iteration of that loop (one token for every request in the batch). All
    requests are queued before the scheduler starts, so they form one batch, as the
    closed loop of our arm keeps ``concurrency`` requests in flight. The step boundaries are
    read from the scheduler's public ``stats()['total_tokens_gen']``; the path copies the
    logits to the host every step, so host and device are in lockstep and the wall clock
    between step boundaries is the step time.
    """
    ref_root = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "squish")):
        return {"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}
    sys.path.insert(0, ref_root)
    import numpy as np
    import torch

    try:
        from squish.serving.scheduler import NestedWaitScheduler  # the reference's public scheduler
    except Exception as exc:  # noqa: BLE001
        return {"impl": "reference", "unavailable": f"reference import failed: {exc!r}"[:200]}
    from transformers import AutoModelForCausalLM, Qwen2Config

    C = args.concurrency
    V = 152064
    # the padded length of the last step inside the window
    L_max = args.prompt_max + args.warmup + args.steps + 2
    logits_host = C * L_max * V * 4  # fp32 logits of every position, copied to the host each step
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    host_need = 2 * logits_host + (8 << 30)  # the previous step's array is alive while the next is copied
    host_avail = int(0.92 * host_memory_available()) // max(1, local_world)
    free_dev, _ = torch.cuda.mem_get_info()
    # fp16 weights, the KV the HF forward returns, and at the peak either two fp16 logit
    # tensors (the previous step's output is alive during the forward) plus activations, or
    # the fp16 logits plus their fp32 copy; 10 % margin
    tokens = C * L_max
    kv = tokens * 28 * 2 * 512 * 2
    peak = max(2 * tokens * V * 2 + tokens * 18944 * 2 * 3, tokens * V * (2 + 4))
    dev_need = 1.1 * (15.3e9 + kv + peak)
    why = None
    if host_need > host_avail:
        why = (f"host memory: the stock path copies {C}x{L_max}x{V} fp32 logits to the host every step "
               f"({host_need / 1e9:.0f} GB peak per process), {host_avail / 1e9:.0f} GB available per process")
    elif dev_need > free_dev:
        why = f"device memory: {dev_need / 1e9:.0f} GB needed per step, {free_dev / 1e9:.0f} GB free"
    bad, = reduce([0.0 if why is None else 1.0], "max", world)  # every rank takes the same path
    if bad:
        return {"impl": "reference", "unavailable": why or "another rank lacks the memory for the stock path"}
    malloc_tuned = keep_host_pages()

    cfg = Qwen2Config(vocab_size=V, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                      num_attention_heads=28, num_key_value_heads=4, max_position_embeddings=32768,
                      rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=False, initializer_range=0.02)
    torch.manual_seed(args.seed)
    with torch.device("cuda"):
        model = AutoModelForCausalLM.from_config(cfg, dtype=torch.float16)
    model.eval()

    class TokenIdTokenizer:
        """Prompts are random token ids written as text: encode parses them back.

        ``eos_token_id`` is an id the model cannot produce, so every request runs to
        ``max_tokens``, as ``ignore_eos`` does in our arm."""

        eos_token_id = 1 << 30
        pad_token_id = 1  # nonzero: the scheduler takes `pad_token_id or eos_token_id or 0` as its pad id

        def encode(self, text, add_special_tokens=True):
            return [int(t) for t in text.split()]

        def __call__(self, text):
            return {"input_ids": self.encode(text)}

        def decode(self, ids, skip_special_tokens=True, **kw):
            return " ".join(str(int(i)) for i in ids)

    tok = TokenIdTokenizer()
    # the scheduler pads every row of the batch with this id and feeds it to the embedding:
    # it must be a token of the vocabulary (the EOS id above never is, on purpose)
    pad = tok.pad_token_id or tok.eos_token_id or 0
    if not 0 <= pad < V:
        return {"impl": "reference", "unavailable": f"pad id {pad} outside the vocabulary"}
    rng = np.random.default_rng(1000 + args.seed + rank)

    def prompt_text(n):
        return " ".join(str(int(t)) for t in rng.integers(0, V, n))

    def drain(gen, ttfts, out):
        t_sub = time.perf_counter()
        first = True
        try:
            for _text, fin in gen:
                if first:
                    ttfts.append((time.perf_counter() - t_sub) * 1000)
                    first = False
                if fin is not None:
                    out.append(fin)
                    break
        except Exception as exc:  # noqa: BLE001
            out.append(f"error: {exc!r}")

    # warm-up: one full-length request through the same path, so no cold first token or
    # cold kernel selection lands in the measured batch
    warm = NestedWaitScheduler(model, tok, max_batch_size=C, batch_window_ms=20.0, max_pending=0).start()
    drain(warm.submit_sync(prompt_text(args.prompt_max), max_tokens=4, temperature=0.0, top_p=1.0), [], [])
    warm.stop()
    torch.cuda.synchronize()

    sched = NestedWaitScheduler(model, tok, max_batch_size=C, batch_window_ms=20.0, max_pending=0)
    lens = [int(rng.integers(args.prompt_min, args.prompt_max + 1)) for _ in range(C)]
    texts = [prompt_text(n) for n in lens]
    ttfts, fins = [], []
    threads = []
    for t in texts:
        gen = sched.submit_sync(t, max_tokens=args.output_len, temperature=0.0, top_p=1.0)
        th = threading.Thread(target=drain, args=(gen, ttfts, fins), daemon=True)
        th.start()
        threads.append(th)
    deadline = time.time() + 120
    while sched.stats()["pending_queue"] < C and time.time() < deadline:
        time.sleep(0.005)
    barrier(world)
    sched.start()  # every request is queued: the scheduler forms one batch of C

    def wait_tokens(target):
        while True:
            if sched.stats()["total_tokens_gen"] >= target or fins:
                return time.perf_counter()
            time.sleep(0.0005)

    # The stock path re-forwards the whole padded batch every step (tens of seconds a step at
    # this config), so the window is sized to a time budget: min(W, 3) warm-up steps, then as
    # many of the K requested steps as fit in --ref-budget-s (at least 3). The JSON reports the
    # counts it ran.
    warm = min(args.warmup, 3)
    t_start = time.perf_counter()
    wait_tokens(C * warm)
    per_step, = reduce([(time.perf_counter() - t_start) / max(warm, 1)], "max", world)
    steps = min(args.steps, max(3, int(args.ref_budget_s / max(per_step, 1e-3))))
    clocks = ClockSampler(local, args.clocks != "0")
    clocks.start()
    w0 = time.perf_counter()
    wait_tokens(C * (warm + steps))
    wall = time.perf_counter() - w0
    clk = clocks.stop()
    failed = [f for f in fins if f not in ("length", "stop")]
    bad, = reduce([1.0 if failed else 0.0], "max", world)
    if bad:
        return {"impl": "reference", "unavailable": (f"reference batch ended early: {failed[0]}" if failed else
                                                     "the reference batch ended early on another rank")[:200]}
    tokens = C * steps
    tot, = reduce([tokens], "sum", world)
    mx, = reduce([wall], "max", world)
    all_ttft = gather_list(ttfts, world)
    return {"metric": METRIC, "value": tot / mx, "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": warm, "steps_requested": args.steps, "warmup_requested": args.warmup,
            "ms_per_step": mx * 1000 / steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic: random-init N(0,0.02) weights, random token-id prompts",
            "config": {"model": MODEL_DESC, "global_batch": C * world,
                       "seq_len": f"prompt U[{args.prompt_min},{args.prompt_max}] + {args.output_len} out",
                       "parallelism": f"dp{world}", "concurrency_per_gpu": C,
                       "l2": "no flush: fp16 weights (15 GB) and the padded batch exceed the 126 MB L2 every step",
                       "weights": "fp16 (the reference's INT4 torch loader dequantizes to fp16 before loading)",
                       "path": "squish.serving.scheduler.NestedWaitScheduler.submit_sync -> _generate_batch_torch "
                               "(HF Qwen2ForCausalLM forward of the padded batch every step)"},
            "ttft_ms": {"p50": pct(all_ttft, 50), "p99": pct(all_ttft, 99), "n": len(all_ttft),
                        "source": "every request of the measured batch (submitted together)"},
            "e2e": {"value": tot / mx, "unit": "tokens/s",
                    "h2d_bytes_per_step": C * (max(lens) + warm + steps // 2) * 8,
                    "d2h_bytes_per_step": C * (max(lens) + warm + steps // 2) * V * 4,
                    "api": "NestedWaitScheduler.submit_sync (tokens counted as the iterators yield them)"},
            "timing": "wall clock between step boundaries: the path copies the logits to the host every step, "
                      "so host and device run in lockstep",
            "padded_len": [max(lens) + warm, max(lens) + warm + steps],
            "window": f"{warm} warm-up + {steps} timed steps: the steps of ~{per_step:.0f} s that fit in "
                      f"--ref-budget-s {args.ref_budget_s:.0f}",
            "host_allocator": "glibc: one arena, no mmap, no trim (freed logit pages reused)" if malloc_tuned
            else "default",
            "clocks": clk,
            "impl": "reference"}


def main():
    args = parse()
    if args.impl == "reference":
        # The stock path allocates the fp32 copy of every position's logits (tens of GB) right
        # after a forward whose activations were just freed; without expandable segments the
        # caching allocator cannot place it in the freed (fragmented) space. Allocator setting
        # only: the reference's code runs unchanged.
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
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
