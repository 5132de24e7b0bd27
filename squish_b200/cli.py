"""``squish`` command line (the reference's verbs, squish/cli.py:6715-6975).

    squish serve MODEL       OpenAI + Ollama + LocalAI HTTP server
    squish run MODEL [TEXT]  one-shot generation when TEXT is given, else serve
    squish compress SRC      HF safetensors (or --random-init PRESET) -> npy-dir
    squish convert SRC DST   between npy-dir / squizd
    squish models            local checkpoints and built-in presets
    squish catalog           presets with their sizes
    squish pull NAME         (offline) materialise a preset as a random-init checkpoint
    squish bench MODEL       closed-loop serving load (tok/s, TTFT p50/p99)
    squish doctor            GPU, extension and interconnect checks
    squish config ...        get / set / show / reset / path of ~/.squish/config.json
    squish daemon ...        start / stop / status / ping / reload the UDS daemon
    squish chat | info | search | rm | ps | logs | trace | quality | route | export | eval | push
                             (cli_verbs.py)
    squish version

MODEL is a checkpoint path or a preset name (random-init weights of that architecture).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

from . import config as ucfg

__version__ = "0.1.0"


def _engine_args(p: argparse.ArgumentParser) -> None:
    e = ucfg.load()["engine"]
    p.add_argument("model", nargs="?", default=None, help="checkpoint path or preset name")
    p.add_argument("--device", default=None)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--kv-dtype", "--kv-bits", dest="kv_dtype", default=None,
                   choices=["bf16", "fp16", "int8", "int4", "int2", "k8v4", "auto"],
                   help="auto: INT8 up to 8K-token contexts, INT4 to 16K, INT2 beyond (by --max-model-len)")
    p.add_argument("--max-num-seqs", "--batch-size", dest="max_num_seqs", type=int, default=e["max_num_seqs"])
    p.add_argument("--max-num-batched-tokens", "--chunk-prefill-size", dest="max_num_batched_tokens", type=int,
                   default=e["max_num_batched_tokens"])
    p.add_argument("--max-model-len", "--max-kv-size", dest="max_model_len", type=int, default=e["max_model_len"])
    p.add_argument("--gpu-memory-utilization", type=float, default=e["gpu_memory_utilization"])
    p.add_argument("--no-cuda-graphs", action="store_true")
    p.add_argument("--no-prefix-caching", "--no-block-kv-cache", dest="no_prefix_caching", action="store_true")
    p.add_argument("--chunk-align", type=int, default=0, help="grid-aligned prefill chunks (bit-exact prefix reuse)")
    p.add_argument("--kv-host-gb", type=float, default=0.0, help="host-RAM tier for evicted prefix blocks")
    p.add_argument("--kv-disk-dir", default=None, help="disk tier (persists prefix blocks across restarts)")
    p.add_argument("--compress-prompt", action="store_true", help="extractive compression of long user messages")
    p.add_argument("--compress-ratio", type=float, default=0.5)
    p.add_argument("--compress-min-tokens", type=int, default=256)
    p.add_argument("--compress-preserve-tokens", type=int, default=0)
    p.add_argument("--page-size", type=int, default=None, help="KV page size in tokens (a multiple of 16)")
    p.add_argument("--prompt-logit-cache", type=int, default=64,
                   help="keep the last logits of this many recent prompts: a repeated prompt's first token "
                        "needs no forward pass (0 = off)")
    p.add_argument("--kv-sink-tokens", type=int, default=0, help="attention sinks kept with --kv-window-tokens")
    p.add_argument("--kv-window-tokens", type=int, default=0,
                   help="> 0: attend to the sink pages and the most recent N tokens only; older KV pages are freed")
    p.add_argument("--kv-h2o-budget", type=int, default=0,
                   help="> 0: heavy-hitter eviction keeps at most N tokens per sequence (least-attended pages go)")
    p.add_argument("--kv-h2o-interval", type=int, default=4, help="decode steps between attention-mass refreshes")
    p.add_argument("--kv-h2o-decay", type=float, default=1.0,
                   help="score decay per refresh (1 = accumulated H2O scores; < 1 favours recent queries)")
    p.add_argument("--kv-budget-adaptive", action="store_true",
                   help="share the page pool among running sequences: heavy-hitter budgets shrink under pressure")
    # speculative decoding (the reference serves with prompt lookup on: squish/server.py:5194)
    sp = ucfg.load()["speculative"]
    p.add_argument("--prompt-lookup", dest="prompt_lookup", action="store_true", default=bool(sp["prompt_lookup"]),
                   help="greedy-lossless n-gram drafts from the request's own tokens (default on)")
    p.add_argument("--no-prompt-lookup", dest="prompt_lookup", action="store_false")
    p.add_argument("--prompt-lookup-n", type=int, default=int(sp["prompt_lookup_n"]), help="longest n-gram matched")
    p.add_argument("--prompt-lookup-k", type=int, default=int(sp["prompt_lookup_k"]), help="draft tokens per round")
    p.add_argument("--draft-model", default=sp["draft_model"] or None,
                   help="draft model (checkpoint or preset of the same vocabulary) for draft/verify decoding")
    p.add_argument("--draft-depth", type=int, default=int(sp["draft_depth"]), help="draft tokens per round")
    p.add_argument("--jacobi", action="store_true", help="Jacobi (fixed-point) parallel decoding")
    p.add_argument("--medusa-heads", default=None,
                   help="Medusa head file or directory (medusa_head.{i}.* tensors): tree drafts from extra heads "
                        "on the final hidden state")
    p.add_argument("--medusa-top-k", type=int, default=4, help="Medusa: candidates per head")
    p.add_argument("--redrafter-head", default=None,
                   help="recurrent drafter file or directory (gru.* / proj.* tensors): GRU drafts from the target's features")
    p.add_argument("--eagle-head", default=None,
                   help="EAGLE draft head file or directory (fc / layers.0.* tensors): drafts from a one-layer "
                        "model over the target's features")
    p.add_argument("--spec-branches", type=int, default=1, help="prompt lookup: continuations per draft tree")
    # multi-GPU
    p.add_argument("--tp", type=int, default=1, help="tensor-parallel GPUs (one process per GPU over NVLink)")
    p.add_argument("--offload-layers", type=int, default=0,
                   help="keep the last N layers' weights in host memory, streamed to the GPU each step")
    p.add_argument("--pp", type=int, default=1,
                   help="split the layers over this many GPUs of one process (layer-split fallback)")
    p.add_argument("--ep", type=int, default=0,
                   help="expert-parallel GPUs for MoE models (experts split over ranks; sets --tp)")
    p.add_argument("--dp", type=int, default=1, help="data-parallel replicas (one per GPU) behind a request router")
    p.add_argument("--gpus", type=int, default=0, help="GPUs to use: tp x dp (dp = gpus / tp when --dp is not given)")
    p.add_argument("--tp-mode", default="nvlink", choices=["nvlink", "sp", "nccl"],
                   help="nvlink: fused GEMM + all-reduce over peer memory; sp: sequence parallel (fused GEMM -> "
                        "reduce-scatter, RMSNorm + all-gather, gather-waiting GEMM; MoE layers use the expert "
                        "all-to-all over peer memory); nccl: NCCL")
    p.add_argument("--log-level", default="warning", choices=["debug", "info", "warning", "error", "critical"])
    p.add_argument("--log-format", default="text", choices=["text", "json"], help="json: one JSON object per line")


def _spec(a):
    """SpecConfig from the flags: a draft model wins over an EAGLE head, then Medusa heads, then
    Jacobi, then prompt lookup."""
    from .engine.speculative import SpecConfig

    if getattr(a, "draft_model", None):
        return SpecConfig(method="draft", k=a.draft_depth, draft_model=a.draft_model)
    if getattr(a, "redrafter_head", None):
        return SpecConfig(method="redrafter", k=a.draft_depth, redrafter_head=a.redrafter_head)
    if getattr(a, "eagle_head", None):
        return SpecConfig(method="eagle", k=a.draft_depth, eagle_head=a.eagle_head)
    if getattr(a, "medusa_heads", None):
        return SpecConfig(method="medusa", k=a.draft_depth, medusa_heads=a.medusa_heads,
                          medusa_top_k=getattr(a, "medusa_top_k", 4))
    if getattr(a, "jacobi", False):
        return SpecConfig(method="jacobi", k=a.draft_depth)
    if getattr(a, "prompt_lookup", False):
        return SpecConfig(method="prompt_lookup", k=a.prompt_lookup_k, ngram_max=a.prompt_lookup_n,
                          branches=max(1, a.spec_branches))
    return None


def _parallel(a) -> tuple[int, int]:
    """(tp, dp) from --tp / --ep / --dp / --gpus."""
    tp = max(1, getattr(a, "tp", 1), getattr(a, "ep", 0) or 1)
    dp = max(1, getattr(a, "dp", 1))
    gpus = getattr(a, "gpus", 0) or 0
    if gpus:
        if gpus % tp:
            raise SystemExit(f"--gpus {gpus} is not a multiple of --tp {tp}")
        if dp == 1:
            dp = gpus // tp
        elif dp * tp != gpus:
            raise SystemExit(f"--gpus {gpus} != --tp {tp} x --dp {dp}")
    return tp, dp


def _ecfg(a):
    from .engine.engine import EngineConfig

    tp, _ = _parallel(a)
    return EngineConfig(max_num_seqs=a.max_num_seqs, max_num_batched_tokens=a.max_num_batched_tokens,
                        max_model_len=a.max_model_len, gpu_memory_utilization=a.gpu_memory_utilization,
                        enable_prefix_caching=not a.no_prefix_caching, cuda_graphs=not a.no_cuda_graphs,
                        chunk_align=a.chunk_align, seed=a.seed, kv_host_bytes=int(a.kv_host_gb * (1 << 30)),
                        kv_disk_dir=a.kv_disk_dir, spec=_spec(a), tp=tp, tp_mode=getattr(a, "tp_mode", "nvlink"),
                        prompt_logit_cache=a.prompt_logit_cache, kv_sink_tokens=a.kv_sink_tokens,
                        kv_window_tokens=a.kv_window_tokens, pp=a.pp, offload_layers=a.offload_layers,
                        kv_h2o_budget=getattr(a, "kv_h2o_budget", 0), kv_h2o_interval=getattr(a, "kv_h2o_interval", 4),
                        kv_h2o_decay=getattr(a, "kv_h2o_decay", 1.0),
                        kv_budget_adaptive=getattr(a, "kv_budget_adaptive", False))


def _kv(a):
    if a.kv_dtype == "auto":
        from .kv.planning import auto_kv_mode

        return auto_kv_mode(a.max_model_len)
    return {"fp16": "bf16"}.get(a.kv_dtype, a.kv_dtype)


def _model(a) -> str:
    return a.model or ucfg.get("model.default")


def _logging(a, log_file=None) -> None:
    from .utils.logconfig import configure_logging

    configure_logging(getattr(a, "log_level", "warning"), json_format=getattr(a, "log_format", "text") == "json",
                      log_file=log_file)


def _relaunch_ranks(tp: int) -> int:
    """Start the tensor-parallel ranks: this command again under torch.distributed.run, one
    process per GPU (rank 0 serves HTTP, the others follow its steps)."""
    import socket
    import subprocess

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "squish_b200", *sys.argv[1:]]
    return subprocess.call(cmd)


def _tp_rank_setup(a, tp: int):
    """Join the process group of a tensor-parallel server; returns (rank, device string)."""
    import datetime

    import torch
    import torch.distributed as dist

    rank, local = int(os.environ["RANK"]), int(os.environ.get("LOCAL_RANK", "0"))
    if int(os.environ.get("WORLD_SIZE", "1")) != tp:
        raise SystemExit(f"WORLD_SIZE {os.environ.get('WORLD_SIZE')} != --tp {tp}")
    if torch.cuda.is_available() and (a.device or "cuda").startswith("cuda"):
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        return rank, f"cuda:{local}"
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    return rank, "cpu"


def _build_frontend(a, max_pending: int):
    """Load the model(s) and return (front-end engine, Loaded of replica 0, follower or None).
    One GPU: an AsyncEngine. --dp N: N replicas (cuda:0..N-1) behind a DPRouter. --tp N:
    this process is one rank; rank 0 gets a TPAsyncEngine, the others a follower callable."""
    from .api import load_engine
    from .serving.async_engine import AsyncEngine

    tp, dp = _parallel(a)
    if tp > 1 and dp > 1:
        raise SystemExit("--tp and --dp together are not supported: use one of them")
    if tp > 1:
        from .serving.multi import TPAsyncEngine, TPControl, follow

        rank, dev = _tp_rank_setup(a, tp)
        loaded = load_engine(_model(a), dev, seed=a.seed, kv_dtype=_kv(a), ecfg=_ecfg(a), page_size=a.page_size)
        ctrl = TPControl()
        if rank != 0:
            return None, loaded, lambda: follow(loaded.engine, ctrl)
        aeng = TPAsyncEngine(loaded.engine, ctrl, loaded.tokenizer, max_pending=max_pending, model_name=loaded.name)
        return aeng.start(), loaded, None
    if dp > 1:
        import torch

        from .serving.multi import DPRouter

        base = a.device or ("cuda" if torch.cuda.is_available() else "cpu")
        reps, first = [], None
        for i in range(dp):
            dev = f"cuda:{i}" if base.startswith("cuda") else base
            ld = load_engine(_model(a), dev, seed=a.seed, kv_dtype=_kv(a), ecfg=_ecfg(a), page_size=a.page_size)
            ld.engine.warmup_graphs()  # decode graphs captured before the first request
            first = first or ld
            reps.append(AsyncEngine(ld.engine, ld.tokenizer, max_pending=max_pending, model_name=ld.name))
        return DPRouter(reps, max_pending=max_pending).start(), first, None
    loaded = load_engine(_model(a), a.device, seed=a.seed, kv_dtype=_kv(a), ecfg=_ecfg(a), page_size=a.page_size)
    loaded.engine.warmup_graphs()
    return AsyncEngine(loaded.engine, loaded.tokenizer, max_pending=max_pending, model_name=loaded.name).start(), \
        loaded, None


def cmd_serve(a) -> int:
    import uvicorn

    from .serving.server import ServerState, create_app

    from .cli_verbs import log_path

    _logging(a, log_file=log_path() if os.environ.get("RANK", "0") == "0" else None)
    tp, _ = _parallel(a)
    if tp > 1 and "RANK" not in os.environ:
        return _relaunch_ranks(tp)
    c = ucfg.load()["server"]
    aeng, loaded, follower = _build_frontend(a, c["max_pending"])
    if follower is not None:
        follower()
        return 0
    key = a.api_key if a.api_key is not None else os.environ.get("SQUISH_API_KEY", c["api_key"])
    cp = ({"ratio": a.compress_ratio, "min_tokens": a.compress_min_tokens,
           "preserve_tokens": a.compress_preserve_tokens} if getattr(a, "compress_prompt", False) else None)
    st = ServerState(aeng, loaded.name, api_key=key or None, arch=loaded.engine.cfg.arch, load_time_s=loaded.load_s,
                     compress_prompt=cp)
    print(f"squish: {loaded.name} loaded in {loaded.load_s:.1f}s; listening on http://{a.host or c['host']}:"
          f"{a.port or c['port']}", file=sys.stderr)
    try:
        uvicorn.run(create_app(st), host=a.host or c["host"], port=a.port or c["port"], log_level="warning")
    finally:
        aeng.stop()
    return 0


def cmd_run(a) -> int:
    if not a.text:
        return cmd_serve(a)
    from .api import LLM
    from .engine.sampling import SamplingParams
    from .serving.chat_template import apply_chat_template

    _logging(a)
    llm = LLM(_model(a), a.device, seed=a.seed, kv_dtype=_kv(a), ecfg=_ecfg(a), page_size=a.page_size)
    prompt = apply_chat_template([{"role": "user", "content": " ".join(a.text)}], llm.tokenizer,
                                 arch=llm.engine.cfg.arch)
    p = SamplingParams(max_tokens=a.max_tokens, temperature=a.temperature, top_p=a.top_p,
                       stop_token_ids=[llm.engine.cfg.eos_token_id])
    out = llm.generate([prompt], p)[0]
    print(out["text"])
    return 0


def cmd_compress(a) -> int:
    from .io.convert import compress

    kind = {"int4": "q4a", "int8": "q8", "fp8": "fp8", "nf4": "nf4", "int3": "q3", "int2": "q2", "sqint2": "sqint2",
            "mixed": "mixed", "aqlm": "aqlm", "any4": "any4", "quarot": "quarot",
            "none": "dense"}[a.format]
    out = a.output or (str(Path(a.source).with_name(Path(a.source).name + "-squished")) if a.source else
                       str(ucfg.squish_home() / "models" / a.random_init))
    st = compress(a.source, out, kind=kind, group_size=a.group_size, mse_clip=a.mse, device=a.device,
                  delete_source=a.delete_source, random_preset=a.random_init, seed=a.seed, kv_dtype=a.kv_dtype,
                  hqq=getattr(a, "hqq", False), awq=getattr(a, "awq", False),
                  awq_scales=getattr(a, "awq_scales", None), awq_alpha=getattr(a, "awq_alpha", 0.5),
                  awq_samples=getattr(a, "awq_samples", 16), gptq=getattr(a, "gptq", False),
                  df11=getattr(a, "df11", False))
    print(json.dumps({"output": out, **st}))
    return 0


def cmd_merge_model(a) -> int:
    from .quant.merge import merge_adapter_files

    paths = []
    for spec in a.adapters:  # "domain:path" (the domain is a label) or a bare path
        d, _, p = spec.partition(":")
        path = p if p and not Path(spec).exists() else spec
        if not Path(path).expanduser().exists():
            print(f"adapter path not found: {path}", file=sys.stderr)
            return 2
        paths.append(str(Path(path).expanduser()))
    out = merge_adapter_files(paths, str(Path(a.output_path).expanduser()), a.method)
    print(json.dumps(out))
    return 0


def cmd_convert(a) -> int:
    from .io.convert import load_checkpoint
    from .io.npy_dir import write_npy_dir
    from .io.squizd import write_squizd

    ck, _ = load_checkpoint(a.source, "cpu")
    if a.to == "squizd":
        write_squizd(a.dest, ck, group=a.group_size)
    else:
        write_npy_dir(a.dest, ck)
    print(json.dumps({"output": a.dest, "format": a.to, "tensors": len(ck.tensors)}))
    return 0


def _local_models() -> list[dict]:
    import dataclasses

    from .serving.model_scanner import LocalModelScanner

    extra = ucfg.get("model.models_dir")
    sc = LocalModelScanner(extra_dirs=[Path(extra)] if extra else [])
    return [dataclasses.asdict(m) for m in sc.find_all()]


def cmd_scan(a) -> int:
    from .serving.model_scanner import scan_before_load

    r = scan_before_load(a.path)
    print(json.dumps({"status": r.status, "scanned": r.scanned, "findings": r.findings}, indent=2))
    return 0 if r.status == "clean" else 1


def _catalog() -> list[dict]:
    from .models.config import PRESETS

    rows = []
    for name, (c, q) in sorted(PRESETS.items()):
        rows.append({"name": name, "arch": c.arch, "layers": c.num_layers, "hidden": c.hidden_size,
                     "params_b": round(c.num_params() / 1e9, 2) if hasattr(c, "num_params") else None,
                     "weights": f"int{q.weight_bits} g{q.group_size}", "kv": q.kv_dtype})
    return rows


def cmd_models(a) -> int:
    print(json.dumps({"local": _local_models(), "presets": [r["name"] for r in _catalog()]}, indent=2))
    return 0


def cmd_catalog(a) -> int:
    import dataclasses

    from . import catalog

    es = catalog.search(a.search) if getattr(a, "search", None) else catalog.list_catalog(getattr(a, "tag", None))
    print(json.dumps({"catalog": [dataclasses.asdict(e) for e in es], "presets": _catalog()}, indent=2))
    return 0


def cmd_pull(a) -> int:
    """Materialize a catalog model: from a local checkpoint directory (``--from``: compressed
    to INT4), else as random weights of its architecture preset (no network access here)."""
    from . import catalog
    from .models.config import PRESETS

    e = catalog.resolve(a.name)
    src = getattr(a, "source_dir", None)
    if e is None and not src and a.name.lower() in PRESETS:  # a preset name outside the catalog
        a.source, a.random_init, a.output = None, a.name.lower(), None
        a.format, a.mse, a.delete_source, a.kv_dtype = "int4", False, False, "int4"
        a.group_size = PRESETS[a.name.lower()][1].group_size
        return cmd_compress(a)
    if e is None and not src:
        near = [x.id for x in catalog.suggest(a.name)]
        print(f"squish pull: {a.name!r} is not in the catalog" + (f"; did you mean {', '.join(near)}?" if near else ""),
              file=sys.stderr)
        return 2
    preset = e.preset if e is not None else None
    if src:
        a.source, a.random_init = src, None
    elif preset in PRESETS:
        a.source, a.random_init = None, preset
    else:
        print(f"squish pull: no network access here; download {e.hf_repo} elsewhere and run "
              f"'squish pull {a.name} --from <dir>'", file=sys.stderr)
        return 2
    a.output = None if not src else str(ucfg.squish_home() / "models" / (e.id.replace(":", "-") if e else Path(src).name))
    a.format, a.mse, a.delete_source, a.kv_dtype = "int4", False, False, "int4"
    a.group_size = PRESETS[preset][1].group_size if preset in PRESETS else 64
    return cmd_compress(a)


def cmd_bench(a) -> int:
    import torch

    from .api import load_engine
    from .utils.loadgen import run_load

    loaded = load_engine(_model(a), a.device, seed=a.seed, kv_dtype=_kv(a), ecfg=_ecfg(a), page_size=a.page_size)
    sync = torch.cuda.synchronize if torch.cuda.is_available() and loaded.engine.runner.__class__.__name__ == \
        "CudaRunner" else None
    rows = []
    for c in a.concurrency:
        rows.append(run_load(loaded.engine, num_requests=max(a.requests, c), concurrency=c, prompt_min=a.prompt_min,
                             prompt_max=a.prompt_max, max_tokens=a.max_tokens, seed=a.seed, sync=sync))
        print(json.dumps({"model": loaded.name, **rows[-1]}), flush=True)
    return 0


def nvlink_topology(nvml=None) -> list[dict] | None:
    """Per GPU: NVLink links up and the NVML P2P status toward every other GPU (read-only NVML
    queries; None when NVML is unavailable). ``nvml`` is the pynvml module (a stand-in in tests)."""
    if nvml is None:
        try:
            import pynvml as nvml
        except ImportError:
            return None
    try:
        nvml.nvmlInit()
    except Exception:  # noqa: BLE001 - no driver: nothing to report
        return None
    try:
        n = nvml.nvmlDeviceGetCount()
        hs = [nvml.nvmlDeviceGetHandleByIndex(i) for i in range(n)]
        out = []
        for i, h in enumerate(hs):
            links = 0
            for ln in range(getattr(nvml, "NVML_NVLINK_MAX_LINKS", 18)):
                try:
                    links += int(nvml.nvmlDeviceGetNvLinkState(h, ln) == getattr(nvml, "NVML_FEATURE_ENABLED", 1))
                except Exception:  # noqa: BLE001 - link index past this GPU's links
                    break
            p2p = {}
            for j, hj in enumerate(hs):
                if j == i:
                    continue
                try:
                    st = nvml.nvmlDeviceGetP2PStatus(h, hj, getattr(nvml, "NVML_P2P_CAPS_INDEX_NVLINK", 3))
                    p2p[j] = st == getattr(nvml, "NVML_P2P_STATUS_OK", 0)
                except Exception:  # noqa: BLE001
                    p2p[j] = None
            out.append({"index": i, "nvlinks_up": links, "nvlink_p2p": p2p})
        return out
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass


def doctor_report() -> dict:
    import torch

    rep: dict = {"python": sys.version.split()[0], "torch": torch.__version__, "cuda_available":
                 torch.cuda.is_available(), "squish_home": str(ucfg.squish_home())}
    try:
        from ._ext import native

        native()
        rep["extension"] = "loaded"
    except Exception as exc:  # noqa: BLE001 - report, do not raise
        rep["extension"] = f"missing: {exc}"
    if torch.cuda.is_available():
        n = torch.cuda.device_count()
        gpus = []
        for i in range(n):
            p = torch.cuda.get_device_properties(i)
            gpus.append({"index": i, "name": p.name, "sm": f"{p.major}.{p.minor}", "sms": p.multi_processor_count,
                         "memory_gb": round(p.total_memory / 2**30, 1), "sm_100a": (p.major, p.minor) == (10, 0)})
        rep["gpus"] = gpus
        if n > 1:
            rep["peer_access"] = all(torch.cuda.can_device_access_peer(0, j) for j in range(1, n))
        rep["nvlink"] = nvlink_topology()
        try:
            rep["nccl"] = ".".join(map(str, torch.cuda.nccl.version()))
        except (AttributeError, RuntimeError):
            rep["nccl"] = None
    return rep


def cmd_doctor(a) -> int:
    rep = doctor_report()
    print(json.dumps(rep, indent=2))
    return 0 if rep.get("extension") == "loaded" else 1


def cmd_config(a) -> int:
    if a.action == "show":
        print(json.dumps(ucfg.load(), indent=2, sort_keys=True))
    elif a.action == "path":
        print(ucfg.config_path())
    elif a.action == "get":
        v = ucfg.get(a.key)
        if v is None:
            print(f"unknown key {a.key}", file=sys.stderr)
            return 1
        print(json.dumps(v))
    elif a.action == "set":
        ucfg.set_value(a.key, a.value)
        print(json.dumps(ucfg.get(a.key)))
    elif a.action == "reset":
        ucfg.reset()
    return 0


def cmd_daemon(a) -> int:
    from . import daemon as d

    if a.action == "start":
        if d.is_running():
            print("squishd already running", file=sys.stderr)
            return 1
        print(f"squishd listening on {d.sock_path()}", file=sys.stderr)
        d.Daemon(default_model=_model(a)).serve_forever()
        return 0
    if not d.is_running():
        print("squishd is not running", file=sys.stderr)
        return 1
    cmd = {"status": "status", "ping": "ping", "stop": "stop", "reload": "reload"}[a.action]
    req = {"_cmd": cmd}
    if a.model:
        req["model"] = a.model
    print(json.dumps(d.request(req), indent=2))
    return 0


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="squish", description="B200-native quantized LLM inference server")
    ap.add_argument("--version", action="version", version=f"squish-b200 {__version__}")
    sub = ap.add_subparsers(dest="cmd")

    for name in ("serve", "run"):
        p = sub.add_parser(name)
        _engine_args(p)
        p.add_argument("--host", default=None)
        p.add_argument("--port", type=int, default=None)
        p.add_argument("--api-key", default=None)
        if name == "run":
            p.add_argument("text", nargs="*")
            p.add_argument("--max-tokens", type=int, default=256)
            p.add_argument("--temperature", type=float, default=0.0)
            p.add_argument("--top-p", type=float, default=1.0)
        p.set_defaults(fn=cmd_serve if name == "serve" else cmd_run)

    p = sub.add_parser("compress")
    p.add_argument("source", nargs="?", default=None)
    p.add_argument("-o", "--output", default=None)
    p.add_argument("--format", default="int4",
                   choices=["int4", "int8", "fp8", "nf4", "any4", "quarot", "int3", "int2", "sqint2", "mixed", "aqlm",
                            "none"],
                   help="mixed: INT4 boundary layers, INT3 attention, SQINT2 gate/up, INT4 elsewhere; any4: NF4 codes "
                        "with a learned 16-level table per tensor; quarot: INT4 of the block-Hadamard rotated weight")
    p.add_argument("--group-size", type=int, default=64)
    p.add_argument("--mse", action="store_true", help="MSE-optimal clipping search (INT4)")
    p.add_argument("--random-init", default=None, metavar="PRESET")
    p.add_argument("--delete-source", action="store_true")
    p.add_argument("--device", default=None)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--kv-dtype", default="int4")
    p.add_argument("--hqq", action="store_true", help="half-quadratic refinement of INT4 / INT2 grids")
    p.add_argument("--awq", action="store_true", help="activation-aware scaling (calibrates on the fp32 model)")
    p.add_argument("--awq-scales", default=None, metavar="DIR", help="apply saved AWQ scales instead")
    p.add_argument("--awq-alpha", type=float, default=0.5)
    p.add_argument("--awq-samples", type=int, default=16)
    p.add_argument("--gptq", action="store_true", help="GPTQ INT4 (calibrates on the fp32 model)")
    p.add_argument("--df11", action="store_true",
                   help="store unquantized tensors losslessly as bf16 with entropy-coded exponents (__pt_df11)")
    p.set_defaults(fn=cmd_compress)

    p = sub.add_parser("merge-model", help="merge LoRA adapters (DARE / TIES / DARE-TIES)")
    p.add_argument("base_model", nargs="?", default=None)
    p.add_argument("--adapters", nargs="+", required=True, metavar="DOMAIN:PATH")
    p.add_argument("--method", default="dare-ties", choices=["dare", "ties", "dare-ties"])
    p.add_argument("--output-path", required=True)
    p.set_defaults(fn=cmd_merge_model)

    p = sub.add_parser("convert")
    p.add_argument("source")
    p.add_argument("dest")
    p.add_argument("--to", default="squizd", choices=["squizd", "npy-dir"])
    p.add_argument("--group-size", type=int, default=64)
    p.set_defaults(fn=cmd_convert)

    sub.add_parser("models").set_defaults(fn=cmd_models)
    p = sub.add_parser("scan", help="static safety scan of model files (nothing is executed)")
    p.add_argument("path")
    p.set_defaults(fn=cmd_scan)
    p = sub.add_parser("catalog", help="known models (built in + ~/.squish/catalog.json) and presets")
    p.add_argument("--search", default=None)
    p.add_argument("--tag", default=None)
    p.set_defaults(fn=cmd_catalog)
    p = sub.add_parser("pull", help="materialize a catalog model (local --from dir, or random weights of its preset)")
    p.add_argument("name")
    p.add_argument("--from", dest="source_dir", default=None, help="local HF checkpoint directory to compress")
    p.add_argument("--device", default=None)
    p.add_argument("--seed", type=int, default=0)
    p.set_defaults(fn=cmd_pull)

    p = sub.add_parser("bench")
    _engine_args(p)
    p.add_argument("--concurrency", type=int, nargs="+", default=[1, 8, 32, 64])
    p.add_argument("--requests", type=int, default=64)
    p.add_argument("--prompt-min", type=int, default=128)
    p.add_argument("--prompt-max", type=int, default=2048)
    p.add_argument("--max-tokens", type=int, default=256)
    p.set_defaults(fn=cmd_bench)

    sub.add_parser("doctor").set_defaults(fn=cmd_doctor)
    p = sub.add_parser("config")
    p.add_argument("action", choices=["show", "get", "set", "reset", "path"], nargs="?", default="show")
    p.add_argument("key", nargs="?")
    p.add_argument("value", nargs="?")
    p.set_defaults(fn=cmd_config)
    p = sub.add_parser("daemon")
    p.add_argument("action", choices=["start", "stop", "status", "ping", "reload"], nargs="?", default="status")
    p.add_argument("--model", default=None)
    p.set_defaults(fn=cmd_daemon)
    sub.add_parser("version").set_defaults(fn=lambda a: print(f"squish-b200 {__version__}") or 0)
    from .cli_verbs import add_parsers

    add_parsers(sub)
    return ap


def main(argv: list[str] | None = None) -> int:
    ap = build_parser()
    a = ap.parse_args(argv)
    if not getattr(a, "fn", None):
        ap.print_help()
        return 0
    return int(a.fn(a) or 0)


if __name__ == "__main__":
    sys.exit(main())
