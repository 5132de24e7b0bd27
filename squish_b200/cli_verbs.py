"""The ``squish`` verbs beyond serving and conversion (the reference's squish/cli.py):

  chat MODEL           interactive chat with a local model, or with a running server (--url)
  info MODEL           architecture, quantization and on-disk size of a checkpoint or preset
  search QUERY         presets and local models whose name or architecture matches
  rm NAME              delete a local model directory (asks unless --yes)
  ps                   what a running server has loaded (GET /api/ps)
  logs                 the last lines of the server log (--follow to stream)
  trace [view|reset|obs]  slowest spans, clearing them, or the observability report;
                       --chrome PATH saves Chrome trace JSON
  quality              rolling latency / error report of a running server (GET /v1/quality)
  route PROMPT         the prompt router's decision for a prompt (POST /v1/route)
  export MODEL DEST    write a checkpoint as SQUIZD or an npy-dir
  eval MODEL           perplexity of a text file (or of seeded random tokens) under the
                       model's fp32 reference forward
  push                 uploading needs network access; reports that and exits 2

Client verbs talk to ``--host``/``--port`` (the user config's server address by default).
References: squish/cli.py cmd_chat (:1990), cmd_info (:1348), cmd_search (:1320), cmd_rm
(:844), cmd_ps (:5817), cmd_logs (:5936), cmd_trace (:5981), cmd_quality (:6399), cmd_route
(:6452), cmd_export (:2260), cmd_eval (:2393), cmd_push (:981).
"""
from __future__ import annotations

import collections
import json
import math
import shutil
import sys
import time
import urllib.error
import urllib.request
from pathlib import Path

from . import config as ucfg


def log_path() -> Path:
    return ucfg.squish_home() / "logs" / "server.log"


def _base(a) -> str:
    c = ucfg.load()["server"]
    return f"http://{getattr(a, 'host', None) or c['host']}:{getattr(a, 'port', None) or c['port']}"


def _http(a, path: str, method: str = "GET", body: dict | None = None, raw: bool = False):
    data = json.dumps(body).encode() if body is not None else None
    req = urllib.request.Request(_base(a) + path, data=data, method=method,
                                 headers={"Content-Type": "application/json", "Accept": "application/json"})
    key = getattr(a, "api_key", None)
    if key:
        req.add_header("Authorization", f"Bearer {key}")
    with urllib.request.urlopen(req, timeout=getattr(a, "timeout", 10)) as r:
        out = r.read()
    return out if raw else json.loads(out or b"null")


def _no_server(a, e) -> int:
    print(f"no squish server at {_base(a)} ({e}); start one with: squish serve <model>", file=sys.stderr)
    return 1


# ----------------------------------------------------------------------------- client verbs
def cmd_ps(a) -> int:
    try:
        d = _http(a, "/api/ps")
    except (urllib.error.URLError, OSError) as e:
        return _no_server(a, e)
    models = d.get("models", [])
    if not models:
        print(f"server at {_base(a)} has no model loaded")
    for m in models:
        det = m.get("details", {})
        print(json.dumps({"name": m.get("name"), "size_gb": round(m.get("size", 0) / 1e9, 2),
                          "family": det.get("family"), "quantization": det.get("quantization_level"),
                          "expires_at": m.get("expires_at")}))
    return 0


def cmd_quality(a) -> int:
    try:
        d = _http(a, f"/v1/quality?window={a.window}")
    except (urllib.error.URLError, OSError) as e:
        return _no_server(a, e)
    print(json.dumps(d, indent=2))
    return 0


def cmd_route(a) -> int:
    try:
        d = _http(a, "/v1/route", "POST", {"prompt": " ".join(a.prompt)})
    except (urllib.error.URLError, OSError) as e:
        return _no_server(a, e)
    print(json.dumps(d, indent=2))
    return 0


def cmd_trace(a) -> int:
    try:
        if a.action == "reset":
            print(json.dumps(_http(a, "/v1/trace", "DELETE")))
            return 0
        if a.action == "obs":
            print(json.dumps(_http(a, "/v1/obs-report"), indent=2))
            return 0
        tr = _http(a, "/v1/trace")
    except (urllib.error.URLError, OSError) as e:
        return _no_server(a, e)
    if a.chrome:
        Path(a.chrome).write_text(json.dumps(tr))
        print(f"Chrome trace written to {a.chrome} (open in chrome://tracing or Perfetto)")
        return 0
    events = tr.get("traceEvents", tr if isinstance(tr, list) else [])
    spans = [e for e in events if e.get("ph") == "X"]
    spans.sort(key=lambda e: -float(e.get("dur", 0)))
    for e in spans[: a.top]:
        print(f"{float(e.get('dur', 0)) / 1000:10.3f} ms  {e.get('name')}")
    if not spans:
        print("no spans recorded (start the server with SQUISH_TRACE=1)")
    return 0


def cmd_logs(a) -> int:
    p = Path(a.file) if a.file else log_path()
    if not p.exists():
        print(f"no log file at {p}; `squish serve` writes one there", file=sys.stderr)
        return 1
    with open(p, errors="replace") as fh:
        for line in collections.deque(fh, a.lines):
            print(line, end="")
        if not a.follow:
            return 0
        try:  # pragma: no cover - interactive
            while True:
                line = fh.readline()
                if line:
                    print(line, end="", flush=True)
                else:
                    time.sleep(0.2)
        except KeyboardInterrupt:
            return 0


def cmd_push(a) -> int:
    print("squish push: this build has no network access; copy the checkpoint directory to the target host "
          "(or upload it to a model hub) with your own tools", file=sys.stderr)
    return 2


# ----------------------------------------------------------------------------- local verbs
def _model_info(model: str) -> dict:
    from .models.config import PRESETS, get_preset

    if model.lower() in PRESETS:
        cfg, q = get_preset(model)
        src = {"kind": "preset (random-init weights of the architecture)"}
    else:
        p = Path(model).expanduser()
        if not p.exists():
            raise FileNotFoundError(f"{model!r} is neither a checkpoint path nor a preset")
        from .io.convert import load_checkpoint

        ck, _ = load_checkpoint(str(p), "cpu")
        cfg, q = ck.config, ck.quant
        files = [f for f in p.rglob("*") if f.is_file()] if p.is_dir() else [p]
        kinds = collections.Counter(t.kind for t in ck.tensors.values() if hasattr(t, "kind"))
        src = {"kind": "checkpoint", "path": str(p), "files": len(files),
               "size_gb": round(sum(f.stat().st_size for f in files) / 1e9, 3), "tensor_formats": dict(kinds)}
    return {"name": cfg.name, "arch": cfg.arch, "layers": cfg.num_layers, "hidden": cfg.hidden_size,
            "heads": cfg.num_heads, "kv_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
            "ffn": cfg.intermediate_size, "vocab": cfg.vocab_size, "experts": cfg.num_experts,
            "params_b": round(cfg.num_params() / 1e9, 3),
            "weights": f"int{q.weight_bits} g{q.group_size}", "kv": f"{q.kv_dtype} g{q.kv_group}",
            "page_size": q.page_size, **src}


def cmd_info(a) -> int:
    try:
        print(json.dumps(_model_info(a.model), indent=2))
    except FileNotFoundError as e:
        print(str(e), file=sys.stderr)
        return 1
    return 0


def _local_models() -> list[dict]:
    import dataclasses

    from .serving.model_scanner import LocalModelScanner

    extra = ucfg.get("model.models_dir")
    sc = LocalModelScanner(extra_dirs=[Path(extra)] if extra else [])
    return [dataclasses.asdict(m) for m in sc.find_all()]


def cmd_search(a) -> int:
    from .models.config import PRESETS

    from . import catalog

    q = a.query.lower()
    hits = [{"name": e.id, "source": "catalog", "repo": e.hf_repo, "params": e.params, "preset": e.preset}
            for e in catalog.search(a.query)]
    hits += [{"name": n, "source": "preset", "arch": c.arch, "params_b": round(c.num_params() / 1e9, 2)}
             for n, (c, _) in sorted(PRESETS.items()) if q in n or q in c.arch]
    for m in _local_models():
        if q in json.dumps(m).lower():
            hits.append({"name": m.get("name"), "source": "local", "path": m.get("path")})
    for h in hits:
        print(json.dumps(h))
    if not hits:
        print(f"nothing matches {a.query!r}", file=sys.stderr)
        return 1
    return 0


def cmd_rm(a) -> int:
    root = ucfg.squish_home() / "models"
    p = Path(a.name).expanduser()
    if not p.is_absolute() or not p.exists():
        p = root / a.name
    p = p.resolve()
    if not p.exists():
        print(f"no local model {a.name!r} under {root}", file=sys.stderr)
        return 1
    if root.resolve() not in p.parents:
        print(f"refusing to delete {p}: it is not under {root}", file=sys.stderr)
        return 2
    if not a.yes:
        ans = input(f"delete {p}? [y/N] ").strip().lower()
        if ans not in ("y", "yes"):
            print("kept")
            return 1
    shutil.rmtree(p) if p.is_dir() else p.unlink()
    print(json.dumps({"removed": str(p)}))
    return 0


def cmd_export(a) -> int:
    from .io.convert import load_checkpoint
    from .io.npy_dir import write_npy_dir
    from .io.squizd import write_squizd

    ck, _ = load_checkpoint(a.model, "cpu")
    if a.format == "squizd":
        write_squizd(a.dest, ck, group=a.group_size)
    else:
        write_npy_dir(a.dest, ck)
    print(json.dumps({"output": a.dest, "format": a.format, "tensors": len(ck.tensors)}))
    return 0


def perplexity(model: str, tokens: list[int], window: int = 512, device: str = "cpu", seed: int = 0) -> dict:
    """Mean negative log-likelihood and perplexity of ``tokens`` under the model's fp32
    reference forward (dequantized weights, quantized KV round trip), in windows of
    ``window`` tokens (each window predicts its tokens 1.. from the ones before)."""
    import torch

    from .models.config import PRESETS, get_preset
    from .models.reference import ReferenceModel
    from .models.weights import random_checkpoint

    if model.lower() in PRESETS:
        cfg, q = get_preset(model)
        ck = random_checkpoint(cfg, q, seed=seed, device=device)
    else:
        from .io.convert import load_checkpoint

        ck, _ = load_checkpoint(model, device)
    ref = ReferenceModel(ck)
    nll, n = 0.0, 0
    with torch.no_grad():
        for s in range(0, max(len(tokens) - 1, 0), window):
            chunk = tokens[s:s + window + 1]
            if len(chunk) < 2:
                break
            logits = ref.forward(chunk[:-1], ref.new_cache(), 0).float()
            lp = torch.log_softmax(logits, -1)
            tgt = torch.tensor(chunk[1:], dtype=torch.long, device=lp.device)
            nll -= float(lp.gather(1, tgt[:, None]).sum())
            n += len(chunk) - 1
    mean = nll / max(n, 1)
    return {"tokens": n, "nll": mean, "perplexity": math.exp(min(mean, 700.0))}


def cmd_eval(a) -> int:
    import numpy as np

    if a.text:
        from .api import load_engine  # noqa: F401  (tokenizer loading mirrors serving)
        from .serving.tokenizer import load_tokenizer

        tok_dir = a.model if Path(a.model).is_dir() else None
        info = _model_info(a.model)
        tok = load_tokenizer(tok_dir, vocab_size=info["vocab"], eos_token_id=None)
        tokens = tok.encode(Path(a.text).read_text())[: a.max_tokens]
    else:
        info = _model_info(a.model)
        tokens = np.random.default_rng(a.seed).integers(0, info["vocab"], a.max_tokens).tolist()
    out = perplexity(a.model, tokens, window=a.window, device=a.device or "cpu", seed=a.seed)
    print(json.dumps({"model": info["name"], "source": a.text or f"{a.max_tokens} random tokens", **out}))
    return 0


# ----------------------------------------------------------------------------- chat
def _chat_remote(a) -> int:
    history = []
    print(f"chatting with {_base(a)} (empty line or Ctrl-D to quit)", file=sys.stderr)
    for line in sys.stdin:
        line = line.rstrip("\n")
        if not line:
            break
        history.append({"role": "user", "content": line})
        try:
            d = _http(a, "/v1/chat/completions", "POST", {"model": "default", "messages": history,
                                                          "max_tokens": a.max_tokens, "temperature": a.temperature})
        except (urllib.error.URLError, OSError) as e:
            return _no_server(a, e)
        reply = d["choices"][0]["message"]["content"] or ""
        print(reply, flush=True)
        history.append({"role": "assistant", "content": reply})
    return 0


def cmd_chat(a) -> int:
    if a.url:
        a.host, _, port = a.url.replace("http://", "").rstrip("/").partition(":")
        a.port = int(port or 11435)
        return _chat_remote(a)
    from .api import LLM
    from .engine.sampling import SamplingParams
    from .serving.chat_template import apply_chat_template

    llm = LLM(a.model or ucfg.get("model.default"), a.device, seed=a.seed)
    eos = llm.engine.cfg.eos_token_id
    history = []
    print(f"squish chat: {llm.loaded.name} (empty line or Ctrl-D to quit)", file=sys.stderr)
    for line in sys.stdin:
        line = line.rstrip("\n")
        if not line:
            break
        history.append({"role": "user", "content": line})
        prompt = apply_chat_template(history, llm.tokenizer, arch=llm.engine.cfg.arch)
        out = llm.generate([prompt], SamplingParams(max_tokens=a.max_tokens, temperature=a.temperature,
                                                    stop_token_ids=[eos]))[0]
        print(out["text"], flush=True)
        history.append({"role": "assistant", "content": out["text"]})
    return 0


def add_parsers(sub) -> None:
    def client(p):
        p.add_argument("--host", default=None)
        p.add_argument("--port", type=int, default=None)
        p.add_argument("--api-key", default=None)
        p.add_argument("--timeout", type=float, default=10.0)

    p = sub.add_parser("chat", help="interactive chat (local model, or a server with --url)")
    p.add_argument("model", nargs="?", default=None)
    p.add_argument("--url", default=None, help="chat with a running server, e.g. http://127.0.0.1:11435")
    p.add_argument("--device", default=None)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--max-tokens", type=int, default=256)
    p.add_argument("--temperature", type=float, default=0.7)
    p.add_argument("--api-key", default=None)
    p.add_argument("--timeout", type=float, default=300.0)
    p.set_defaults(fn=cmd_chat)
    p = sub.add_parser("info", help="architecture, quantization and size of a model")
    p.add_argument("model")
    p.set_defaults(fn=cmd_info)
    p = sub.add_parser("search", help="find presets and local models")
    p.add_argument("query")
    p.set_defaults(fn=cmd_search)
    p = sub.add_parser("rm", help="delete a local model")
    p.add_argument("name")
    p.add_argument("-y", "--yes", action="store_true")
    p.set_defaults(fn=cmd_rm)
    p = sub.add_parser("ps", help="what a running server has loaded")
    client(p)
    p.set_defaults(fn=cmd_ps)
    p = sub.add_parser("logs", help="the server log")
    p.add_argument("-n", "--lines", type=int, default=50)
    p.add_argument("-f", "--follow", action="store_true")
    p.add_argument("--file", default=None)
    p.set_defaults(fn=cmd_logs)
    p = sub.add_parser("trace", help="span traces of a running server")
    p.add_argument("action", nargs="?", default="view", choices=["view", "reset", "obs"])
    p.add_argument("--chrome", default=None, metavar="PATH")
    p.add_argument("--top", type=int, default=20)
    client(p)
    p.set_defaults(fn=cmd_trace)
    p = sub.add_parser("quality", help="latency / error report of a running server")
    p.add_argument("--window", type=int, default=300)
    client(p)
    p.set_defaults(fn=cmd_quality)
    p = sub.add_parser("route", help="the prompt router's decision")
    p.add_argument("prompt", nargs="+")
    client(p)
    p.set_defaults(fn=cmd_route)
    p = sub.add_parser("export", help="write a checkpoint as SQUIZD or an npy-dir")
    p.add_argument("model")
    p.add_argument("dest")
    p.add_argument("--format", default="squizd", choices=["squizd", "npy-dir"])
    p.add_argument("--group-size", type=int, default=64)
    p.set_defaults(fn=cmd_export)
    p = sub.add_parser("eval", help="perplexity under the fp32 reference forward")
    p.add_argument("model")
    p.add_argument("--text", default=None, help="text file (default: seeded random tokens)")
    p.add_argument("--max-tokens", type=int, default=1024)
    p.add_argument("--window", type=int, default=512)
    p.add_argument("--device", default=None)
    p.add_argument("--seed", type=int, default=0)
    p.set_defaults(fn=cmd_eval)
    p = sub.add_parser("push", help="upload a model (needs network access)")
    p.add_argument("name", nargs="?")
    p.set_defaults(fn=cmd_push)


__all__ = ["add_parsers", "perplexity", "log_path"]
