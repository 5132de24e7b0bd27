"""Persistent user configuration: ``$SQUISH_HOME/config.json`` (default ``~/.squish``).

Same file, keys and defaults as the reference (squish/config.py:1-183): a flat JSON object
addressed with dot keys (``server.port``), defaults port 11435, host 127.0.0.1, api_key
"squish". ``SQUISH_HOME`` moves the whole directory, ``SQUISH_CONFIG_DIR`` only the config
file. Writes go through a temporary file and ``os.replace`` so a crash never leaves a
half-written config.
"""
from __future__ import annotations

import copy
import json
import os
from pathlib import Path
from typing import Any

DEFAULTS: dict[str, Any] = {
    "server": {"host": "127.0.0.1", "port": 11435, "api_key": "squish", "max_pending": 256},
    "model": {"default": "qwen2.5-7b", "models_dir": ""},
    "engine": {"max_num_seqs": 64, "max_num_batched_tokens": 2048, "max_model_len": 4096,
               "gpu_memory_utilization": 0.85, "kv_dtype": "int4", "page_size": 16, "cuda_graphs": True,
               "prefix_caching": True},
    "speculative": {"prompt_lookup": True, "prompt_lookup_n": 3, "prompt_lookup_k": 4, "draft_model": "",
                    "draft_depth": 4},
    "telemetry": {"trace": False, "trace_file": ""},
}


def squish_home() -> Path:
    return Path(os.environ.get("SQUISH_HOME") or Path.home() / ".squish")


def config_path() -> Path:
    d = os.environ.get("SQUISH_CONFIG_DIR")
    return (Path(d) if d else squish_home()) / "config.json"


def _merge(base: dict, over: dict) -> dict:
    out = copy.deepcopy(base)
    for k, v in over.items():
        out[k] = _merge(out[k], v) if isinstance(v, dict) and isinstance(out.get(k), dict) else v
    return out


def load() -> dict:
    p = config_path()
    if p.exists():
        try:
            return _merge(DEFAULTS, json.loads(p.read_text()))
        except (json.JSONDecodeError, OSError):
            pass
    return copy.deepcopy(DEFAULTS)


def save(cfg: dict) -> Path:
    p = config_path()
    p.parent.mkdir(parents=True, exist_ok=True)
    tmp = p.with_suffix(".json.tmp")
    tmp.write_text(json.dumps(cfg, indent=2, sort_keys=True))
    os.replace(tmp, p)
    return p


def get(key: str, default: Any = None, cfg: dict | None = None) -> Any:
    node: Any = cfg if cfg is not None else load()
    for part in key.split("."):
        if not isinstance(node, dict) or part not in node:
            return default
        node = node[part]
    return node


def _coerce(value: str) -> Any:
    lo = value.lower()
    if lo in ("true", "false"):
        return lo == "true"
    for cast in (int, float):
        try:
            return cast(value)
        except ValueError:
            pass
    return value


def set_value(key: str, value: Any) -> dict:
    cfg = load()
    node = cfg
    parts = key.split(".")
    for part in parts[:-1]:
        node = node.setdefault(part, {})
        if not isinstance(node, dict):
            raise KeyError(f"{key}: {part} is not a section")
    node[parts[-1]] = _coerce(value) if isinstance(value, str) else value
    save(cfg)
    return cfg


def reset() -> dict:
    save(copy.deepcopy(DEFAULTS))
    return load()
