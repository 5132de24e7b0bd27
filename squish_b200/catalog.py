"""Model catalog: the models this package knows by name, their sizes, and name resolution.

Entries are built from the built-in architecture presets (exact parameter counts, raw bf16 and
INT4 footprints computed from the configs) plus an optional user catalog file
(``~/.squish/catalog.json``, a JSON list of entry objects; its entries override built-in ones
of the same id), which stands in for the reference's remote catalog refresh: this package
makes no network requests. The reference's catalog (squish/catalog.py:199-263 entries,
:790-981 list / search / suggest / resolve) names models ``family:size`` (``qwen2.5:7b``); the
same canonical form, the same user spellings (``Qwen2.5-7B-Instruct``, ``qwen2.5-7b-int4``) and
the preset names resolve here.
"""
from __future__ import annotations

import dataclasses
import json
import re
from dataclasses import dataclass, field
from pathlib import Path


@dataclass
class CatalogEntry:
    id: str                           # canonical "family:size", e.g. "qwen2.5:7b"
    name: str                         # display name
    hf_repo: str                      # the upstream checkpoint repository
    params: str                       # "7.6B"
    params_b: float
    context: int
    size_gb: float                    # raw bf16 weights
    int4_size_gb: float               # INT4 codes + group scales (the serving format)
    preset: str | None = None         # built-in architecture preset (random init offline)
    tags: list[str] = field(default_factory=list)
    moe: bool = False
    active_params_b: float | None = None
    grammar_trigger: str | None = None  # opening tag of the family's tool-call format
    notes: str = ""

    @property
    def dir_name(self) -> str:
        return self.hf_repo.split("/")[-1]


# preset -> (id, display name, upstream repository, tags, tool-call opening tag)
_KNOWN = {
    "qwen2.5-0.5b": ("qwen2.5:0.5b", "Qwen2.5 0.5B Instruct", "Qwen/Qwen2.5-0.5B-Instruct", ["small", "fast", "draft"],
                     "<tool_call>"),
    "qwen2.5-1.5b": ("qwen2.5:1.5b", "Qwen2.5 1.5B Instruct", "Qwen/Qwen2.5-1.5B-Instruct", ["small", "fast"],
                     "<tool_call>"),
    "qwen2.5-7b": ("qwen2.5:7b", "Qwen2.5 7B Instruct", "Qwen/Qwen2.5-7B-Instruct", ["general", "tools"],
                   "<tool_call>"),
    "qwen3-8b": ("qwen3:8b", "Qwen3 8B", "Qwen/Qwen3-8B", ["general", "reasoning", "tools"], "<tool_call>"),
    "qwen3-30b-a3b": ("qwen3:30b-a3b", "Qwen3 30B-A3B (MoE)", "Qwen/Qwen3-30B-A3B", ["moe", "reasoning", "tools"],
                      "<tool_call>"),
    "llama-3.1-8b": ("llama3.1:8b", "Llama 3.1 8B Instruct", "meta-llama/Llama-3.1-8B-Instruct", ["general"], None),
    "llama-3-70b": ("llama3:70b", "Llama 3 70B Instruct", "meta-llama/Meta-Llama-3-70B-Instruct", ["large"], None),
}

_SIZE_RE = re.compile(r"[-_:](\d+(?:\.\d+)?[bm](?:-a\d+(?:\.\d+)?b)?)"
                      r"(?:[-_](?:instruct|chat|it|base))?"
                      r"(?:[-_](?:int2|int3|int4|int8|q4|q8|bf16|fp16|fp32|squished))?$", re.I)


def _fmt_params(b: float) -> str:
    return f"{b:.1f}B" if b >= 1 else f"{b * 1000:.0f}M"


def _from_preset(preset: str) -> CatalogEntry | None:
    from .models.config import PRESETS

    if preset not in PRESETS or preset not in _KNOWN:
        return None
    cfg, q = PRESETS[preset]
    eid, name, repo, tags, trig = _KNOWN[preset]
    n = cfg.num_params()
    # INT4 codes (half a byte per weight) + one bf16 (scale, zero) pair per group of the
    # quantized matrices (everything but the embedding table, which is kept dense here)
    emb = cfg.vocab_size * cfg.hidden_size
    quant = n - emb
    int4 = quant * 0.5 + quant / q.group_size * 4 + emb * 2
    active = None
    if cfg.is_moe:
        dense = n - cfg.num_layers * cfg.num_experts * 3 * cfg.hidden_size * cfg.moe_intermediate_size
        active = (dense + cfg.num_layers * cfg.num_experts_per_tok * 3 * cfg.hidden_size
                  * cfg.moe_intermediate_size) / 1e9
    return CatalogEntry(id=eid, name=name, hf_repo=repo, params=_fmt_params(n / 1e9), params_b=round(n / 1e9, 3),
                        context=cfg.max_position, size_gb=round(n * 2 / 1e9, 2), int4_size_gb=round(int4 / 1e9, 2),
                        preset=preset, tags=list(tags), moe=cfg.is_moe,
                        active_params_b=None if active is None else round(active, 2), grammar_trigger=trig)


def user_catalog_path() -> Path:
    from .config import squish_home

    return squish_home() / "catalog.json"


def load_catalog(path: str | Path | None = None) -> dict[str, CatalogEntry]:
    """Built-in entries, then the user's catalog file (when present) merged over them."""
    cat = {e.id: e for e in (_from_preset(p) for p in _KNOWN) if e is not None}
    p = Path(path) if path is not None else user_catalog_path()
    if p.is_file():
        names = {f.name for f in dataclasses.fields(CatalogEntry)}
        for d in json.loads(p.read_text()):
            base = dataclasses.asdict(cat[d["id"]]) if d.get("id") in cat else {}
            base.update({k: v for k, v in d.items() if k in names})
            cat[base["id"]] = CatalogEntry(**base)
    return cat


def list_catalog(tag: str | None = None, path=None) -> list[CatalogEntry]:
    """Entries by parameter count, optionally those carrying ``tag``."""
    es = [e for e in load_catalog(path).values() if tag is None or tag.lower() in (t.lower() for t in e.tags)]
    return sorted(es, key=lambda e: (e.params_b, e.id))


def search(query: str, path=None) -> list[CatalogEntry]:
    """Case-insensitive substring match on id, name, tags, parameter string and repository."""
    q = query.lower()
    return [e for e in list_catalog(path=path)
            if q in e.id or q in e.name.lower() or q in e.params.lower() or q in e.hf_repo.lower()
            or any(q in t.lower() for t in e.tags)]


def normalize_name(name: str) -> str:
    """User spelling -> canonical ``family:size``: lower case, the repository owner, a trailing
    variant (``-instruct``) and quantization suffix (``-int4``) dropped, the separator before the
    size replaced by a colon (``Qwen/Qwen2.5-7B-Instruct`` -> ``qwen2.5:7b``). Names without a
    recognisable size come back lower-cased."""
    n = name.strip().lower().split("/")[-1]
    m = _SIZE_RE.search(n)
    if m:
        return f"{n[:m.start()]}:{m.group(1)}"
    return n


def resolve(name: str, path=None) -> CatalogEntry | None:
    """The entry for an id, a user spelling of it, a preset name or an upstream repository."""
    cat = load_catalog(path)
    key = name.strip().lower()
    if key in cat:
        return cat[key]
    norm = normalize_name(name)
    if norm in cat:
        return cat[norm]
    for e in cat.values():
        if key in (e.preset or "", e.hf_repo.lower(), e.dir_name.lower()):
            return e
    # family spellings without the dot or with "llama-3" for "llama3"
    squashed = norm.replace("-", "").replace(".", "")
    for e in cat.values():
        if e.id.replace("-", "").replace(".", "") == squashed:
            return e
    return None


def suggest(query: str, max_results: int = 3, path=None) -> list[CatalogEntry]:
    """Close matches for an unknown name: the normalized query and its parts (separator-split and
    letter / number runs) scored against ids (substring of the whole id 10, a part inside the id
    3, inside the display name 1)."""
    norm = normalize_name(query)
    parts = {p for p in re.split(r"[:\-_]", norm) + re.findall(r"[a-z]+|\d+(?:\.\d+)?[bm]?", norm) if len(p) >= 2}
    scored = []
    for e in load_catalog(path).values():
        score = 10 if (norm in e.id or e.id in norm) else 0
        for p in parts:
            score += 3 * (p in e.id) + (p in e.name.lower())
        if score:
            scored.append((-score, e.params_b, e))
    return [e for _, _, e in sorted(scored, key=lambda x: (x[0], x[1]))[:max_results]]
