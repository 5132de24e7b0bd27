"""Activation-aware weight scaling (AWQ, Lin et al. 2023) at convert time.

Calibration runs forward passes of the fp32 model (``models/reference.py`` on the GPU when one
is present) over calibration token sequences and records, for the input of every norm-fed
projection group, the mean absolute activation per input channel; on CUDA tensors the
statistics are one kernel per forward step (``csrc/quantize.cu``, ``_C.channel_abs_mean``,
double accumulators). Scales are ``s = clip(mean_abs, 1e-4) ** alpha`` (optionally floored at
``min_scale``), as in squish/quant/awq.py:329-346.

Application (squish/quant/awq.py:536-676) keeps ``(x / s) @ (W * s)^T == x @ W^T``: the
columns of every projection fed by a norm are multiplied by s and the norm's gamma is divided
by s, once per norm, with one scale per norm (the channel-wise mean of its members' scales).
Only norm-fed projections are scaled (q/k/v after ``input_layernorm``; gate/up after
``post_attention_layernorm``); ``o_proj`` and ``down_proj`` are left alone. In a MoE layer the
router (``mlp.gate``) reads the same normalised input, so it is scaled with the experts --
without that the identity would not hold for the routing logits.

Scale files keep the reference's layout (``{safe}.awq.npy`` per linear layer, ``awq_index.json``,
``.awq_ready``), so scales computed by either tool load in the other.
"""
from __future__ import annotations

import json
import re
from pathlib import Path

import numpy as np
import torch

from .._ext import native

_ATTN = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj")
_MLP = ("mlp.gate_proj", "mlp.up_proj")

# Generic calibration prose (written for this package) used when no texts are given.
DEFAULT_CALIBRATION_TEXTS = [
    "The river rose through the night, and by morning the lower fields were under a sheet of grey water.",
    "To compute the determinant of a triangular matrix, multiply the entries on its main diagonal.",
    "def merge(a, b):\n    out = []\n    while a and b:\n        out.append(a.pop(0) if a[0] < b[0] else b.pop(0))\n"
    "    return out + a + b",
    "Customer support transcript: the user reports that the export button does nothing in the web app.",
    "In 1887 the observatory installed a new refractor, and the first survey of the southern sky began.",
    "Mix the flour and salt, add warm water slowly, and knead the dough until it is smooth and elastic.",
    "SELECT region, SUM(amount) FROM orders WHERE created_at >= '2024-01-01' GROUP BY region;",
    "Photosynthesis converts light energy into chemical energy stored in glucose and other sugars.",
]


class ActivationStats:
    """Per-norm running sum of per-call mean |x| per channel (float64) and the call count."""

    def __init__(self):
        self.acc: dict[str, torch.Tensor] = {}
        self.count: dict[str, int] = {}

    def __call__(self, name: str, x: torch.Tensor) -> None:
        if not name.endswith("layernorm"):
            return  # AWQ scales only norm-fed projections
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        a = self.acc.get(name)
        if a is None:
            a = self.acc[name] = torch.zeros(x2.shape[1], dtype=torch.float64, device=x2.device)
        if x2.is_cuda:
            native().channel_abs_mean(x2 if x2.dtype in (torch.float32, torch.bfloat16) else x2.float(), a)
        else:
            a += x2.float().abs().mean(0).double()
        self.count[name] = self.count.get(name, 0) + 1

    def mean(self, name: str) -> np.ndarray:
        return (self.acc[name] / max(1, self.count[name])).float().cpu().numpy()


def calibration_tokens(vocab: int, n_samples: int = 16, seq_len: int = 256, tokenizer=None, texts=None,
                       seed: int = 0) -> list[list[int]]:
    """Token sequences for calibration: the tokenizer's encoding of ``texts`` (cycled to
    ``n_samples``) when a tokenizer is given, else seeded uniform random ids."""
    if tokenizer is not None:
        texts = texts or DEFAULT_CALIBRATION_TEXTS
        out = []
        for i in range(n_samples):
            ids = tokenizer.encode(texts[i % len(texts)])[:seq_len]
            if ids:
                out.append([t for t in ids if 0 <= t < vocab])
        return out
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (seq_len,), generator=g).tolist() for _ in range(n_samples)]


def collect_activation_scales(ck, tokens: list[list[int]], alpha: float = 0.5, min_scale: float = 0.0,
                              device: str | torch.device | None = None) -> dict[str, np.ndarray]:
    """Run ``tokens`` through the fp32 model of checkpoint ``ck``; return linear-layer name ->
    per-input-channel scale (float32)."""
    from ..models.reference import ReferenceModel

    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    model = ReferenceModel(ck, device=dev)
    stats = ActivationStats()
    model.tap = stats
    for seq in tokens:
        if seq:
            model.forward(seq, model.new_cache(), 0)
    cfg = ck.config
    scales: dict[str, np.ndarray] = {}
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        for norm, members in (("input_layernorm", _ATTN), ("post_attention_layernorm", _MLP)):
            if p + norm not in stats.acc:
                continue
            s = np.clip(stats.mean(p + norm), 1e-4, None) ** alpha
            if min_scale > 0.0:
                s = np.maximum(s, min_scale)
            for m in members:
                scales[p + m] = s.astype(np.float32)
    return scales


def _norm_of(name: str) -> str | None:
    """The norm whose output feeds weight ``name`` (None when it is not norm-fed)."""
    m = re.match(r"(.*\.layers\.\d+\.)(self_attn\.[qkv]_proj|mlp\.(?:experts\.\d+\.)?(?:gate|up)_proj|mlp\.gate)"
                 r"\.weight$", name)
    if not m:
        return None
    return m.group(1) + ("input_layernorm.weight" if m.group(2).startswith("self_attn") else
                         "post_attention_layernorm.weight")


def _scale_for(layer_path: str, scales: dict) -> np.ndarray | None:
    if layer_path in scales:
        return scales[layer_path]
    best = max((k for k in scales if layer_path.endswith(k)), key=len, default=None)
    return scales[best] if best else None


def prepare_awq_application(scales: dict, names) -> dict[str, tuple[str, np.ndarray]]:
    """tensor name -> ("mul", s) for norm-fed projection weights (columns times s) or
    ("div", s) for their norms (gamma / s), s being the mean of the norm's members' scales.
    MoE routers and experts take their layer's ``mlp.gate_proj`` / ``mlp.up_proj`` scale."""
    names = list(names)
    groups: dict[str, list[tuple[str, np.ndarray]]] = {}
    for n in names:
        norm = _norm_of(n)
        if norm is None or norm not in names:
            continue
        path = n[: -len(".weight")]
        s = _scale_for(path, scales)
        if s is None and ".mlp." in path:
            root = path[: path.index(".mlp.")]
            s = _scale_for(root + ".mlp.gate_proj", scales)
            if s is None:
                s = _scale_for(root + ".mlp.up_proj", scales)
        if s is None:
            continue
        groups.setdefault(norm, []).append((n, np.asarray(s, dtype=np.float32)))
    ops: dict[str, tuple[str, np.ndarray]] = {}
    for norm, members in groups.items():
        s = np.stack([m[1] for m in members]).mean(0).astype(np.float32)
        ops[norm] = ("div", s)
        for n, _ in members:
            ops[n] = ("mul", s)
    return ops


def apply_op(t: torch.Tensor, op: tuple[str, np.ndarray]) -> torch.Tensor:
    kind, s = op
    st = torch.from_numpy(s).to(t.device, torch.float32)
    if kind == "div":
        return (t.float() / st).to(t.dtype)
    if t.shape[-1] != st.shape[0]:
        raise ValueError(f"AWQ scale of {st.shape[0]} channels does not match a weight of {t.shape[-1]} columns")
    return (t.float() * st).to(t.dtype)


def apply_awq_to_weights(weights: dict[str, torch.Tensor], scales: dict) -> dict[str, torch.Tensor]:
    """Apply scales in place to a flat name -> fp tensor dict; returns it."""
    for name, op in prepare_awq_application(scales, weights.keys()).items():
        weights[name] = apply_op(weights[name], op)
    return weights


def save_awq_scales(scales: dict, output_dir: str | Path) -> None:
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    index = {}
    for name, s in scales.items():
        fn = name.replace("/", "_").replace(".", "__") + ".awq.npy"
        np.save(str(out / fn), np.asarray(s, dtype=np.float32))
        index[name] = fn
    (out / "awq_index.json").write_text(json.dumps(index, indent=2))
    (out / ".awq_ready").touch()


def load_awq_scales(awq_dir: str | Path) -> dict[str, np.ndarray]:
    d = Path(awq_dir)
    if not d.exists():
        return {}
    idx = d / "awq_index.json"
    if idx.exists():
        return {k: np.load(str(d / f)) for k, f in json.loads(idx.read_text()).items() if (d / f).exists()}
    return {p.name[: -len(".awq.npy")].replace("__", ".").replace("_", "/"): np.load(str(p))
            for p in sorted(d.glob("*.awq.npy"))}
