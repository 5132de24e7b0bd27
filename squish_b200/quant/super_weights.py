"""Super-weight detection: the few scalar weights whose loss collapses a model.

Rule of the reference's SuperWeightCalibrator (squish/quant/super_weight_calibrator.py:150-300,
after Yu et al., arXiv:2411.07191): view each tensor as 2-D (rows x last dim), compute
``ratio = |w| / (mean(|row|) + 1e-9)``, and report elements above ``threshold`` (100 for
matrices, ``threshold_1d`` = 5 for vectors), the top ``max_per_tensor`` by ratio (8; no limit
for vectors), skipping embeddings / LM head and matrices narrower than ``min_2d_cols``. The
scan runs as tensor ops on the tensor's device.

Use in ``squish compress``: INT4-asymmetric groups keep their own min and max exactly (the
grid's end points), so a super weight survives quantization unless the MSE clip search clips
it; rows holding a super weight are therefore re-quantized without clipping (``protect``).
"""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from pathlib import Path

import torch


@dataclass(frozen=True, order=True)
class SuperWeightCoord:
    tensor_name: str
    row: int
    col: int
    value: float
    ratio: float
    original_shape: tuple = field(compare=False, default=())

    @property
    def coord_key(self) -> str:
        return f"{self.tensor_name}[{self.row},{self.col}]"


@dataclass
class SuperWeightConfig:
    threshold: float = 100.0
    threshold_1d: float = 5.0
    max_per_tensor: int = 8
    max_per_tensor_1d: int = 0
    skip_patterns: list = field(default_factory=lambda: ["embed_tokens", "lm_head", "embed_positions"])
    min_2d_cols: int = 64


class SuperWeightCalibrator:
    def __init__(self, config: SuperWeightConfig | None = None):
        self.config = config or SuperWeightConfig()

    def scan_tensor(self, name: str, t: torch.Tensor) -> list[SuperWeightCoord]:
        cfg = self.config
        if t.dim() == 0 or any(p in name for p in cfg.skip_patterns):
            return []
        is_1d = t.dim() == 1
        flat = t.detach().float().reshape(1, -1) if is_1d else t.detach().float().reshape(-1, t.shape[-1])
        if not is_1d and flat.shape[1] < cfg.min_2d_cols:
            return []
        a = flat.abs()
        ratio = a / (a.mean(1, keepdim=True) + 1e-9)
        thr = cfg.threshold_1d if is_1d else cfg.threshold
        hit = (ratio > thr).nonzero()
        if hit.numel() == 0:
            return []
        r = ratio[hit[:, 0], hit[:, 1]]
        order = torch.argsort(r, descending=True)
        limit = cfg.max_per_tensor_1d if is_1d else cfg.max_per_tensor
        if limit > 0:
            order = order[:limit]
        hit, r = hit[order].cpu(), r[order].cpu()
        vals = flat[hit[:, 0], hit[:, 1]].cpu() if hit.numel() else torch.empty(0)
        return [SuperWeightCoord(name, int(h[0]), int(h[1]), float(v), float(rt), tuple(t.shape))
                for h, v, rt in zip(hit, vals, r)]

    def scan_weights(self, weights: dict) -> list[SuperWeightCoord]:
        out = []
        for name, t in weights.items():
            out += self.scan_tensor(name, torch.as_tensor(t))
        return sorted(out, key=lambda c: -c.ratio)


def calibrate_from_dir(model_dir: str, config: SuperWeightConfig | None = None,
                       device: str | None = None) -> list[SuperWeightCoord]:
    """Scan every tensor of the safetensors shards in ``model_dir`` (one tensor in memory at a time)."""
    from safetensors import safe_open

    cal = SuperWeightCalibrator(config)
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    out = []
    for shard in sorted(Path(model_dir).glob("*.safetensors")):
        with safe_open(str(shard), "pt", device="cpu") as f:
            for n in f.keys():
                out += cal.scan_tensor(n, f.get_tensor(n).to(dev))
    return sorted(out, key=lambda c: -c.ratio)


def save_coords(coords: list[SuperWeightCoord], path: str | Path) -> None:
    Path(path).write_text(json.dumps([dict(asdict(c), original_shape=list(c.original_shape)) for c in coords],
                                     indent=1))


def load_coords(path: str | Path) -> list[SuperWeightCoord]:
    return [SuperWeightCoord(**dict(d, original_shape=tuple(d.get("original_shape", ()))))
            for d in json.loads(Path(path).read_text())]


def protect(t, w: torch.Tensor, rows: set[int]):
    """Re-quantize ``rows`` of an MSE-clipped INT4 tensor ``t`` without clipping (their super
    weights then stay at the groups' exact end points)."""
    if not rows or t.kind != "q4a":
        return t
    from ..models.weights import quantize_q4a

    idx = torch.tensor(sorted(rows), dtype=torch.long)
    sub = quantize_q4a(w[idx.to(w.device)], t.group, mse_clip=False)
    t.packed[idx] = sub.packed.to(t.packed.device)
    t.scales[idx] = sub.scales.to(t.scales.device)
    t.offsets[idx] = sub.offsets.to(t.offsets.device)
    return t
