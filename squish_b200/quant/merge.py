"""Model and adapter merging: SLERP, DARE and TIES (torch, any device).

Semantics of the reference's merge kernels (squish_quant_rs/src/lib.rs:2563-2686) and of its
``merge-model`` command (squish/cli.py:5663-5770):

* ``slerp(a, b, t)``: spherical interpolation of the two tensors seen as flat vectors (angle
  from the normalised dot product; a plain lerp when the angle is below 1e-6).
* ``dare(base, delta, density, seed)``: keep each delta element with probability ``density``
  (a deterministic per-element hash of (seed, index), so a merge is reproducible) and rescale
  the kept ones by 1/density.
* ``ties(base, deltas, trim_fraction, t)``: per model, drop delta elements whose magnitude is
  below that model's ``trim_fraction`` quantile; elect the sign of the sum of surviving signs;
  average the surviving elements that agree with it; add ``t`` times that mean.
* ``merge_adapters(dicts, method)``: "dare" (drop 99%, rescale, average), "ties" (majority
  sign vote, average the aligned deltas), "dare-ties" (both).
"""
from __future__ import annotations

import math
from pathlib import Path

import torch


def slerp(a: torch.Tensor, b: torch.Tensor, t: float) -> torch.Tensor:
    if a.shape != b.shape:
        raise ValueError("a and b must have the same shape")
    af, bf = a.float().reshape(-1), b.float().reshape(-1)
    na, nb = af.norm().clamp_min(1e-10), bf.norm().clamp_min(1e-10)
    dot = float(((af / na) * (bf / nb)).sum().clamp(-1.0, 1.0))
    theta = math.acos(dot)
    if abs(theta) < 1e-6:
        out = af * (1 - t) + bf * t
    else:
        st = math.sin(theta)
        out = af * (math.sin((1 - t) * theta) / st) + bf * (math.sin(t * theta) / st)
    return out.reshape(a.shape).to(a.dtype)


def _hash_uniform(n: int, seed: int, device) -> torch.Tensor:
    """Uniform [0, 1) per element index: SplitMix64 finaliser of (seed + index * golden ratio),
    in int64 arithmetic (wrapping), top 24 bits."""
    i = torch.arange(n, dtype=torch.int64, device=device)
    z = i * -7046029254386353131 + seed  # 0x9E3779B97F4A7C15 as a signed int64; products wrap

    def shr(v, k):  # logical shift right of an int64 bit pattern
        return (v >> k) & ((1 << (64 - k)) - 1)

    z = (z ^ shr(z, 30)) * -4658895280553007687  # 0xBF58476D1CE4E5B9
    z = (z ^ shr(z, 27)) * -7723592293110705685  # 0x94D049BB133111EB
    z = z ^ shr(z, 31)
    return shr(z, 40).double().div_(float(1 << 24)).float()


def dare(base: torch.Tensor, delta: torch.Tensor, density: float, seed: int = 0) -> torch.Tensor:
    if base.shape != delta.shape:
        raise ValueError("base and delta must match")
    if not 0.0 < density <= 1.0:
        raise ValueError("density must be in (0, 1]")
    keep = _hash_uniform(base.numel(), seed, base.device).reshape(base.shape) < density
    return (base.float() + torch.where(keep, delta.float() / density, torch.zeros((), device=base.device))
            ).to(base.dtype)


def ties(base: torch.Tensor, deltas: list[torch.Tensor] | torch.Tensor, trim_fraction: float = 0.2,
         t: float = 1.0) -> torch.Tensor:
    d = torch.stack([x.float().reshape(-1) for x in deltas]) if isinstance(deltas, (list, tuple)) \
        else deltas.float().reshape(deltas.shape[0], -1)
    n = d.shape[1]
    if base.numel() != n:
        raise ValueError("base / deltas shape mismatch")
    k = min(int(math.ceil(n * trim_fraction)), max(n - 1, 0))
    thr = d.abs().sort(dim=1).values[:, k:k + 1]
    kept = d.abs() >= thr
    sgn = torch.where(kept, torch.sign(d), torch.zeros((), device=d.device)).sum(0)
    agree = kept & (torch.sign(d) == torch.sign(sgn)[None])
    cnt = agree.sum(0)
    mean = torch.where(agree, d, torch.zeros((), device=d.device)).sum(0) / cnt.clamp_min(1)
    out = base.float().reshape(-1) + torch.where(cnt > 0, t * mean, torch.zeros((), device=d.device))
    return out.reshape(base.shape).to(base.dtype)


def merge_adapters(adapters: list[dict[str, torch.Tensor]], method: str = "dare-ties", drop: float = 0.99,
                   seed: int = 0) -> tuple[dict[str, torch.Tensor], int]:
    """Merge flat adapter (delta) dicts; returns (merged dict, number of sign-conflicted elements)."""
    if method not in ("dare", "ties", "dare-ties"):
        raise ValueError(f"unknown merge method {method!r}")
    keys = sorted(set().union(*[a.keys() for a in adapters]))
    merged, conflicts = {}, 0
    for j, key in enumerate(keys):
        ds = [a[key].float() for a in adapters if key in a]
        if method in ("dare", "dare-ties"):
            ds = [dare(torch.zeros_like(d), d, 1.0 - drop, seed + 7919 * j + i) for i, d in enumerate(ds)]
        st = torch.stack(ds)
        if method in ("ties", "dare-ties") and len(ds) > 1:
            maj = torch.sign(torch.sign(st).sum(0))
            conflicts += int((torch.sign(st) != maj[None]).any(0).sum())
            st = st * (torch.sign(st) == maj[None])
        merged[key] = st.mean(0).to(adapters[0][key].dtype if key in adapters[0] else ds[0].dtype)
    return merged, conflicts


def merge_adapter_files(paths: list[str], out_dir: str, method: str = "dare-ties") -> dict:
    """``squish merge-model``: safetensors adapters -> ``out_dir/adapter_model.safetensors``."""
    from safetensors.torch import load_file, save_file

    files = []
    for p in paths:
        q = Path(p)
        if q.is_dir():
            cands = sorted(q.glob("*.safetensors"))
            if not cands:
                raise FileNotFoundError(f"no .safetensors adapter in {q}")
            q = cands[0]
        files.append(q)
    merged, conflicts = merge_adapters([load_file(str(f)) for f in files], method)
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    save_file({k: v.contiguous() for k, v in merged.items()}, str(out / "adapter_model.safetensors"))
    return {"output": str(out / "adapter_model.safetensors"), "tensors": len(merged), "sign_conflicts": conflicts}
