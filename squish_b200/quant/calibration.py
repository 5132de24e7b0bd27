"""Calibration statistics and Wanda pruning scores (tensor ops on any device).

Same definitions as the reference's research kernels (squish_quant_rs/src/lib.rs):
  calib_absmax      per channel, max |x| over the samples                       (:2964)
  calib_percentile  per channel, |x| sorted ascending at index floor(p/100 * (n - 1))  (:2986)
  calib_aciq        per channel, sigma * max(1, sqrt(2 ln n + 1)) (unbiased sigma), >= 1e-6  (:3013)
  wanda_importance  |W[o, i]| * norm[i] (norm: the input channel's activation norm)   (:3682)
  wanda_nm_mask     per row, in every block of m inputs keep the n most important  (:3714)
Activations come from ``ReferenceModel.tap`` (``collect_input_norms``). No sparse GEMM uses the
N:M masks here; ``wanda_prune`` zeroes the pruned weights before quantization.
"""
from __future__ import annotations

import math

import torch


def calib_absmax(acts: torch.Tensor) -> torch.Tensor:
    return acts.float().abs().amax(0)


def calib_percentile(acts: torch.Tensor, percentile: float) -> torch.Tensor:
    a = acts.float().abs().sort(0).values
    n = a.shape[0]
    p = min(max(float(percentile), 0.0), 100.0)
    idx = min(int(p / 100.0 * max(n - 1, 0)), max(n - 1, 0))
    return a[idx]


def calib_aciq(acts: torch.Tensor) -> torch.Tensor:
    x = acts.float()
    n = x.shape[0]
    sigma = x.std(0, unbiased=True) if n > 1 else torch.zeros(x.shape[1], device=x.device)
    return (sigma * max(1.0, math.sqrt(2.0 * math.log(n) + 1.0))).clamp_min(1e-6)


def wanda_importance(w: torch.Tensor, norm: torch.Tensor) -> torch.Tensor:
    return w.float().abs() * norm.float().to(w.device)[None, :]


def wanda_nm_mask(importance: torch.Tensor, n: int, m: int) -> torch.Tensor:
    """uint8 [out, in]: 1 for the ``n`` largest scores of each ``m``-wide block of a row."""
    out_f, in_f = importance.shape
    pad = (-in_f) % m
    imp = torch.nn.functional.pad(importance.float(), (0, pad), value=-math.inf)
    blocks = imp.reshape(out_f, -1, m)
    keep = torch.zeros_like(blocks, dtype=torch.uint8)
    k = min(n, m)
    top = blocks.topk(k, dim=-1).indices
    keep.scatter_(-1, top, 1)
    # pad slots score -inf, so a narrower last block keeps min(n, its width) real entries
    return keep.reshape(out_f, -1)[:, :in_f].contiguous()


def wanda_prune(w: torch.Tensor, norm: torch.Tensor, n: int = 2, m: int = 4) -> torch.Tensor:
    return w * wanda_nm_mask(wanda_importance(w, norm), n, m).to(w.dtype)


def collect_input_norms(ck, tokens: list[list[int]], device=None) -> dict[str, torch.Tensor]:
    """tap name -> L2 norm of each input channel over all calibration tokens (the Wanda norm)."""
    from ..models.reference import ReferenceModel

    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    model = ReferenceModel(ck, device=dev)
    sq: dict[str, torch.Tensor] = {}

    def tap(name, x):
        x2 = x.reshape(-1, x.shape[-1]).float()
        sq[name] = sq.get(name, 0) + (x2 * x2).sum(0)

    model.tap = tap
    for seq in tokens:
        if seq:
            model.forward(seq, model.new_cache(), 0)
    return {k: v.sqrt() for k, v in sq.items()}
