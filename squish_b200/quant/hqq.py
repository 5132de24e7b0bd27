"""Half-Quadratic Quantization (HQQ, Badri & Shaji, arXiv:2309.15531): calibration-free
affine weight quantization at any level count in [2, 256] (1 to 8 bits, fractional widths
included: ``levels = max(2, round(2 ** bits))``).

Same algorithm and container as the reference's HQQQuantizer (squish/quant/hqq.py:60-316):
per group a min/max affine grid, then ``max_iter`` alternating half-quadratic updates of the
scale (proximal weight ``lambda_scale``), the zero point (mean residual) and the codes. CUDA
tensors run one warp per group in ``csrc/quantize.cu`` (``_C.hqq``); CPU tensors run the torch
restatement below, which is also the oracle of the GPU test.

The decode ``x = zero + code * scale`` is exactly the INT4-asymmetric (and INT2) form, so an
HQQ result with <= 16 levels is stored and served as ``q4a`` (<= 4 levels: ``q2`` too) by
:meth:`HQQTensor.to_qtensor` -- the tcgen05 GEMM runs it with no HQQ-specific kernel.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .._ext import native
from ..models.weights import QTensor

__all__ = ["HQQConfig", "HQQTensor", "HQQQuantizer", "hqq_quantize"]


def grid_levels(bits: float) -> int:
    return max(2, round(2.0 ** bits))


@dataclass
class HQQConfig:
    bits: float = 4.0
    group_size: int = 128      # -1: the whole row (axis 0) or column (axis 1)
    lambda_scale: float = 1.0
    max_iter: int = 10
    axis: int = 0              # 0: groups along a row, 1: along a column

    def __post_init__(self) -> None:
        self.bits = float(self.bits)
        if not 1.0 <= self.bits <= 8.0:
            raise ValueError(f"bits must be in [1.0, 8.0]; got {self.bits}")
        if self.group_size != -1 and self.group_size < 1:
            raise ValueError(f"group_size must be >= 1 or -1 (full row); got {self.group_size}")
        if self.lambda_scale <= 0:
            raise ValueError(f"lambda_scale must be positive; got {self.lambda_scale}")
        if self.max_iter < 1:
            raise ValueError(f"max_iter must be >= 1; got {self.max_iter}")
        if self.axis not in (0, 1):
            raise ValueError(f"axis must be 0 or 1; got {self.axis}")

    @property
    def n_levels(self) -> int:
        return grid_levels(self.bits)


@dataclass
class HQQTensor:
    codes: np.ndarray   # uint8, the original shape
    scale: np.ndarray   # float32 [other_dim, groups]
    zero: np.ndarray    # float32 [other_dim, groups]
    shape: tuple
    config: HQQConfig

    def nbytes(self) -> int:
        return int(self.codes.nbytes + self.scale.nbytes + self.zero.nbytes)

    def to_qtensor(self, kind: str = "q4a") -> QTensor:
        """The GEMM-servable form: ``q4a`` (<= 16 levels) or ``q2`` (<= 4 levels), axis 0 only,
        the group dividing the row."""
        cfg = self.config
        rows, cols = self.shape
        g = cfg.group_size if cfg.group_size != -1 else cols
        if cfg.axis != 0 or cols % g:
            raise ValueError("only row-wise HQQ with a group dividing the row maps onto a GEMM format")
        c = torch.from_numpy(self.codes.astype(np.int64))
        s, z = torch.from_numpy(self.scale), torch.from_numpy(self.zero)
        if kind == "q4a":
            if cfg.n_levels > 16:
                raise ValueError(f"{cfg.n_levels} levels do not fit 4-bit codes")
            packed = (c[:, 0::2] | (c[:, 1::2] << 4)).to(torch.uint8)
            return QTensor("q4a", (rows, cols), packed=packed, scales=s, offsets=z, group=g)
        if kind == "q2":
            if cfg.n_levels > 4:
                raise ValueError(f"{cfg.n_levels} levels do not fit 2-bit codes")
            c4 = c.view(rows, cols // 4, 4)
            packed = (c4[..., 0] | (c4[..., 1] << 2) | (c4[..., 2] << 4) | (c4[..., 3] << 6)).to(torch.uint8)
            return QTensor("q2", (rows, cols), packed=packed, scales=s, offsets=z, group=g)
        raise ValueError(f"unknown target kind {kind!r}")


def hqq_torch(w: torch.Tensor, group: int, levels: int, lam: float, iters: int):
    """Torch restatement (any device): w [R, C] with C % group == 0 -> (codes uint8 [R, C],
    scale [R, C/group], zero [R, C/group])."""
    r, c = w.shape
    wg = w.float().reshape(r, c // group, group)
    qmax = float(levels - 1)
    mn = wg.amin(-1, keepdim=True)
    mx = wg.amax(-1, keepdim=True)
    sc = (mx - mn).clamp_min(1e-6) / qmax
    z = mn
    q = torch.clamp(torch.round((wg - z) / sc), 0, qmax)
    for _ in range(iters):
        c2 = (q * q).sum(-1, keepdim=True) + lam
        sc = ((q * (wg - z)).sum(-1, keepdim=True) + lam * sc) / c2
        z = (wg - q * sc).mean(-1, keepdim=True)
        q = torch.clamp(torch.round((wg - z) / sc.abs().clamp_min(1e-8)), 0, qmax)
    return q.reshape(r, c).to(torch.uint8), sc.squeeze(-1), z.squeeze(-1)


def hqq_quantize(w: torch.Tensor, group: int, levels: int, lam: float = 1.0, iters: int = 10):
    """(codes, scale, zero) of a 2-D tensor whose width ``group`` divides: the CUDA kernel for
    CUDA tensors with group <= 512, else the torch restatement."""
    if w.is_cuda and group <= 512:
        x = w.detach()
        x = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
        return tuple(native().hqq(x.contiguous(), group, levels, float(lam), int(iters)))
    return hqq_torch(w.detach(), group, levels, lam, iters)


class HQQQuantizer:
    """encode / decode / error metrics with the reference class's interface."""

    def __init__(self, config: HQQConfig | None = None, device: str | torch.device | None = None) -> None:
        self.config = config or HQQConfig()
        self.device = torch.device(device) if device is not None else None

    def encode(self, weight) -> HQQTensor:
        W = torch.as_tensor(np.asarray(weight, dtype=np.float32)) if not isinstance(weight, torch.Tensor) \
            else weight.detach().float()
        if W.dim() != 2:
            raise ValueError(f"weight must be 2-D; got shape {tuple(W.shape)}")
        cfg = self.config
        shape = tuple(W.shape)
        if cfg.axis == 1:
            W = W.T
        other, dim = W.shape
        g = cfg.group_size if cfg.group_size != -1 else dim
        n_groups = max(1, -(-dim // g))
        if n_groups * g > dim:  # zero-pad the last group (the pad takes part in the group's fit)
            W = torch.nn.functional.pad(W, (0, n_groups * g - dim))
        if self.device is not None:
            W = W.to(self.device)
        codes, scale, zero = hqq_quantize(W.contiguous(), g, cfg.n_levels, cfg.lambda_scale, cfg.max_iter)
        codes = codes[:, :dim].cpu()
        if cfg.axis == 1:
            codes = codes.T
        return HQQTensor(codes=codes.contiguous().numpy().astype(np.uint8), scale=scale.float().cpu().numpy(),
                         zero=zero.float().cpu().numpy(), shape=shape, config=cfg)

    def decode(self, tensor: HQQTensor) -> np.ndarray:
        cfg = tensor.config
        codes = tensor.codes.astype(np.float32)
        rows, cols = tensor.shape
        if cfg.axis == 1:
            codes = codes.T
        other, dim = codes.shape
        g = cfg.group_size if cfg.group_size != -1 else dim
        n_groups = tensor.scale.shape[-1]
        pad = np.zeros((other, n_groups * g), dtype=np.float32)
        pad[:, :dim] = codes
        w = pad.reshape(other, n_groups, g) * tensor.scale[:, :, None] + tensor.zero[:, :, None]
        w = w.reshape(other, -1)[:, :dim]
        return (w.T if cfg.axis == 1 else w).astype(np.float32)

    @staticmethod
    def relative_error(original, reconstructed) -> float:
        o = np.asarray(original, dtype=np.float32)
        n = float(np.linalg.norm(o))
        return 0.0 if n == 0 else float(np.linalg.norm(o - np.asarray(reconstructed, dtype=np.float32))) / n

    @staticmethod
    def quantisation_error_db(original, reconstructed) -> float:
        o = np.asarray(original, dtype=np.float32)
        noise = float(np.mean((o - np.asarray(reconstructed, dtype=np.float32)) ** 2)) + 1e-20
        return 10.0 * float(np.log10(float(np.mean(o ** 2)) / noise))

    def __repr__(self) -> str:
        c = self.config
        return f"HQQQuantizer(bits={c.bits}, group_size={c.group_size}, max_iter={c.max_iter})"
