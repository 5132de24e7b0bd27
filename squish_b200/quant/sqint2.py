"""SQINT2: Hadamard-rotated INT2 weights (NF2 grid with a Lloyd refinement, optional low-rank
residual), after the reference's squish/quant/sqint2.py.

Reference pipeline (sqint2.py:747-895): W_rot = H_left W H_right^T with H a sign-randomised
Sylvester Hadamard for power-of-two sizes and a dense random orthogonal matrix (QR of a
Gaussian) otherwise; per-group NF2 quantisation of W_rot (values {-1.5, -0.5, 0.5, 1.5} after an
asymmetric per-group rescale, one global Lloyd sweep, the grid re-fitted to the refined end
points); optional rank-r SVD and sparse corrections of the rotated residual. At inference the
reference dequantises W_rot and rotates back with dense matrices.

Here the rotation is chosen so that the GPU never materialises a weight: only the input side
is rotated, with R = blockdiag(H_b / sqrt(b)) D -- a +-1 sign vector D and Sylvester
Hadamard blocks of b = the largest power of two (<= 4096) dividing the input width. Then
W x = W_rot (R x): the activations go through the O(b log b) butterfly kernel of
``csrc/hadamard.cu`` and the rotated weights run in the tcgen05 INT2 GEMM unchanged (the NF2
decode (v - zp) * scale is affine in the 2-bit code, i.e. exactly the INT2 format
x = z + q s with z = (-1.5 - zp) scale). Tensors carrying a low-rank residual, and
reference-format files with a left rotation or a dense QR rotation, are decompressed at load
and re-encoded INT4, like INT3 with a MiLo compensator.

Files: the reference's ``__sqint2_idx / _scales / _zp / _meta`` (+ ``_L / _R``, sparse COO)
set. Files written here carry format version 2 in ``meta[0]`` (the reference refuses versions
above its 1.0 instead of mis-decoding them) and the rotation block in ``meta[11]``; the sign
vector is re-derived from ``meta[4]`` (seed).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from ..models.weights import QTensor

NF2_VALUES = np.array([-1.5, -0.5, 0.5, 1.5], dtype=np.float32)
REF_VERSION = 1.0
OUR_VERSION = 2.0
MAX_BLOCK = 4096


@dataclass
class SQINT2Config:
    group_size: int = 32
    seed: int = 42
    refine_iters: int = 1
    residual_rank: int = 0
    residual_factor_dtype: str = "fp16"

    def __post_init__(self) -> None:
        if self.group_size < 4 or self.group_size % 4:
            raise ValueError(f"group_size must be a positive multiple of 4, got {self.group_size}")
        if self.refine_iters < 0 or self.residual_rank < 0:
            raise ValueError("refine_iters and residual_rank must be >= 0")
        if self.residual_factor_dtype not in ("fp16", "fp32"):
            raise ValueError("residual_factor_dtype must be fp16 or fp32")


# ------------------------------------------------------------------------------ rotation
def rotation_block(k: int) -> int:
    b = k & -k  # largest power of two dividing k
    return min(b, MAX_BLOCK)


def rotation_signs(k: int, seed: int) -> torch.Tensor:
    """+-1 float32 [k]: bit 63 of SplitMix64(seed + 1 + j * golden) per position j."""
    j = torch.arange(k, dtype=torch.int64)
    z = j * -7046029254386353131 + (seed + 1)

    def shr(v, n):
        return (v >> n) & ((1 << (64 - n)) - 1)

    z = (z ^ shr(z, 30)) * -4658895280553007687
    z = (z ^ shr(z, 27)) * -7723592293110705685
    z = z ^ shr(z, 31)
    return torch.where(z < 0, -1.0, 1.0).float()


def fwht_blocks(x: torch.Tensor, b: int) -> torch.Tensor:
    """Unnormalised Sylvester Walsh-Hadamard transform of every length-b block of the last dim."""
    shape = x.shape
    k = shape[-1]
    y = x.reshape(-1, k // b, b)
    h = 1
    while h < b:
        y = y.reshape(y.shape[0], k // b, b // (2 * h), 2, h)
        a, c = y[..., 0, :], y[..., 1, :]
        y = torch.stack([a + c, a - c], dim=-2)
        h *= 2
    return y.reshape(shape)


def rotate(x: torch.Tensor, signs: torch.Tensor, b: int) -> torch.Tensor:
    """R x = blockdiag(H_b / sqrt(b)) (signs * x) along the last dim (torch; any device)."""
    if x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2:
        from .._ext import native

        return native().hadamard_rows(x.contiguous(), signs.to(x.device).float().contiguous(), b)
    return fwht_blocks(x.float() * signs.to(x.device), b) / math.sqrt(b)


def unrotate(x: torch.Tensor, signs: torch.Tensor, b: int) -> torch.Tensor:
    """R^T x = signs * (blockdiag(H_b / sqrt(b)) x) (H is symmetric)."""
    return fwht_blocks(x.float(), b) / math.sqrt(b) * signs.to(x.device)


# ------------------------------------------------------------------------------ NF2
def nf2_quantise_groups(groups: torch.Tensor, refine_iters: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(M, gs) float -> (indices uint8 (M, gs), scale (M,), zp (M,)) with the reference's rules."""
    g = groups.float()
    xmin, xmax = g.amin(1), g.amax(1)
    span = xmax - xmin
    safe = span > 0
    scale = torch.where(safe, span / 3.0, torch.ones_like(span))
    zp = torch.where(safe, -1.5 - xmin / scale, torch.zeros_like(span))
    resc = g / scale[:, None] + zp[:, None]
    cb = torch.tensor(NF2_VALUES, device=g.device)

    def assign(c):
        return (resc[..., None] - c).abs().argmin(-1)

    idx = assign(cb)
    for _ in range(refine_iters):
        new = cb.clone()
        fr, fi = resc.reshape(-1), idx.reshape(-1)
        for k in range(4):
            m = fi == k
            if bool(m.any()):
                new[k] = fr[m].mean()
        cb = new.sort().values
        idx = assign(cb)
    if refine_iters > 0:
        lo, hi = float(cb[0]), float(cb[-1])
        if hi - lo > 0:
            new_scale = (hi - lo) / 3.0 * scale
            ok = new_scale > 0
            dec_lo = (lo - zp) * scale
            zp = torch.where(ok, -1.5 - dec_lo / torch.where(ok, new_scale, torch.ones_like(new_scale)), zp)
            scale = torch.where(ok, new_scale, scale)
    const = ~safe
    if bool(const.any()):
        idx[const] = 1
        scale = torch.where(const, torch.ones_like(scale), scale)
        zp = torch.where(const, -0.5 - xmin, zp)
    return idx.to(torch.uint8), scale, zp


def _pack2(idx: torch.Tensor) -> torch.Tensor:
    i = idx.to(torch.int64).reshape(idx.shape[0], -1, 4)
    return (i[..., 0] | (i[..., 1] << 2) | (i[..., 2] << 4) | (i[..., 3] << 6)).to(torch.uint8)


def _unpack2(p: torch.Tensor, cols: int) -> torch.Tensor:
    q = p.to(torch.int64)
    return torch.stack([(q >> (2 * j)) & 3 for j in range(4)], -1).reshape(p.shape[0], -1)[:, :cols]


# ------------------------------------------------------------------------------ compress
def compress_weight(w: torch.Tensor, cfg: SQINT2Config | None = None) -> QTensor:
    """A weight [N, K] -> an INT2 ``q2`` QTensor in the rotated frame, carrying the rotation
    (``extra['rot_signs']``, ``extra['rot_block']``) and, with ``residual_rank``, the low-rank
    residual factors (``extra['sq_L']`` [N, r], ``extra['sq_R']`` [r, K])."""
    cfg = cfg or SQINT2Config()
    n, k = w.shape
    if k % cfg.group_size:
        raise ValueError(f"input width {k} is not a multiple of the group size {cfg.group_size}")
    b = rotation_block(k)
    signs = rotation_signs(k, cfg.seed)
    wr = fwht_blocks(w.float() * signs.to(w.device), b) / math.sqrt(b)
    grp = wr.reshape(-1, cfg.group_size)
    idx, scale, zp = nf2_quantise_groups(grp, cfg.refine_iters)
    gpr = k // cfg.group_size
    s = scale.reshape(n, gpr)
    z = ((-1.5 - zp) * scale).reshape(n, gpr)  # affine form: x = z + q * s
    extra = {"rot_signs": signs, "rot_block": b, "seed": cfg.seed}
    if cfg.residual_rank > 0:
        deq = (z.repeat_interleave(cfg.group_size, 1) + idx.reshape(n, k).float() * s.repeat_interleave(
            cfg.group_size, 1))
        U, S, Vh = torch.linalg.svd(wr - deq, full_matrices=False)
        r = min(cfg.residual_rank, S.numel())
        dt = torch.float16 if cfg.residual_factor_dtype == "fp16" else torch.float32
        extra["sq_L"] = (U[:, :r] * S[:r]).to(dt).cpu()
        extra["sq_R"] = Vh[:r].to(dt).cpu()
    return QTensor("q2", (n, k), packed=_pack2(idx.reshape(n, k)).cpu(), scales=s.float().cpu(),
                   offsets=z.float().cpu(), group=cfg.group_size, extra=extra)


def is_rotated(t: QTensor) -> bool:
    return bool(t.extra) and "rot_signs" in t.extra


def dequantize_rotated(t: QTensor, base: torch.Tensor) -> torch.Tensor:
    """Original-frame weights from the rotated-frame dequantisation ``base`` [N, K]."""
    wr = base.float()
    if "sq_L" in t.extra:
        wr = wr + t.extra["sq_L"].float() @ t.extra["sq_R"].float()
    return unrotate(wr, t.extra["rot_signs"], int(t.extra["rot_block"]))


# ------------------------------------------------------------------------------ files
def _ref_hadamard(dim: int, rng: np.random.Generator) -> np.ndarray:
    """The reference's rotation construction (sqint2.py:384-420), needed to decode its files."""
    if dim & (dim - 1) == 0:
        h = np.array([[1.0]], dtype=np.float32)
        while h.shape[0] < dim:
            h = np.block([[h, h], [h, -h]])
        h /= np.sqrt(dim)
        return (h * rng.choice([-1.0, 1.0], size=(dim,)).astype(np.float32)[None, :]).astype(np.float32)
    q, _ = np.linalg.qr(rng.standard_normal((dim, dim)).astype(np.float32))
    return q.astype(np.float32)


def write_files(name_key: str, t: QTensor) -> dict[str, np.ndarray]:
    """npy-dir files of a rotated ``q2`` tensor in the SQINT2 file set (format version 2)."""
    n, k = t.shape
    s = t.scales.float().numpy()
    zp = (-1.5 - t.offsets.float().numpy() / s).astype(np.float32)
    meta = np.zeros(16, dtype=np.float64)
    meta[0], meta[1], meta[2], meta[3] = OUR_VERSION, k, n, t.group
    meta[4] = float(t.extra.get("seed", 42))
    meta[6], meta[7] = 0.0, 1.0  # right (input) rotation only
    meta[11] = float(t.extra["rot_block"])
    out = {f"{name_key}__sqint2_idx": t.packed.numpy().astype(np.uint8), f"{name_key}__sqint2_scales": s,
           f"{name_key}__sqint2_zp": zp, f"{name_key}__sqint2_meta": meta,
           f"{name_key}__shape": np.asarray(t.shape, dtype=np.int64)}
    if "sq_L" in t.extra:
        meta[8] = t.extra["sq_L"].shape[1]
        meta[9] = 1.0 if t.extra["sq_L"].dtype == torch.float16 else 0.0
        out[f"{name_key}__sqint2_L"] = t.extra["sq_L"].numpy()
        out[f"{name_key}__sqint2_R"] = t.extra["sq_R"].numpy()
    return out


def read_files(load, key: str, shape) -> QTensor:
    """A SQINT2 tensor from its files (``load(suffix)`` returns the array). Version-2 files
    become rotated ``q2`` tensors; reference (version-1) files are decoded with the reference's
    rotations and returned dense (the engine re-encodes them INT4)."""
    meta = np.asarray(load("__sqint2_meta"), dtype=np.float64)
    ver = float(meta[0])
    k, n, gs, seed = int(meta[1]), int(meta[2]), int(meta[3]), int(meta[4])
    idx_packed = torch.from_numpy(np.array(load("__sqint2_idx"), dtype=np.uint8))
    scales = np.array(load("__sqint2_scales"), dtype=np.float32)
    zp = np.array(load("__sqint2_zp"), dtype=np.float32)
    rank = int(meta[8])
    L = R = None
    if rank > 0:
        L = torch.from_numpy(np.array(load("__sqint2_L"))).float()
        R = torch.from_numpy(np.array(load("__sqint2_R"))).float()
    if ver == OUR_VERSION:
        b = int(meta[11])
        s = torch.from_numpy(scales)
        z = torch.from_numpy((-1.5 - zp) * scales)
        extra = {"rot_signs": rotation_signs(k, seed), "rot_block": b, "seed": seed}
        if L is not None:
            extra["sq_L"], extra["sq_R"] = L, R
        return QTensor("q2", (n, k), packed=idx_packed, scales=s, offsets=z, group=gs, extra=extra)
    if ver != REF_VERSION:
        raise ValueError(f"unsupported SQINT2 file version {ver}")
    k_pad = -(-k // gs) * gs
    idx = _unpack2(idx_packed, k_pad).numpy()
    wr = ((NF2_VALUES[idx].reshape(n, -1, gs) - zp[:, :, None]) * scales[:, :, None]).reshape(n, k_pad)
    if L is not None:
        wr = wr + (L @ R).numpy()
    if meta[10] > 0:  # sparse COO corrections
        try:
            rows, cols, vals = load("__sqint2_srows"), load("__sqint2_scols"), load("__sqint2_svals")
            wr = wr.copy()
            wr[np.asarray(rows), np.asarray(cols)] += np.asarray(vals, dtype=np.float32)
        except FileNotFoundError:
            pass
    hl = _ref_hadamard(n, np.random.default_rng(seed)) if meta[6] else None
    hr = _ref_hadamard(k_pad, np.random.default_rng(seed + 1)) if meta[7] else None
    w = wr.astype(np.float32)
    if hl is not None:
        w = hl.T @ w
    if hr is not None:
        w = w @ hr
    w = torch.from_numpy(np.ascontiguousarray(w[:, :k]))
    return QTensor("dense", tuple(shape) if shape else (n, k), data=w)


def snr_db(w: torch.Tensor, w_hat: torch.Tensor) -> float:
    noise = float(((w.float() - w_hat.float()) ** 2).mean()) + 1e-20
    return 10.0 * math.log10(float((w.float() ** 2).mean()) / noise)


def save_layer(t: QTensor, tensor_dir: str | Path, key: str) -> None:
    for suf, a in write_files(key, t).items():
        np.save(str(Path(tensor_dir) / f"{suf}.npy"), a)
