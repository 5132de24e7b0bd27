"""Weight codecs of the npy-dir format (quantize / dequantize), on top of the C++ CPU kernels.

Each codec restates a reference quantizer (squish_quant_rs/src/lib.rs, squish/quant/*):
INT8 symmetric, INT4 asymmetric (+ MSE clip search), INT4 symmetric legacy, NF4, INT3
(8 values per 3 bytes, with the optional low-rank compensator of MiLo), INT2 asymmetric,
and AQLM additive codebooks (quant/aqlm.py).
"""
from __future__ import annotations

import numpy as np
import torch

from .._ext import native
from ..models.weights import QTensor


def dequantize_qtensor(t: QTensor) -> torch.Tensor:
    C = native().cpu
    k = t.kind
    if k == "q4a":
        w = C.dequantize_int4_asym(t.packed.cpu(), t.scales.cpu().float(), t.offsets.cpu().float(), t.group)
        if t.extra and "rot_signs" in t.extra:  # QuaRot: stored in the rotated frame
            from .sqint2 import unrotate

            w = unrotate(w, t.extra["rot_signs"], int(t.extra["rot_block"]))
        return w
    if k == "nf4":
        lv = (t.extra or {}).get("levels")
        if lv is not None:  # any4: codes index a learned 16-level table
            p = t.packed.cpu()
            codes = torch.stack([p & 0xF, p >> 4], dim=-1).reshape(p.shape[0], -1).long()
            # the GEMM multiplies bf16 levels by bf16 scales: match its table precision
            levels = lv.float().cpu().to(torch.bfloat16).float()
            return levels[codes] * t.scales.cpu().float().repeat_interleave(t.group, dim=1)[:, : codes.shape[1]]
        return C.dequantize_nf4(t.packed.cpu(), t.scales.cpu().float(), t.group)
    if k == "q8":
        return C.dequantize_int8(t.packed.cpu(), t.scales.cpu().float())
    if k == "fp8":
        return C.dequantize_fp8(t.packed.cpu().contiguous(), t.scales.cpu().float().contiguous(), 0)
    if k == "q2":
        w = C.dequantize_int2(t.packed.cpu(), t.scales.cpu().float(), t.offsets.cpu().float(), t.group)
        if t.extra and "rot_signs" in t.extra:  # SQINT2: stored in the rotated frame
            from .sqint2 import dequantize_rotated

            w = dequantize_rotated(t, w)
        return w
    if k == "q3":
        w = C.unpack_int3(t.packed.cpu(), t.scales.cpu().float(), t.group, t.shape[-1])
        if t.offsets is not None:
            w = w + t.offsets.cpu().float().repeat_interleave(t.group, dim=1)[:, : w.shape[1]]
        ex = t.extra or {}
        if "lra" in ex:  # low-rank compensator: W += A @ B
            w = w + ex["lra"].float() @ ex["lrb"].float()
        return w
    if k == "aqlm":
        from .aqlm import aqlm_dequantize

        return aqlm_dequantize(t)
    raise ValueError(f"unknown tensor kind {k!r}")


_GPU_CODEC = {"q8": 0, "nf4": 2, "q3": 3, "q2": 4, "fp8": 5}
_FP8 = {"e4m3": (0, 5, 448.0), "e5m2": (1, 6, 57344.0)}


def quantize_fp8(w: torch.Tensor, fmt: str = "e4m3", group: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """FP8 codes (uint8) and fp32 scales of a 2-D tensor: one scale for the whole tensor
    (``group=0``: absmax / largest finite, the reference's quantize_fp8_e4m3_f32 /
    quantize_fp8_e5m2_f32, squish_quant_rs/src/lib.rs:1012-1091) or one per ``group`` columns.
    Codes round to nearest even and saturate (the hardware cvt.rn.satfinite conversion); CUDA
    tensors are encoded by the GPU kernel, others by the C++ CPU library, bit-identically."""
    cpu_fmt, codec, fmax = _FP8[fmt]
    x = w.detach()
    fixed = 0.0
    g = group if group > 0 else x.shape[1]
    if group <= 0:
        am = float(x.abs().max()) if x.numel() else 0.0
        fixed = 1.0 if am == 0.0 else am / fmax
    if x.is_cuda:
        x = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
        return tuple(native().quantize_codec(x.contiguous(), codec, g, fixed))
    return tuple(native().cpu.quantize_fp8(x.float().contiguous(), cpu_fmt, g, fixed))


_FP6 = {"e3m2": (3, 2), "e2m3": (2, 3)}


def fp6_encode(x: torch.Tensor, fmt: str = "e3m2") -> torch.Tensor:
    """Pack a float tensor (numel a multiple of 4) as FP6 codes, 4 values per 3 bytes (the
    reference's fp6_encode_f32 layout, squish_quant_rs/src/lib.rs:2410); no scaling."""
    e, m = _FP6[fmt]
    return native().cpu.fp6_encode(x.detach().float().cpu().reshape(-1).contiguous(), e, m)


def fp6_decode(packed: torch.Tensor, n: int, fmt: str = "e3m2") -> torch.Tensor:
    e, m = _FP6[fmt]
    return native().cpu.fp6_decode(packed.cpu().contiguous(), n, e, m)


def quantize_fp6(w: torch.Tensor, fmt: str = "e3m2", group: int = 32) -> tuple[torch.Tensor, torch.Tensor]:
    """FP6 with one fp32 scale per ``group`` values of each row (absmax / largest FP6 value):
    (packed bytes, scales [rows, cols / group])."""
    e, m = _FP6[fmt]
    fmax = (1 + ((1 << m) - 1) / (1 << m)) * 2.0 ** ((1 << e) - 1 - ((1 << (e - 1)) - 1))
    x = w.detach().float().cpu()
    r, c = x.shape
    if c % group or group % 4:
        raise ValueError("group must divide the row and be a multiple of 4")
    g = x.reshape(r, c // group, group)
    am = g.abs().amax(-1)
    sc = torch.where(am > 0, am / fmax, torch.ones_like(am))
    return fp6_encode((g / sc[..., None]).reshape(-1), fmt), sc


def dequantize_fp6(packed: torch.Tensor, scales: torch.Tensor, shape: tuple, fmt: str = "e3m2") -> torch.Tensor:
    r, c = shape
    g = c // scales.shape[1]
    return (fp6_decode(packed, r * c, fmt).reshape(r, c // g, g) * scales.float()[..., None]).reshape(r, c)


def dequantize_fp8(codes: torch.Tensor, scales: torch.Tensor, fmt: str = "e4m3") -> torch.Tensor:
    """fp32 reconstruction of :func:`quantize_fp8` output (on the CPU)."""
    sc = scales.float().cpu()
    if sc.dim() < 2:
        sc = sc.reshape(1, 1).expand(codes.shape[0], 1)
    return native().cpu.dequantize_fp8(codes.cpu().contiguous(), sc.contiguous(), _FP8[fmt][0])


def quantize(w: torch.Tensor, kind: str, group: int, mse_clip: bool = False, hqq: bool = False,
             hqq_iters: int = 10) -> QTensor:
    """Quantize a 2-D weight to ``kind`` (q4a | q8 | fp8 | nf4 | any4 | quarot | q2 | sqint2 | q3 | aqlm |
    dense).
    ``hqq``: refine the INT4 / INT2 affine grids by half-quadratic quantization (quant/hqq.py)."""
    from ..models.weights import pick_group, quantize_q4a

    C = native().cpu
    if hqq and kind in ("q4a", "q2"):
        from .hqq import HQQConfig, HQQTensor, hqq_quantize

        g = pick_group(w.shape[1], group)
        lv = 16 if kind == "q4a" else 4
        codes, sc, z = hqq_quantize(w.detach() if w.is_cuda else w.detach().float(), g, lv, 1.0, hqq_iters)
        ht = HQQTensor(codes.cpu().numpy(), sc.float().cpu().numpy(), z.float().cpu().numpy(), tuple(w.shape),
                       HQQConfig(bits=4 if kind == "q4a" else 2, group_size=g, max_iter=hqq_iters))
        return ht.to_qtensor(kind)
    if kind == "q4a":
        return quantize_q4a(w, group, mse_clip)
    if kind == "sqint2":
        from .sqint2 import SQINT2Config, compress_weight

        return compress_weight(w.detach(), SQINT2Config(group_size=pick_group(w.shape[1], group)))
    if kind == "dense":
        return QTensor("dense", tuple(w.shape), data=w)
    g = pick_group(w.shape[1], group)
    if w.is_cuda and kind in _GPU_CODEC:
        # the GPU quantizers (csrc/quantize.cu) produce the CPU library's layouts bit for bit
        out = native().quantize_codec(w.detach().contiguous() if w.dtype in (torch.float32, torch.bfloat16)
                                      else w.detach().float().contiguous(), _GPU_CODEC[kind], g, 0.0)
        out = [t.cpu() for t in out]
        if kind == "q2":
            return QTensor("q2", tuple(w.shape), packed=out[0], scales=out[1], offsets=out[2], group=g)
        return QTensor(kind, tuple(w.shape), packed=out[0], scales=out[1], group=g)
    wf = w.detach().float().cpu().contiguous()
    if kind == "q8":
        q, s = C.quantize_int8(wf, g)
        return QTensor("q8", tuple(wf.shape), packed=q, scales=s, group=g)
    if kind == "fp8":
        q, s = C.quantize_fp8(wf, 0, g, 0.0)
        return QTensor("fp8", tuple(wf.shape), packed=q, scales=s, group=g)
    if kind == "nf4":
        p, s = C.quantize_nf4(wf, g)
        return QTensor("nf4", tuple(wf.shape), packed=p, scales=s, group=g)
    if kind == "any4":
        from .research import quantize_any4

        return quantize_any4(wf, g)
    if kind == "quarot":
        from .research import quarot_quantize
        from .sqint2 import rotation_block

        return quarot_quantize(wf, g, bits=4, block=rotation_block(wf.shape[1]))
    if kind == "q2":
        p, s, z = C.quantize_int2(wf, g)
        return QTensor("q2", tuple(wf.shape), packed=p, scales=s, offsets=z, group=g)
    if kind == "q3":
        p, s = C.pack_int3(wf, g)
        return QTensor("q3", tuple(wf.shape), packed=p, scales=s, group=g)
    if kind == "aqlm":
        from .aqlm import aqlm_quantize

        return aqlm_quantize(wf)
    raise ValueError(f"unknown quantization kind {kind!r}")
