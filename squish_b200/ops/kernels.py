"""Python wrappers of the native kernels.

Every wrapper launches on the current CUDA stream and allocates nothing when the
caller provides the output: scratch memory (split-K partials, tile counters, the
decode split partials, the sampler's fp32 row buffer) lives in a per-device
:class:`Workspace`, so whole decode steps can be captured in CUDA graphs.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np
import torch

from .._ext import native

# KV page formats understood by the attention kernels (csrc/kv_format.cuh)
KV_FORMATS = {"bf16": (0, 0), "int8": (1, 1), "int4": (2, 2), "int2": (3, 3), "k8v4": (4, 5)}
KV_BITS = {0: 16, 1: 8, 2: 4, 3: 2, 4: 8, 5: 4}
KV_ASYM = {4, 5}


class Workspace:
    """Per-device scratch buffers shared by all kernels of one stream."""

    GEMM_WS_FLOATS = 12 * 1024 * 1024
    GEMM_COUNTERS = 1 << 16

    def __init__(self, device: torch.device):
        self.device = device
        self.gemm_ws = torch.empty(self.GEMM_WS_FLOATS, dtype=torch.float32, device=device)
        self.gemm_counters = torch.zeros(self.GEMM_COUNTERS, dtype=torch.int32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self._attn_o = torch.empty(0, dtype=torch.float32, device=device)
        self._attn_lse = torch.empty(0, dtype=torch.float32, device=device)
        self._sampler = torch.empty(0, dtype=torch.float32, device=device)
        self._dq = torch.empty(0, dtype=torch.bfloat16, device=device)  # expanded weights (large-M GEMMs)
        self._rot = torch.empty(0, dtype=torch.bfloat16, device=device)  # rotated activations (SQINT2)
        # set once a CUDA graph has captured these buffers: growing one then would leave the
        # graph writing to freed memory, so it becomes an error instead
        self.frozen = False

    def _grow_check(self, what: str) -> None:
        if self.frozen:
            raise RuntimeError(f"workspace {what} buffer would grow after CUDA-graph capture; reserve it up front")

    def attn_buffers(self, b: int, hq: int, splits: int, d: int):
        need = b * hq * splits * d
        if self._attn_o.numel() < need or self._attn_lse.numel() < need // d:
            self._grow_check("attention")
            self._attn_o = torch.empty(max(need, 1 << 20), dtype=torch.float32, device=self.device)
            self._attn_lse = torch.empty(max(need // d, 1 << 16), dtype=torch.float32, device=self.device)
        return self._attn_o, self._attn_lse

    def reserve_attn(self, b: int, hq: int, splits: int, d: int):
        self.attn_buffers(b, hq, splits, d)

    def sampler_buffer(self, rows: int, vocab: int):
        need = rows * vocab
        if self._sampler.numel() < need:
            self._grow_check("sampler")
            self._sampler = torch.empty(need, dtype=torch.float32, device=self.device)
        return self._sampler

    def dq_buffer(self, elems: int) -> torch.Tensor | None:
        """bf16 scratch for one expanded weight matrix; None if it would have to grow after capture."""
        if self._dq.numel() < elems:
            if self.frozen:
                return None
            self._dq = torch.empty(elems, dtype=torch.bfloat16, device=self.device)
        return self._dq

    def rot_buffer(self, m: int, k: int) -> torch.Tensor:
        """bf16 [m, k] scratch for Hadamard-rotated activations (one linear at a time)."""
        if self._rot.numel() < m * k:
            self._grow_check("rotation")
            self._rot = torch.empty(m * k, dtype=torch.bfloat16, device=self.device)
        return self._rot[: m * k].view(m, k)

    def check(self) -> None:
        """Raise if any kernel recorded an error: a bounded wait that timed out (1-5) or an
        index outside its pool (6: a KV page or cache slot; the access was skipped)."""
        code = int(self.status.item())
        if code != 0:
            self.status.zero_()
            what = "index outside its pool" if code == 6 else "bounded wait timed out"
            raise RuntimeError(f"squish_b200 kernel reported status {code} ({what})")


_WORKSPACES: dict[int, Workspace] = {}

# Number of this package's kernels launched from Python (a CUDA-graph replay adds the
# count recorded while it was captured). Read by the benchmark as its launch count.
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


def workspace(device: torch.device | None = None) -> Workspace:
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _WORKSPACES.get(idx)
    if ws is None:
        ws = Workspace(torch.device("cuda", idx))
        _WORKSPACES[idx] = ws
    return ws


@dataclass
class Int4Weight:
    """An INT4 asymmetric group-quantized weight in the tile-major device layout."""

    wq: torch.Tensor  # int32 [Np/128, KB, 1024 + gpk*128]: nibbles then (scale, zero) pairs per tile
    sz: torch.Tensor  # unused (empty)
    n: int
    k: int
    group: int
    bias: torch.Tensor | None = None
    fmt: int = 0  # WF_INT4 | WF_NF4 | WF_INT8 | WF_INT2 | WF_INT3 | WF_AQLM | WF_FP8
    codebook: torch.Tensor | None = None  # WF_AQLM: [books, 256, 8] bf16; WF_NF4 (any4): [16] bf16 levels
    # optional resident bf16 expansion [n, 64 * ceil(k / 64)] for large-M GEMMs (the exact
    # values the quantized GEMM computes with); None = expand per call
    dense: torch.Tensor | None = None
    # SQINT2: the weight is stored rotated (W R^T) and the input is rotated first,
    # R x = blockdiag(H_b / sqrt(b)) (rot * x) (csrc/hadamard.cu)
    rot: torch.Tensor | None = None  # float32 [k] signs
    rot_block: int = 0
    # low-rank residual W += A B (MiLo INT3 compensator; SQINT2 residual in the rotated frame):
    # y += (x B^T) A^T after the GEMM, on the (rotated) input, before any SiLU*up epilogue
    lr_a: torch.Tensor | None = None  # [n, r] (rows in the weight's row order)
    lr_b: torch.Tensor | None = None  # [r, k]

    @property
    def nbytes(self) -> int:
        return self.wq.numel() * 4 + self.sz.numel() * 4


def prepare_int4_weight(packed: torch.Tensor, scales: torch.Tensor, offsets: torch.Tensor, k: int, group: int,
                        device, bias: torch.Tensor | None = None) -> Int4Weight:
    """Upload an npy-dir INT4 asymmetric weight (``__q4a/__s4a/__z4a``) and repack it on the GPU."""
    dev = torch.device(device)
    p = packed.to(dev, torch.uint8).contiguous()
    s = scales.to(dev, torch.float32).contiguous()
    z = offsets.to(dev, torch.float32).contiguous()
    wq, sz = native().repack_int4(p, s, z, int(k), int(group))
    b = None if bias is None else bias.to(dev, torch.bfloat16).contiguous()
    return Int4Weight(wq=wq, sz=sz, n=int(packed.shape[0]), k=int(k), group=int(group), bias=b)


WF_INT4, WF_NF4, WF_INT8, WF_INT2, WF_INT3, WF_AQLM, WF_FP8 = 0, 1, 2, 3, 4, 5, 6
_NIB_POS = (0, 16, 4, 20, 8, 24, 12, 28)  # bit of value j in an 8-value word (pairs share a 16-bit shift)


def _bf16_bits(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).view(torch.int16).to(torch.int64) & 0xFFFF


def repack_codes(codes: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, k: int, group: int,
                 fmt: int) -> torch.Tensor:
    """Tile-major device layout of a quantized weight for the GEMM kernel, any WF_* format.

    ``codes`` (N, K) holds one code per weight (uint8: INT4 / NF4 index 0..15, INT2 0..3,
    INT8 two's complement). Per (128-row block, 64-column k-block) tile: the codes as
    [2 halves][128 rows][32 values] packed into words (INT4/NF4: 8 per word in the kernel's
    interleaved nibble order; INT2: 16 per word, value 2e at bit 2e and 2e+1 at 16+2e; INT8:
    4 bytes little-endian), then (scale | zero << 16) bf16 pairs [groups per k-block][128].
    Padding rows and columns get zero scales, so they dequantize to 0.
    """
    dev = codes.device
    n = codes.shape[0]
    npad = (n + 255) // 256 * 256
    kb = (k + 63) // 64
    kp = kb * 64
    gpk = 1 if group >= 64 else 64 // group
    c = torch.zeros(npad, kp, dtype=torch.int64, device=dev)
    c[:n, :k] = codes[:, :k].to(torch.int64) & 0xFF
    v = c.view(npad // 128, 128, kb, 2, 32).permute(0, 2, 3, 1, 4)  # [rb, kb, half, row, 32]
    if fmt in (WF_INT4, WF_NF4):
        pos = torch.tensor(_NIB_POS, dtype=torch.int64, device=dev)
        words = (v.reshape(*v.shape[:4], 4, 8) << pos).sum(-1)
    elif fmt == WF_INT2:
        j = torch.arange(16, device=dev)
        pos = (j % 2) * 16 + (j // 2) * 2
        words = (v.reshape(*v.shape[:4], 2, 16) << pos).sum(-1)
    elif fmt in (WF_INT8, WF_FP8):
        pos = torch.arange(4, device=dev) * 8
        words = (v.reshape(*v.shape[:4], 8, 4) << pos).sum(-1)
    elif fmt == WF_INT3:
        # pair p < 15 in word p // 5 at bits 3(p%5) / 16 + 3(p%5); pair 15 bit-sliced over bits 15 / 31
        ws = []
        for q in range(3):
            acc = torch.zeros_like(v[..., 0])
            for k in range(5):
                pp = 5 * q + k
                acc = acc | (v[..., 2 * pp] << (3 * k)) | (v[..., 2 * pp + 1] << (16 + 3 * k))
            acc = acc | (((v[..., 30] >> q) & 1) << 15) | (((v[..., 31] >> q) & 1) << 31)
            ws.append(acc)
        words = torch.stack(ws, dim=-1)
    elif fmt == WF_AQLM:
        # v holds 32 index bytes per (half, row): 8 groups x 2 books ... packed 4 per word
        pos = torch.arange(4, device=dev) * 8
        words = (v[..., :8].reshape(*v.shape[:4], 2, 4) << pos).sum(-1)
    else:
        raise ValueError(f"unknown weight format {fmt}")
    words = words.reshape(npad // 128, kb, -1)
    g_n = scales.shape[1]
    cols = torch.arange(kb, device=dev)[:, None] * 64 + torch.arange(gpk, device=dev)[None, :] * (64 // gpk)
    gi = torch.clamp(cols // group, max=g_n - 1).reshape(-1)  # [kb * gpk]
    s = torch.zeros(npad, g_n, dtype=torch.float32, device=dev)
    s[:n] = scales.float()
    z = torch.zeros_like(s)
    if zeros is not None:
        z[:n] = zeros.float()
    aux = _bf16_bits(s[:, gi]) | (_bf16_bits(z[:, gi]) << 16)  # [npad, kb*gpk]
    aux = aux.view(npad // 128, 128, kb, gpk).permute(0, 2, 3, 1).reshape(npad // 128, kb, gpk * 128)
    tile = torch.cat([words, aux], dim=-1)
    tile = torch.where(tile >= 2**31, tile - 2**32, tile)
    return tile.to(torch.int32).contiguous()


def _lowrank_factors(t, dev):
    """(A [n, r], B [r, k]) bf16 on the device of a MiLo (``lra``/``lrb``) or SQINT2 residual
    (``sq_L``/``sq_R``) weight, else (None, None)."""
    ex = t.extra or {}
    for a, b in (("lra", "lrb"), ("sq_L", "sq_R")):
        if a in ex and ex[a] is not None and ex[a].numel():
            return (ex[a].to(dev, torch.float32).to(torch.bfloat16).contiguous(),
                    ex[b].to(dev, torch.float32).to(torch.bfloat16).contiguous())
    return None, None


def prepare_weight(t, device, bias: torch.Tensor | None = None) -> Int4Weight:
    """A QTensor in the GEMM's device layout: INT4 asymmetric (repacked on the GPU), NF4,
    INT8 or INT2 (repacked with tensor ops) in their own code formats."""
    dev = torch.device(device)
    k = int(t.shape[1])
    b = None if bias is None else bias.to(dev, torch.bfloat16).contiguous()
    if t.kind == "q4a":
        w = prepare_int4_weight(t.packed, t.scales, t.offsets, k, t.group, dev)
        w.bias = b
        if t.extra and "rot_signs" in t.extra:  # QuaRot: stored rotated, the input is rotated first
            w.rot = t.extra["rot_signs"].to(dev, torch.float32).contiguous()
            w.rot_block = int(t.extra["rot_block"])
        return w
    p = t.packed.to(dev)
    if t.kind == "nf4":
        codes = torch.stack([p & 0xF, p >> 4], dim=-1).reshape(p.shape[0], -1)
        wt = repack_codes(codes, t.scales.to(dev), None, k, t.group, WF_NF4)
        lv = (t.extra or {}).get("levels")
        if lv is not None:  # any4: a learned 16-level table in place of the NormalFloat levels
            return Int4Weight(wq=wt, sz=torch.empty(0, dtype=torch.int32, device=dev), n=int(t.shape[0]), k=k,
                              group=int(t.group), bias=b, fmt=WF_NF4,
                              codebook=lv.to(dev, torch.float32).to(torch.bfloat16).contiguous())
        fmt = WF_NF4
    elif t.kind == "q8":
        wt = repack_codes(p.view(torch.uint8), t.scales.to(dev), None, k, t.group, WF_INT8)
        fmt = WF_INT8
    elif t.kind == "fp8":
        wt = repack_codes(p.view(torch.uint8), t.scales.to(dev), None, k, t.group, WF_FP8)
        fmt = WF_FP8
    elif t.kind == "q2":
        codes = torch.stack([(p >> (2 * i)) & 3 for i in range(4)], dim=-1).reshape(p.shape[0], -1)
        wt = repack_codes(codes, t.scales.to(dev), t.offsets.to(dev), k, t.group, WF_INT2)
        fmt = WF_INT2
        if t.extra and "rot_signs" in t.extra:
            lr = _lowrank_factors(t, dev)
            return Int4Weight(wq=wt, sz=torch.empty(0, dtype=torch.int32, device=dev), n=int(t.shape[0]), k=k,
                              group=int(t.group), bias=b, fmt=fmt,
                              rot=t.extra["rot_signs"].to(dev, torch.float32).contiguous(),
                              rot_block=int(t.extra["rot_block"]), lr_a=lr[0], lr_b=lr[1])
    elif t.kind == "q3":
        lr = _lowrank_factors(t, dev)
        bb = p.to(torch.int64).view(p.shape[0], -1, 3)
        bits = bb[..., 0] | (bb[..., 1] << 8) | (bb[..., 2] << 16)  # 8 codes of 3 bits
        q = torch.stack([(bits >> (3 * j)) & 7 for j in range(8)], dim=-1).reshape(p.shape[0], -1)[:, :k]
        u = torch.where(q >= 4, q - 8, q) + 4  # two's complement code -> q + 4 in [0, 7]
        z = t.offsets.to(dev) if t.offsets is not None else None
        wt = repack_codes(u, t.scales.to(dev), z, k, t.group, WF_INT3)
        return Int4Weight(wq=wt, sz=torch.empty(0, dtype=torch.int32, device=dev), n=int(t.shape[0]), k=k,
                          group=int(t.group), bias=b, fmt=WF_INT3, lr_a=lr[0], lr_b=lr[1])
    elif t.kind == "aqlm":
        cb = t.scales.float()
        scale, size, gs = float(cb[0]), int(cb[1]), int(cb[2])
        idx = t.packed.to(dev).long()  # [N, groups, books]
        books = idx.shape[2]
        if gs != 8 or books > 2 or size > 256:
            raise ValueError("AQLM GEMM format needs 8-column groups, <= 2 books of <= 256 codes")
        n_rows, groups = idx.shape[0], idx.shape[1]
        b2 = torch.zeros(n_rows, groups, 2, dtype=torch.int64, device=dev)
        b2[:, :, :books] = idx
        per_kb = b2.view(n_rows, groups * 2)  # 16 index bytes per 64 columns, (group, book) order
        # repack_codes expects one code per column: spread the 16 bytes of a k-block over the
        # first 8 "columns" of each 32-column half
        kb = (k + 63) // 64
        cols = torch.zeros(n_rows, kb * 64, dtype=torch.int64, device=dev)
        pk = torch.zeros(n_rows, kb * 16, dtype=torch.int64, device=dev)
        pk[:, : per_kb.shape[1]] = per_kb
        pk = pk.view(n_rows, kb, 2, 8)
        cols.view(n_rows, kb, 2, 32)[..., :8] = pk
        sc = torch.full((n_rows, kb), scale, dtype=torch.float32, device=dev)
        wt = repack_codes(cols, sc, None, kb * 64, 64, WF_AQLM)
        cbk = torch.zeros(books, 256, 8, dtype=torch.float32, device=dev)
        cbk[:, :size] = cb[3:].to(dev).view(books, size, gs)
        return Int4Weight(wq=wt, sz=torch.empty(0, dtype=torch.int32, device=dev), n=int(t.shape[0]), k=k, group=64,
                          bias=b, fmt=WF_AQLM, codebook=cbk.to(torch.bfloat16).contiguous())
    else:
        raise ValueError(f"no GEMM code format for weight kind {t.kind!r}")
    return Int4Weight(wq=wt, sz=torch.empty(0, dtype=torch.int32, device=dev), n=int(t.shape[0]), k=k,
                      group=int(t.group), bias=b, fmt=fmt)


def gemm_plan(m: int, n: int, k: int, group: int = 64, fmt: int = 0):
    bn, nt, splits, kps, tiles = native().gemm_plan(m, n, k, group, fmt)
    return {"bn": bn, "nt": nt, "splits": splits, "kb_per_split": kps, "tiles": tiles}


EPI_PLAIN, EPI_SILU_MUL = 0, 1


def w4a16_linear(x: torch.Tensor, w: Int4Weight, out: torch.Tensor | None = None,
                 residual: torch.Tensor | None = None, silu_mul: bool = False,
                 ws: Workspace | None = None, trace: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ dequant(w)^T (+bias) (+residual); with ``silu_mul`` the weight rows are
    interleaved gate/up blocks of 64 and y = silu(gate) * up has N/2 columns."""
    ws = ws or workspace(x.device)
    m = x.shape[0]
    if w.rot is not None:
        x = native().hadamard_rows(x, w.rot, w.rot_block, ws.rot_buffer(m, w.k))
        _count()
    if w.lr_a is not None:
        return _lowrank_linear(x, w, out, residual, silu_mul, ws, trace)
    return _linear_core(x, w, out, residual, silu_mul, ws, trace)


def _lowrank_term(x: torch.Tensor, w: Int4Weight) -> torch.Tensor:
    """(x B^T) A^T in fp32 (two skinny library GEMMs, rank r)."""
    return (x.float() @ w.lr_b.float().T) @ w.lr_a.float().T


def _lowrank_linear(x, w, out, residual, silu_mul, ws, trace):
    """A quantized GEMM plus its low-rank residual. With the SiLU*up epilogue the correction
    must precede the activation: plain GEMM into [m, n], add, then SiLU(gate) * up."""
    m = x.shape[0]
    if not silu_mul:
        y = _linear_core(x, w, out, residual, False, ws, trace)
        y.add_(_lowrank_term(x, w).to(y.dtype))
        return y
    if residual is not None:
        raise ValueError("a residual cannot follow the SiLU*up epilogue")
    full = _linear_core(x, w, None, None, False, ws, trace).float() + _lowrank_term(x, w)
    g, u = full.view(m, w.n // 128, 2, 64).unbind(2)
    act = (torch.nn.functional.silu(g) * u).reshape(m, w.n // 2).to(torch.bfloat16)
    if out is None:
        return act
    out.copy_(act)
    return out


def _linear_core(x, w, out, residual, silu_mul, ws, trace):
    m = x.shape[0]
    ncols = w.n // 2 if silu_mul else w.n
    if out is None:
        out = torch.empty((m, ncols), dtype=torch.bfloat16, device=x.device)
    if m >= DQ_GEMM_MIN_M and trace is None:
        # many token tiles: expand the weights to bf16 once, then a bf16 tensor-core GEMM
        if w.dense is not None:
            return bf16_linear(x, w.dense[:, : w.k], out, w.bias, residual, silu_mul, ws)
        kpad = (w.k + 63) // 64 * 64
        buf = ws.dq_buffer(w.n * kpad)
        if buf is not None:
            wd = dequant_weight(w, buf[: w.n * kpad].view(w.n, kpad))
            return bf16_linear(x, wd[:, : w.k], out, w.bias, residual, silu_mul, ws)
    native().w4a16_gemm(x, w.wq, w.sz, w.n, w.k, w.group, out, w.bias, residual,
                        EPI_SILU_MUL if silu_mul else EPI_PLAIN, ws.gemm_ws, ws.gemm_counters, ws.status, trace,
                        w.fmt, w.codebook)
    _count()
    return out


# Token count from which a quantized linear layer expands its weights to bf16 and runs the bf16
# tensor-core GEMM instead of dequantizing inside the GEMM (measured crossover on B200).
DQ_GEMM_MIN_M = int(os.environ.get("SQ_DQ_GEMM_MIN_M", "384"))


def dequant_weight(w: Int4Weight, out: torch.Tensor | None = None) -> torch.Tensor:
    """The bf16 values of a tile-major quantized weight, [n, 64 * ceil(k / 64)] (the GEMM's exact
    operand values; columns >= k hold padding)."""
    kpad = (w.k + 63) // 64 * 64
    if out is None:
        out = torch.empty((w.n, kpad), dtype=torch.bfloat16, device=w.wq.device)
    native().dequant_weight(w.wq, w.n, w.k, w.group, w.fmt, w.codebook, out)
    _count()
    return out


def bf16_linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, bias: torch.Tensor | None = None,
                residual: torch.Tensor | None = None, silu_mul: bool = False,
                ws: Workspace | None = None) -> torch.Tensor:
    """y = x @ w^T (+bias) (+residual) on the persistent tcgen05 bf16 GEMM; with ``silu_mul`` the
    rows of w are interleaved gate/up blocks of 64 and y = silu(gate) * up."""
    ws = ws or workspace(x.device)
    n = w.shape[0]
    if out is None:
        out = torch.empty((x.shape[0], n // 2 if silu_mul else n), dtype=torch.bfloat16, device=x.device)
    native().bf16_gemm(x, w, out, bias, residual, EPI_SILU_MUL if silu_mul else EPI_PLAIN, ws.gemm_ws,
                       ws.gemm_counters, ws.status)
    _count()
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None,
            row_idx: torch.Tensor | None = None) -> torch.Tensor:
    rows = x.shape[0] if row_idx is None else row_idx.numel()
    if out is None:
        out = torch.empty((rows, x.shape[1]), dtype=torch.bfloat16, device=x.device)
    native().rmsnorm(x, weight, out, row_idx, float(eps))
    _count()
    return out


def rope_kv_write(qkv, positions, cos_sin, q_out, slot_mapping, k_codes, k_scales, v_codes, v_scales,
                  hq: int, hkv: int, d: int, page_size: int, group: int, fmt_k: int, fmt_v: int,
                  q_norm=None, k_norm=None, norm_eps: float = 1e-6, ws: Workspace | None = None,
                  had_k=None, had_v=None) -> None:
    """A slot past the pools is not written; it records SQ_ERR_BOUNDS in the workspace status.
    With ``had_k`` / ``had_v`` (+-1 signs [d], :func:`kv_hadamard_signs`) q and k are written as
    H (s_k * x) / sqrt(d) and v as s_v * (H v) / sqrt(d)."""
    ws = ws or workspace(qkv.device)
    native().rope_kv_write(qkv, positions, cos_sin, q_out, slot_mapping, k_codes, k_scales, v_codes, v_scales,
                           hq, hkv, d, page_size, group, fmt_k, fmt_v, q_norm, k_norm, float(norm_eps), ws.status,
                           had_k, had_v)
    _count()


def kv_hadamard_signs(d: int, seed: int = 0x4B56) -> tuple[torch.Tensor, torch.Tensor]:
    """The +-1 sign vectors (s_k, s_v), float32 [d], of the Hadamard-rotated KV cache: a fixed
    function of (d, seed), so every rank, the oracle and a restarted server agree. Randomized
    Hadamard rotation of K and V before quantization, as the reference's HadamardKVCache
    (squish/kv/kv_cache.py:2769-2860), with separate signs for K and V."""
    g = np.random.default_rng(seed + d)
    s = np.where(g.random((2, d)) < 0.5, -1.0, 1.0).astype(np.float32)
    return torch.from_numpy(s[0].copy()), torch.from_numpy(s[1].copy())


def sylvester(d: int) -> torch.Tensor:
    """Sylvester-ordered Hadamard matrix H_d / sqrt(d) (symmetric, orthonormal), float64."""
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < d:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h / math.sqrt(d)


def page_mass(q, k_codes, k_scales, block_tables, seq_lens, mass, hq: int, hkv: int, d: int, page_size: int,
              group: int, fmt_k: int, sm_scale: float, ws: Workspace | None = None) -> None:
    """mass[page] += the softmax attention probability of decode row b's query heads on the
    keys of that page (summed over heads), for every row of ``seq_lens`` (kv_score.cu)."""
    ws = ws or workspace(q.device)
    native().page_mass(q, k_codes, k_scales, block_tables, seq_lens, mass, hq, hkv, d, page_size, group, fmt_k,
                       float(sm_scale), ws.status)
    _count()


MAX_DECODE_SPLITS = 64


def decode_splits(batch: int, hkv: int, max_ctx: int, num_sms: int = 148) -> tuple[int, int]:
    """Split count for flash-decoding: aim for ~2 CTAs per SM, >= 8 tiles (128 keys) per split
    (measured on B200 at 64 x 1300 keys: 1-2 splits 43 us, 3: 46, 6: 51, 12: 67)."""
    tiles = max(1, math.ceil(max_ctx / 16))
    base = max(1, batch * hkv)
    want = max(1, (2 * num_sms + base - 1) // base)
    splits = max(1, min(want, tiles // 8 if tiles >= 16 else 1, MAX_DECODE_SPLITS))
    tps = math.ceil(tiles / splits)
    splits = math.ceil(tiles / tps)
    return splits, tps


def paged_decode_attention(q, k_codes, k_scales, v_codes, v_scales, block_tables, seq_lens, out, hq, hkv, d,
                           page_size, group, fmt_k, fmt_v, sm_scale, max_ctx: int, ws: Workspace | None = None,
                           splits: tuple[int, int] | None = None):
    ws = ws or workspace(q.device)
    b = seq_lens.shape[0]
    s, tps = splits or decode_splits(b, hkv, max_ctx)
    o_part, lse = ws.attn_buffers(b, hq, s, d)
    native().paged_decode_attention(q, k_codes, k_scales, v_codes, v_scales, block_tables, seq_lens, out, o_part,
                                    lse, hq, hkv, d, page_size, group, fmt_k, fmt_v, float(sm_scale), s, tps,
                                    ws.status)
    _count(2 if s > 1 else 1)
    return out


def paged_prefill_attention(q, k_codes, k_scales, v_codes, v_scales, block_tables, tile_seq, tile_q0, q_start,
                            q_len, ctx_len, n_tiles, out, hq, hkv, d, page_size, group, fmt_k, fmt_v, sm_scale,
                            tree_mask=None, ws: Workspace | None = None, trace: torch.Tensor | None = None):
    """Causal attention of prefill chunks over their paged context; ``tree_mask`` (int32 per
    query row, bit j = may attend chunk token j, 0 = causal) turns a chunk into a token tree.
    Head dim 128 with 3..16 query heads per KV head runs on the tcgen05 kernel."""
    ws = ws or workspace(q.device)
    native().paged_prefill_attention(q, k_codes, k_scales, v_codes, v_scales, block_tables, tile_seq, tile_q0,
                                     q_start, q_len, ctx_len, int(n_tiles), out, hq, hkv, d, page_size, group,
                                     fmt_k, fmt_v, float(sm_scale), tree_mask, ws.status, trace)
    _count()
    return out


def sample(logits, out_tokens, temperature=None, top_p=None, top_k=None, min_p=None, rep_penalty=None, hist=None,
           allow_mask=None, seed: int = 0, step=None, out_logprob=None, ws: Workspace | None = None):
    ws = ws or workspace(logits.device)
    work = ws.sampler_buffer(logits.shape[0], logits.shape[1])
    native().sample(logits, temperature, top_p, top_k, min_p, rep_penalty, hist, allow_mask, int(seed), step,
                    out_tokens, out_logprob, work)
    _count()
    return out_tokens


# ----------------------------------------------------------------------------- mixture of experts
def moe_tile(tokens: int, top_k: int, experts: int) -> int:
    """Token tile of the grouped GEMM for ``tokens`` routed tokens: the smallest of 16/32/64/128
    that covers the mean rows per expert (padding per expert is at most one tile)."""
    avg = tokens * top_k / max(experts, 1)
    for bn in (16, 32, 64):
        if avg <= bn:
            return bn
    return 128


def moe_padded_rows(tokens: int, top_k: int, experts: int, bn: int) -> int:
    rows = tokens * top_k + experts * (bn - 1)
    return (rows + bn - 1) // bn * bn


def moe_route(logits: torch.Tensor, top_k: int, renorm: bool, ids: torch.Tensor, weights: torch.Tensor) -> None:
    native().moe_route(logits, top_k, renorm, ids, weights)
    _count()


def moe_align(ids: torch.Tensor, experts: int, bn: int, sorted_slot: torch.Tensor, slot_pos: torch.Tensor,
              tile_expert: torch.Tensor, num_tiles: torch.Tensor, counts: torch.Tensor | None = None,
              wait_flags: torch.Tensor | None = None, wait_expect: int = 0, status: torch.Tensor | None = None) -> None:
    """Expert-sorted, tile-padded slot layout of the routed ids (one CTA). With ``wait_flags`` the
    kernel first waits (bounded) until every entry reached ``wait_expect`` and clears them (the
    expert-parallel receiver's dispatch arrivals; a timeout is recorded in ``status``)."""
    native().moe_align(ids, experts, bn, sorted_slot, slot_pos, tile_expert, num_tiles, counts, wait_flags,
                       int(wait_expect), status)
    _count()


def moe_gather(x: torch.Tensor, sorted_slot: torch.Tensor, num_tiles: torch.Tensor, bn: int, top_k: int,
               xs: torch.Tensor) -> None:
    native().moe_gather(x, sorted_slot, num_tiles, bn, top_k, xs)
    _count()


def moe_combine(ys: torch.Tensor, slot_pos: torch.Tensor, weights: torch.Tensor, top_k: int, h: torch.Tensor) -> None:
    native().moe_combine(ys, slot_pos, weights, top_k, h)
    _count()


@dataclass
class GroupedInt4Weight:
    """Per-expert INT4 weights stacked in the tile-major layout: wq [E, words per expert]."""

    wq: torch.Tensor
    n: int
    k: int
    group: int


def stack_int4_experts(ws: list[Int4Weight]) -> GroupedInt4Weight:
    wq = torch.stack([w.wq.reshape(-1) for w in ws]).contiguous()
    return GroupedInt4Weight(wq=wq, n=ws[0].n, k=ws[0].k, group=ws[0].group)


def w4a16_grouped_linear(xs: torch.Tensor, w: GroupedInt4Weight, out: torch.Tensor, tile_expert: torch.Tensor,
                         num_tiles: torch.Tensor, bn: int, silu_mul: bool = False,
                         ws: Workspace | None = None) -> torch.Tensor:
    ws = ws or workspace(xs.device)
    native().w4a16_grouped_gemm(xs, w.wq, w.n, w.k, w.group, out, EPI_SILU_MUL if silu_mul else EPI_PLAIN,
                                tile_expert, num_tiles, bn, ws.gemm_ws, ws.gemm_counters, ws.status)
    _count()
    return out


# ----------------------------------------------------------------------------- speculative decoding
MAX_TREE_NODES = 32
TREE_META_INTS = 2 + 3 * MAX_TREE_NODES


def tree_verify(logits: torch.Tensor, meta: torch.Tensor, temperature: torch.Tensor, step: torch.Tensor, seed: int,
                out: torch.Tensor, draft_logits: torch.Tensor | None = None, ws: Workspace | None = None) -> torch.Tensor:
    """Walk each group's draft tree against its target logits rows (greedy or rejection
    sampling); out[g] = (n_accepted, final token, accepted node indices...)."""
    ws = ws or workspace(logits.device)
    scratch = ws.sampler_buffer(meta.shape[0], logits.shape[1])
    native().tree_verify(logits, draft_logits, meta, temperature, step, int(seed), scratch, out)
    _count()
    return out


def kv_compact(layer_ptrs: torch.Tensor, src: torch.Tensor, dst: torch.Tensor, hkv: int, page_size: int,
               kc_bytes: int, vc_bytes: int, ks_n: int, vs_n: int) -> None:
    native().kv_compact(layer_ptrs, src, dst, hkv, page_size, kc_bytes, vc_bytes, ks_n, vs_n)
    _count()
