"""Plain PyTorch fp32 references of the CUDA kernels (test oracles)."""
from __future__ import annotations

import math

import torch


def unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    """(N, K/2) uint8, low nibble = even column -> (N, K) int64."""
    p = packed.to(torch.int64)
    out = torch.empty(p.shape[0], p.shape[1] * 2, dtype=torch.int64, device=p.device)
    out[:, 0::2] = p & 0xF
    out[:, 1::2] = (p >> 4) & 0xF
    return out


def dequant_int4_as_kernel(packed, scales, offsets, group: int) -> torch.Tensor:
    """What the W4A16 kernel multiplies with: bf16(q * bf16(scale) + bf16(zero)) in fp32."""
    q = unpack_nibbles(packed).float()
    s = scales.to(torch.bfloat16).float().repeat_interleave(group, dim=1)[:, : q.shape[1]]
    z = offsets.to(torch.bfloat16).float().repeat_interleave(group, dim=1)[:, : q.shape[1]]
    return (q * s + z).to(torch.bfloat16).float()


def rope_cos_sin(max_pos: int, d: int, theta: float) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], dim=1).float()


def apply_rope(x: torch.Tensor, pos: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """x [..., T, H, D] neox rotate-half with cos/sin table [max_pos, D]."""
    d = x.shape[-1]
    cs = cos_sin[pos.long()]
    c, s = cs[:, : d // 2].unsqueeze(1), cs[:, d // 2:].unsqueeze(1)
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor, scale: float) -> torch.Tensor:
    """q [Tq, Hq, D], k/v [Tk, Hkv, D], causal by absolute position (key j visible to query i iff j <= q_pos[i])."""
    hq, hkv = q.shape[1], k.shape[1]
    g = hq // hkv
    kk = k.repeat_interleave(g, dim=1)
    vv = v.repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kk.float()) * scale
    kpos = torch.arange(k.shape[0], device=q.device)
    mask = kpos[None, :] > q_pos[:, None]
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, vv.float())


def sm_scale(d: int) -> float:
    return 1.0 / math.sqrt(d)
