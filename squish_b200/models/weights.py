"""Quantized checkpoint container and random initialisation.

A :class:`Checkpoint` maps HF tensor names to entries in the same representation the
reference's npy-dir format stores (squish/convert.py:283-540):

  * ``Q4A``  — INT4 asymmetric group quantized: ``packed`` (N, K/2) uint8 with the low
    nibble = even column, ``scales`` and ``offsets`` (N, K/g) float32
    (``__q4a/__s4a/__z4a``);
  * ``DENSE`` — an unquantized tensor (norms, biases, embeddings, routers; ``__pt``).

Random initialisation draws every linear weight from N(0, 0.02) with a seeded
generator and quantizes it (on the GPU for large models, with the C++ CPU quantizer
for small ones); RMSNorm weights are ones and biases zeros, as HF initialises them.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .._ext import native
from .config import ModelConfig, QuantConfig


@dataclass
class QTensor:
    kind: str  # "q4a" | "dense"
    shape: tuple
    packed: torch.Tensor | None = None
    scales: torch.Tensor | None = None
    offsets: torch.Tensor | None = None
    group: int = 0
    data: torch.Tensor | None = None
    extra: dict | None = None  # INT3 low-rank compensator (lra, lrb)

    def dequantize(self) -> torch.Tensor:
        """fp32 reconstruction on the CPU for the CPU-decoded kinds, on the tensor's device
        for INT4 asymmetric."""
        if self.kind == "dense":
            return self.data.float()
        if self.kind != "q4a":
            from ..quant.codecs import dequantize_qtensor

            return dequantize_qtensor(self)
        p = self.packed.to(torch.int64)
        q = torch.empty(p.shape[0], p.shape[1] * 2, dtype=torch.float32, device=p.device)
        q[:, 0::2] = (p & 0xF).float()
        q[:, 1::2] = ((p >> 4) & 0xF).float()
        s = self.scales.float().repeat_interleave(self.group, dim=1)[:, : q.shape[1]]
        o = self.offsets.float().repeat_interleave(self.group, dim=1)[:, : q.shape[1]]
        w = o + q * s
        if self.extra and "rot_signs" in self.extra:  # QuaRot: stored in the rotated frame (W R^T)
            from ..quant.sqint2 import unrotate

            w = unrotate(w, self.extra["rot_signs"], int(self.extra["rot_block"]))
        return w


@dataclass
class Checkpoint:
    config: ModelConfig
    quant: QuantConfig
    tensors: dict[str, QTensor] = field(default_factory=dict)

    def __getitem__(self, name: str) -> QTensor:
        return self.tensors[name]

    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def nbytes(self) -> int:
        n = 0
        for t in self.tensors.values():
            for a in (t.packed, t.scales, t.offsets, t.data):
                if a is not None:
                    n += a.numel() * a.element_size()
        return n


def linear_names(cfg: ModelConfig) -> list[tuple[str, tuple[int, int]]]:
    """(name, (out, in)) of every linear weight of the architecture, in load order."""
    h, d = cfg.hidden_size, cfg.head_dim
    out = []
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        out += [(p + "self_attn.q_proj.weight", (cfg.num_heads * d, h)),
                (p + "self_attn.k_proj.weight", (cfg.num_kv_heads * d, h)),
                (p + "self_attn.v_proj.weight", (cfg.num_kv_heads * d, h)),
                (p + "self_attn.o_proj.weight", (h, cfg.num_heads * d))]
        if cfg.is_moe:
            f = cfg.moe_intermediate_size
            for e in range(cfg.num_experts):
                q = p + f"mlp.experts.{e}."
                out += [(q + "gate_proj.weight", (f, h)), (q + "up_proj.weight", (f, h)),
                        (q + "down_proj.weight", (h, f))]
        else:
            f = cfg.intermediate_size
            out += [(p + "mlp.gate_proj.weight", (f, h)), (p + "mlp.up_proj.weight", (f, h)),
                    (p + "mlp.down_proj.weight", (h, f))]
    return out


def pick_group(cols: int, group: int) -> int:
    """Largest group <= ``group`` that divides ``cols`` (the reference falls back through
    smaller powers of two, squish/convert.py:269-280)."""
    for g in (group, 128, 64, 32, 16, 8, 4):
        if g <= group and cols % g == 0 and cols >= 2 * g:
            return g
    return cols


def quantize_q4a(w: torch.Tensor, group: int, mse_clip: bool = False) -> QTensor:
    """Quantize a 2-D weight with the INT4 asymmetric group codec (GPU kernel on CUDA
    tensors, the C++ CPU kernel otherwise)."""
    g = pick_group(w.shape[1], group)
    if w.is_cuda:
        packed, scales, offsets = native().quantize_int4_asym(w.contiguous(), g, 8 if mse_clip else 1)
    elif mse_clip:
        packed, scales, offsets = native().cpu.quantize_int4_asym_mse(w.float().contiguous(), g, 8)
    else:
        packed, scales, offsets = native().cpu.quantize_int4_asym(w.float().contiguous(), g)
    return QTensor("q4a", tuple(w.shape), packed=packed, scales=scales, offsets=offsets, group=g)


def random_checkpoint(cfg: ModelConfig, q: QuantConfig, seed: int = 0, device: str | torch.device = "cpu",
                      dense_dtype: torch.dtype = torch.float32) -> Checkpoint:
    """Random-init weights N(0, 0.02) of the architecture, quantized per ``q``.

    On CPU the draw order is deterministic per tensor name order (one generator seeded
    with ``seed``); on CUDA each tensor uses its own generator seeded by (seed, index),
    so large models are generated and quantized on the device without host copies.
    """
    dev = torch.device(device)
    ck = Checkpoint(cfg, q)
    gen = torch.Generator(device=dev).manual_seed(seed)
    h = cfg.hidden_size

    def draw(shape):
        if dev.type == "cuda":
            return torch.randn(shape, generator=gen, device=dev, dtype=torch.bfloat16) * 0.02
        return torch.randn(shape, generator=gen) * 0.02

    emb = draw((cfg.vocab_size, h))
    ck.tensors["model.embed_tokens.weight"] = QTensor("dense", tuple(emb.shape), data=emb.to(dense_dtype))
    for name, shape in linear_names(cfg):
        w = draw(shape)
        ck.tensors[name] = quantize_q4a(w, q.group_size, q.mse_clip) if q.weight_bits == 4 else \
            QTensor("dense", shape, data=w.to(dense_dtype))
        del w
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        for n in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            ck.tensors[p + n] = QTensor("dense", (h,), data=torch.ones(h, dtype=dense_dtype, device=dev))
        if cfg.qkv_bias:
            for n, sz in (("q_proj", cfg.q_size), ("k_proj", cfg.kv_size), ("v_proj", cfg.kv_size)):
                ck.tensors[p + f"self_attn.{n}.bias"] = QTensor("dense", (sz,),
                                                                data=torch.zeros(sz, dtype=dense_dtype, device=dev))
        if cfg.qk_norm:
            for n in ("q_norm", "k_norm"):
                ck.tensors[p + f"self_attn.{n}.weight"] = QTensor(
                    "dense", (cfg.head_dim,), data=torch.ones(cfg.head_dim, dtype=dense_dtype, device=dev))
        if cfg.is_moe:
            r = draw((cfg.num_experts, h))
            ck.tensors[p + "mlp.gate.weight"] = QTensor("dense", tuple(r.shape), data=r.to(dense_dtype))
    ck.tensors["model.norm.weight"] = QTensor("dense", (h,), data=torch.ones(h, dtype=dense_dtype, device=dev))
    if cfg.tie_embeddings:
        lm = emb
    else:
        lm = draw((cfg.vocab_size, h))
    if q.quantize_lm_head and q.weight_bits == 4:
        ck.tensors["lm_head.weight"] = quantize_q4a(lm, q.group_size, q.mse_clip)
    else:
        ck.tensors["lm_head.weight"] = QTensor("dense", tuple(lm.shape), data=lm.to(dense_dtype))
    return ck
