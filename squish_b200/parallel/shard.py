"""Tensor-parallel sharding of a checkpoint (Megatron layout, one shard per rank).

  * q/k/v projections and their biases: column parallel by attention head (each rank keeps
    Hq/tp query heads and the KV heads they use; with tp > Hkv a KV head is replicated
    over tp/Hkv ranks);
  * o_proj: row parallel (the input columns of the rank's query heads);
  * gate/up: column parallel (F/tp rows each); down: row parallel (the same F/tp columns);
  * embeddings, norms, q/k norms: replicated; LM head: vocabulary rows split evenly.

Row-parallel outputs are partial sums: the runner all-reduces them (fused GEMM+all-reduce
over NVLink, or NCCL). The local shard is a regular Checkpoint of a local ModelConfig, so
the single-GPU runner code runs it unchanged.

Mixture-of-experts layers use expert parallelism over the same ranks: attention is
tensor-parallel as above, the router is replicated, rank r keeps experts
[r E/tp, (r+1) E/tp), computes the MoE output of the routed slots that land on its
experts, and the partial outputs are all-reduced like a row-parallel projection.
"""
from __future__ import annotations

import dataclasses

import torch

from ..models.config import ModelConfig
from ..models.weights import Checkpoint, QTensor


def _rows(t: QTensor, r0: int, r1: int) -> QTensor:
    if t.kind == "dense":
        return QTensor("dense", (r1 - r0,) + tuple(t.shape[1:]), data=t.data[r0:r1].contiguous())
    from ..models.decoder import gemm_extra_ok

    rot_only = bool(t.extra) and gemm_extra_ok(t)
    if t.kind not in ("q4a", "q8", "fp8", "nf4", "q2", "q3") or (t.extra and not rot_only):
        t = _to_q4a(t)
        rot_only = False
    # a row slice keeps the input rotation of an SQINT2 weight (it acts on the columns) and the
    # level table of an any4 weight
    return dataclasses.replace(t, shape=(r1 - r0, t.shape[1]), packed=t.packed[r0:r1].contiguous(),
                               scales=t.scales[r0:r1].contiguous(),
                               offsets=None if t.offsets is None else t.offsets[r0:r1].contiguous(),
                               extra=t.extra if rot_only else None)


def _to_q4a(t: QTensor) -> QTensor:
    from ..quant.codecs import quantize

    return quantize(t.dequantize().float(), "q4a", t.group or 64)


def _cols(t: QTensor, c0: int, c1: int) -> QTensor:
    if t.kind == "dense":
        return QTensor("dense", (t.shape[0], c1 - c0), data=t.data[:, c0:c1].contiguous())
    if t.kind != "q4a" or t.extra:  # (an input rotation does not survive a column slice)
        t = _to_q4a(t)
    g = t.group
    if c0 % g or c1 % g or c0 % 2:
        raise ValueError(f"column shard [{c0}, {c1}) is not aligned to the quantization group {g}")
    return dataclasses.replace(t, shape=(t.shape[0], c1 - c0), packed=t.packed[:, c0 // 2:c1 // 2].contiguous(),
                               scales=t.scales[:, c0 // g:c1 // g].contiguous(),
                               offsets=t.offsets[:, c0 // g:c1 // g].contiguous())


def _vec(t: QTensor, r0: int, r1: int) -> QTensor:
    return QTensor("dense", (r1 - r0,), data=t.data[r0:r1].contiguous())


def kv_heads_of(rank: int, tp: int, hkv: int) -> tuple[int, int]:
    """[first, last) KV heads held by ``rank``."""
    if tp <= hkv:
        if hkv % tp:
            raise ValueError(f"{hkv} KV heads do not split over {tp} ranks")
        n = hkv // tp
        return rank * n, rank * n + n
    if tp % hkv:
        raise ValueError(f"{tp} ranks do not replicate {hkv} KV heads evenly")
    h = rank * hkv // tp
    return h, h + 1


def local_config(cfg: ModelConfig, tp: int) -> ModelConfig:
    if cfg.num_heads % tp:
        raise ValueError(f"{cfg.num_heads} query heads do not split over {tp} ranks")
    hkv = max(1, cfg.num_kv_heads // tp)
    if cfg.is_moe:
        # attention tensor-parallel, experts split over the same ranks (expert parallelism)
        if cfg.num_experts % tp:
            raise ValueError(f"{cfg.num_experts} experts do not split over {tp} ranks")
        return dataclasses.replace(cfg, name=f"{cfg.name}-tp{tp}", num_heads=cfg.num_heads // tp, num_kv_heads=hkv,
                                   num_local_experts=cfg.num_experts // tp)
    if cfg.intermediate_size % tp:
        raise ValueError(f"FFN width {cfg.intermediate_size} does not split over {tp} ranks")
    return dataclasses.replace(cfg, name=f"{cfg.name}-tp{tp}", num_heads=cfg.num_heads // tp, num_kv_heads=hkv,
                               intermediate_size=cfg.intermediate_size // tp)


def vocab_shard(vocab: int, rank: int, tp: int) -> tuple[int, int]:
    """Even vocabulary split, rounded to multiples of 8 (16-byte rows of bf16 logits)."""
    per = ((vocab + tp - 1) // tp + 7) // 8 * 8
    return min(vocab, rank * per), min(vocab, (rank + 1) * per)


def shard_checkpoint(ck: Checkpoint, rank: int, tp: int) -> Checkpoint:
    cfg = ck.config
    lc = local_config(cfg, tp)
    out = Checkpoint(lc, dataclasses.replace(ck.quant))
    t = ck.tensors
    d = cfg.head_dim
    hq_l = cfg.num_heads // tp
    q0, q1 = rank * hq_l * d, (rank + 1) * hq_l * d
    k0h, k1h = kv_heads_of(rank, tp, cfg.num_kv_heads)
    k0, k1 = k0h * d, k1h * d
    f_l = cfg.intermediate_size // tp if not cfg.is_moe else 0
    f0, f1 = rank * f_l, (rank + 1) * f_l
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        out.tensors[a + "q_proj.weight"] = _rows(t[a + "q_proj.weight"], q0, q1)
        out.tensors[a + "k_proj.weight"] = _rows(t[a + "k_proj.weight"], k0, k1)
        out.tensors[a + "v_proj.weight"] = _rows(t[a + "v_proj.weight"], k0, k1)
        if cfg.qkv_bias:
            out.tensors[a + "q_proj.bias"] = _vec(t[a + "q_proj.bias"], q0, q1)
            out.tensors[a + "k_proj.bias"] = _vec(t[a + "k_proj.bias"], k0, k1)
            out.tensors[a + "v_proj.bias"] = _vec(t[a + "v_proj.bias"], k0, k1)
        out.tensors[a + "o_proj.weight"] = _cols(t[a + "o_proj.weight"], q0, q1)
        for n in ("q_norm.weight", "k_norm.weight"):
            if a + n in t:
                out.tensors[a + n] = t[a + n]
        m = p + "mlp."
        if cfg.is_moe:
            e_loc = cfg.num_experts // tp
            lc.expert_offset = rank * e_loc
            out.tensors[m + "gate.weight"] = t[m + "gate.weight"]  # the router sees every expert
            for e in range(rank * e_loc, (rank + 1) * e_loc):
                for n in ("gate_proj", "up_proj", "down_proj"):
                    out.tensors[m + f"experts.{e}.{n}.weight"] = t[m + f"experts.{e}.{n}.weight"]
        else:
            out.tensors[m + "gate_proj.weight"] = _rows(t[m + "gate_proj.weight"], f0, f1)
            out.tensors[m + "up_proj.weight"] = _rows(t[m + "up_proj.weight"], f0, f1)
            out.tensors[m + "down_proj.weight"] = _cols(t[m + "down_proj.weight"], f0, f1)
        for n in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            out.tensors[p + n] = t[p + n]
    out.tensors["model.embed_tokens.weight"] = t["model.embed_tokens.weight"]
    out.tensors["model.norm.weight"] = t["model.norm.weight"]
    v0, v1 = vocab_shard(cfg.vocab_size, rank, tp)
    out.tensors["lm_head.weight"] = _rows(t["lm_head.weight"], v0, v1)
    return out
