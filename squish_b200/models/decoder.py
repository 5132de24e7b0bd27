"""Decoder forward over the paged KV cache.

:class:`StepInputs` is one engine iteration, flattened: decode sequences first (one
token each), then prefill chunks. :class:`CudaRunner` runs it with the sm_100a kernels:

  embed -> [RMSNorm -> W4A16 qkv(+bias) -> RoPE+KV-quant write -> paged attention
  (decode split-K kernel | prefill causal kernel) -> W4A16 o_proj (+residual in the
  epilogue) -> RMSNorm -> W4A16 gate_up with the SiLU*up epilogue -> W4A16 down_proj
  (+residual)] x L -> RMSNorm of the logit rows -> W4A16 lm_head -> fused sampler.

Activation buffers are allocated once for the step token budget, so decode steps
can be captured in CUDA graphs (engine/cuda_graph.py). :class:`TorchPagedRunner` is the
same step in plain PyTorch on the CPU (dequantized weights, the C++ KV codec), used as
the oracle of the engine path in CPU tests.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import ops
from .._ext import native
from ..kv.paged import KVPools
from ..ops.kernels import KV_FORMATS, Int4Weight
from .config import ModelConfig, QuantConfig
from .reference import rope_table
from .weights import Checkpoint, QTensor


@dataclass
class StepInputs:
    input_ids: np.ndarray          # int32 [T]
    positions: np.ndarray          # int32 [T]
    slot_mapping: np.ndarray       # int32 [T]
    num_decode: int
    decode_seq_lens: np.ndarray    # int32 [Bd]
    prefill_q_start: np.ndarray    # int32 [Bp] (relative to the first prefill row)
    prefill_q_len: np.ndarray      # int32 [Bp]
    prefill_ctx_len: np.ndarray    # int32 [Bp]
    tile_seq: np.ndarray           # int32 [n_tiles]
    tile_q0: np.ndarray            # int32 [n_tiles]
    block_tables: np.ndarray       # int32 [Bd + Bp, max_pages]
    logits_rows: np.ndarray        # int32 [B]
    temperature: np.ndarray        # f32 [B]
    top_p: np.ndarray              # f32 [B]
    top_k: np.ndarray              # int32 [B]
    min_p: np.ndarray              # f32 [B]
    rep_penalty: np.ndarray        # f32 [B]
    rng_step: np.ndarray           # int32 [B]
    hist: np.ndarray | None = None  # int32 [B, H] recent tokens for the repetition penalty
    seed: int = 0
    max_decode_ctx: int = 0
    all_logits: bool = False       # also return the logits of every logit row (spec verify)
    allow_mask: np.ndarray | None = None  # int32 [B, ceil(V/32)] grammar bitmask (bit set = token allowed)
    # speculative verification: logits_rows = the B sample rows, then every tree node's row
    tree_mask: np.ndarray | None = None    # int32 [T] ancestor bits within the chunk (0 = causal)
    verify_meta: np.ndarray | None = None  # int32 [G, TREE_META_INTS] (row0 relative to the first node row)
    verify_temp: np.ndarray | None = None  # f32 [G]
    verify_step: np.ndarray | None = None  # int32 [G]
    verify_preds: bool = False             # also return the greedy token of every node row (Jacobi)
    draft_logits: object = None            # device tensor of draft-model rows (q of the rejection test)

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])

    @property
    def num_prefill(self) -> int:
        return int(self.prefill_q_len.shape[0])

    @property
    def num_sample_rows(self) -> int:
        return int(self.temperature.shape[0])

    @property
    def num_verify(self) -> int:
        return 0 if self.verify_meta is None else int(self.verify_meta.shape[0])

    def h2d_bytes(self) -> int:
        n = 0
        for v in self.__dict__.values():
            if isinstance(v, np.ndarray):
                n += v.nbytes
        return n


def prefill_tiles(q_len: np.ndarray, tile: int = 32) -> tuple[np.ndarray, np.ndarray]:
    seq, q0 = [], []
    for i, ql in enumerate(q_len.tolist()):
        for s in range(0, ql, tile):
            seq.append(i)
            q0.append(s)
    return np.asarray(seq, dtype=np.int32), np.asarray(q0, dtype=np.int32)


# ----------------------------------------------------------------------------- device weights
@dataclass
class LayerWeights:
    ln1: torch.Tensor
    ln2: torch.Tensor
    qkv: Int4Weight
    o: Int4Weight
    gate_up: Int4Weight | None
    down: Int4Weight | None
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None
    moe: object | None = None


# stored kinds the GEMM decodes natively (others, and INT3 with a low-rank term, are re-encoded INT4)
GEMM_KINDS = ("q4a", "nf4", "q8", "fp8", "q2", "q3", "aqlm")


def _rotation(t: QTensor):
    """(signs, block) of an SQINT2 tensor stored in the rotated frame, else None."""
    return (t.extra["rot_signs"], int(t.extra["rot_block"])) if t.extra and "rot_signs" in t.extra else None


def _same_rotation(parts: list[QTensor]) -> bool:
    r0 = _rotation(parts[0])
    for p in parts[1:]:
        r = _rotation(p)
        if (r is None) != (r0 is None) or (r is not None and (r[1] != r0[1] or not torch.equal(r[0], r0[0]))):
            return False
    return True


def _levels(t: QTensor):
    return (t.extra or {}).get("levels")


def _same_levels(parts: list[QTensor]) -> bool:
    l0 = _levels(parts[0])
    return all((_levels(p) is None) == (l0 is None) and (l0 is None or torch.equal(_levels(p), l0))
               for p in parts[1:])


def _same_kind(parts: list[QTensor], group: int) -> list[QTensor]:
    """Tensors fused into one GEMM must share a native kind, group and input rotation; otherwise
    all are re-encoded as INT4."""
    k0 = parts[0].kind
    # AQLM tensors carry their own codebooks, so they cannot share one fused GEMM; any4 tensors
    # (NF4 codes with a learned level table) only when their tables agree
    if (k0 in GEMM_KINDS and all(p.kind == k0 and p.group == parts[0].group and gemm_extra_ok(p) for p in parts)
            and not (k0 == "aqlm" and len(parts) > 1) and _same_rotation(parts) and _same_levels(parts)):
        return parts
    return [_as_q4a(p, group) for p in parts]


_LOWRANK_KEYS = (("lra", "lrb"), ("sq_L", "sq_R"))


def _lowrank(t: QTensor):
    """(keys, A [N, r], B [r, K]) of a low-rank residual W += A B, or None."""
    ex = t.extra or {}
    for ka, kb in _LOWRANK_KEYS:
        if ka in ex and ex[ka] is not None:
            return (ka, kb), ex[ka].float(), ex[kb].float()
    return None


def _merged_extra(parts: list[QTensor], rows) -> dict | None:
    """Extras of a fused weight: the shared rotation / level table, and the parts' low-rank
    residuals as one block-diagonal factor pair (``rows(As)`` arranges the A row blocks the way
    the fused weight arranges the parts' rows)."""
    p0 = parts[0]
    ex = {}
    if _rotation(p0):
        ex.update({k: p0.extra[k] for k in ("rot_signs", "rot_block", "seed") if k in p0.extra})
    if _levels(p0) is not None:
        ex["levels"] = _levels(p0)
    lrs = [_lowrank(p) for p in parts]
    if any(lr is not None for lr in lrs):
        keys = next(lr[0] for lr in lrs if lr is not None)
        ranks = [0 if lr is None else lr[1].shape[1] for lr in lrs]
        R = sum(ranks)
        As, Bs, c = [], [], 0
        for p, lr, r in zip(parts, lrs, ranks):
            a = torch.zeros(p.shape[0], R)
            if lr is not None:
                a[:, c:c + r] = lr[1]
                Bs.append(lr[2])
            As.append(a)
            c += r
        ex[keys[0]], ex[keys[1]] = rows(As), torch.cat(Bs)
    return ex or None


def _cat_rows(parts: list[QTensor]) -> QTensor:
    def cat(name):
        xs = [getattr(p, name) for p in parts]
        return None if xs[0] is None else torch.cat(xs)

    return QTensor(parts[0].kind, (sum(p.shape[0] for p in parts), parts[0].shape[1]), packed=cat("packed"),
                   scales=cat("scales"), offsets=cat("offsets"), group=parts[0].group,
                   extra=_merged_extra(parts, torch.cat))


_cat_q4a = _cat_rows


def _interleave_gate_up(gate: QTensor, up: QTensor) -> QTensor:
    """Rows [g0:64, u0:64, g64:128, u64:128, ...] (F padded to a multiple of 64 with zero
    rows, whose zero scales make them 0), the layout the SiLU*up GEMM epilogue expects."""
    f = gate.shape[0]
    fp = (f + 63) // 64 * 64

    def pad(t, fill=0):
        if t.shape[0] == fp:
            return t
        z = torch.full((fp - f,) + tuple(t.shape[1:]), fill, dtype=t.dtype, device=t.device)
        return torch.cat([t, z])

    def inter(a, b):
        if a is None:
            return None
        a, b = pad(a), pad(b)
        return torch.stack([a.view(fp // 64, 64, -1), b.view(fp // 64, 64, -1)], 1).reshape(2 * fp, -1)

    return QTensor(gate.kind, (2 * fp, gate.shape[1]), packed=inter(gate.packed, up.packed),
                   scales=inter(gate.scales, up.scales), offsets=inter(gate.offsets, up.offsets), group=gate.group,
                   extra=_merged_extra([gate, up], lambda As: inter(As[0], As[1])))


def _as_q4a(t: QTensor, group: int) -> QTensor:
    """Stored kinds without a GEMM code format (INT3, AQLM, dense) are decoded once at load
    and re-encoded as INT4 asymmetric group ``group``."""
    if t.kind == "q4a" and not t.extra:
        return t
    from ..quant.codecs import quantize

    return quantize(t.dequantize().float(), "q4a", group)


def gemm_extra_ok(t: QTensor) -> bool:
    """Extras the GEMM path handles as stored: an input rotation (SQINT2 INT2, QuaRot INT4),
    an any4 level table on NF4 codes, a low-rank residual (SQINT2 residual, MiLo INT3
    compensator: two skinny GEMMs after the quantized one)."""
    if not t.extra:
        return True
    keys = set(t.extra)
    if t.kind == "q2":
        return keys <= {"rot_signs", "rot_block", "seed", "sq_L", "sq_R"} and (
            "rot_signs" in keys or not keys & {"sq_L", "sq_R"})
    if t.kind == "q4a":
        return keys <= {"rot_signs", "rot_block", "seed"}
    if t.kind == "q3":
        return keys <= {"lra", "lrb"}
    return t.kind == "nf4" and keys <= {"levels"}


def _native(t: QTensor, group: int) -> QTensor:
    """Kinds the GEMM decodes as stored (with the extras of ``gemm_extra_ok``); others are
    re-encoded as INT4."""
    return t if t.kind in GEMM_KINDS and gemm_extra_ok(t) else _as_q4a(t, group)


def _to_int4(t: QTensor, device, bias: torch.Tensor | None = None, group: int = 64) -> Int4Weight:
    return ops.kernels.prepare_weight(_native(t, group), device, bias=bias)


def _dense(t: QTensor, device, dtype=torch.bfloat16) -> torch.Tensor:
    return t.data.to(device=device, dtype=dtype).contiguous()


class CudaRunner:
    """Runs engine steps on one GPU with the sm_100a kernels."""

    def __init__(self, ck: Checkpoint, device, num_pages: int, max_num_tokens: int = 4096, max_num_seqs: int = 256,
                 max_model_len: int = 4096, pools: KVPools | None = None, free_checkpoint: bool = False,
                 spec_rows: int = 0, prefill_weight_cache: bool = False, offload_layers: int = 0):
        self.cfg: ModelConfig = ck.config
        self.qcfg: QuantConfig = ck.quant
        self.device = torch.device(device)
        cfg, dev = self.cfg, self.device
        self.max_num_tokens = max_num_tokens
        self.max_num_seqs = max_num_seqs
        self.spec_rows = spec_rows
        self.prefill_weight_cache = prefill_weight_cache
        self.max_model_len = max_model_len
        self.ws = ops.Workspace(dev)  # owned by this runner: its CUDA graphs capture these buffers
        self.fk, self.fv = KV_FORMATS[self.qcfg.kv_dtype]
        self.F = cfg.intermediate_size
        self.F_pad = (self.F + 63) // 64 * 64
        t = ck.tensors
        self.embed = _dense(t["model.embed_tokens.weight"], dev)
        self.layers: list[LayerWeights] = []
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            g = self.qcfg.group_size
            qkv = _cat_rows(_same_kind([_native(t[p + f"self_attn.{n}_proj.weight"], g) for n in "qkv"], g))
            bias = None
            if cfg.qkv_bias:
                bias = torch.cat([t[p + f"self_attn.{n}.bias"].data.float() for n in ("q_proj", "k_proj", "v_proj")])
            lw = LayerWeights(ln1=_dense(t[p + "input_layernorm.weight"], dev),
                              ln2=_dense(t[p + "post_attention_layernorm.weight"], dev),
                              qkv=_to_int4(qkv, dev, bias), o=_to_int4(t[p + "self_attn.o_proj.weight"], dev),
                              gate_up=None, down=None)
            if cfg.qk_norm:
                lw.q_norm = _dense(t[p + "self_attn.q_norm.weight"], dev)
                lw.k_norm = _dense(t[p + "self_attn.k_norm.weight"], dev)
            if cfg.is_moe:
                from .moe import MoELayer, MoEScratch

                if i == 0:
                    self.moe_scratch = MoEScratch(cfg, max_num_tokens, dev)
                lw.moe = MoELayer.from_checkpoint(ck, i, dev, self.moe_scratch)
            else:
                gu = _same_kind([_native(t[p + "mlp.gate_proj.weight"], g), _native(t[p + "mlp.up_proj.weight"], g)], g)
                lw.gate_up = _to_int4(_interleave_gate_up(gu[0], gu[1]), dev)
                lw.down = _to_int4(t[p + "mlp.down_proj.weight"], dev)
            self.layers.append(lw)
            if free_checkpoint:
                for k in list(t):
                    if k.startswith(p):
                        del t[k]
        self.norm = _dense(t["model.norm.weight"], dev)
        lm = t["lm_head.weight"]
        self.lm_head_q = _to_int4(lm, dev, group=self.qcfg.group_size) if lm.kind != "dense" else None
        self.lm_head_dense = _dense(lm, dev) if lm.kind == "dense" else None
        self.cos_sin = rope_table(cfg, max(max_model_len, 16) + 1).to(dev)
        self.pools = pools or KVPools(cfg, self.qcfg, num_pages, dev)
        self.sm_scale = 1.0 / math.sqrt(cfg.head_dim)
        # attention mass per KV page, refreshed on the steps the engine marks (H2O-style eviction)
        self.score_step = False
        self.page_mass_buf = torch.zeros(0, dtype=torch.float32, device=dev)  # sized at the first scoring step
        self.had_k = self.had_v = self.had_v_row = None
        if getattr(self.qcfg, "kv_hadamard", False):
            sk, sv = ops.kernels.kv_hadamard_signs(cfg.head_dim)
            self.had_k, self.had_v = sk.to(dev), sv.to(dev)
            self.had_v_row = sv.repeat(cfg.num_heads).to(dev)  # un-rotation of the [T, Hq * D] output
        self.offload = None
        if offload_layers > 0:
            self._offload_setup(offload_layers)
        self._alloc_buffers()

    # ------------------------------------------------------------------ weight offload
    _OFF_NAMES = ("qkv", "o", "gate_up", "down")

    def _offload_setup(self, n: int) -> None:
        """Keep the quantized weights of the last ``n`` layers in pinned host memory and stream
        each one into one of two device staging sets just ahead of its use (a copy stream,
        events both ways), so a model larger than HBM runs with only two layers' weights
        resident for those layers. The reference pages layers between tiers with numpy copies
        (squish/io/split_loader.py, squish/io/model_shard_loader.py)."""
        import dataclasses

        if any(lw.moe is not None for lw in self.layers):
            raise ValueError("weight offload covers dense decoder layers")
        L = len(self.layers)
        n = min(n, L)
        first = L - n
        host, staged = {}, [{}, {}]
        for li in range(first, L):
            lw = self.layers[li]
            host[li] = {}
            for name in self._OFF_NAMES:
                w = getattr(lw, name)
                if w.dense is not None or w.rot is not None:
                    raise ValueError("offloaded layers stream their quantized codes only")
                host[li][name] = w.wq.to("cpu").pin_memory()
                for b in range(min(2, n)):
                    if name not in staged[b]:
                        staged[b][name] = torch.empty_like(w.wq)
        for k, li in enumerate(range(first, L)):
            lw = self.layers[li]
            for name in self._OFF_NAMES:
                setattr(lw, name, dataclasses.replace(getattr(lw, name), wq=staged[k % 2][name]))
        torch.cuda.empty_cache()
        self.offload = {"first": first, "host": host, "staged": staged, "stream": torch.cuda.Stream(self.device),
                        "copied": [torch.cuda.Event(), torch.cuda.Event()],
                        "done": [torch.cuda.Event(), torch.cuda.Event()]}

    def _offload_fetch(self, li: int) -> None:
        """Queue the copy of offloaded layer li into its staging set, after the layer that last
        used that set has finished."""
        o = self.offload
        b = (li - o["first"]) % 2
        cs = o["stream"]
        if li - o["first"] >= 2:
            cs.wait_event(o["done"][b])
        else:
            cs.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(cs):
            for name in self._OFF_NAMES:
                o["staged"][b][name].copy_(o["host"][li][name], non_blocking=True)
            o["copied"][b].record(cs)

    # ------------------------------------------------------------------ buffers
    def _alloc_buffers(self):
        cfg, dev, T = self.cfg, self.device, self.max_num_tokens
        bf = torch.bfloat16
        self.h = torch.empty(T, cfg.hidden_size, dtype=bf, device=dev)
        self.x = torch.empty(T, cfg.hidden_size, dtype=bf, device=dev)
        self.qkv = torch.empty(T, cfg.q_size + 2 * cfg.kv_size, dtype=bf, device=dev)
        self.q = torch.empty(T, cfg.q_size, dtype=bf, device=dev)
        self.attn = torch.empty(T, cfg.q_size, dtype=bf, device=dev)
        f_act = self.F_pad if not cfg.is_moe else 0
        self.act = torch.empty(T, max(f_act, 8), dtype=bf, device=dev)
        B = self.max_num_seqs
        R = B + min(T, self.spec_rows)  # logit rows: samples + speculative tree nodes
        self.xs = torch.empty(R, cfg.hidden_size, dtype=bf, device=dev)
        self.logits = torch.empty(R, cfg.vocab_size, dtype=bf, device=dev)
        self.tokens = torch.empty(B + T, dtype=torch.int32, device=dev)
        self.tokens_host = torch.empty(B + T, dtype=torch.int32, pin_memory=True)
        self.vout = torch.zeros(B, 2 + ops.kernels.MAX_TREE_NODES, dtype=torch.int32, device=dev)
        self.prefill_cache_bytes = 0
        if T >= ops.kernels.DQ_GEMM_MIN_M:
            allw = ws = [w for lw in self.layers for w in (lw.qkv, lw.o, lw.gate_up, lw.down)
                         if isinstance(w, ops.Int4Weight)]
            if ws and self.prefill_weight_cache and dev.type == "cuda":
                # resident bf16 expansions: prefill GEMMs skip the per-step expansion (HBM for time).
                # A runner whose row-parallel GEMMs run elsewhere (tensor parallel: fused with the
                # all-reduce) caches only the column-parallel weights.
                if type(self)._row_parallel is not CudaRunner._row_parallel:
                    ws = [w for lw in self.layers for w in (lw.qkv, lw.gate_up) if isinstance(w, ops.Int4Weight)]
                need = sum(w.n * ((w.k + 63) // 64 * 64) * 2 for w in ws)
                free, _ = torch.cuda.mem_get_info(dev)
                if need > free // 2:  # keep at least half of what is free for the KV cache
                    self.prefill_weight_cache = False
                    self.ws.dq_buffer(max(w.n * ((w.k + 63) // 64 * 64) for w in allw))
                    ws = []
                for w in ws:
                    w.dense = ops.dequant_weight(w)
                    self.prefill_cache_bytes += w.dense.numel() * 2
            elif ws:
                # bf16 expansion buffer of the large-M GEMM path, sized for the largest layer weight
                self.ws.dq_buffer(max(w.n * ((w.k + 63) // 64 * 64) for w in ws))
        self.vout_host = torch.zeros(B, 2 + ops.kernels.MAX_TREE_NODES, dtype=torch.int32, pin_memory=True)
        self._layer_ptrs = None
        self.last_verify = None
        self.last_preds = None
        self.max_pages = (self.max_model_len + self.qcfg.page_size - 1) // self.qcfg.page_size
        # one packed int32 staging area for all per-step metadata
        self.meta_cap = (9 * T + 16 * B + B * self.max_pages + B * 64 + B * ((cfg.vocab_size + 31) // 32) + 1024 +
                         B * (ops.kernels.TREE_META_INTS + 2))
        self.meta_host = torch.empty(self.meta_cap, dtype=torch.int32, pin_memory=True)
        self.meta_dev = torch.empty(self.meta_cap, dtype=torch.int32, device=dev)
        self.ws.reserve_attn(B, cfg.num_heads, 64, cfg.head_dim)
        self.ws.sampler_buffer(R, cfg.vocab_size)
        rot_k = [w.k for lw in self.layers for w in (lw.qkv, lw.o, lw.gate_up, lw.down, self.lm_head_q)
                 if w is not None and getattr(w, "rot", None) is not None]
        if rot_k:  # SQINT2 input rotations: one scratch for the largest activation block
            self.ws.rot_buffer(max(T, R), max(rot_k))

    # ------------------------------------------------------------------ metadata upload
    def upload(self, st: StepInputs) -> dict:
        """Pack all per-step arrays into one pinned buffer, one H2D copy; return device views."""
        arrays = {
            "ids": st.input_ids, "pos": st.positions, "slots": st.slot_mapping, "dlens": st.decode_seq_lens,
            "qs": st.prefill_q_start, "ql": st.prefill_q_len, "ctx": st.prefill_ctx_len, "tseq": st.tile_seq,
            "tq0": st.tile_q0, "rows": st.logits_rows, "temp": st.temperature.view(np.int32),
            "topp": st.top_p.view(np.int32), "topk": st.top_k, "minp": st.min_p.view(np.int32),
            "rep": st.rep_penalty.view(np.int32), "step": st.rng_step,
        }
        bt = st.block_tables
        if st.hist is not None:
            arrays["hist"] = st.hist.reshape(-1)
        if st.allow_mask is not None:
            arrays["mask"] = st.allow_mask.reshape(-1)
        if st.tree_mask is not None:
            arrays["tmask"] = st.tree_mask
        if st.verify_meta is not None:
            arrays["vmeta"] = st.verify_meta.reshape(-1)
            arrays["vtemp"] = st.verify_temp.view(np.int32)
            arrays["vstep"] = st.verify_step
        host = self.meta_host.numpy()
        off = 0
        offs = {}
        for k, a in arrays.items():
            n = a.size
            host[off:off + n] = a.reshape(-1)
            offs[k] = (off, n)
            off += n
        nb = bt.size
        host[off:off + nb] = bt.reshape(-1)
        offs["bt"] = (off, nb)
        off += nb
        if off > self.meta_cap:
            raise ValueError("step metadata exceeds the staging buffer")
        self.meta_dev[:off].copy_(self.meta_host[:off], non_blocking=True)
        d = {k: self.meta_dev[o:o + n] for k, (o, n) in offs.items()}
        for k in ("temp", "topp", "minp", "rep"):
            d[k] = d[k].view(torch.float32)
        d["bt"] = d["bt"].view(bt.shape[0], bt.shape[1]) if bt.size else d["bt"].view(0, max(bt.shape[1], 1))
        if "hist" in d:
            d["hist"] = d["hist"].view(st.hist.shape[0], st.hist.shape[1])
        if "mask" in d:
            d["mask"] = d["mask"].view(st.allow_mask.shape[0], st.allow_mask.shape[1])
        if "vmeta" in d:
            d["vmeta"] = d["vmeta"].view(st.verify_meta.shape[0], st.verify_meta.shape[1])
            d["vtemp"] = d["vtemp"].view(torch.float32)
        return d

    # ------------------------------------------------------------------ forward
    # layer split: a callable(st, T) that runs the earlier stages and leaves the hidden state of
    # the step's T tokens in self.h[:T] (set by LayerSplitRunner), instead of the embedding
    upstream = None

    def forward(self, st: StepInputs, m: dict) -> torch.Tensor:
        self.run_layers(st, m)
        B = st.logits_rows.shape[0]
        xs = ops.rmsnorm(self.h[:st.num_tokens], self.norm, self.cfg.rms_eps, out=self.xs[:B], row_idx=m["rows"])
        return self._lm_head(xs, B)

    def run_layers(self, st: StepInputs, m: dict) -> None:
        """Embedding (or the upstream stages) and this runner's decoder layers, in place on self.h."""
        cfg = self.cfg
        T, Bd = st.num_tokens, st.num_decode
        ws = self.ws
        h, x = self.h[:T], self.x[:T]
        if self.upstream is not None:
            self.upstream(st, T)
        else:
            torch.index_select(self.embed, 0, m["ids"], out=h)
        hkv = cfg.num_kv_heads
        dsplit = ops.kernels.decode_splits(max(Bd, 1), hkv, max(st.max_decode_ctx, 1)) if Bd else (1, 1)
        o = self.offload
        if o is not None:
            self._offload_fetch(o["first"])
        for li, lw in enumerate(self.layers):
            if o is not None and li >= o["first"]:
                b = (li - o["first"]) % 2
                if li + 1 < len(self.layers):
                    self._offload_fetch(li + 1)  # the next layer streams in while this one computes
                torch.cuda.current_stream(self.device).wait_event(o["copied"][b])
            ops.rmsnorm(h, lw.ln1, cfg.rms_eps, out=x)
            qkv = ops.w4a16_linear(x, lw.qkv, out=self.qkv[:T], ws=ws)
            attn = self._attention(li, lw, qkv, st, m, dsplit)
            self._row_parallel(attn, lw.o, h)
            ops.rmsnorm(h, lw.ln2, cfg.rms_eps, out=x)
            if lw.moe is not None:
                lw.moe.forward(x, h, ws)
            else:
                act = ops.w4a16_linear(x, lw.gate_up, out=self.act[:T], silu_mul=True, ws=ws)
                self._row_parallel(act[:, : self.F], lw.down, h)
            if o is not None and li >= o["first"]:
                o["done"][(li - o["first"]) % 2].record(torch.cuda.current_stream(self.device))

    def _attention(self, li: int, lw, qkv: torch.Tensor, st: StepInputs, m: dict, dsplit) -> torch.Tensor:
        """RoPE + KV write, then decode and prefill attention of layer li over the paged cache."""
        cfg, ws = self.cfg, self.ws
        T, Bd, Bp = st.num_tokens, st.num_decode, st.num_prefill
        hq, hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        ps, grp = self.qcfg.page_size, self.qcfg.kv_group
        bt = m["bt"]
        kc, ks, vc, vs = self.pools.layers[li]
        q = self.q[:T]
        ops.rope_kv_write(qkv, m["pos"], self.cos_sin, q, m["slots"], kc, ks, vc, vs, hq, hkv, d, ps, grp,
                          self.fk, self.fv, lw.q_norm, lw.k_norm, cfg.rms_eps, ws=ws, had_k=self.had_k,
                          had_v=self.had_v)
        attn = self.attn[:T]
        if Bd:
            ops.paged_decode_attention(q[:Bd], kc, ks, vc, vs, bt[:Bd], m["dlens"], attn[:Bd], hq, hkv, d, ps, grp,
                                       self.fk, self.fv, self.sm_scale, st.max_decode_ctx, ws=ws, splits=dsplit)
            if self.score_step:
                ops.kernels.page_mass(q[:Bd].view(Bd, hq * d), kc, ks, bt[:Bd], m["dlens"], self.page_mass_buf, hq,
                                      hkv, d, ps, grp, self.fk, self.sm_scale, ws=ws)
        if Bp:
            tm = m["tmask"][Bd:] if "tmask" in m else None
            ops.paged_prefill_attention(q[Bd:], kc, ks, vc, vs, bt[Bd:], m["tseq"], m["tq0"], m["qs"], m["ql"],
                                        m["ctx"], st.tile_seq.shape[0], attn[Bd:], hq, hkv, d, ps, grp, self.fk,
                                        self.fv, self.sm_scale, tree_mask=tm, ws=ws)
        if self.had_v_row is not None:  # values were stored rotated: o = H (s_v * o_rot) / sqrt(D)
            native().hadamard_rows(attn, self.had_v_row, d, attn)
        return attn

    # hooks overridden by the tensor-parallel runner
    def _row_parallel(self, x: torch.Tensor, w: Int4Weight, h: torch.Tensor) -> None:
        """h += x @ w^T (residual fused into the GEMM epilogue)."""
        ops.w4a16_linear(x, w, out=h, residual=h, ws=self.ws)

    def _lm_head(self, xs: torch.Tensor, B: int) -> torch.Tensor:
        if self.lm_head_q is not None:
            return ops.w4a16_linear(xs, self.lm_head_q, out=self.logits[:B], ws=self.ws)
        return torch.matmul(xs, self.lm_head_dense.T, out=self.logits[:B])

    def sample(self, st: StepInputs, m: dict, logits: torch.Tensor) -> torch.Tensor:
        B = logits.shape[0]
        greedy = bool((st.temperature <= 0).all()) and st.hist is None
        out = self.tokens[:B]
        if greedy and not (st.rep_penalty != 1).any():
            ops.sample(logits, out, allow_mask=m.get("mask"), ws=self.ws)
        else:
            ops.sample(logits, out, temperature=m["temp"], top_p=m["topp"], top_k=m["topk"], min_p=m["minp"],
                       rep_penalty=m["rep"], hist=m.get("hist"), allow_mask=m.get("mask"), seed=st.seed,
                       step=m["step"], ws=self.ws)
        return out

    def logit_row(self, i: int) -> torch.Tensor:
        """The logits row the last step sampled its i-th token from."""
        return self.logits[i]

    @torch.inference_mode()
    def sample_row(self, row: torch.Tensor, temperature: float, top_p: float, top_k: int, min_p: float,
                   rep_penalty: float, hist: np.ndarray | None, seed: int, step: int) -> int:
        """Sample one token from a stored logits row with the step sampler's semantics."""
        out = self.tokens[-1:]
        lg = row[None]
        if temperature <= 0 and hist is None:
            ops.sample(lg, out, ws=self.ws)
        else:
            dev = self.device
            f32 = lambda v: torch.tensor([v], dtype=torch.float32, device=dev)  # noqa: E731
            i32 = lambda v: torch.tensor([v], dtype=torch.int32, device=dev)  # noqa: E731
            h = None if hist is None else torch.from_numpy(hist).to(dev)
            ops.sample(lg, out, temperature=f32(temperature), top_p=f32(top_p), top_k=i32(top_k), min_p=f32(min_p),
                       rep_penalty=f32(rep_penalty), hist=h, seed=seed, step=i32(step), ws=self.ws)
        return int(out.item())

    def sample_full(self, st: StepInputs, m: dict, logits: torch.Tensor) -> torch.Tensor:
        """The sampler with every per-row parameter bound (no host-side branching: graph-safe)."""
        out = self.tokens[: logits.shape[0]]
        ops.sample(logits, out, temperature=m["temp"], top_p=m["topp"], top_k=m["topk"], min_p=m["minp"],
                   rep_penalty=m["rep"], hist=m.get("hist"), seed=st.seed, step=m["step"], ws=self.ws)
        return out

    # ------------------------------------------------------------------ device-side step timing
    timing = False
    _events: list = []
    sync_wait_s = 0.0  # host time spent waiting for the device at the end of steps

    def sync(self) -> None:
        t = time.perf_counter()
        torch.cuda.current_stream(self.device).synchronize()
        self.sync_wait_s += time.perf_counter() - t

    def timer_start(self) -> None:
        if self.timing:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._events.append([e, None])

    def timer_stop(self) -> None:
        if self.timing:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._events[-1][1] = e

    def device_time_ms(self, reset: bool = True) -> float:
        """Sum of the device intervals (H2D metadata copy .. sampled-token D2H) of timed steps."""
        torch.cuda.synchronize(self.device)
        t = sum(a.elapsed_time(b) for a, b in self._events if b is not None)
        if reset:
            self._events = []
        return t

    @torch.inference_mode()
    def execute(self, st: StepInputs) -> np.ndarray:
        self.timer_start()
        if self.score_step:
            n = self.pools.layers[0][0].shape[0]
            if self.page_mass_buf.numel() != n:  # (the page pool is sized after the weights load)
                self.page_mass_buf = torch.zeros(n, dtype=torch.float32, device=self.device)
            self.page_mass_buf.zero_()
        m = self.upload(st)
        logits = self.forward(st, m)
        nS = st.num_sample_rows
        toks = self.sample(st, m, logits[:nS]) if nS else self.tokens[:0]
        B = toks.shape[0]
        self.tokens_host[:B].copy_(toks, non_blocking=True)
        G = st.num_verify
        if G:
            vl = logits[nS:]
            ops.kernels.tree_verify(vl, m["vmeta"], m["vtemp"], m["vstep"], st.seed, self.vout[:G],
                                    draft_logits=st.draft_logits, ws=self.ws)
            self.vout_host[:G].copy_(self.vout[:G], non_blocking=True)
            if st.verify_preds:
                nv = vl.shape[0]
                preds = self.tokens[B:B + nv]
                ops.sample(vl, preds, ws=self.ws)
                self.tokens_host[B:B + nv].copy_(preds, non_blocking=True)
        self.timer_stop()
        self.sync()
        self.last_logits = logits if st.all_logits else None
        self.last_hidden = self.xs[:logits.shape[0]]  # every logits row: sampled, then verified nodes
        if G:
            self.last_verify = self.vout_host[:G].numpy().copy()
            nv = logits.shape[0] - nS
            self.last_preds = self.tokens_host[B:B + nv].numpy().copy() if st.verify_preds else None
        return self.tokens_host[:B].numpy().copy()

    def kv_compact(self, src: list[int], dst: list[int]) -> None:
        """Move accepted tree nodes' KV rows (every layer) from ``src`` to ``dst`` cache slots."""
        if not src:
            return
        if self._layer_ptrs is None:
            rows = [[kc.data_ptr(), ks.data_ptr(), vc.data_ptr(), vs.data_ptr()] for kc, ks, vc, vs in self.pools.layers]
            self._layer_ptrs = torch.tensor(rows, dtype=torch.int64, device=self.device)
        kc, ks, vc, vs = self.pools.layers[0]
        pair = torch.tensor([src, dst], dtype=torch.int32).to(self.device, non_blocking=False)
        ops.kernels.kv_compact(self._layer_ptrs, pair[0], pair[1], self.cfg.num_kv_heads, self.qcfg.page_size,
                               kc.shape[-1], vc.shape[-1], ks.shape[-1], vs.shape[-1])


# ----------------------------------------------------------------------------- CPU oracle of the step
def layer_slice(ck: Checkpoint, a: int, b: int) -> Checkpoint:
    """The checkpoint of decoder layers [a, b) (renumbered from 0) plus the embedding, final norm
    and LM head (tensors shared, not copied)."""
    import dataclasses

    pre = "model.layers."
    tensors = {}
    for k, v in ck.tensors.items():
        if not k.startswith(pre):
            tensors[k] = v
            continue
        i, rest = k[len(pre):].split(".", 1)
        if a <= int(i) < b:
            tensors[f"{pre}{int(i) - a}.{rest}"] = v
    return Checkpoint(dataclasses.replace(ck.config, num_layers=b - a), ck.quant, tensors)


class LayerSplitRunner:
    """The decoder layers split in contiguous ranges over several GPUs of one process, the
    reference's only multi-device mode (HF ``device_map="auto"``, squish/backend.py:295): stage
    i holds layers [b_i, b_i+1) and their KV pages on its device, the hidden state of the
    step's tokens moves to the next device once per stage, and the last stage applies the final
    norm, the LM head and the sampler. Every stage keeps its own copy of the embedding and
    head tensors (only the first / last use them). The engine talks to the last stage; steps
    run eagerly (no CUDA graphs)."""

    def __init__(self, ck: Checkpoint, devices: list, num_pages: int, **kw):
        L, S = ck.config.num_layers, len(devices)
        if S < 2 or S > L:
            raise ValueError(f"layer split needs 2..{L} stages, got {S}")
        bounds = [round(i * L / S) for i in range(S + 1)]
        self.bounds = bounds
        self.stages = [CudaRunner(layer_slice(ck, bounds[i], bounds[i + 1]), d, num_pages, **kw)
                       for i, d in enumerate(devices)]
        self.cfg = ck.config
        for k in range(1, S):
            self.stages[k].upstream = self._feeder(k)

    def _feeder(self, k: int):
        def run(st: StepInputs, T: int) -> None:
            prev, cur = self.stages[k - 1], self.stages[k]
            prev.run_layers(st, prev.upload(st))
            # (a cross-device copy is ordered after the source device's current stream)
            cur.h[:T].copy_(prev.h[:T], non_blocking=True)
        return run

    @property
    def last(self) -> CudaRunner:
        return self.stages[-1]

    _own = ("stages", "bounds", "cfg")

    def __getattr__(self, name):  # the engine-facing surface is the last stage's
        if name in LayerSplitRunner._own:
            raise AttributeError(name)
        return getattr(self.stages[-1], name)

    def __setattr__(self, name, value):
        if name in LayerSplitRunner._own:
            object.__setattr__(self, name, value)
        else:
            setattr(self.stages[-1], name, value)

    @property
    def pools_all(self) -> list:
        return [s.pools for s in self.stages]

    def execute(self, st: StepInputs) -> np.ndarray:
        return self.last.execute(st)

    def kv_compact(self, src, dst) -> None:
        for s in self.stages:
            s.kv_compact(src, dst)


class TorchPagedRunner:
    """The same step semantics as CudaRunner in plain PyTorch on the CPU (fp32)."""

    def __init__(self, ck: Checkpoint, num_pages: int, max_model_len: int = 2048):
        from .reference import ReferenceModel

        self.ref = ReferenceModel(ck)
        self.cfg, self.qcfg = ck.config, ck.quant
        cfg, q = self.cfg, self.qcfg
        self.ps = q.page_size
        # dense (dequantized) page pools [P, Hkv, PS, D]
        self.k = torch.zeros(cfg.num_layers, num_pages, cfg.num_kv_heads, self.ps, cfg.head_dim)
        self.v = torch.zeros_like(self.k)
        self.cos_sin = rope_table(cfg, max_model_len + 1)
        self.last_logits = None
        self.logits = None
        self.last_verify = self.last_preds = None
        self.score_step = False
        self.page_mass_buf = torch.zeros(num_pages)

    def kv_compact(self, src: list[int], dst: list[int]) -> None:
        for a, b in zip(src, dst):
            self.k[:, b // self.ps, :, b % self.ps] = self.k[:, a // self.ps, :, a % self.ps]
            self.v[:, b // self.ps, :, b % self.ps] = self.v[:, a // self.ps, :, a % self.ps]

    @torch.no_grad()
    def execute(self, st: StepInputs) -> np.ndarray:
        from .reference import _rms, _rope

        cfg, w = self.cfg, self.ref.w
        T = st.num_tokens
        if self.score_step:
            self.page_mass_buf.zero_()
        ids = torch.from_numpy(st.input_ids.astype(np.int64))
        pos = torch.from_numpy(st.positions.astype(np.int64))
        slots = torch.from_numpy(st.slot_mapping.astype(np.int64))
        cs = self.cos_sin[pos]
        h = w["model.embed_tokens.weight"][ids]
        hq, hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        Bd = st.num_decode
        # per-row (sequence index, visible context length) for attention
        seq_rows = []
        for i in range(Bd):
            seq_rows.append((i, int(st.decode_seq_lens[i]), i, 1))
        for j in range(st.num_prefill):
            seq_rows.append((Bd + j, int(st.prefill_ctx_len[j]), Bd + int(st.prefill_q_start[j]),
                             int(st.prefill_q_len[j])))
        for li in range(cfg.num_layers):
            p = f"model.layers.{li}."
            x = _rms(h, w[p + "input_layernorm.weight"], cfg.rms_eps)
            qv = x @ w[p + "self_attn.q_proj.weight"].T
            kv = x @ w[p + "self_attn.k_proj.weight"].T
            vv = x @ w[p + "self_attn.v_proj.weight"].T
            if cfg.qkv_bias:
                qv = qv + w[p + "self_attn.q_proj.bias"]
                kv = kv + w[p + "self_attn.k_proj.bias"]
                vv = vv + w[p + "self_attn.v_proj.bias"]
            qv, kv, vv = qv.view(T, hq, d), kv.view(T, hkv, d), vv.view(T, hkv, d)
            if cfg.qk_norm:
                qv = _rms(qv, w[p + "self_attn.q_norm.weight"], cfg.rms_eps)
                kv = _rms(kv, w[p + "self_attn.k_norm.weight"], cfg.rms_eps)
            qv, kv, vv = self.ref.rotate_kv(_rope(qv, cs), _rope(kv, cs), vv)
            kq = self.ref._kv_roundtrip(kv, self.ref.fk)
            vq = self.ref._kv_roundtrip(vv, self.ref.fv)
            valid = slots >= 0
            pg, off = slots[valid] // self.ps, slots[valid] % self.ps
            self.k[li, pg, :, off] = kq[valid]
            self.v[li, pg, :, off] = vq[valid]
            attn = torch.zeros(T, hq * d)
            for (bt_row, ctx, r0, n) in seq_rows:
                npg = (ctx + self.ps - 1) // self.ps
                pages = torch.from_numpy(st.block_tables[bt_row, :npg].astype(np.int64))
                K = self.k[li, pages].permute(0, 2, 1, 3).reshape(-1, hkv, d)[:ctx]
                V = self.v[li, pages].permute(0, 2, 1, 3).reshape(-1, hkv, d)[:ctx]
                K = K.repeat_interleave(hq // hkv, dim=1)
                V = V.repeat_interleave(hq // hkv, dim=1)
                qq = qv[r0:r0 + n]
                s = torch.einsum("qhd,khd->hqk", qq, K) / math.sqrt(d)
                qpos = torch.arange(ctx - n, ctx)
                bad = torch.arange(ctx)[None, :] > qpos[:, None]
                if st.tree_mask is not None:
                    for i in range(n):
                        tm = int(st.tree_mask[r0 + i]) & 0xFFFFFFFF
                        if tm:
                            for j in range(n):
                                if not (tm >> j) & 1:
                                    bad[i, ctx - n + j] = True
                s = s.masked_fill(bad[None], float("-inf"))
                pr = torch.softmax(s, -1)
                if self.score_step and bt_row < Bd:  # attention mass per page (H2O-style scores)
                    per_key = pr.sum((0, 1))
                    self.page_mass_buf.index_add_(0, pages.repeat_interleave(self.ps)[:ctx], per_key)
                o = torch.einsum("hqk,khd->qhd", pr, V)
                attn[r0:r0 + n] = self.ref.unrotate_out(o).reshape(n, hq * d)
            h = h + self.ref._rp(attn, w[p + "self_attn.o_proj.weight"])
            x = _rms(h, w[p + "post_attention_layernorm.weight"], cfg.rms_eps)
            h = h + self.ref._mlp(p, x)
        rows = torch.from_numpy(st.logits_rows.astype(np.int64))
        xs = _rms(h[rows], w["model.norm.weight"], cfg.rms_eps)
        logits = self.ref._head(xs, w["lm_head.weight"])
        self.logits = logits.to(torch.bfloat16)
        self.last_logits = logits
        self.last_hidden = xs
        nS = st.num_sample_rows
        self.last_verify = self.last_preds = None
        if st.num_verify:
            from ..engine.speculative import MAX_TREE_NODES, DraftTree, tree_verify_ref

            vl = logits[nS:]
            res = np.zeros((st.num_verify, 2 + MAX_TREE_NODES), dtype=np.int32)
            for g_, meta in enumerate(st.verify_meta):
                r0_, n_ = int(meta[0]), int(meta[1])
                par = meta[2:2 + n_].tolist()
                tok = meta[2 + MAX_TREE_NODES:2 + MAX_TREE_NODES + n_].tolist()
                qr = meta[2 + 2 * MAX_TREE_NODES:2 + 2 * MAX_TREE_NODES + n_].tolist()
                tree = DraftTree(tok, par, qr)
                path, fin = tree_verify_ref(vl[r0_:r0_ + n_], tree, float(st.verify_temp[g_]), int(st.seed),
                                            int(st.verify_step[g_]), st.draft_logits)
                res[g_, 0], res[g_, 1] = len(path), fin
                res[g_, 2:2 + len(path)] = path
            self.last_verify = res
            if st.verify_preds:
                self.last_preds = vl.argmax(-1).numpy().astype(np.int32)
        out = np.empty(nS, dtype=np.int32)
        for i in range(nS):
            out[i] = self._sample(logits[i], None if st.allow_mask is None else st.allow_mask[i],
                                  float(st.temperature[i]), float(st.top_p[i]), int(st.top_k[i]),
                                  float(st.rep_penalty[i]), None if st.hist is None else st.hist[i], int(st.seed),
                                  int(st.rng_step[i]))
        return out

    @staticmethod
    def _sample(row, mask, temperature, top_p, top_k, rep_penalty, hist, seed, step) -> int:
        lg = row.clone()
        if mask is not None:
            bits = np.unpackbits(mask.view(np.uint8), bitorder="little")[: lg.shape[0]]
            lg[torch.from_numpy(bits == 0)] = float("-inf")
        if hist is not None and rep_penalty != 1.0:
            for t in set(t for t in hist.tolist() if t >= 0):
                lg[t] = lg[t] / rep_penalty if lg[t] > 0 else lg[t] * rep_penalty
        if temperature <= 0:
            return int(lg.argmax())
        g = torch.Generator().manual_seed(seed * 1000003 + step)
        pr = torch.softmax(lg / temperature, -1)
        if top_k > 0:
            kth = pr.topk(top_k).values[-1]
            pr = torch.where(pr >= kth, pr, torch.zeros_like(pr))
        if top_p < 1.0:
            sp, si = pr.sort(descending=True)
            cum = sp.cumsum(0)
            cut = int((cum < top_p).sum()) + 1
            keep = torch.zeros_like(pr)
            keep[si[:cut]] = pr[si[:cut]]
            pr = keep
        return int(torch.multinomial(pr / pr.sum(), 1, generator=g))

    def logit_row(self, i: int) -> torch.Tensor:
        return self.last_logits[i]

    def sample_row(self, row, temperature, top_p, top_k, min_p, rep_penalty, hist, seed, step) -> int:
        return self._sample(row, None, temperature, top_p, top_k, rep_penalty, None if hist is None else hist[0],
                            seed, step)
