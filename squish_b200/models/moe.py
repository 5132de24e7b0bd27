"""Mixture-of-experts FFN (Qwen3-MoE: softmax router, top-k experts, renormalised weights)
on the sm_100a kernels.

One step of a layer:

    logits = x . Wg^T                      (bf16 GEMM, [T, E])
    route  -> top-k ids and weights        (moe.cu, one warp per token)
    align  -> expert-sorted, tile-padded slot layout + each token tile's expert
    gather -> X_sorted                     (rows of x in slot order, padding rows zero)
    grouped INT4 GEMM gate_up (SiLU*up epilogue) -> act_sorted
    grouped INT4 GEMM down                       -> y_sorted
    combine: h[t] += sum_k w[t, k] * y_sorted[pos(t, k)]

All shapes are fixed by the token count T, so the sequence is CUDA-graph capturable: the
per-expert counts never leave the device. The reference's router is numpy / Rust
(squish_quant_rs/src/lib.rs:2688,2727); its experts run through mlx_lm.
"""
from __future__ import annotations

import torch

from .. import ops
from ..ops import kernels as K_
from .config import ModelConfig
from .weights import Checkpoint


class MoEScratch:
    """Step buffers shared by every MoE layer of a runner (layers run one after another)."""

    def __init__(self, cfg: ModelConfig, max_tokens: int, device):
        dev = torch.device(device)
        E, K, H = cfg.num_experts, cfg.num_experts_per_tok, cfg.hidden_size
        El = cfg.num_local_experts or E
        F = (cfg.moe_intermediate_size + 63) // 64 * 64
        T = max(max_tokens, 1)
        bn = K_.moe_tile(T, K, El)
        P = K_.moe_padded_rows(T, K, El, bn)
        i32 = torch.int32
        self.max_tokens = T
        self.logits = torch.empty(T, E, dtype=torch.bfloat16, device=dev)
        self.ids = torch.empty(T * K, dtype=i32, device=dev)
        self.w = torch.empty(T * K, dtype=torch.float32, device=dev)
        self.sorted_slot = torch.empty(P, dtype=i32, device=dev)
        self.slot_pos = torch.empty(T * K, dtype=i32, device=dev)
        self.tile_expert = torch.empty(P // 16, dtype=i32, device=dev)
        self.num_tiles = torch.zeros(1, dtype=i32, device=dev)
        self.counts = torch.zeros(El, dtype=i32, device=dev)
        self.part = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)  # expert-parallel partial output
        self.xs = torch.empty(P, H, dtype=torch.bfloat16, device=dev)
        self.act = torch.empty(P, F, dtype=torch.bfloat16, device=dev)
        self.ys = torch.empty(P, H, dtype=torch.bfloat16, device=dev)


def _interleave(gate, up):
    from .decoder import _interleave_gate_up

    return _interleave_gate_up(gate, up)


class MoELayer:
    def __init__(self, cfg: ModelConfig, gate_w: torch.Tensor, gate_up: K_.GroupedInt4Weight,
                 down: K_.GroupedInt4Weight, scratch: MoEScratch | None = None):
        self.cfg = cfg
        self.gate_w = gate_w  # [E, H] bf16
        self.gate_up = gate_up
        self.down = down
        self.scratch = scratch
        self.E, self.K = cfg.num_experts, cfg.num_experts_per_tok
        self.E_local = cfg.num_local_experts or cfg.num_experts
        self.offset = cfg.expert_offset
        self.F = cfg.moe_intermediate_size
        # expert parallelism: callable(partial, h) adding the all-reduced partial to h
        self.ep_reduce = None

    @classmethod
    def from_checkpoint(cls, ck: Checkpoint, layer: int, device, scratch: MoEScratch | None = None) -> "MoELayer":
        from .decoder import _as_q4a

        cfg, t = ck.config, ck.tensors
        dev = torch.device(device)
        p = f"model.layers.{layer}.mlp."
        g = ck.quant.group_size
        gu, dn = [], []
        e0 = cfg.expert_offset
        for e in range(e0, e0 + (cfg.num_local_experts or cfg.num_experts)):
            q = p + f"experts.{e}."
            w = _interleave(_as_q4a(t[q + "gate_proj.weight"], g), _as_q4a(t[q + "up_proj.weight"], g))
            gu.append(ops.prepare_int4_weight(w.packed, w.scales, w.offsets, w.shape[1], w.group, dev))
            d = _as_q4a(t[q + "down_proj.weight"], g)
            dn.append(ops.prepare_int4_weight(d.packed, d.scales, d.offsets, d.shape[1], d.group, dev))
        gate_w = t[p + "gate.weight"].data.to(dev, torch.bfloat16).contiguous()
        return cls(cfg, gate_w, K_.stack_int4_experts(gu), K_.stack_int4_experts(dn), scratch)

    def forward(self, x: torch.Tensor, h: torch.Tensor, ws=None) -> None:
        """h[:T] += MoE(x[:T]) in place."""
        sc = self.scratch
        T = x.shape[0]
        if T == 0:
            return
        if sc is None or T > sc.max_tokens:
            sc = self.scratch = MoEScratch(self.cfg, max(T, sc.max_tokens if sc else 0), x.device)
        E, K = self.E_local, self.K
        bn = K_.moe_tile(T, K, E)
        P = K_.moe_padded_rows(T, K, E, bn)
        TK = T * K
        logits = torch.mm(x, self.gate_w.t(), out=sc.logits[:T])
        K_.moe_route(logits, K, self.cfg.norm_topk_prob, sc.ids[:TK], sc.w[:TK])
        if self.offset:
            sc.ids[:TK].sub_(self.offset)  # global -> local expert ids; others fall outside [0, E_local)
        K_.moe_align(sc.ids[:TK], E, bn, sc.sorted_slot[:P], sc.slot_pos[:TK], sc.tile_expert[: P // bn],
                     sc.num_tiles, sc.counts)
        K_.moe_gather(x, sc.sorted_slot[:P], sc.num_tiles, bn, K, sc.xs[:P])
        act = K_.w4a16_grouped_linear(sc.xs[:P], self.gate_up, sc.act[:P, : self.gate_up.n // 2],
                                      sc.tile_expert[: P // bn], sc.num_tiles, bn, silu_mul=True, ws=ws)
        K_.w4a16_grouped_linear(act[:, : self.F], self.down, sc.ys[:P], sc.tile_expert[: P // bn], sc.num_tiles, bn,
                                ws=ws)
        if self.ep_reduce is None:
            K_.moe_combine(sc.ys[:P], sc.slot_pos[:TK], sc.w[:TK], K, h)
        else:
            part = sc.part[:T]
            part.zero_()
            K_.moe_combine(sc.ys[:P], sc.slot_pos[:TK], sc.w[:TK], K, part)
            self.ep_reduce(part, h)

    def forward_a2a(self, comm, x_own: torch.Tensor, T: int, ws=None) -> int:
        """Expert-parallel step with the all-to-all over peer memory (sequence-parallel layout,
        csrc/ep_a2a.cu): route this rank's owned rows x_own [own, H], dispatch each row to the
        ranks holding its experts, run the local experts over the tp x R received row slots and
        send the weighted sums back to the row owners' reduce-scatter blocks. Returns the
        arrivals per source that the owners' tp_rs_norm_ag waits for."""
        sc = self.scratch
        R = comm.sp_rows(T)
        Tr = comm.tp * R
        if sc is None or Tr > sc.max_tokens:
            sc = self.scratch = MoEScratch(self.cfg, max(Tr, sc.max_tokens if sc else 0), x_own.device)
        E, K = self.E_local, self.K
        own = x_own.shape[0]
        logits = torch.mm(x_own, self.gate_w.t(), out=sc.logits[:own]) if own else None
        comm.ep_dispatch(x_own, logits, self.cfg.norm_topk_prob, sc.ids, sc.w, T)  # routes, then sends
        bn = K_.moe_tile(Tr, K, E)
        P = K_.moe_padded_rows(Tr, K, E, bn)
        TK = Tr * K
        comm.ep_align(T, bn, sc.sorted_slot[:P], sc.slot_pos[:TK], sc.tile_expert[: P // bn], sc.num_tiles,
                      sc.counts)
        K_.moe_gather(comm.ep_x[:Tr], sc.sorted_slot[:P], sc.num_tiles, bn, K, sc.xs[:P])
        act = K_.w4a16_grouped_linear(sc.xs[:P], self.gate_up, sc.act[:P, : self.gate_up.n // 2],
                                      sc.tile_expert[: P // bn], sc.num_tiles, bn, silu_mul=True, ws=ws)
        K_.w4a16_grouped_linear(act[:, : self.F], self.down, sc.ys[:P], sc.tile_expert[: P // bn], sc.num_tiles, bn,
                                ws=ws)
        return comm.ep_combine(sc.ys[:P], sc.slot_pos[:TK], T)
