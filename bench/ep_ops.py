#!/usr/bin/env python
"""Per-layer timing of an expert-parallel MoE block in three collective formulations (torchrun,
one process per GPU):

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 bench/ep_ops.py [--rows 16,64,256]

Layer shape: Qwen3-30B-A3B (hidden 2048, 128 experts, top-8, expert FFN 768, INT4 g64 experts,
random weights); rank r holds experts [r E / tp, (r + 1) E / tp). Every mode starts from the
attention output already summed into the residual and ends with RMSNorm(h) of all T rows on
every rank (the next layer's input), so the modes do the same math:

  allreduce  every rank holds all T rows: route all of them, run the local experts over the
             slots that land here, all-reduce the partial output into h (one-shot peer-memory
             all-reduce for <= 256 rows), RMSNorm
  a2a        rank r owns T / tp rows: route the owned rows, dispatch each row to the ranks
             holding its experts (P2P stores, csrc/ep_a2a.cu), local experts over the received
             rows, combine back into the owners' reduce-scatter blocks, fused residual add +
             RMSNorm + all-gather (tp_rs_norm_ag)
  nccl       the a2a data movement with NCCL: the same dispatch / combine kernels write into
             local send buffers, torch.distributed.all_to_all_single moves them, then a torch
             residual add, RMSNorm and all_gather_into_tensor

CUDA events per rank after warm-up; the JSON lines report the max over ranks of the mean
per-iteration time.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from squish_b200 import ops  # noqa: E402
from squish_b200._ext import native  # noqa: E402
from squish_b200.models.config import ModelConfig  # noqa: E402
from squish_b200.models.moe import MoELayer, MoEScratch  # noqa: E402
from squish_b200.ops import kernels as K_  # noqa: E402
from squish_b200.parallel.comm import TPComm  # noqa: E402


def expert_layer(cfg: ModelConfig, rank: int, tp: int, dev) -> MoELayer:
    """Random INT4 experts of this rank and the replicated router."""
    import dataclasses

    E, H, F = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
    El = E // tp
    lc = dataclasses.replace(cfg, num_local_experts=El, expert_offset=rank * El)
    gu, dn = [], []
    for e in range(rank * El, (rank + 1) * El):
        g = torch.Generator().manual_seed(1000 + e)
        w = torch.randn(2 * F, H, generator=g) * 0.02
        p, s, z = native().cpu.quantize_int4_asym(w, 64)
        gu.append(ops.prepare_int4_weight(p, s, z, H, 64, dev))
        w = torch.randn(H, F, generator=g) * 0.02
        p, s, z = native().cpu.quantize_int4_asym(w, 64)
        dn.append(ops.prepare_int4_weight(p, s, z, F, 64, dev))
    gate = (torch.randn(E, H, generator=torch.Generator().manual_seed(7)) * 0.02).to(torch.bfloat16).to(dev)
    return MoELayer(lc, gate, K_.stack_int4_experts(gu), K_.stack_int4_experts(dn), None)


def timed(fn, iters, warm=10):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1000 / iters  # us


class NcclA2A:
    """The all-to-all data movement over NCCL with the same dispatch / combine kernels."""

    def __init__(self, layer: MoELayer, tp: int, rank: int, Tmax: int, H: int, dev):
        self.layer, self.tp, self.rank, self.H = layer, tp, rank, H
        R = -(-Tmax // tp)
        K = layer.K
        self.R, self.K = R, K
        bf, i32, f32 = torch.bfloat16, torch.int32, torch.float32
        self.send_x, self.recv_x = torch.empty(tp * R, H, dtype=bf, device=dev), torch.empty(tp * R, H, dtype=bf,
                                                                                            device=dev)
        self.send_ids, self.recv_ids = torch.empty(tp * R * K, dtype=i32, device=dev), torch.empty(
            tp * R * K, dtype=i32, device=dev)
        self.send_w, self.recv_w = torch.empty(tp * R * K, dtype=f32, device=dev), torch.empty(tp * R * K, dtype=f32,
                                                                                             device=dev)
        self.send_y, self.recv_y = torch.empty(tp * R, H, dtype=bf, device=dev), torch.empty(tp * R, H, dtype=bf,
                                                                                            device=dev)
        self.dummy = torch.zeros(2 * tp, dtype=i32, device=dev)
        self.zero_seq = torch.zeros(1, dtype=i32, device=dev)
        self.xg = torch.empty(tp * R, H, dtype=bf, device=dev)
        self.scratch = MoEScratch(layer.cfg, tp * R, dev)
        i64 = dict(dtype=torch.int64, device=dev)
        self.flag_ptrs = torch.tensor([self.dummy.data_ptr() + 4 * d for d in range(tp)], **i64)
        self._cache = {}

    def _ptrs(self, base: torch.Tensor, per_rank: int, esize: int, shift: bool) -> torch.Tensor:
        # dispatch writes slot (rank R + t) of destination d: point it at send block d
        key = (base.data_ptr(), per_rank, esize, shift)
        if key not in self._cache:  # built once per shape (no host copies in the timed loop)
            off = [(d - (self.rank if shift else 0)) * per_rank * esize for d in range(self.tp)]
            self._cache[key] = torch.tensor([base.data_ptr() + o for o in off], dtype=torch.int64, device=base.device)
        return self._cache[key]

    def run(self, x_own, h, lnw, T, ws):
        L, tp, R, K, H = self.layer, self.tp, -(-T // self.tp), self.K, self.H
        sc = self.scratch
        own = x_own.shape[0]
        logits = torch.mm(x_own, L.gate_w.t(), out=sc.logits[:own]) if own else None
        sx, sid, sw = self.send_x[: tp * R], self.send_ids[: tp * R * K], self.send_w[: tp * R * K]
        native().ep_dispatch(x_own, logits, L.cfg.norm_topk_prob, sc.ids, sc.w, own, R, K, L.E_local, self.rank, tp,
                             self._ptrs(sx, R * H, 2, True), self._ptrs(sid, R * K, 4, True),
                             self._ptrs(sw, R * K, 4, True), self.flag_ptrs)
        rx, rid, rw = self.recv_x[: tp * R], self.recv_ids[: tp * R * K], self.recv_w[: tp * R * K]
        dist.all_to_all_single(rx, sx)
        dist.all_to_all_single(rid, sid)
        dist.all_to_all_single(rw, sw)
        Tr, E = tp * R, L.E_local
        bn = K_.moe_tile(Tr, K, E)
        P = K_.moe_padded_rows(Tr, K, E, bn)
        K_.moe_align(rid, E, bn, sc.sorted_slot[:P], sc.slot_pos[: Tr * K], sc.tile_expert[: P // bn], sc.num_tiles,
                     sc.counts)
        K_.moe_gather(rx, sc.sorted_slot[:P], sc.num_tiles, bn, K, sc.xs[:P])
        act = K_.w4a16_grouped_linear(sc.xs[:P], L.gate_up, sc.act[:P, : L.gate_up.n // 2], sc.tile_expert[: P // bn],
                                      sc.num_tiles, bn, silu_mul=True, ws=ws)
        K_.w4a16_grouped_linear(act[:, : L.F], L.down, sc.ys[:P], sc.tile_expert[: P // bn], sc.num_tiles, bn, ws=ws)
        sy = self.send_y[: tp * R]
        native().ep_combine(sc.ys[:P], sc.slot_pos[: Tr * K], rw, R, K, tp, T,
                            self._ptrs(sy, R * H, 2, False), H, self.flag_ptrs, 0, self.zero_seq)
        ry = self.recv_y[: tp * R]
        dist.all_to_all_single(ry, sy)
        r0 = self.rank * R
        if own:
            hv = h[r0:r0 + own]
            hv.copy_((hv.float() + ry.view(tp, R, H)[:, :own].float().sum(0)).to(h.dtype))
        xn = self.xg[:R]  # this rank's block of the gather input
        xn.zero_()
        if own:
            ops.rmsnorm(h[r0:r0 + own], lnw, 1e-6, out=xn[:own])
        full = torch.empty(tp * R, H, dtype=h.dtype, device=h.device)
        dist.all_gather_into_tensor(full, xn)
        return full[:T]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", default="16,64,256", help="token rows T per step")
    ap.add_argument("--modes", default="allreduce,a2a,nccl")
    ap.add_argument("--iters", type=int, default=100)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = ModelConfig("qwen3-30b-a3b-moe-layer", "qwen3_moe", 151936, 2048, 1, 32, 4, 128, 6144, 1e-6, 1e6,
                      qk_norm=True, num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768)
    H = cfg.hidden_size
    rows = [int(x) for x in a.rows.split(",")]
    Tmax = max(rows)
    layer = expert_layer(cfg, rank, world, dev)
    ws = ops.Workspace(dev)
    lnw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    out = []
    for mode in a.modes.split(","):
        comm = TPComm("sp" if mode == "a2a" else "nvlink", Tmax, H, 64, 1024, device=dev) if mode != "nccl" else None
        if mode == "a2a":
            comm.setup_ep(layer.K, layer.E_local)
            layer.scratch = MoEScratch(layer.cfg, world * comm.sp_rows_max, dev)
            layer.ep_reduce = None
        elif mode == "allreduce":
            layer.scratch = MoEScratch(layer.cfg, Tmax, dev)
            layer.ep_reduce = lambda part, h, c=comm: c.allreduce_add(part, h)
        else:
            nc = NcclA2A(layer, world, rank, Tmax, H, dev)
        for T in rows:
            g = torch.Generator().manual_seed(T)
            x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
            h = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16).to(dev)
            xn = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
            R = -(-T // world)
            r0, own = rank * R, max(0, min(R, T - rank * R))
            if mode == "allreduce":
                def block():
                    layer.forward(x, h, ws)
                    ops.rmsnorm(h, lnw, 1e-6, out=xn)
            elif mode == "a2a":
                def block():
                    comm.xg[r0:r0 + own].copy_(x[r0:r0 + own])  # the owned rows of the layer input
                    e = layer.forward_a2a(comm, comm.xg[r0:r0 + own], T, ws)
                    comm.rs_norm_ag(h, lnw, 1e-6, T, e)
                    comm.ag_wait(T)
            else:
                def block():
                    nc.run(x[r0:r0 + own], h, lnw, T, ws)
            t_block = timed(block, a.iters)
            if comm is not None:
                comm.check()
            t = torch.tensor([t_block], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out.append({"mode": mode, "ep": world, "rows": T, "hidden": H, "experts": cfg.num_experts,
                        "top_k": cfg.num_experts_per_tok, "block_us": round(float(t[0]), 2)})
        torch.cuda.synchronize()
        dist.barrier()
        if comm is not None:
            comm.close()
    if rank == 0:
        for r in out:
            print(json.dumps(r))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
