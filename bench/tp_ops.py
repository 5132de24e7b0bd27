#!/usr/bin/env python
"""Per-op timing of one tensor-parallel half layer in each collective mode (torchrun, one
process per GPU):

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 bench/tp_ops.py [--hidden 8192] [--rows 16,64]

A half layer is: row-parallel GEMM (o_proj shard: [M, hidden / tp] x [hidden, hidden / tp]^T)
-> the collective -> RMSNorm -> column-parallel GEMM (qkv shard, hidden -> qkv_out / tp).

  nccl    INT4 GEMM into a scratch, NCCL all_reduce, residual add, RMSNorm, next GEMM
  nvlink  GEMM whose epilogue pushes partial tiles to every rank + flag-synchronised reduce
          (residual fused), RMSNorm, next GEMM
  sp      GEMM with reduce-scatter routing, fused partial sum + residual + RMSNorm + all-gather,
          next GEMM waiting for the gather in its producer

Every rank times the same ops with CUDA events (after warm-up); the JSON line reports the max
over ranks of the mean per-iteration time of the whole block and of the row-parallel GEMM
alone (no collective), so block - gemm_alone is what the collective adds.
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
from squish_b200.parallel.comm import TPComm  # noqa: E402


def weight(n, k, seed, dev):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    p, s, z = native().cpu.quantize_int4_asym(w, 128)
    return ops.prepare_int4_weight(p, s, z, k, 128, dev)


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--qkv", type=int, default=10240, help="full qkv output width")
    ap.add_argument("--rows", default="16,64", help="token rows M")
    ap.add_argument("--modes", default="nccl,nvlink,sp")
    ap.add_argument("--iters", type=int, default=200)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    H = a.hidden
    ms = [int(x) for x in a.rows.split(",")]
    w_o = weight(H, H // world, 1 + rank, dev)
    w_qkv = weight(a.qkv // world, H, 100 + rank, dev)
    lnw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    ws = ops.Workspace(dev)
    out = []
    for mode in a.modes.split(","):
        comm = TPComm(mode, max(ms), H, 64, 1024, device=dev)
        for M in ms:
            x = torch.randn(M, H // world, device=dev).to(torch.bfloat16)
            h = torch.randn(M, H, device=dev).to(torch.bfloat16)
            xn = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
            y = torch.empty(M, a.qkv // world, dtype=torch.bfloat16, device=dev)
            tmp = torch.empty(M, H, dtype=torch.bfloat16, device=dev)

            def gemm_only():
                ops.w4a16_linear(x, w_o, out=tmp, ws=ws)

            if mode == "nccl":
                def block():
                    ops.w4a16_linear(x, w_o, out=tmp, ws=ws)
                    dist.all_reduce(tmp)
                    h.add_(tmp)
                    ops.rmsnorm(h, lnw, 1e-5, out=xn)
                    ops.w4a16_linear(xn, w_qkv, out=y, ws=ws)
            elif mode == "nvlink":
                def block():
                    comm.gemm_allreduce(x, w_o, h, ws)
                    ops.rmsnorm(h, lnw, 1e-5, out=xn)
                    ops.w4a16_linear(xn, w_qkv, out=y, ws=ws)
            else:
                def block():
                    e = comm.gemm_rs(x, w_o, ws)
                    comm.rs_norm_ag(h, lnw, 1e-5, M, e)
                    comm.gemm_ag(w_qkv, y, M, False, ws)

            t_gemm = timed(gemm_only, a.iters)
            t_block = timed(block, a.iters)
            comm.check()
            t = torch.tensor([t_gemm, t_block], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out.append({"mode": mode, "tp": world, "m": M, "hidden": H, "gemm_alone_us": round(float(t[0]), 2),
                        "block_us": round(float(t[1]), 2)})
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
    if rank == 0:
        for r in out:
            print(json.dumps(r))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
