#!/usr/bin/env python
"""Run the paged prefill (or, with --decode B, decode) attention a few times on one shape (a
small, self-terminating case for ncu), Qwen2.5-7B heads (28 query / 4 KV heads, d 128), INT4
KV pages.

    python bench/prof_attn.py --lens 2048 --iters 3
    python bench/prof_attn.py --decode 64 --lens 1300 --iters 3
"""
import argparse
import math
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from squish_b200 import ops  # noqa: E402
from squish_b200.kv.paged import kv_row_bytes  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--lens", default="2048", help="comma-separated prompt lengths (one chunk each)")
    ap.add_argument("--hq", type=int, default=28)
    ap.add_argument("--hkv", type=int, default=4)
    ap.add_argument("--kv", default="int4")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--trace", action="store_true", help="print the pipeline timeline of the heaviest CTA")
    ap.add_argument("--decode", type=int, default=0, help="decode batch: B sequences of --lens context, 1 query each")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    lens = [int(x) for x in a.lens.split(",")]
    if a.decode:
        lens = lens[:1] * a.decode
    d, ps, grp = 128, 16, 32
    fk, fv = ops.KV_FORMATS[a.kv]
    cbk, nsk = kv_row_bytes(fk, d, grp)
    cbv, nsv = kv_row_bytes(fv, d, grp)
    B = len(lens)
    pages_per = math.ceil(max(lens) / ps)
    npg = B * pages_per + 1
    kc = torch.randint(0, 255, (npg, a.hkv, ps, cbk), dtype=torch.uint8, device=dev)
    vc = torch.randint(0, 255, (npg, a.hkv, ps, cbv), dtype=torch.uint8, device=dev)
    ks = (torch.rand(npg, a.hkv, ps, max(nsk, 1), device=dev) * 0.1).half()
    vs = (torch.rand(npg, a.hkv, ps, max(nsv, 1), device=dev) * 0.1).half()
    bt = torch.randperm(npg - 1, device=dev)[: B * pages_per].view(B, pages_per).int()
    ql = torch.tensor(lens, dtype=torch.int32)
    qs = torch.cat([torch.zeros(1, dtype=torch.int32), ql.cumsum(0)[:-1].int()])
    tseq, tq0 = [], []
    for i, n in enumerate(lens):
        for s0 in range(0, n, 32):
            tseq.append(i)
            tq0.append(s0)
    if a.decode:
        qd = torch.randn(B, a.hq * d, device=dev, dtype=torch.bfloat16)
        od = torch.empty_like(qd)
        for _ in range(a.iters):
            ops.paged_decode_attention(qd, kc, ks, vc, vs, bt, ql.to(dev), od, a.hq, a.hkv, d, ps, grp, fk, fv,
                                       1 / math.sqrt(d), max(lens))
        torch.cuda.synchronize()
        ops.workspace(dev).check()
        print("ok decode", B, "x", lens[0])
        return
    T = int(ql.sum())
    q = torch.randn(T, a.hq * d, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    args = (torch.tensor(tseq, dtype=torch.int32, device=dev), torch.tensor(tq0, dtype=torch.int32, device=dev),
            qs.to(dev), ql.to(dev), ql.to(dev), len(tseq))
    for _ in range(a.iters):
        ops.paged_prefill_attention(q, kc, ks, vc, vs, bt, *args, out, a.hq, a.hkv, d, ps, grp, fk, fv,
                                    1 / math.sqrt(d))
    torch.cuda.synchronize()
    if a.trace:
        tr = torch.zeros(16 * 32, dtype=torch.int64, device=dev)
        ops.paged_prefill_attention(q, kc, ks, vc, vs, bt, *args, out, a.hq, a.hkv, d, ps, grp, fk, fv,
                                    1 / math.sqrt(d), trace=tr)
        torch.cuda.synchronize()
        t = tr.view(16, 32).cpu()
        base = int(t[9, 0])
        names = ["load", "staged", "K_st", "V_st", "S_iss", "S_rdy", "P_rdy", "PV_iss", "O_resc"]
        print("setup at 0, epilogue done at", int(t[10, 0]) - base, "cycles")
        for j in range(32):
            if t[0, j] == 0 and t[4, j] == 0:
                break
            print(j, " ".join(f"{n}={int(t[e, j]) - base if t[e, j] else '-'}" for e, n in enumerate(names)))
    ops.workspace(dev).check()
    print("ok", T, "tokens", len(tseq), "tiles")


if __name__ == "__main__":
    main()
