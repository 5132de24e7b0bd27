#!/usr/bin/env python
"""Run one W4A16 GEMM shape a few times (a small, self-terminating case for ncu).

    python bench/prof_gemm.py --m 64 --n 37888 --k 3584 --iters 5
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from squish_b200 import ops  # noqa: E402
from squish_b200._ext import native  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=64)
    ap.add_argument("--n", type=int, default=37888)
    ap.add_argument("--k", type=int, default=3584)
    ap.add_argument("--group", type=int, default=64)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--silu", action="store_true")
    ap.add_argument("--trace", action="store_true", help="print per-k-block role timestamps of CTA 0")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    w = torch.randn(a.n, a.k, device=dev, dtype=torch.bfloat16) * 0.02
    p, s, o = native().quantize_int4_asym(w, a.group, 1)
    wt = ops.prepare_int4_weight(p, s, o, a.k, a.group, dev)
    del w, p, s, o
    x = torch.randn(a.m, a.k, device=dev, dtype=torch.bfloat16)
    for _ in range(a.iters):
        y = ops.w4a16_linear(x, wt, silu_mul=a.silu)
    torch.cuda.synchronize()
    if a.trace:
        tr = torch.zeros(16 * 64, dtype=torch.int64, device=dev)
        ops.w4a16_linear(x, wt, silu_mul=a.silu, trace=tr)
        torch.cuda.synchronize()
        t = tr.view(16, 64).cpu()
        base = int(t[t > 0].min())
        names = ["w_issue", "x_issue", "mma_xfull", "mma_afull", "dq_wfull", "dq_aempty", "dq_afull", "acc_full",
                 "dq_lds", "dq_arrw", "dq_sts", "dq_fence", "mma_iss", "mma_cmt", "setup_done", "exit"]
        for i in range(min(64, (a.k + 63) // 64)):
            print(i, " ".join(f"{n}={(int(t[j, i]) - base) if t[j, i] > 0 else -1}" for j, n in enumerate(names)
                               if (j not in (7, 14, 15) or i == 0) and t[j, i] > 0))
    ops.workspace(dev).check()
    print("plan", ops.gemm_plan(a.m, a.n, a.k), "ok", tuple(y.shape))


if __name__ == "__main__":
    main()
