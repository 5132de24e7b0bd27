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
    ops.workspace(dev).check()
    print("plan", ops.gemm_plan(a.m, a.n, a.k), "ok", tuple(y.shape))


if __name__ == "__main__":
    main()
