#!/usr/bin/env python
"""Time the SQINT2 activation rotation (csrc/hadamard.cu) with CUDA events, and run it a few
times as a small, self-terminating case for ncu.

    python bench/prof_hadamard.py --m 64 --k 18944 --iters 3
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from squish_b200._ext import native  # noqa: E402
from squish_b200.quant.sqint2 import rotation_block, rotation_signs  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=64)
    ap.add_argument("--k", type=int, default=18944)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--time", action="store_true", help="CUDA-event timing over 200 launches in a graph")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    b = rotation_block(a.k)
    s = rotation_signs(a.k, 0).to(dev)
    # several input/output pairs so timed launches do not re-read the same lines from L2
    n = max(1, int(256e6 // (4 * a.m * a.k)))
    xs = [torch.randn(a.m, a.k, device=dev, dtype=torch.bfloat16) for _ in range(n)]
    ys = [torch.empty_like(x) for x in xs]
    for i in range(a.iters):
        native().hadamard_rows(xs[i % n], s, b, ys[i % n])
    torch.cuda.synchronize()
    if a.time:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(200):
                native().hadamard_rows(xs[i % n], s, b, ys[i % n])
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / 200 * 1e3
        byts = 4 * a.m * a.k  # bf16 read + bf16 write
        print(f"m={a.m} k={a.k} block={b}: {us:.2f} us/launch, {byts / us / 1e3:.0f} GB/s")
    print("ok", b)


if __name__ == "__main__":
    main()
