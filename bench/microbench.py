#!/usr/bin/env python
"""Per-kernel timings of the decoder's hot ops at a model's shapes, with roofline fractions.

    python bench/microbench.py [--model qwen2.5-7b] [--json out.json]

Each op is timed with CUDA events on the launching stream after warm-up, median of
``--iters`` launches (inputs larger than L2 where it matters: weight streams of tens of
MB; the INT4 weights rotate over ``--copies`` copies so every launch reads from HBM).
Fractions use the measured peaks in MEASURED_PEAKS.json (copy bandwidth, cuBLAS bf16)
when present.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from squish_b200 import ops  # noqa: E402
from squish_b200._ext import native  # noqa: E402
from squish_b200.models.config import get_preset  # noqa: E402


def peaks():
    p = os.path.join(os.path.dirname(HERE), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], "of measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "of fallback"


def time_op(fn, iters=20, warmup=5, inner=8):
    """Device time of one call: ``inner`` back-to-back calls are captured in a CUDA graph
    (no host launch cost between them), the graph is replayed ``iters`` times, and the
    median replay time / inner is returned."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        for _ in range(inner):
            fn()
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) / inner)
    ts.sort()
    return ts[len(ts) // 2]


def rand_int4(n, k, group, dev, copies):
    ws = []
    for c in range(copies):
        w = torch.randn(n, k, device=dev, dtype=torch.bfloat16) * 0.02
        p, s, o = native().quantize_int4_asym(w, group, 1)
        ws.append(ops.prepare_int4_weight(p, s, o, k, group, dev))
        del w, p, s, o
    return ws


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--copies", type=int, default=8, help="weight copies cycled (their total exceeds L2)")
    ap.add_argument("--json", default=None)
    ap.add_argument("--ms", default="1,16,64,128,512,2048")
    ap.add_argument("--ops", default="qkv,o_proj,gate_up,down,lm_head", help="GEMM shapes to time")
    ap.add_argument("--no-attn", action="store_true", help="skip the attention timings")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    cfg, q = get_preset(args.model)
    hbm, tflops, tag = peaks()
    h, f = cfg.hidden_size, cfg.intermediate_size
    shapes = {"qkv": (cfg.q_size + 2 * cfg.kv_size, h), "o_proj": (h, cfg.q_size), "gate_up": (2 * f, h),
              "down": (h, f), "lm_head": (cfg.vocab_size, h)}
    rows = []
    ms = [int(x) for x in args.ms.split(",")]
    for name, (n, k) in shapes.items():
        if name not in args.ops.split(","):
            continue
        wb = n * k // 2
        copies = max(2, min(args.copies, -(-384 * 2**20 // wb)))  # > 3x L2 of weights in the rotation
        wts = rand_int4(n, k, q.group_size, dev, copies)
        for m in ms:
            if name == "lm_head" and m > 256:
                continue
            x = torch.randn(m, k, device=dev, dtype=torch.bfloat16)
            y = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
            it = [0]

            def fn():
                ops.w4a16_linear(x, wts[it[0] % copies], out=y)
                it[0] += 1

            t = time_op(fn, args.iters, inner=copies)
            extra = {}
            if m >= ops.kernels.DQ_GEMM_MIN_M and name != "lm_head":
                # the large-M route (expand + bf16 GEMM) against its parts, the fused kernel and cuBLAS
                saved = ops.kernels.DQ_GEMM_MIN_M
                ops.kernels.DQ_GEMM_MIN_M = 1 << 30
                extra["fused_ms"] = time_op(fn, args.iters, inner=copies)
                ops.kernels.DQ_GEMM_MIN_M = saved
                wd = ops.dequant_weight(wts[0])
                extra["expand_ms"] = time_op(lambda: ops.dequant_weight(wts[0], out=wd), args.iters)
                extra["bf16_gemm_ms"] = time_op(lambda: ops.bf16_linear(x, wd[:, :k], out=y), args.iters)
                extra["cublas_ms"] = time_op(lambda: torch.mm(x, wd[:, :k].t(), out=y), args.iters)
                del wd
            wbytes = n * k / 2 + n * (k // q.group_size) * 4
            bytes_ = wbytes + m * k * 2 + m * n * 2
            flops = 2.0 * m * n * k
            t_bw = bytes_ / (hbm * 1e9) * 1e3
            t_fl = flops / (tflops * 1e12) * 1e3
            roof = max(t_bw, t_fl)
            plan = ops.gemm_plan(m, n, k)
            rows.append({"op": f"w4a16 {name}", "m": m, "n": n, "k": k, "ms": t, "GB/s": bytes_ / t / 1e6,
                         "TFLOP/s": flops / t / 1e9, "roofline_ms": roof, "frac": roof / t,
                         "bound": "hbm" if t_bw > t_fl else "tensor", "plan": plan, **extra})
        del wts
        torch.cuda.empty_cache()
    if not args.no_attn:
        rows += other_ops(args, cfg, q, dev, hbm, tflops)
    for r in rows:
        print(json.dumps(r))
    print(json.dumps({"peaks": {"hbm_gbs": hbm, "bf16_tflops": tflops, "basis": tag}}))
    if args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f, indent=1)


def other_ops(args, cfg, q, dev, hbm, tflops):
    """Attention, RMSNorm, RoPE + KV write and sampler timings."""
    rows = []
    h = cfg.hidden_size
    # attention (INT4 g32 pages)
    from squish_b200.kv.paged import kv_row_bytes

    hq, hkv, d, ps, grp = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, 16, q.kv_group
    fk, fv = ops.KV_FORMATS[q.kv_dtype]
    for B, ctx in ((1, 2048), (64, 1300), (64, 2300)):
        pages_per = math.ceil(ctx / ps)
        npg = B * pages_per + 1
        cbk, nsk = kv_row_bytes(fk, d, grp)
        cbv, nsv = kv_row_bytes(fv, d, grp)
        kc = torch.randint(0, 255, (npg, hkv, ps, cbk), dtype=torch.uint8, device=dev)
        vc = torch.randint(0, 255, (npg, hkv, ps, cbv), dtype=torch.uint8, device=dev)
        ks = (torch.rand(npg, hkv, ps, max(nsk, 1), device=dev) * 0.1).half()
        vs = (torch.rand(npg, hkv, ps, max(nsv, 1), device=dev) * 0.1).half()
        bt = torch.randperm(npg - 1, device=dev)[: B * pages_per].view(B, pages_per).int()
        lens = torch.full((B,), ctx, dtype=torch.int32, device=dev)
        qd = torch.randn(B, hq * d, device=dev, dtype=torch.bfloat16)
        out = torch.empty_like(qd)

        def fa():
            ops.paged_decode_attention(qd, kc, ks, vc, vs, bt, lens, out, hq, hkv, d, ps, grp, fk, fv,
                                       1 / math.sqrt(d), ctx)

        t = time_op(fa, args.iters)
        kv_bytes = B * ctx * hkv * (cbk + cbv + 2 * (nsk + nsv))
        rows.append({"op": "decode_attn", "B": B, "ctx": ctx, "ms": t, "GB/s": kv_bytes / t / 1e6,
                     "roofline_ms": kv_bytes / (hbm * 1e9) * 1e3, "frac": kv_bytes / (hbm * 1e9) * 1e3 / t,
                     "splits": ops.kernels.decode_splits(B, hkv, ctx)})
    # prefill attention: one 2048-token prompt and 8 x 256
    for lens_ in ([2048], [256] * 8, [1100, 900]):
        B = len(lens_)
        pages_per = math.ceil(max(lens_) / ps)
        npg = B * pages_per + 1
        kc = torch.randint(0, 255, (npg, hkv, ps, cbk), dtype=torch.uint8, device=dev)
        vc = torch.randint(0, 255, (npg, hkv, ps, cbv), dtype=torch.uint8, device=dev)
        ks = (torch.rand(npg, hkv, ps, max(nsk, 1), device=dev) * 0.1).half()
        vs = (torch.rand(npg, hkv, ps, max(nsv, 1), device=dev) * 0.1).half()
        bt = torch.arange(B * pages_per, device=dev).view(B, pages_per).int()
        ql = torch.tensor(lens_, dtype=torch.int32)
        qs = torch.cat([torch.zeros(1, dtype=torch.int32), ql.cumsum(0)[:-1].int()])
        tseq, tq0 = [], []
        for i, l in enumerate(lens_):
            for s0 in range(0, l, 32):
                tseq.append(i)
                tq0.append(s0)
        T = int(ql.sum())
        qp = torch.randn(T, hq * d, device=dev, dtype=torch.bfloat16)
        out = torch.empty_like(qp)
        tseq_d = torch.tensor(tseq, dtype=torch.int32, device=dev)
        tq0_d = torch.tensor(tq0, dtype=torch.int32, device=dev)
        ql_d, qs_d = ql.to(dev), qs.to(dev)

        def fp():
            ops.paged_prefill_attention(qp, kc, ks, vc, vs, bt, tseq_d, tq0_d, qs_d, ql_d, ql_d, len(tseq), out, hq,
                                        hkv, d, ps, grp, fk, fv, 1 / math.sqrt(d))

        t = time_op(fp, args.iters)
        flops = sum(4.0 * hq * d * l * (l + 1) / 2 for l in lens_)
        rows.append({"op": "prefill_attn", "lens": lens_, "ms": t, "TFLOP/s": flops / t / 1e9,
                     "roofline_ms": flops / (tflops * 1e12) * 1e3, "frac": flops / (tflops * 1e12) * 1e3 / t})
    # norm, rope, sampler
    for T in (64, 2048):
        x = torch.randn(T, h, device=dev, dtype=torch.bfloat16)
        w = torch.ones(h, device=dev, dtype=torch.bfloat16)
        y = torch.empty_like(x)
        t = time_op(lambda: ops.rmsnorm(x, w, 1e-6, out=y), args.iters)
        rows.append({"op": "rmsnorm", "T": T, "ms": t, "GB/s": 2 * x.numel() * 2 / t / 1e6})
        qkv = torch.randn(T, hq * d + 2 * hkv * d, device=dev, dtype=torch.bfloat16)
        pos = torch.arange(T, dtype=torch.int32, device=dev)
        from squish_b200.models.reference import rope_table

        cs = rope_table(cfg, 4096).to(dev)
        qo = torch.empty(T, hq, d, device=dev, dtype=torch.bfloat16)
        npg = T // 16 + 1
        kc = torch.zeros(npg, hkv, ps, cbk, dtype=torch.uint8, device=dev)
        vc = torch.zeros(npg, hkv, ps, cbv, dtype=torch.uint8, device=dev)
        ks = torch.zeros(npg, hkv, ps, max(nsk, 1), dtype=torch.float16, device=dev)
        vs = torch.zeros(npg, hkv, ps, max(nsv, 1), dtype=torch.float16, device=dev)
        t = time_op(lambda: ops.rope_kv_write(qkv, pos, cs, qo, pos, kc, ks, vc, vs, hq, hkv, d, ps, grp, fk, fv),
                    args.iters)
        rows.append({"op": "rope_kv_write", "T": T, "ms": t})
    for B in (1, 64):
        lg = torch.randn(B, cfg.vocab_size, device=dev).bfloat16()
        o = torch.empty(B, dtype=torch.int32, device=dev)
        rows.append({"op": "sampler greedy", "B": B, "ms": time_op(lambda: ops.sample(lg, o), args.iters)})
        tmp = torch.full((B,), 0.7, device=dev)
        tp = torch.full((B,), 0.9, device=dev)
        rows.append({"op": "sampler top-p", "B": B,
                     "ms": time_op(lambda: ops.sample(lg, o, temperature=tmp, top_p=tp, seed=1), args.iters)})
    return rows


if __name__ == "__main__":
    main()
