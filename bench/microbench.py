#!/usr/bin/env python
"""Per-kernel timings of the decoder's hot ops at a model's shapes, with roofline fractions.

    python bench/microbench.py [--model qwen2.5-7b] [--json out.json]

Small, self-terminating cases of one kernel each (the commands the ncu summaries in
profiles/ run):

    python bench/microbench.py case gemm --m 64 --n 37888 --k 3584 --iters 2
    python bench/microbench.py case attn --decode 64 --lens 1300 --iters 3
    python bench/microbench.py case attn --lens 2048 --iters 3
    python bench/microbench.py case hadamard --m 64 --k 18944 --iters 3 [--time]
    python bench/microbench.py case step --mode decode|prefill [--batch 64 --ctx 1000]

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
    ap.add_argument("--ops", default="qkv,o_proj,gate_up,down,lm_head", help="GEMM shapes to time ('none': skip)")
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
        if name not in args.ops.split(",") or args.ops == "none":
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


# ----------------------------------------------------------------------------- single-kernel cases
def case_gemm(a):
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


def case_attn(a):
    from squish_b200.kv.paged import kv_row_bytes

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
    qs = torch.cat([torch.zeros(1, dtype=torch.int32), ql.cumsum(0)[:-1].int()])
    tseq, tq0 = [], []
    for i, n in enumerate(lens):
        for s0 in range(0, n, 32):
            tseq.append(i)
            tq0.append(s0)
    T = int(ql.sum())
    q = torch.randn(T, a.hq * d, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    args = (torch.tensor(tseq, dtype=torch.int32, device=dev), torch.tensor(tq0, dtype=torch.int32, device=dev),
            qs.to(dev), ql.to(dev), ql.to(dev), len(tseq))
    for _ in range(a.iters):
        ops.paged_prefill_attention(q, kc, ks, vc, vs, bt, *args, out, a.hq, a.hkv, d, ps, grp, fk, fv,
                                    1 / math.sqrt(d))
    torch.cuda.synchronize()
    ops.workspace(dev).check()
    print("ok", T, "tokens", len(tseq), "tiles")


def case_hadamard(a):
    from squish_b200.quant.sqint2 import rotation_block, rotation_signs

    dev = torch.device("cuda", 0)
    b = rotation_block(a.k)
    s = rotation_signs(a.k, 0).to(dev)
    n = max(1, int(256e6 // (4 * a.m * a.k)))  # several pairs: timed launches do not re-read L2
    xs = [torch.randn(a.m, a.k, device=dev, dtype=torch.bfloat16) for _ in range(n)]
    ys = [torch.empty_like(x) for x in xs]
    for i in range(a.iters):
        native().hadamard_rows(xs[i % n], s, b, ys[i % n])
    torch.cuda.synchronize()
    if a.time:
        it = [0]

        def fn():
            native().hadamard_rows(xs[it[0] % n], s, b, ys[it[0] % n])
            it[0] += 1

        us = time_op(fn, 20, inner=max(8, n)) * 1e3
        print(f"m={a.m} k={a.k} block={b}: {us:.2f} us/launch, {4 * a.m * a.k / us / 1e3:.0f} GB/s")
    print("ok", b)


def case_step(a):
    import numpy as np

    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.engine.sampling import SamplingParams

    eng = LLMEngine.from_preset(a.model, device="cuda", seed=0, ecfg=EngineConfig(
        max_num_seqs=a.batch + 1, max_num_batched_tokens=2048, max_model_len=a.ctx + 512,
        cuda_graphs=not a.no_graphs))
    rng = np.random.default_rng(0)
    for _ in range(a.batch):
        eng.add_request(rng.integers(0, eng.cfg.vocab_size, a.ctx).tolist(),
                        SamplingParams(max_tokens=400, ignore_eos=True))
    while any(r.in_prefill for r in eng.scheduler.running) or eng.scheduler.waiting:
        eng.step()
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    if a.mode == "prefill":
        eng.add_request(rng.integers(0, eng.cfg.vocab_size, a.ctx).tolist(), SamplingParams(max_tokens=4))
    # ncu --profile-from-start off sees only the steps inside this window
    torch.cuda.profiler.start()
    for _ in range(a.steps):
        eng.step()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print("ok", eng.stats.graph_steps, eng.stats.mixed_steps)


def case_main(argv):
    ap = argparse.ArgumentParser(prog="microbench.py case")
    sub = ap.add_subparsers(dest="kind", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--m", type=int, default=64)
    g.add_argument("--n", type=int, default=37888)
    g.add_argument("--k", type=int, default=3584)
    g.add_argument("--group", type=int, default=64)
    g.add_argument("--iters", type=int, default=5)
    g.add_argument("--silu", action="store_true")
    t = sub.add_parser("attn")
    t.add_argument("--lens", default="2048", help="comma-separated prompt lengths (one chunk each)")
    t.add_argument("--hq", type=int, default=28)
    t.add_argument("--hkv", type=int, default=4)
    t.add_argument("--kv", default="int4")
    t.add_argument("--iters", type=int, default=3)
    t.add_argument("--decode", type=int, default=0, help="decode batch: B sequences of --lens context")
    h = sub.add_parser("hadamard")
    h.add_argument("--m", type=int, default=64)
    h.add_argument("--k", type=int, default=18944)
    h.add_argument("--iters", type=int, default=3)
    h.add_argument("--time", action="store_true")
    st = sub.add_parser("step")
    st.add_argument("--model", default="qwen2.5-7b")
    st.add_argument("--batch", type=int, default=64)
    st.add_argument("--ctx", type=int, default=1000)
    st.add_argument("--mode", default="decode", choices=["decode", "prefill"])
    st.add_argument("--steps", type=int, default=2)
    st.add_argument("--no-graphs", action="store_true")
    a = ap.parse_args(argv)
    {"gemm": case_gemm, "attn": case_attn, "hadamard": case_hadamard, "step": case_step}[a.kind](a)


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "case":
        case_main(sys.argv[2:])
    else:
        main()
