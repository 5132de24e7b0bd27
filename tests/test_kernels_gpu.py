"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch

from squish_b200 import ops
from squish_b200._ext import native
from squish_b200.models.config import get_preset

from ._refs import apply_rope, attention, dequant_int4_as_kernel, rope_cos_sin, sm_scale

pytestmark = pytest.mark.gpu

C = native()


def _rand_int4(n, k, group, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    packed, scales, offsets = C.cpu.quantize_int4_asym(w, group)
    return packed, scales, offsets


@pytest.mark.parametrize(
    "m,n,k,group",
    [
        (1, 256, 256, 32),
        (5, 384, 512, 64),
        (16, 1024, 1024, 64),
        (33, 512, 688, 16),
        (64, 3584, 3584, 64),
        (16, 1024, 7168, 64),  # 16-way split-K cluster (non-portable size)
        (48, 640, 8960, 128),
        (100, 640, 1024, 128),
        (300, 1024, 896, 64),
        (1024, 2048, 512, 32),
        (700, 4096, 1024, 64),
    ],
)
def test_w4a16_gemm_matches_fp32(cuda, m, n, k, group):
    packed, scales, offsets = _rand_int4(n, k, group, seed=m + n)
    w = ops.prepare_int4_weight(packed, scales, offsets, k, group, cuda)
    x = (torch.randn(m, k) * 0.5).to(torch.bfloat16)
    y = ops.w4a16_linear(x.to(cuda), w)
    torch.cuda.synchronize()
    ref = x.float() @ dequant_int4_as_kernel(packed, scales, offsets, group).T
    torch.testing.assert_close(y.float().cpu(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())
    ops.workspace(cuda).check()


@pytest.mark.parametrize("n,k,group", [(384, 512, 64), (1000, 688, 16), (256, 1024, 32), (640, 896, 128)])
def test_dequant_weight_matches_kernel_values(cuda, n, k, group):
    packed, scales, offsets = _rand_int4(n, k, group, seed=n + k)
    w = ops.prepare_int4_weight(packed, scales, offsets, k, group, cuda)
    wd = ops.dequant_weight(w)
    torch.cuda.synchronize()
    assert wd.shape == (n, (k + 63) // 64 * 64)
    ref = dequant_int4_as_kernel(packed, scales, offsets, group)
    torch.testing.assert_close(wd[:, :k].float().cpu(), ref, rtol=0, atol=1e-6 + 2e-3 * ref.abs().max().item())


@pytest.mark.parametrize(
    "m,n,k",
    [(1, 256, 64), (130, 300, 200), (257, 512, 4096), (2048, 1024, 512), (700, 37888 // 8, 3584)],
)
def test_bf16_gemm_matches_fp32(cuda, m, n, k):
    g = torch.Generator().manual_seed(m * 7 + n)
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
    res = torch.randn(m, n, generator=g).to(torch.bfloat16)
    y = ops.bf16_linear(x.to(cuda), w.to(cuda), bias=bias.to(cuda), residual=res.to(cuda))
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T + bias.float() + res.float()
    torch.testing.assert_close(y.float().cpu(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())
    ops.workspace(cuda).check()


@pytest.mark.parametrize("m,f,k", [(333, 384, 520), (64, 256, 4096)])  # the second splits K 8 ways
def test_bf16_gemm_silu_and_strided_weight(cuda, m, f, k):
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16)
    wpad = (torch.randn(2 * f, k + 56, generator=g) * 0.05).to(torch.bfloat16)  # row stride > k
    w = wpad[:, :k]
    y = ops.bf16_linear(x.to(cuda), wpad.to(cuda)[:, :k], silu_mul=True)
    y2 = ops.bf16_linear(x.to(cuda), wpad.to(cuda)[:, :k], silu_mul=True)
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "split-K reduction must be deterministic"
    h = (x.float() @ w.float().T).view(m, f // 64, 2, 64)
    ref = torch.nn.functional.silu(h[:, :, 0].reshape(m, f)) * h[:, :, 1].reshape(m, f)
    torch.testing.assert_close(y.float().cpu(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())


def test_w4a16_large_m_paths_agree(cuda, monkeypatch):
    """The expanded-weight path (m >= DQ_GEMM_MIN_M) and the fused path give the same result."""
    n, k, group, m = 1024, 2048, 64, 512
    packed, scales, offsets = _rand_int4(n, k, group, seed=11)
    w = ops.prepare_int4_weight(packed, scales, offsets, k, group, cuda)
    x = (torch.randn(m, k) * 0.5).to(torch.bfloat16).to(cuda)
    y_dq = ops.w4a16_linear(x, w)
    monkeypatch.setattr(ops.kernels, "DQ_GEMM_MIN_M", 1 << 30)
    y_fused = ops.w4a16_linear(x, w)
    torch.cuda.synchronize()
    torch.testing.assert_close(y_dq.float(), y_fused.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("m", [3, 64, 257])
def test_w4a16_bias_residual_and_determinism(cuda, m):
    n, k, group = 768, 1024, 64
    packed, scales, offsets = _rand_int4(n, k, group, seed=7)
    bias = torch.randn(n) * 0.1
    w = ops.prepare_int4_weight(packed, scales, offsets, k, group, cuda, bias=bias)
    x = (torch.randn(m, k) * 0.5).to(torch.bfloat16).to(cuda)
    res = (torch.randn(m, n)).to(torch.bfloat16).to(cuda)
    y1 = ops.w4a16_linear(x, w, residual=res)
    y2 = ops.w4a16_linear(x, w, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2), "split-K reduction must be deterministic"
    ref = x.float().cpu() @ dequant_int4_as_kernel(packed, scales, offsets, group).T
    ref = ref + bias.to(torch.bfloat16).float() + res.float().cpu()
    torch.testing.assert_close(y1.float().cpu(), ref, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("m", [2, 48, 200, 300])
def test_w4a16_silu_mul_epilogue(cuda, m):
    f, k, group = 640, 512, 64
    gate = torch.randn(f, k) * 0.05
    up = torch.randn(f, k) * 0.05
    # interleave 64-row blocks: [gate 0:64, up 0:64, gate 64:128, up 64:128, ...]
    blocks = []
    for j in range(0, f, 64):
        blocks += [gate[j:j + 64], up[j:j + 64]]
    wf = torch.cat(blocks, 0)
    packed, scales, offsets = C.cpu.quantize_int4_asym(wf, group)
    w = ops.prepare_int4_weight(packed, scales, offsets, k, group, cuda)
    x = (torch.randn(m, k)).to(torch.bfloat16)
    y = ops.w4a16_linear(x.to(cuda), w, silu_mul=True)
    torch.cuda.synchronize()
    wd = dequant_int4_as_kernel(packed, scales, offsets, group)
    h = x.float() @ wd.T  # [m, 2f] interleaved
    h = h.view(m, f // 64, 2, 64)
    g_, u_ = h[:, :, 0].reshape(m, f), h[:, :, 1].reshape(m, f)
    ref = torch.nn.functional.silu(g_) * u_
    torch.testing.assert_close(y.float().cpu(), ref, rtol=3e-2, atol=3e-2 * ref.abs().max().item())


def test_rmsnorm(cuda):
    x = torch.randn(37, 3584).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(3584)).to(torch.bfloat16)
    y = ops.rmsnorm(x.to(cuda), w.to(cuda), 1e-6)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    torch.testing.assert_close(y.float().cpu(), ref, rtol=1e-2, atol=1e-2)
    idx = torch.tensor([3, 0, 36], dtype=torch.int32)
    y2 = ops.rmsnorm(x.to(cuda), w.to(cuda), 1e-6, row_idx=idx.to(cuda))
    torch.testing.assert_close(y2.float().cpu(), ref[idx.long()], rtol=1e-2, atol=1e-2)


def _make_pools(num_pages, hkv, ps, d, fmt_k, fmt_v, group, device):
    def pool(fmt):
        cb = d * ops.kernels.KV_BITS[fmt] // 8
        ns = 0 if fmt == 0 else (d // group) * (2 if fmt in ops.kernels.KV_ASYM else 1)
        return (torch.zeros(num_pages, hkv, ps, cb, dtype=torch.uint8, device=device),
                torch.zeros(num_pages, hkv, ps, max(ns, 1), dtype=torch.float16, device=device))
    kc, ks = pool(fmt_k)
    vc, vs = pool(fmt_v)
    return kc, ks, vc, vs


def _dequant_pool(codes, scales, fmt, group, d):
    """Dequantize every row of a pool with the C++ CPU codec (oracle)."""
    shp = codes.shape
    c = codes.reshape(-1, shp[-1]).cpu()
    if fmt == 0:
        return c.view(torch.bfloat16).float().reshape(*shp[:-1], d)
    s = scales.reshape(-1, scales.shape[-1]).cpu().float()
    return C.cpu.kv_dequantize(c, s, fmt, group, d).reshape(*shp[:-1], d)


@pytest.mark.parametrize("kvfmt,group", [("int4", 32), ("int4", 128), ("k8v4", 64), ("int8", 64), ("int2", 32),
                                         ("bf16", 32)])
def test_rope_kv_write_matches_codec(cuda, kvfmt, group):
    hq, hkv, d, ps = 8, 2, 128, 16
    fk, fv = ops.KV_FORMATS[kvfmt]
    t = 21
    qkv = (torch.randn(t, (hq + 2 * hkv) * d)).to(torch.bfloat16)
    pos = torch.randint(0, 500, (t,), dtype=torch.int32)
    cs = rope_cos_sin(512, d, 10000.0)
    slots = torch.randperm(4 * ps)[:t].to(torch.int32)
    kc, ks, vc, vs = _make_pools(4, hkv, ps, d, fk, fv, group, cuda)
    q_out = torch.empty(t, hq, d, dtype=torch.bfloat16, device=cuda)
    ops.rope_kv_write(qkv.to(cuda), pos.to(cuda), cs.to(cuda), q_out, slots.to(cuda), kc, ks, vc, vs,
                      hq, hkv, d, ps, group, fk, fv)
    torch.cuda.synchronize()
    x = qkv.float().view(t, hq + 2 * hkv, d)
    q_ref = apply_rope(x[:, :hq], pos, cs)
    k_ref = apply_rope(x[:, hq:hq + hkv], pos, cs)
    v_ref = x[:, hq + hkv:]
    torch.testing.assert_close(q_out.float().cpu(), q_ref, rtol=1e-2, atol=1e-2)
    kd = _dequant_pool(kc, ks, fk, group, d)
    vd = _dequant_pool(vc, vs, fv, group, d)
    page, off = slots.long() // ps, slots.long() % ps
    k_got = kd[page, :, off]  # [t, hkv, d]
    v_got = vd[page, :, off]
    # the quantization error bound: half a step per group (plus bf16 input rounding)
    steps = {"int4": 1 / 7.5, "k8v4": 1 / 15, "int8": 1 / 127, "int2": 1 / 1.5, "bf16": 0.0}[kvfmt]
    for got, ref in ((k_got, k_ref), (v_got, v_ref)):
        amax = ref.abs().amax(-1, keepdim=True)
        bound = amax * steps * 0.5 + 2e-2 * amax + 1e-3
        if kvfmt == "k8v4":
            bound = (ref.amax(-1, keepdim=True) - ref.amin(-1, keepdim=True)) / 15 * 0.51 + 1e-2
        assert ((got - ref).abs() <= bound).all(), f"{kvfmt}: max err {(got - ref).abs().max()}"


def _fill_random_cache(num_pages, hkv, ps, d, fk, fv, group, device, seed=0):
    """Write random K/V rows into every pool slot through the CPU codec; return pools + dense K/V."""
    g = torch.Generator().manual_seed(seed)
    kc, ks, vc, vs = _make_pools(num_pages, hkv, ps, d, fk, fv, group, device)
    rows = num_pages * hkv * ps
    dense = []
    for fmt, codes, scales in ((fk, kc, ks), (fv, vc, vs)):
        x = torch.randn(rows, d, generator=g)
        if fmt == 0:
            xb = x.to(torch.bfloat16)
            codes.copy_(xb.view(torch.uint8).reshape(codes.shape).to(device))
            dense.append(xb.float().reshape(num_pages, hkv, ps, d))
        else:
            c, s = C.cpu.kv_quantize(x, fmt, group)
            codes.copy_(c.reshape(codes.shape).to(device))
            scales.copy_(s.to(torch.float16).reshape(scales.shape).to(device))
            dense.append(C.cpu.kv_dequantize(c, s, fmt, group, d).reshape(num_pages, hkv, ps, d))
    return kc, ks, vc, vs, dense[0], dense[1]


def _gather(dense, bt_row, n_tok, ps):
    pages = bt_row[: (n_tok + ps - 1) // ps].long()
    x = dense[pages]  # [np, hkv, ps, d]
    x = x.permute(0, 2, 1, 3).reshape(-1, x.shape[1], x.shape[3])
    return x[:n_tok]


@pytest.mark.parametrize("kvfmt,hq,hkv,d", [("int4", 28, 4, 128), ("k8v4", 64, 8, 128), ("bf16", 8, 2, 64),
                                            ("int8", 14, 2, 64), ("int2", 32, 4, 128)])
@pytest.mark.parametrize("lens", [[1, 17, 300], [2048, 5, 64, 1000], [33]])
def test_paged_decode_attention(cuda, kvfmt, hq, hkv, d, lens):
    torch.manual_seed(sum(lens) + hq)
    ps, group = 16, 32 if kvfmt != "k8v4" else 64
    fk, fv = ops.KV_FORMATS[kvfmt]
    max_pages = max((l + ps - 1) // ps for l in lens)
    num_pages = sum((l + ps - 1) // ps for l in lens) + 3
    kc, ks, vc, vs, kd, vd = _fill_random_cache(num_pages, hkv, ps, d, fk, fv, group, cuda)
    perm = torch.randperm(num_pages)
    bt = torch.zeros(len(lens), max_pages, dtype=torch.int32)
    o = 0
    for i, l in enumerate(lens):
        n = (l + ps - 1) // ps
        bt[i, :n] = perm[o:o + n].to(torch.int32)
        o += n
    q = torch.randn(len(lens), hq * d).to(torch.bfloat16)
    out = torch.empty(len(lens), hq * d, dtype=torch.bfloat16, device=cuda)
    seq = torch.tensor(lens, dtype=torch.int32)
    ops.paged_decode_attention(q.to(cuda), kc, ks, vc, vs, bt.to(cuda), seq.to(cuda), out, hq, hkv, d, ps, group,
                               fk, fv, sm_scale(d), max_ctx=max(lens))
    torch.cuda.synchronize()
    for i, l in enumerate(lens):
        k = _gather(kd, bt[i], l, ps).to(torch.bfloat16).float()
        v = _gather(vd, bt[i], l, ps).to(torch.bfloat16).float()
        ref = attention(q[i].float().view(1, hq, d), k, v, torch.tensor([l - 1]), sm_scale(d))
        # P is rounded to bf16 before the PV product; over 2k keys that is ~1e-2 absolute
        torch.testing.assert_close(out[i].float().cpu().view(1, hq, d), ref, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("kvfmt,hq,hkv,d,group", [("int4", 28, 4, 128, 128), ("int4", 28, 4, 128, 64),
                                                  ("int4", 14, 2, 64, 32), ("int4", 8, 8, 128, 32),
                                                  ("k8v4", 64, 8, 128, 32), ("k8v4", 32, 8, 128, 128),
                                                  ("k8v4", 16, 4, 64, 64), ("int4", 36, 4, 128, 32)])
@pytest.mark.parametrize("legacy", [False, True])
def test_paged_decode_attention_token_major(cuda, monkeypatch, kvfmt, hq, hkv, d, group, legacy):
    """The token-major decode kernel (keys multiplied as codes, scales applied after the MMA)
    and the head-major one it replaces, on every group size / head count the first covers
    (36 / 4 = 9 query heads per KV head falls back to the head-major kernel)."""
    if legacy:
        monkeypatch.setenv("SQ_DECODE_LEGACY", "1")
    lens = [1, 15, 16, 17, 300, 2048, 777]
    torch.manual_seed(hq * 7 + group)
    ps = 16
    fk, fv = ops.KV_FORMATS[kvfmt]
    max_pages = max((l + ps - 1) // ps for l in lens)
    num_pages = sum((l + ps - 1) // ps for l in lens) + 3
    kc, ks, vc, vs, kd, vd = _fill_random_cache(num_pages, hkv, ps, d, fk, fv, group, cuda, seed=group + d)
    perm = torch.randperm(num_pages)
    bt = torch.zeros(len(lens), max_pages, dtype=torch.int32)
    o = 0
    for i, l in enumerate(lens):
        n = (l + ps - 1) // ps
        bt[i, :n] = perm[o:o + n].to(torch.int32)
        o += n
    q = torch.randn(len(lens), hq * d).to(torch.bfloat16)
    out = torch.full((len(lens), hq * d), float("nan"), dtype=torch.bfloat16, device=cuda)
    seq = torch.tensor(lens, dtype=torch.int32)
    for splits in (None, (1, max_pages)):
        ops.paged_decode_attention(q.to(cuda), kc, ks, vc, vs, bt.to(cuda), seq.to(cuda), out, hq, hkv, d, ps,
                                   group, fk, fv, sm_scale(d), max_ctx=max(lens), splits=splits)
        torch.cuda.synchronize()
        for i, l in enumerate(lens):
            k = _gather(kd, bt[i], l, ps).to(torch.bfloat16).float()
            v = _gather(vd, bt[i], l, ps).to(torch.bfloat16).float()
            ref = attention(q[i].float().view(1, hq, d), k, v, torch.tensor([l - 1]), sm_scale(d))
            torch.testing.assert_close(out[i].float().cpu().view(1, hq, d), ref, rtol=2e-2, atol=3e-2)


SHORT_SEQS = [(40, 40), (70, 200), (1, 1), (130, 130), (16, 48)]
LONG_SEQS = [(300, 1100), (600, 600), (5, 900), (257, 257)]  # several 128-key tiles, partial last tiles


# head dim 128 with 3..16 query heads per KV head runs the tcgen05 kernel (4, 8 or 16 head slots)
@pytest.mark.parametrize("kvfmt,hq,hkv,d,seqs", [
    ("int4", 28, 4, 128, SHORT_SEQS), ("int4", 28, 4, 128, LONG_SEQS), ("k8v4", 16, 2, 128, SHORT_SEQS),
    ("int4", 32, 8, 128, LONG_SEQS), ("int8", 64, 4, 128, LONG_SEQS), ("int2", 12, 4, 128, SHORT_SEQS),
    ("bf16", 8, 2, 64, SHORT_SEQS)])
def test_paged_prefill_attention(cuda, kvfmt, hq, hkv, d, seqs):
    torch.manual_seed(hq + d + len(seqs))
    ps, group = 16, 32 if kvfmt != "k8v4" else 64
    fk, fv = ops.KV_FORMATS[kvfmt]
    # (chunk length, total context after the chunk): fresh prompts and chunked continuations
    max_pages = max((c + ps - 1) // ps for _, c in seqs)
    num_pages = sum((c + ps - 1) // ps for _, c in seqs) + 2
    kc, ks, vc, vs, kd, vd = _fill_random_cache(num_pages, hkv, ps, d, fk, fv, group, cuda, seed=3)
    perm = torch.randperm(num_pages)
    bt = torch.zeros(len(seqs), max_pages, dtype=torch.int32)
    o = 0
    for i, (_, c) in enumerate(seqs):
        n = (c + ps - 1) // ps
        bt[i, :n] = perm[o:o + n].to(torch.int32)
        o += n
    q_len = torch.tensor([s[0] for s in seqs], dtype=torch.int32)
    ctx = torch.tensor([s[1] for s in seqs], dtype=torch.int32)
    q_start = torch.cumsum(torch.cat([torch.zeros(1, dtype=torch.int32), q_len[:-1]]), 0).to(torch.int32)
    tile_seq, tile_q0 = [], []
    for i, (ql, _) in enumerate(seqs):
        for q0 in range(0, ql, 32):
            tile_seq.append(i)
            tile_q0.append(q0)
    t = int(q_len.sum())
    q = torch.randn(t, hq * d).to(torch.bfloat16)
    out = torch.zeros(t, hq * d, dtype=torch.bfloat16, device=cuda)
    ops.paged_prefill_attention(q.to(cuda), kc, ks, vc, vs, bt.to(cuda), torch.tensor(tile_seq, dtype=torch.int32,
                                device=cuda), torch.tensor(tile_q0, dtype=torch.int32, device=cuda),
                                q_start.to(cuda), q_len.to(cuda), ctx.to(cuda), len(tile_seq), out, hq, hkv, d, ps,
                                group, fk, fv, sm_scale(d))
    torch.cuda.synchronize()
    for i, (ql, c) in enumerate(seqs):
        k = _gather(kd, bt[i], c, ps).to(torch.bfloat16).float()
        v = _gather(vd, bt[i], c, ps).to(torch.bfloat16).float()
        qs = int(q_start[i])
        qpos = torch.arange(c - ql, c)
        ref = attention(q[qs:qs + ql].float().view(ql, hq, d), k, v, qpos, sm_scale(d))
        # P is rounded to bf16 before the PV product (as in any bf16 flash kernel)
        torch.testing.assert_close(out[qs:qs + ql].float().cpu().view(ql, hq, d), ref, rtol=2e-2, atol=5e-2)
    ops.workspace(cuda).check()


def test_sampler_greedy_and_filters(cuda):
    b, v = 6, 152064
    logits = torch.randn(b, v) * 3
    logits[torch.arange(b), logits.argmax(-1)] += 1.0  # a unique maximum (bf16 ties are common)
    logits = logits.to(torch.bfloat16).to(cuda)
    out = torch.empty(b, dtype=torch.int32, device=cuda)
    ops.sample(logits, out)
    torch.cuda.synchronize()
    assert torch.equal(out.long(), logits.float().argmax(-1))
    # top_k = 1 and tiny top_p both collapse to the argmax
    temp = torch.full((b,), 0.8, device=cuda)
    ops.sample(logits, out, temperature=temp, top_k=torch.ones(b, dtype=torch.int32, device=cuda), seed=3)
    assert torch.equal(out.long(), logits.float().argmax(-1))
    ops.sample(logits, out, temperature=temp, top_p=torch.full((b,), 1e-6, device=cuda), seed=4)
    assert torch.equal(out.long(), logits.float().argmax(-1))
    # grammar mask: only token 5 allowed
    mask = torch.zeros(b, (v + 31) // 32, dtype=torch.int32, device=cuda)
    mask[:, 0] = 1 << 5
    ops.sample(logits, out, temperature=temp, allow_mask=mask, seed=5)
    assert (out == 5).all()


def test_sampler_distribution(cuda):
    # 4-token vocabulary, many rows with different rng steps: empirical frequencies ~ softmax(x / T)
    rows, v = 4000, 64
    base = torch.full((v,), -30.0)
    base[:4] = torch.tensor([1.0, 0.5, 0.0, -1.0])
    logits = base.repeat(rows, 1).to(torch.bfloat16).to(cuda)
    out = torch.empty(rows, dtype=torch.int32, device=cuda)
    temp = torch.full((rows,), 0.7, device=cuda)
    step = torch.arange(rows, dtype=torch.int32, device=cuda)
    ops.sample(logits, out, temperature=temp, seed=11, step=step)
    freq = torch.bincount(out.long().cpu(), minlength=v)[:4].float() / rows
    ref = torch.softmax(base[:4].to(torch.bfloat16).float() / 0.7, 0)
    assert (freq - ref).abs().max() < 0.03, (freq, ref)
    # top_k = 2 renormalises over the two best
    ops.sample(logits, out, temperature=temp, top_k=torch.full((rows,), 2, dtype=torch.int32, device=cuda), seed=12,
               step=step)
    freq = torch.bincount(out.long().cpu(), minlength=v)[:4].float() / rows
    ref2 = torch.softmax(base[:2].to(torch.bfloat16).float() / 0.7, 0)
    assert freq[2:].sum() == 0 and (freq[:2] - ref2).abs().max() < 0.03
    # top_p: the smallest head of the sorted distribution whose mass reaches top_p, renormalised
    full = torch.softmax(base[:4].to(torch.bfloat16).float() / 0.7, 0)
    for tp, keep in ((0.8, 2), (0.9, 3), (0.5, 1)):
        assert full[:keep].sum() >= tp and (keep == 1 or full[: keep - 1].sum() < tp)
        ops.sample(logits, out, temperature=temp, top_p=torch.full((rows,), tp, device=cuda), seed=13, step=step)
        freq = torch.bincount(out.long().cpu(), minlength=v)[:4].float() / rows
        ref3 = full[:keep] / full[:keep].sum()
        assert freq[keep:].sum() == 0 and (freq[:keep] - ref3).abs().max() < 0.03, (tp, freq, ref3)


@pytest.mark.parametrize("legacy", [False, True])
def test_out_of_pool_indices_are_skipped_and_reported(cuda, monkeypatch, legacy):
    """A block-table entry or cache slot outside the KV pools is never dereferenced: the kernel
    reads an empty (or the first) page instead, records SQ_ERR_BOUNDS (6) in the workspace
    status, and the workspace check raises; sequences with valid tables are unaffected."""
    if legacy:
        monkeypatch.setenv("SQ_DECODE_LEGACY", "1")
        monkeypatch.setenv("SQ_PREFILL_ATTN_LEGACY", "1")
    ps, group, hq, hkv, d = 16, 32, 28, 4, 128
    fk, fv = ops.KV_FORMATS["int4"]
    lens = [40, 300]
    num_pages = sum((l + ps - 1) // ps for l in lens) + 1
    kc, ks, vc, vs, kd, vd = _fill_random_cache(num_pages, hkv, ps, d, fk, fv, group, cuda, seed=9)
    bt = torch.zeros(2, 19, dtype=torch.int32)
    bt[0, :3] = torch.tensor([0, 1, 2])
    bt[1, :19] = torch.arange(3, 22)
    bt[1, 5] = num_pages + 7  # outside the pool
    ws = ops.workspace(cuda)
    ws.status.zero_()
    q = torch.randn(2, hq * d).to(torch.bfloat16)
    out = torch.full((2, hq * d), float("nan"), dtype=torch.bfloat16, device=cuda)
    ops.paged_decode_attention(q.to(cuda), kc, ks, vc, vs, bt.to(cuda), torch.tensor(lens, dtype=torch.int32,
                               device=cuda), out, hq, hkv, d, ps, group, fk, fv, sm_scale(d), max(lens))
    torch.cuda.synchronize()
    assert int(ws.status.item()) == 6
    assert bool(torch.isfinite(out.float()).all())
    k = _gather(kd, bt[0], lens[0], ps).to(torch.bfloat16).float()
    v = _gather(vd, bt[0], lens[0], ps).to(torch.bfloat16).float()
    ref = attention(q[0].float().view(1, hq, d), k, v, torch.tensor([lens[0] - 1]), sm_scale(d))
    torch.testing.assert_close(out[0].float().cpu().view(1, hq, d), ref, rtol=2e-2, atol=3e-2)
    with pytest.raises(RuntimeError, match="status 6"):
        ws.check()
    # prefill chunk of the second sequence over the same bad table
    ql = 32
    qp = torch.randn(ql, hq * d).to(torch.bfloat16).to(cuda)
    outp = torch.zeros(ql, hq * d, dtype=torch.bfloat16, device=cuda)
    i32 = dict(dtype=torch.int32, device=cuda)
    ops.paged_prefill_attention(qp, kc, ks, vc, vs, bt[1:].to(cuda), torch.zeros(1, **i32), torch.zeros(1, **i32),
                                torch.zeros(1, **i32), torch.tensor([ql], **i32), torch.tensor([lens[1]], **i32), 1,
                                outp, hq, hkv, d, ps, group, fk, fv, sm_scale(d))
    torch.cuda.synchronize()
    assert int(ws.status.item()) == 6 and bool(torch.isfinite(outp.float()).all())
    ws.status.zero_()
    # KV write to a slot past the pool: nothing written, status recorded
    before = [t.clone() for t in (kc, ks, vc, vs)]
    qkv = torch.randn(2, (hq + 2 * hkv) * d, dtype=torch.bfloat16, device=cuda)
    from squish_b200.models.reference import rope_table

    cfg, _ = get_preset("qwen2.5-7b")
    cs = rope_table(cfg, 64).to(cuda)
    slots = torch.tensor([num_pages * ps + 3, -1], **i32)
    ops.rope_kv_write(qkv, torch.tensor([5, 6], **i32), cs, torch.empty(2, hq, d, dtype=torch.bfloat16, device=cuda),
                      slots, kc, ks, vc, vs, hq, hkv, d, ps, group, fk, fv)
    torch.cuda.synchronize()
    assert int(ws.status.item()) == 6
    assert all(torch.equal(a, b) for a, b in zip(before, (kc, ks, vc, vs)))
    ws.status.zero_()


@pytest.mark.parametrize("kv,d,hq,hkv", [("int4", 128, 28, 4), ("k8v4", 64, 8, 2), ("bf16", 32, 8, 2)])
def test_page_attention_mass(cuda, kv, d, hq, hkv):
    """Attention mass per KV page (H2O scores): for each decode row, the softmax probabilities
    of all query heads over the row's keys, summed per page, accumulated into mass[page];
    against fp32 on the CPU from the same pages decoded by the CPU codec."""
    from squish_b200.kv.paged import kv_row_bytes

    ps, group = 16, 32
    fk, _ = ops.KV_FORMATS[kv]
    cb, ns = kv_row_bytes(fk, d, group)
    lens = [37, 300, 16, 129]
    B = len(lens)
    npg = sum(-(-n // ps) for n in lens) + 3
    g = torch.Generator().manual_seed(5)
    if fk == 0:
        kc = torch.randn(npg, hkv, ps, d, generator=g).to(torch.bfloat16).view(torch.uint8).reshape(npg, hkv, ps, cb)
        ks = torch.zeros(npg, hkv, ps, 1, dtype=torch.float16)
    else:
        kc = torch.randint(0, 256, (npg, hkv, ps, cb), generator=g, dtype=torch.uint8)
        ks = (torch.rand(npg, hkv, ps, max(ns, 1), generator=g) * 0.2 + 0.05).half()
    perm = torch.randperm(npg, generator=g)
    maxp = max(-(-n // ps) for n in lens)
    bt = torch.zeros(B, maxp, dtype=torch.int32)
    o = 0
    for b, n in enumerate(lens):
        k = -(-n // ps)
        bt[b, :k] = perm[o:o + k].int()
        o += k
    q = (torch.randn(B, hq * d, generator=g) * 0.5).to(torch.bfloat16)
    mass = torch.zeros(npg, device=cuda)
    ops.kernels.page_mass(q.to(cuda), kc.to(cuda), ks.to(cuda), bt.to(cuda), torch.tensor(lens, dtype=torch.int32,
                          device=cuda), mass, hq, hkv, d, ps, group, fk, 1 / math.sqrt(d))
    torch.cuda.synchronize()
    ops.workspace(cuda).check()
    if fk == 0:
        K = kc.view(torch.bfloat16).float().reshape(npg, hkv, ps, d)
    else:
        # (the kernel, like the attention kernels, computes with the bf16 dequantized keys)
        K = C.cpu.kv_dequantize(kc.reshape(-1, cb).contiguous(), ks.reshape(-1, ks.shape[-1]).float().contiguous(),
                                fk, group, d).reshape(npg, hkv, ps, d).to(torch.bfloat16).float()
    want = torch.zeros(npg, dtype=torch.float64)
    for b, n in enumerate(lens):
        pos = torch.arange(n)
        pages = bt[b, pos // ps].long()
        Kb = K[pages, :, pos % ps].double()                       # [n, hkv, d]
        Kb = Kb.repeat_interleave(hq // hkv, dim=1)               # [n, hq, d]
        s = torch.einsum("hd,nhd->hn", q[b].double().view(hq, d), Kb) / math.sqrt(d)
        want.index_add_(0, pages, torch.softmax(s, -1).sum(0))
    got = mass.double().cpu()
    assert torch.allclose(got, want, rtol=2e-2, atol=2e-3), (got - want).abs().max()
    assert abs(float(got.sum()) - hq * B) < 1e-2 * hq * B  # each head's probabilities sum to 1
