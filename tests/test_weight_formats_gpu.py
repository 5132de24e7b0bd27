"""The INT4 GEMM kernel's other code formats (NF4, any4 learned 4-bit tables, QuaRot rotated
INT4, INT8, INT2) against a plain PyTorch fp32
reference of the same dequantized weight, the tensor-op repack against the CUDA INT4
repack, and an engine whose linear layers are NF4 / INT8 / INT2 against the CPU oracle."""
import dataclasses

import numpy as np
import pytest
import torch

from squish_b200 import ops
from squish_b200.ops import kernels as K
from squish_b200.quant.codecs import quantize

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind,group", [("nf4", 64), ("nf4", 32), ("q8", 64), ("q8", 32), ("q2", 64), ("q2", 128),
                                        ("q3", 64), ("q3", 32), ("aqlm", 8), ("fp8", 64), ("fp8", 32),
                                        ("any4", 64), ("any4", 32)])
@pytest.mark.parametrize("m", [1, 37, 64, 300, 512])
def test_gemm_formats_match_fp32(cuda, kind, group, m):
    g = torch.Generator().manual_seed(m + group)
    n, k = 640, 1024
    w = torch.randn(n, k, generator=g) * 0.05
    t = quantize(w, kind, group)
    dw = K.prepare_weight(t, cuda)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    y = ops.w4a16_linear(x.to(cuda), dw)
    torch.cuda.synchronize()
    ref = x.float() @ t.dequantize().float().T
    err = (y.float().cpu() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err


def test_tensor_op_repack_equals_cuda_int4_repack(cuda):
    g = torch.Generator().manual_seed(5)
    w = torch.randn(384, 704, generator=g) * 0.05
    t = quantize(w, "q4a", 64)
    a = K.prepare_int4_weight(t.packed, t.scales, t.offsets, 704, t.group, cuda).wq
    p = t.packed.to(cuda)
    codes = torch.stack([p & 0xF, p >> 4], dim=-1).reshape(p.shape[0], -1)
    b = K.repack_codes(codes, t.scales.to(cuda), t.offsets.to(cuda), 704, t.group, K.WF_INT4)
    assert torch.equal(a, b)


@pytest.mark.parametrize("m", [1, 64, 512])
def test_quarot_rotated_int4_gemm_matches_fp32(cuda, m):
    """QuaRot INT4 weights (stored as W R^T): the runner rotates the input with the same
    block Hadamard and the GEMM computes (W R^T)(R x) = W x."""
    from squish_b200.quant.research import quarot_quantize

    g = torch.Generator().manual_seed(m)
    w = torch.randn(640, 1024, generator=g) * 0.05
    w[:, 7] *= 30
    t = quarot_quantize(w, 64, bits=4, block=128, seed=3)
    dw = K.prepare_weight(t, cuda)
    assert dw.rot is not None and dw.rot_block == 128
    x = torch.randn(m, 1024, generator=g).to(torch.bfloat16)
    y = ops.w4a16_linear(x.to(cuda), dw)
    torch.cuda.synchronize()
    ref = x.float() @ t.dequantize().float().T
    err = (y.float().cpu() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err


@pytest.mark.parametrize("m", [1, 64, 512])
def test_lowrank_residual_gemms_match_fp32(cuda, m):
    """Quantized GEMM + low-rank residual: a MiLo INT3 weight (plain and as an interleaved
    gate/up pair under the SiLU*up epilogue) and an SQINT2 weight with a rotated-frame residual."""
    from squish_b200.models.decoder import _interleave_gate_up
    from squish_b200.quant.research import milo_int3
    from squish_b200.quant.sqint2 import SQINT2Config, compress_weight

    g = torch.Generator().manual_seed(m)
    x = torch.randn(m, 512, generator=g).to(torch.bfloat16)
    xf = x.float()

    def check(y, ref):
        err = (y.float().cpu() - ref).abs().max().item()
        assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err

    t = milo_int3(torch.randn(384, 512, generator=g) * 0.05, 32, 8)
    dw = K.prepare_weight(t, cuda)
    assert dw.lr_a is not None and dw.lr_a.shape == (384, 8)
    check(ops.w4a16_linear(x.to(cuda), dw), xf @ t.dequantize().T)
    gate = milo_int3(torch.randn(192, 512, generator=g) * 0.05, 32, 4)
    up = milo_int3(torch.randn(192, 512, generator=g) * 0.05, 32, 4)
    gu = K.prepare_weight(_interleave_gate_up(gate, up), cuda)
    want = torch.nn.functional.silu(xf @ gate.dequantize().T) * (xf @ up.dequantize().T)
    check(ops.w4a16_linear(x.to(cuda), gu, silu_mul=True), want)
    s2 = compress_weight(torch.randn(256, 512, generator=g) * 0.05, SQINT2Config(group_size=32, residual_rank=4))
    ds = K.prepare_weight(s2, cuda)
    assert ds.rot is not None and ds.lr_a is not None
    check(ops.w4a16_linear(x.to(cuda), ds), xf @ s2.dequantize().T)


@pytest.mark.parametrize("kind", ["nf4", "q8", "q2", "q3", "aqlm", "fp8", "any4", "milo"])
def test_engine_with_format_weights_matches_oracle(cuda, kind):
    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.engine.sampling import SamplingParams
    from squish_b200.models.config import get_preset
    from squish_b200.models.reference import ReferenceModel
    from squish_b200.models.weights import linear_names, random_checkpoint

    from .test_engine_gpu import _teacher_forced_ok

    cfg, q = get_preset("tiny-llama")
    cfg = dataclasses.replace(cfg, intermediate_size=512)

    def ck():
        c = random_checkpoint(cfg, q, seed=0)
        for name, _ in linear_names(cfg):
            w = c.tensors[name].dequantize().float()
            if kind == "aqlm":
                from squish_b200.quant.aqlm import aqlm_quantize

                c.tensors[name] = aqlm_quantize(w, iters=2)
            elif kind == "milo":  # INT3 + low-rank compensator
                from squish_b200.quant.research import milo_int3

                c.tensors[name] = milo_int3(w, 32, 4)
            else:
                c.tensors[name] = quantize(w, kind, 32)
        return c

    ref = ReferenceModel(ck())
    eng = LLMEngine.from_checkpoint(ck(), cuda, EngineConfig(max_num_seqs=2, max_model_len=256, num_pages=32))
    prompt = np.random.default_rng(2).integers(0, cfg.vocab_size, 30).tolist()
    out = eng.generate([prompt], SamplingParams(max_tokens=8, ignore_eos=True))[0]
    ok, worst = _teacher_forced_ok(ref, prompt, out)
    assert ok, (worst, out)
    o = eng.runner.layers[0].o
    assert o.fmt == {"nf4": K.WF_NF4, "q8": K.WF_INT8, "q2": K.WF_INT2, "q3": K.WF_INT3, "aqlm": K.WF_AQLM,
                     "fp8": K.WF_FP8, "any4": K.WF_NF4, "milo": K.WF_INT3}[kind]
    if kind == "any4":  # served by the NF4 path with the tensor's learned table
        assert o.codebook is not None and o.codebook.numel() == 16
    if kind == "milo":  # the compensator runs after the INT3 GEMM (fused qkv / gate_up too)
        assert o.lr_a is not None and eng.runner.layers[0].qkv.lr_a is not None
        assert eng.runner.layers[0].gate_up.lr_a is not None


@pytest.mark.parametrize("codec,group", [(0, 64), (0, 0), (1, 32), (2, 64), (3, 32), (4, 64)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gpu_quantizers_match_cpu_library(codec, group, dtype):
    """csrc/quantize.cu reproduces the CPU library's codes and scales (same float arithmetic)."""
    from squish_b200._ext import native

    C = native()
    g = torch.Generator().manual_seed(codec * 7 + group)
    x = (torch.randn(96, 512, generator=g) * 0.03).to(dtype)
    xf = x.float()
    got = [t.cpu() for t in C.quantize_codec(x.cuda(), codec, group)]
    if codec == 0:
        want = C.cpu.quantize_int8(xf, group)
    elif codec == 1:
        want = C.cpu.quantize_int4_sym(xf, group)
    elif codec == 2:
        want = C.cpu.quantize_nf4(xf, group)
    elif codec == 3:
        want = C.cpu.pack_int3(xf, group)
    else:
        want = C.cpu.quantize_int2(xf, group)
    assert len(got) == len(want)
    for a, b in zip(got, want):
        assert a.shape == b.shape and a.dtype == b.dtype
        if a.dtype.is_floating_point:
            torch.testing.assert_close(a, b, rtol=1e-6, atol=0)
        else:
            # codes: identical except where a value sits on a rounding boundary (fused multiply-add
            # contraction can differ between the compilers); allow a few
            assert (a != b).float().mean().item() < 1e-3


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("group", [0, 64])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gpu_fp8_codec_matches_cpu_library(fmt, group, dtype):
    """The GPU FP8 encoder (hardware cvt.rn.satfinite) and the C++ software encoder agree bit
    for bit, per group and per tensor."""
    from squish_b200.quant.codecs import quantize_fp8

    g = torch.Generator().manual_seed(group + len(fmt))
    x = (torch.randn(64, 512, generator=g) * torch.logspace(-5, 1, 512)[None, :]).to(dtype)
    cg, sg = quantize_fp8(x.cuda(), fmt, group)
    cc, sc = quantize_fp8(x.float(), fmt, group)
    torch.testing.assert_close(sg.cpu(), sc, rtol=1e-6, atol=0)
    assert torch.equal(cg.cpu(), cc)


@pytest.mark.parametrize("levels,group", [(16, 64), (4, 128), (6, 32), (256, 512)])
def test_hqq_kernel_matches_torch(levels, group):
    """The one-warp-per-group HQQ kernel against the torch restatement (fp32 sums in another
    order: scales agree to 1e-4, codes except on rounding boundaries)."""
    from squish_b200.quant.hqq import hqq_quantize, hqq_torch

    g = torch.Generator().manual_seed(levels + group)
    w = torch.randn(128, 1024, generator=g) * 0.02
    c1, s1, z1 = hqq_quantize(w.cuda(), group, levels, 1.0, 10)
    c2, s2, z2 = hqq_torch(w, group, levels, 1.0, 10)
    torch.testing.assert_close(s1.cpu(), s2, rtol=1e-3, atol=1e-6)
    torch.testing.assert_close(z1.cpu(), z2, rtol=1e-3, atol=1e-5)
    assert (c1.cpu() != c2).float().mean().item() < 2e-3


def test_channel_abs_mean_kernel():
    from squish_b200._ext import native

    g = torch.Generator().manual_seed(1)
    acc = torch.zeros(896, dtype=torch.float64, device="cuda")
    xs = [torch.randn(n, 896, generator=g) * torch.linspace(0.1, 5, 896) for n in (1, 70, 300)]
    for x in xs:
        native().channel_abs_mean(x.cuda(), acc)
        native().channel_abs_mean(x.to(torch.bfloat16).cuda(), acc)
    want = sum(x.abs().mean(0).double() + x.to(torch.bfloat16).float().abs().mean(0).double() for x in xs)
    torch.testing.assert_close(acc.cpu(), want, rtol=1e-5, atol=1e-6)


def test_awq_calibration_on_gpu_matches_cpu():
    """AWQ statistics collected by the GPU forward (channel kernel) equal the CPU forward's."""
    from squish_b200.models.config import get_preset
    from squish_b200.models.weights import random_checkpoint
    from squish_b200.quant.awq import calibration_tokens, collect_activation_scales

    cfg, q = get_preset("tiny-llama")
    ck = random_checkpoint(cfg, q, seed=3)
    toks = calibration_tokens(cfg.vocab_size, 3, 40, seed=1)
    a = collect_activation_scales(ck, toks, device="cuda")
    b = collect_activation_scales(ck, toks, device="cpu")
    assert a.keys() == b.keys() and len(a) == 5 * cfg.num_layers
    for k in a:
        np.testing.assert_allclose(a[k], b[k], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("d", [3, 8, 16, 64])
def test_kmeans_kernels_match_torch(d):
    """csrc/kmeans.cu: assignment equals the torch nearest-centroid search; Lloyd from the same
    seeds reaches the CPU fit's inertia; ADC equals the table sum."""
    from squish_b200.quant import pq

    g = torch.Generator().manual_seed(d)
    x = torch.randn(20000, d, generator=g)
    c = torch.randn(300, d, generator=g)
    a_gpu, dist_gpu = pq.assign(x.cuda(), c.cuda())
    a_cpu, dist_cpu = pq._sqdist_min(x.double(), c.double())
    agree = (a_gpu.cpu() == a_cpu).float().mean().item()
    assert agree > 0.999, agree
    torch.testing.assert_close(dist_gpu.cpu().double(), dist_cpu.double(), rtol=1e-4, atol=1e-4)
    init = pq.kmeans_pp_init(x, 64, seed=3)
    cg, ag = pq.kmeans(x.cuda(), 64, iters=15, init=init)
    cc, ac = pq.kmeans(x, 64, iters=15, init=init)
    inert = lambda xx, cc_, aa: ((xx - cc_[aa]) ** 2).sum().item()  # noqa: E731
    ig, ic = inert(x, cg.cpu(), ag.cpu()), inert(x, cc, ac)
    assert abs(ig - ic) <= 2e-3 * ic, (ig, ic)
    codes = torch.randint(0, 256, (50000, 8), generator=g, dtype=torch.uint8)
    lut = torch.rand(8, 256, generator=g)
    got = pq.pq_adc_search(codes.cuda(), lut.cuda()).cpu()
    torch.testing.assert_close(got, pq.pq_adc_search(codes, lut), rtol=1e-5, atol=1e-5)


def test_aqlm_gpu_fit_serves_in_gemm(cuda):
    from squish_b200.quant.aqlm import aqlm_quantize

    g = torch.Generator().manual_seed(9)
    w = torch.randn(256, 512, generator=g) * 0.02
    t = aqlm_quantize(w.cuda(), iters=5)
    dw = K.prepare_weight(t, cuda)
    x = torch.randn(16, 512, generator=g).to(torch.bfloat16)
    y = ops.w4a16_linear(x.to(cuda), dw)
    ref = x.float() @ t.dequantize().float().T
    assert (y.float().cpu() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item() + 1e-2


@pytest.mark.parametrize("k,b", [(3584, 512), (1024, 1024), (4096, 4096), (96, 32)])
def test_hadamard_kernel_matches_torch(k, b):
    from squish_b200.quant.sqint2 import fwht_blocks, rotation_signs

    g = torch.Generator().manual_seed(k)
    x = torch.randn(70, k, generator=g).to(torch.bfloat16)
    s = rotation_signs(k, 3)
    from squish_b200._ext import native

    y = native().hadamard_rows(x.cuda(), s.cuda(), b).cpu().float()
    ref = fwht_blocks(x.float() * s, b) / b ** 0.5
    torch.testing.assert_close(y, ref, rtol=1e-2, atol=1e-2)
    # strided rows into a larger output buffer
    out = torch.zeros(80, k, dtype=torch.bfloat16, device="cuda")
    native().hadamard_rows(x.cuda(), s.cuda(), b, out)
    assert torch.equal(out[:70].cpu(), y.to(torch.bfloat16)) and out[70:].abs().sum().item() == 0


@pytest.mark.parametrize("m", [1, 37, 300, 500])
def test_sqint2_linear_matches_fp32(cuda, m):
    """An SQINT2 weight (rotated INT2 in the tcgen05 GEMM, input rotated by the kernel) against
    x @ W^T with W the unrotated dequantisation, in the fused-dequant (small M) and expanded
    (large M) paths."""
    from squish_b200.quant.sqint2 import SQINT2Config, compress_weight

    g = torch.Generator().manual_seed(m)
    n, k = 640, 1536
    w = torch.randn(n, k, generator=g) * 0.02
    t = compress_weight(w, SQINT2Config(group_size=64))
    dw = K.prepare_weight(t, cuda)
    assert dw.rot is not None and dw.rot_block == 512
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    y = ops.w4a16_linear(x.to(cuda), dw)
    torch.cuda.synchronize()
    ref = x.float() @ t.dequantize().float().T
    err = (y.float().cpu() - ref).abs().max().item()
    assert err <= 3e-2 * ref.abs().max().item() + 1e-2, err


def test_engine_with_sqint2_weights_matches_oracle(cuda):
    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.engine.sampling import SamplingParams
    from squish_b200.models.config import get_preset
    from squish_b200.models.reference import ReferenceModel
    from squish_b200.models.weights import linear_names, random_checkpoint

    from .test_engine_gpu import _teacher_forced_ok

    cfg, q = get_preset("tiny-llama")
    cfg = dataclasses.replace(cfg, intermediate_size=512)

    def ck():
        c = random_checkpoint(cfg, q, seed=0)
        for name, _ in linear_names(cfg):
            c.tensors[name] = quantize(c.tensors[name].dequantize().float(), "sqint2", 32)
        return c

    ref = ReferenceModel(ck())
    eng = LLMEngine.from_checkpoint(ck(), cuda, EngineConfig(max_num_seqs=2, max_model_len=256, num_pages=32))
    assert eng.runner.layers[0].qkv.rot is not None and eng.runner.layers[0].gate_up.rot is not None
    prompt = np.random.default_rng(3).integers(0, cfg.vocab_size, 30).tolist()
    out = eng.generate([prompt], SamplingParams(max_tokens=8, ignore_eos=True))[0]
    ok, worst = _teacher_forced_ok(ref, prompt, out)
    assert ok, (worst, out)


def test_engine_with_mixed_precision_checkpoint(cuda, tmp_path, monkeypatch):
    """compress --format mixed (INT4 boundary layers, INT3 attention, SQINT2 gate/up) runs in the
    engine with every projection in its own GEMM code format, matching the CPU oracle."""
    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.engine.sampling import SamplingParams
    from squish_b200.io.convert import compress, load_checkpoint
    from squish_b200.models import config as C
    from squish_b200.models.reference import ReferenceModel

    from .test_engine_gpu import _teacher_forced_ok

    cfg, q = C.get_preset("tiny-llama")
    cfg = dataclasses.replace(cfg, name="tiny-llama-6l", num_layers=6, intermediate_size=512)
    monkeypatch.setitem(C.PRESETS, "tiny-llama-6l", (cfg, q))
    compress(None, str(tmp_path / "m"), kind="mixed", random_preset="tiny-llama-6l", device="cpu", group_size=32,
             log=lambda *_: None)
    ck, _ = load_checkpoint(str(tmp_path / "m"), "cpu")
    ref = ReferenceModel(ck)
    eng = LLMEngine.from_checkpoint(load_checkpoint(str(tmp_path / "m"), "cpu")[0], cuda,
                                    EngineConfig(max_num_seqs=2, max_model_len=256, num_pages=32))
    L = eng.runner.layers
    assert L[0].qkv.fmt == K.WF_INT4 and L[2].qkv.fmt == K.WF_INT3 and L[2].gate_up.fmt == K.WF_INT2
    assert L[2].gate_up.rot is not None and L[2].down.fmt == K.WF_INT4
    prompt = np.random.default_rng(4).integers(0, cfg.vocab_size, 30).tolist()
    out = eng.generate([prompt], SamplingParams(max_tokens=8, ignore_eos=True))[0]
    ok, worst = _teacher_forced_ok(ref, prompt, out)
    assert ok, (worst, out)
