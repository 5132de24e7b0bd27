"""C++ CPU reference kernels vs numpy restatements of the reference's quantizers.

The numpy functions below restate, in this repository's own code, the semantics of
squish/quant/quantizer.py:632 (`_quantized_matmul_int4_numpy`), the Rust quantizers in
squish_quant_rs/src/lib.rs (56, 402, 1125-1255, 1440-1550) and the KV codecs of
squish/kv/kv_cache.py:78-375 and squish/kv/k8v4_codec.py:64-137.
"""
import numpy as np
import pytest
import torch

from squish_b200._ext import native

C = native()


def np_round_half_away(x):
    return np.sign(x) * np.floor(np.abs(x) + 0.5)


def np_int4_asym(w, g):
    n, d = w.shape
    grp = w.reshape(n, d // g, g)
    mn, mx = grp.min(-1), grp.max(-1)
    sc = np.where(mx == mn, 1.0, (mx - mn) / 15.0).astype(np.float32)
    q = np.clip(np_round_half_away((grp - mn[..., None]) / sc[..., None]), 0, 15).astype(np.uint8).reshape(n, d)
    packed = (q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)
    return packed.astype(np.uint8), sc, mn.astype(np.float32)


def np_quantized_matmul_int4(w_codes, scales, offsets, x, group_size):
    out_f, n_packed = w_codes.shape
    in_f = n_packed * 2
    w = np.empty((out_f, in_f), dtype=np.float32)
    w[:, 0::2] = (w_codes & 0x0F).astype(np.float32)
    w[:, 1::2] = ((w_codes >> 4) & 0x0F).astype(np.float32)
    w_hat = np.repeat(offsets, group_size, axis=1) + w * np.repeat(scales, group_size, axis=1)
    return x.astype(np.float32) @ w_hat.T


@pytest.mark.parametrize("n,d,g", [(8, 64, 32), (33, 256, 64), (5, 688, 16)])
def test_int4_asym_quantizer_matches_rust_semantics(n, d, g):
    rng = np.random.default_rng(0)
    w = rng.standard_normal((n, d)).astype(np.float32)
    p, s, o = C.cpu.quantize_int4_asym(torch.from_numpy(w), g)
    rp, rs, ro = np_int4_asym(w, g)
    assert np.array_equal(p.numpy(), rp)
    np.testing.assert_allclose(s.numpy(), rs, rtol=1e-6)
    np.testing.assert_allclose(o.numpy(), ro, rtol=1e-6)
    deq = C.cpu.dequantize_int4_asym(p, s, o, g).numpy()
    assert np.abs(deq - w).max() <= (rs.max() * 0.5 + 1e-5)


def test_fused_int4_matmul_matches_numpy_oracle():
    rng = np.random.default_rng(1)
    w = rng.standard_normal((96, 256)).astype(np.float32) * 0.02
    x = rng.standard_normal((3, 256)).astype(np.float32)
    p, s, o = C.cpu.quantize_int4_asym(torch.from_numpy(w), 32)
    got = C.cpu.quantized_matmul_int4(p, s, o, torch.from_numpy(x), 32).numpy()
    ref = np_quantized_matmul_int4(p.numpy(), s.numpy(), o.numpy(), x, 32)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)


def test_int4_mse_clip_never_worse_than_plain():
    rng = np.random.default_rng(2)
    w = rng.standard_normal((64, 128)).astype(np.float32)
    w[::7, 3] *= 25  # outliers
    wt = torch.from_numpy(w)
    plain = C.cpu.dequantize_int4_asym(*C.cpu.quantize_int4_asym(wt, 32), 32).numpy()
    mse = C.cpu.dequantize_int4_asym(*C.cpu.quantize_int4_asym_mse(wt, 32, 8), 32).numpy()
    assert ((mse - w) ** 2).mean() <= ((plain - w) ** 2).mean() + 1e-9


def test_int8_symmetric():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((10, 128)).astype(np.float32)
    q, s = C.cpu.quantize_int8(torch.from_numpy(w), 64)
    grp = w.reshape(10, 2, 64)
    am = np.abs(grp).max(-1)
    rs = np.where(am == 0, 1.0, am / 127.0)
    rq = np.clip(np_round_half_away(grp / rs[..., None]), -127, 127).astype(np.int8).reshape(10, 128)
    assert np.array_equal(q.numpy(), rq)
    np.testing.assert_allclose(C.cpu.dequantize_int8(q, s).numpy(), w, atol=rs.max() / 2 + 1e-6)


def test_int3_pack_roundtrip_and_layout():
    rng = np.random.default_rng(4)
    w = rng.standard_normal((4, 64)).astype(np.float32)
    p, s = C.cpu.pack_int3(torch.from_numpy(w), 32)
    assert p.shape == (4, 24)
    u = C.cpu.unpack_int3(p, s, 32, 64).numpy()
    grp = w.reshape(4, 2, 32)
    sc = np.abs(grp).max(-1) / 3.0
    q = np.clip(np_round_half_away(grp / sc[..., None]), -3, 3)
    np.testing.assert_allclose(u, (q * sc[..., None]).reshape(4, 64), rtol=1e-6)
    # value j of a chunk sits at bits 3j..3j+2 of the little-endian 24-bit word
    bits = int(p[0, 0]) | (int(p[0, 1]) << 8) | (int(p[0, 2]) << 16)
    v0 = (bits & 7) - 8 if bits & 4 else bits & 7
    assert v0 == int(q[0, 0, 0])


def test_int2_asym_and_nf4():
    rng = np.random.default_rng(5)
    w = rng.standard_normal((6, 128)).astype(np.float32)
    p, s, o = C.cpu.quantize_int2(torch.from_numpy(w), 32)
    d = C.cpu.dequantize_int2(p, s, o, 32).numpy()
    assert np.abs(d - w).max() <= s.numpy().max() * 0.5 + 1e-5
    pn, sn = C.cpu.quantize_nf4(torch.from_numpy(w), 64)
    dn = C.cpu.dequantize_nf4(pn, sn, 64).numpy()
    assert np.corrcoef(dn.ravel(), w.ravel())[0, 1] > 0.98


@pytest.mark.parametrize("fmt,name", [(2, "int4"), (3, "int2"), (1, "int8")])
def test_kv_codecs_match_reference_semantics(fmt, name):
    rng = np.random.default_rng(6)
    x = rng.standard_normal((50, 128)).astype(np.float32)
    codes, scales = C.cpu.kv_quantize(torch.from_numpy(x), fmt, 128)
    d = C.cpu.kv_dequantize(codes, scales, fmt, 128, 128).numpy()
    am = np.abs(x).max(-1, keepdims=True)
    qmax = {"int4": 7.5, "int2": 1.5, "int8": 127.0}[name]
    s = np.maximum(am, 1e-8) / qmax
    if name == "int8":
        ref = np.clip(np.round(x / s), -128, 127) * s
    else:
        ref = (np.clip(np.round(x / s + qmax), 0, 2 * qmax) - qmax) * s
    # scales are stored in fp16: the reconstruction is within half a step of x, and equal
    # to the fp32-scale reference except where fp16 rounding moved a rounding boundary
    assert (np.abs(d - x) <= s * 0.5 * (1 + 2e-3) + 1e-6).all()
    assert np.mean(np.isclose(d, ref, atol=float(s.max()) * 0.1)) > 0.99


def test_k8v4_codec():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((20, 128)).astype(np.float32)
    for fmt, qmax in ((4, 255), (5, 15)):
        codes, scales = C.cpu.kv_quantize(torch.from_numpy(x), fmt, 64)
        d = C.cpu.kv_dequantize(codes, scales, fmt, 64, 128).numpy()
        grp = x.reshape(20, 2, 64)
        step = (grp.max(-1) - grp.min(-1)) / qmax
        assert (np.abs(d - x).reshape(20, 2, 64) <= step[..., None] * 0.51 + 1e-3).all()
