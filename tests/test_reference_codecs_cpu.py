"""This package's codecs against the reference's own numpy code, imported from the installed
reference (baseline/_ref) and run directly, bit for bit where the format defines the bits:

  * KV codecs: per-token INT8 / INT4 / INT2 (squish/kv/kv_cache.py:78-375) and the k8v4
    group codec (squish/kv/k8v4_codec.py:64-137), with this package's C++ codec in its
    float32-scale mode (the reference arithmetic);
  * weight codecs: per-row / per-group symmetric INT8 (squish/quant/quantizer.py:163-200);
  * the fused INT4 matmul oracle ``_quantized_matmul_int4_numpy`` (quantizer.py:632) against
    the C++ ``quantized_matmul_int4``;
  * an npy-dir written by the reference's ``write_npy_dir`` (squish/convert.py:936) from its
    numpy quantization paths, loaded by this package's reader.
"""
import json
import os
import sys

import numpy as np
import pytest
import torch

from squish_b200._ext import native

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "squish")):
        pytest.skip("the reference is not installed in baseline/_ref")
    sys.path.insert(0, REF)
    try:
        import squish.kv.k8v4_codec as k8v4
        import squish.kv.kv_cache as kvc
        import squish.quant.quantizer as qz
    finally:
        sys.path.remove(REF)
    return {"kvc": kvc, "k8v4": k8v4, "qz": qz}


def _rows(n=257, d=128, seed=0, scale=1.0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((n, d)) * scale).astype(np.float16)
    x[3] = 0  # an all-zero row (the 1e-8 floor)
    x[5, :7] = 60.0  # an outlier row
    return x


def test_kv_int4_int2_int8_match_reference(ref):
    kvc, C = ref["kvc"], native().cpu
    x = _rows()
    xf = torch.from_numpy(x.astype(np.float32))
    d = x.shape[1]
    for fmt, qf, levels in ((2, kvc._quantize_int4_per_channel, 7.5), (3, kvc._quantize_int2_per_channel, 1.5)):
        packed, scale = qf(x)
        codes, scales = C.kv_quantize(xf, fmt, d, fp16_scales=False)
        assert np.array_equal(codes.numpy(), packed), f"fmt {fmt}: codes differ"
        assert np.array_equal(scales.numpy()[:, 0], scale), f"fmt {fmt}: scales differ"
    q8, s8 = kvc._quantize_int8_per_channel(x)
    codes, scales = C.kv_quantize(xf, 1, d, fp16_scales=False)
    assert np.array_equal(codes.numpy().view(np.int8), q8)
    np.testing.assert_allclose(scales.numpy()[:, 0] * 127.0, s8, rtol=1e-6)
    # decoding: same levels (reference returns fp16)
    packed, scale = kvc._quantize_int4_per_channel(x)
    ref_dec = kvc._dequantize_int4_per_channel(packed, scale, d).astype(np.float32)
    ours = C.kv_dequantize(torch.from_numpy(packed), torch.from_numpy(scale[:, None].copy()), 2, d, d).numpy()
    np.testing.assert_array_equal(ours.astype(np.float16).astype(np.float32), ref_dec)


@pytest.mark.parametrize("group", [32, 64, 128])
def test_k8v4_matches_reference(ref, group):
    k8v4, C = ref["k8v4"], native().cpu
    x = _rows(seed=group)
    xf = torch.from_numpy(x.astype(np.float32))
    for bits, fmt in ((8, 4), (4, 5)):
        pay = k8v4.quantize_array(x.astype(np.float32), bits, group)
        codes, scales = C.kv_quantize(xf, fmt, group, fp16_scales=False)
        assert np.array_equal(codes.numpy(), pay["q"]), f"{bits}-bit codes differ"
        ng = x.shape[1] // group
        sz = scales.numpy().reshape(-1, ng, 2)
        assert np.array_equal(sz[..., 0], pay["scale"]) and np.array_equal(sz[..., 1], pay["zero"])
        dec = C.kv_dequantize(codes, scales, fmt, group, x.shape[1]).numpy()
        np.testing.assert_allclose(dec, k8v4.dequantize_array(pay, dtype=np.float32), rtol=0, atol=1e-6)


def test_kv_fp16_scale_mode_stays_within_one_level(ref):
    """The device pools store fp16 scales and choose codes under them: at most one level away
    from the reference's float32-scale codes, and only on a small fraction of values."""
    kvc, C = ref["kvc"], native().cpu
    x = _rows(n=1024, seed=7)
    packed, _ = kvc._quantize_int4_per_channel(x)
    codes, _ = C.kv_quantize(torch.from_numpy(x.astype(np.float32)), 2, x.shape[1])
    a = np.stack([packed & 15, packed >> 4], -1).astype(int)
    b = np.stack([codes.numpy() & 15, codes.numpy() >> 4], -1).astype(int)
    diff = np.abs(a - b)
    assert diff.max() <= 1 and diff.mean() < 0.01


@pytest.mark.parametrize("group", [0, 64])
def test_int8_weight_codec_matches_reference(ref, group):
    qz, C = ref["qz"], native().cpu
    rng = np.random.default_rng(group)
    w = (rng.standard_normal((96, 320)) * 0.02).astype(np.float32)
    w[7] = 0
    r = qz._quantize_numpy(w, group)
    q, s = C.quantize_int8(torch.from_numpy(w), group)
    assert np.array_equal(q.numpy(), r.quantized)
    np.testing.assert_array_equal(s.numpy().reshape(r.scales.shape), r.scales)


def test_fused_int4_matmul_matches_reference_oracle(ref):
    qz, C = ref["qz"], native().cpu
    rng = np.random.default_rng(3)
    out_f, in_f, g = 48, 256, 32
    codes = rng.integers(0, 256, (out_f, in_f // 2), dtype=np.uint8)
    scales = rng.uniform(0.001, 0.02, (out_f, in_f // g)).astype(np.float32)
    offsets = rng.uniform(-0.1, 0.0, (out_f, in_f // g)).astype(np.float32)
    x = rng.standard_normal((5, in_f)).astype(np.float32)
    want = qz._quantized_matmul_int4_numpy(codes, scales, offsets, x, g)
    got = C.quantized_matmul_int4(torch.from_numpy(codes), torch.from_numpy(scales), torch.from_numpy(offsets),
                                  torch.from_numpy(x), g).numpy()
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


def test_reference_written_npy_dir_loads(ref, tmp_path):
    """An npy-dir the reference's own convert code produced: ``quantize_tensor`` (its default
    INT8 grouped-64 path and its float16 passthrough, numpy backend) and ``write_npy_dir``
    (squish/convert.py:283-540, :936), read by this package: the same dequantized values."""
    from pathlib import Path

    sys.path.insert(0, REF)
    try:
        import squish.convert as rconv
    finally:
        sys.path.remove(REF)
    qz = ref["qz"]
    rng = np.random.default_rng(11)
    weights = {"model.layers.0.mlp.down_proj.weight": (rng.standard_normal((64, 192)) * 0.02).astype(np.float32),
               "model.layers.0.self_attn.q_proj.weight": (rng.standard_normal((32, 128)) * 0.02).astype(np.float32),
               "model.norm.weight": rng.standard_normal(96).astype(np.float32)}
    npz, manifest = {}, {}
    for name, w in weights.items():
        files = rconv.quantize_tensor(name, w, outlier_threshold=1e9, passthrough_patterns=["norm"])
        key = rconv.safe_key(name)
        manifest[name] = key
        for suf, a in files.items():
            npz[key + suf] = a
    out = tmp_path / "ref_npy"
    rconv.write_npy_dir(Path(out), npz, manifest)
    from squish_b200.io.npy_dir import read_tensor, tensor_dir

    td = tensor_dir(out)
    for name, w in weights.items():
        t = read_tensor(td, manifest[name])
        if name.endswith("norm.weight"):
            assert t.kind == "dense"
            np.testing.assert_array_equal(t.data.float().numpy().reshape(-1), w.astype(np.float16).astype(np.float32))
            continue
        assert t.kind == "q8"
        r = qz._quantize_numpy(w, 64)
        want = qz._reconstruct_numpy(r)
        np.testing.assert_allclose(t.dequantize().float().numpy(), want, rtol=1e-6, atol=1e-7)
