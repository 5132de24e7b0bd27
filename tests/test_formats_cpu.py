"""Checkpoint formats: npy-dir round trip, resumable compress, MLX 4-bit, GGUF import, SQUIZD.

Mirrors the reference's format tests (tests/test_convert_unit.py, tests/test_gguf_loader.py,
tests/test_squizd_format.py): each format is written, read back, and the dequantized
weights compared with the source.
"""
import json
import struct

import numpy as np
import pytest
import torch

from squish_b200.io import convert, gguf, npy_dir, squizd
from squish_b200.models.config import ModelConfig, QuantConfig
from squish_b200.models.weights import Checkpoint, QTensor, random_checkpoint
from squish_b200.quant.codecs import quantize


def _tiny_cfg(**kw):
    base = dict(name="t", arch="llama", vocab_size=64, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2,
                head_dim=16, intermediate_size=128, tie_embeddings=True)
    base.update(kw)
    return ModelConfig(**base)


def _same(a: Checkpoint, b: Checkpoint, atol=0.0):
    assert set(a.tensors) == set(b.tensors)
    for n in a.tensors:
        x, y = a[n].dequantize().float(), b[n].dequantize().float()
        torch.testing.assert_close(x, y, atol=atol, rtol=0, msg=n)


def test_npy_dir_round_trip(tmp_path):
    cfg = _tiny_cfg()
    ck = random_checkpoint(cfg, QuantConfig(group_size=32))
    ck.tensors["model.layers.0.mlp.down_proj.weight"] = quantize(torch.randn(64, 128) * 0.02, "q8", 32)
    ck.tensors["model.layers.1.mlp.down_proj.weight"] = quantize(torch.randn(64, 128) * 0.02, "nf4", 32)
    ck.tensors["model.layers.1.mlp.up_proj.weight"] = quantize(torch.randn(128, 64) * 0.02, "q2", 32)
    n = npy_dir.write_npy_dir(tmp_path / "m", ck)
    assert n > 0 and (tmp_path / "m" / "tensors" / ".manifest_ready").exists()
    assert npy_dir.detect_format(tmp_path / "m") == "npy-dir"
    back, tok = convert.load_checkpoint(str(tmp_path / "m"))
    assert back.config.hidden_size == 64 and back.config.tie_embeddings
    # dense tensors are stored as fp16 (__pt)
    for name in ck.tensors:
        tol = 1e-3 if ck[name].kind == "dense" else 0.0
        torch.testing.assert_close(back[name].dequantize(), ck[name].dequantize().float(), atol=tol, rtol=0)
    assert back["model.layers.0.mlp.down_proj.weight"].kind == "q8"


def test_npy_dir_reference_suffixes(tmp_path):
    """Files with the reference's legacy suffixes: __q4/__s4 (x = (q - 7) s) and __q/__s INT8."""
    td = tmp_path / "tensors"
    td.mkdir()
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 15, (8, 32), dtype=np.uint8)
    s4 = rng.random((8, 1), dtype=np.float32)
    np.save(td / "w__q4.npy", npy_dir.pack_nibbles(codes))
    np.save(td / "w__s4.npy", s4)
    np.save(td / "w__shape.npy", np.array([8, 32]))
    t = npy_dir.read_tensor(td, "w")
    want = (codes.astype(np.float32) - 7.0) * s4
    np.testing.assert_allclose(t.dequantize().numpy(), want, rtol=0, atol=1e-6)
    q = rng.integers(-127, 127, (4, 16), dtype=np.int8)
    s = rng.random(4, dtype=np.float32)
    np.save(td / "v__q.npy", q)
    np.save(td / "v__s.npy", s)
    np.testing.assert_allclose(npy_dir.read_tensor(td, "v").dequantize().numpy(), q * s[:, None], atol=1e-6)


def test_compress_random_preset_resumes(tmp_path):
    out = tmp_path / "c"
    logs = []
    st = convert.compress(None, str(out), random_preset="tiny-llama", group_size=32, device="cpu", log=logs.append)
    assert st["n_quantized"] > 0 and st["n_passthrough"] > 0
    prog = json.loads((out / "_compress_progress.json").read_text())
    assert "random-init" in prog["completed_shards"]
    st2 = convert.compress(None, str(out), random_preset="tiny-llama", group_size=32, device="cpu")
    assert st2["skipped_shards"] == 1 and st2["n_quantized"] == 0
    ck, _ = convert.load_checkpoint(str(out))
    assert ck.config.num_layers == 4 and ck["model.layers.0.self_attn.q_proj.weight"].kind == "q4a"


def test_compress_hf_safetensors_shards(tmp_path):
    from safetensors.torch import save_file

    from squish_b200.models.config import to_hf_config

    cfg = _tiny_cfg()
    src = tmp_path / "hf"
    src.mkdir()
    (src / "config.json").write_text(json.dumps(to_hf_config(cfg)))
    g = torch.Generator().manual_seed(0)
    w = {"model.embed_tokens.weight": torch.randn(64, 64, generator=g), "model.norm.weight": torch.ones(64)}
    for i in range(2):
        p = f"model.layers.{i}."
        w.update({p + "self_attn.q_proj.weight": torch.randn(64, 64, generator=g) * 0.02,
                  p + "self_attn.k_proj.weight": torch.randn(32, 64, generator=g) * 0.02,
                  p + "self_attn.v_proj.weight": torch.randn(32, 64, generator=g) * 0.02,
                  p + "self_attn.o_proj.weight": torch.randn(64, 64, generator=g) * 0.02,
                  p + "mlp.gate_proj.weight": torch.randn(128, 64, generator=g) * 0.02,
                  p + "mlp.up_proj.weight": torch.randn(128, 64, generator=g) * 0.02,
                  p + "mlp.down_proj.weight": torch.randn(64, 128, generator=g) * 0.02,
                  p + "input_layernorm.weight": torch.ones(64), p + "post_attention_layernorm.weight": torch.ones(64)})
    names = sorted(w)
    save_file({k: w[k] for k in names[: len(names) // 2]}, str(src / "model-00001-of-00002.safetensors"))
    save_file({k: w[k] for k in names[len(names) // 2:]}, str(src / "model-00002-of-00002.safetensors"))
    out = tmp_path / "out"
    st = convert.compress(str(src), str(out), group_size=32, device="cpu", delete_source=True)
    assert st["shards"] == 2 and not list(src.glob("*.safetensors"))
    ck, _ = convert.load_checkpoint(str(out))
    q = ck["model.layers.1.mlp.down_proj.weight"]
    assert q.kind == "q4a" and q.group == 32
    err = (q.dequantize() - w["model.layers.1.mlp.down_proj.weight"]).abs().max()
    assert err < 0.02 * 4 / 15 + 1e-6  # half a step of the per-group range at most, with margin
    assert ck["model.norm.weight"].kind == "dense"


def test_squish_4bit_mlx_directory(tmp_path):
    from safetensors.numpy import save_file

    from squish_b200.models.config import to_hf_config

    rng = np.random.default_rng(1)
    codes = rng.integers(0, 16, (16, 64), dtype=np.uint32)
    words = np.zeros((16, 8), np.uint32)
    for c in range(64):
        words[:, c // 8] |= codes[:, c] << (4 * (c % 8))
    scales = rng.random((16, 2)).astype(np.float16)
    biases = (rng.random((16, 2)) - 0.5).astype(np.float16)
    d = tmp_path / "mlx"
    d.mkdir()
    save_file({"model.layers.0.mlp.up_proj.weight": words, "model.layers.0.mlp.up_proj.scales": scales,
               "model.layers.0.mlp.up_proj.biases": biases,
               "model.norm.weight": np.ones(64, np.float16)}, str(d / "model.safetensors"))
    (d / "config.json").write_text(json.dumps(to_hf_config(_tiny_cfg())))
    assert npy_dir.detect_format(d) == "squish_4bit"
    ck, _ = convert.load_checkpoint(str(d))
    got = ck["model.layers.0.mlp.up_proj.weight"].dequantize().numpy()
    want = np.repeat(biases.astype(np.float32), 32, 1) + codes.astype(np.float32) * np.repeat(
        scales.astype(np.float32), 32, 1)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5)


def _q4_0_blocks(w: np.ndarray):
    """Reference Q4_0 encoder (llama.cpp block layout): d = max / -8, q = round(x/d) + 8."""
    rows, cols = w.shape
    b = w.reshape(-1, 32)
    idx = np.abs(b).argmax(1)
    mx = b[np.arange(len(b)), idx]
    d = (mx / -8.0).astype(np.float16)
    inv = np.where(d != 0, 1.0 / d.astype(np.float32), 0.0)
    q = np.clip(np.floor(b * inv[:, None] + 8.5), 0, 15).astype(np.uint8)
    packed = q[:, :16] | (q[:, 16:] << 4)
    raw = np.concatenate([d.view(np.uint8).reshape(-1, 2), packed], 1)
    deq = (q.astype(np.float32) - 8.0) * d.astype(np.float32)[:, None]
    return raw, deq.reshape(rows, cols)


def _q8_0_blocks(w: np.ndarray):
    b = w.reshape(-1, 32)
    d = (np.abs(b).max(1) / 127.0).astype(np.float16)
    inv = np.where(d != 0, 1.0 / d.astype(np.float32), 0.0)
    q = np.clip(np.rint(b * inv[:, None]), -127, 127).astype(np.int8)
    raw = np.concatenate([d.view(np.uint8).reshape(-1, 2), q.view(np.uint8)], 1)
    return raw, (q.astype(np.float32) * d.astype(np.float32)[:, None]).reshape(w.shape)


def test_gguf_import_q4_0_q8_0_and_unpermute(tmp_path):
    rng = np.random.default_rng(2)
    hid, nh = 64, 4
    wq = rng.standard_normal((hid, hid)).astype(np.float32)
    wd = rng.standard_normal((hid, 2 * hid)).astype(np.float32)
    emb = rng.standard_normal((32, hid)).astype(np.float32)
    # llama.cpp permutes Q rows per head: (h, 2, d/2) -> (h, d/2, 2)
    perm = wq.reshape(nh, 2, hid // nh // 2, hid).swapaxes(1, 2).reshape(hid, hid)
    raw_q, deq_q = _q4_0_blocks(perm)
    raw_d, deq_d = _q8_0_blocks(wd)
    meta = {"general.architecture": "llama", "general.name": "mini", "llama.block_count": 1,
            "llama.embedding_length": hid, "llama.attention.head_count": nh, "llama.attention.head_count_kv": nh,
            "llama.feed_forward_length": 2 * hid, "llama.rope.freq_base": 10000.0, "llama.context_length": 256}
    p = tmp_path / "mini.gguf"
    gguf.write_gguf_minimal(str(p), meta, {
        "token_embd.weight": (gguf.GGML_F32, emb, (hid, 32)),
        "blk.0.attn_q.weight": (gguf.GGML_Q4_0, raw_q, (hid, hid)),
        "blk.0.ffn_down.weight": (gguf.GGML_Q8_0, raw_d, (2 * hid, hid)),
    })
    assert npy_dir.detect_format(p) == "gguf"
    ck, _ = convert.load_checkpoint(str(p))
    assert ck.config.num_heads == nh and ck.config.tie_embeddings
    q = ck["model.layers.0.self_attn.q_proj.weight"]
    assert q.kind == "q4a" and q.group == 32
    unperm = deq_q.reshape(nh, hid // nh // 2, 2, hid).swapaxes(1, 2).reshape(hid, hid)
    np.testing.assert_allclose(q.dequantize().numpy(), unperm, atol=1e-5)
    d = ck["model.layers.0.mlp.down_proj.weight"]
    assert d.kind == "q8"
    np.testing.assert_allclose(d.dequantize().numpy(), deq_d, atol=1e-5)
    np.testing.assert_allclose(ck["lm_head.weight"].dequantize().numpy(), emb)


def test_gguf_rejects_kquants(tmp_path):
    p = tmp_path / "k.gguf"
    meta = {"general.architecture": "llama", "llama.block_count": 1, "llama.embedding_length": 32,
            "llama.attention.head_count": 2, "llama.feed_forward_length": 64}
    gguf.write_gguf_minimal(str(p), meta, {"blk.0.ffn_up.weight": (12, np.zeros(144, np.uint8), (256, 1))})
    with pytest.raises(ValueError, match="not supported"):
        gguf.read_gguf(str(p))


def test_squizd_round_trip_and_validation(tmp_path):
    cfg = _tiny_cfg(arch="qwen2", qkv_bias=True)
    ck = random_checkpoint(cfg, QuantConfig(group_size=32))
    p = tmp_path / "m.squizd"
    squizd.write_squizd(str(p), ck, group=32)
    info = squizd.validate(str(p), strict=True)
    assert info["layers"] == cfg.num_layers + 1 and info["flags"] & squizd.F_INT4
    assert npy_dir.detect_format(p) == "squizd"
    back, _ = convert.load_checkpoint(str(p))
    assert back.config.qkv_bias and back.config.arch == "qwen2" and back.config.hidden_size == 64
    for name in ck.tensors:
        a, b = ck[name].dequantize().float(), back[name].dequantize().float()
        if ck[name].kind == "dense":
            torch.testing.assert_close(b, a, atol=2e-3, rtol=1e-3)
        else:  # symmetric INT4 storage then INT4 asymmetric on load: two quantization steps
            rng = a.abs().amax(1, keepdim=True)
            assert ((b - a).abs() <= rng / 7 + 1e-6).all(), name
    # corruptions the validator must catch
    raw = bytearray(p.read_bytes())
    bad = tmp_path / "bad.squizd"
    bad.write_bytes(b"XXXX" + bytes(raw[4:]))
    with pytest.raises(ValueError, match="magic"):
        squizd.validate(str(bad))
    r2 = bytearray(raw)
    struct.pack_into("<H", r2, 4, 9)
    bad.write_bytes(bytes(r2))
    with pytest.raises(ValueError, match="version"):
        squizd.validate(str(bad))
    r3 = bytearray(raw)
    struct.pack_into("<I", r3, 6, squizd.F_INT4 | squizd.F_ASTC)
    bad.write_bytes(bytes(r3))
    with pytest.raises(ValueError, match="Apple"):
        squizd.read_squizd(str(bad))
    bad.write_bytes(bytes(raw[: squizd.HEADER + 10]))
    with pytest.raises(ValueError, match="truncated|bounds"):
        squizd.validate(str(bad))


def test_fnv1a64_known_vectors():
    assert squizd.fnv1a64(b"") == 0xCBF29CE484222325
    assert squizd.fnv1a64(b"a") == 0xAF63DC4C8601EC8C


def test_aqlm_codec_round_trip():
    torch.manual_seed(0)
    w = torch.randn(32, 64)
    t = quantize(w, "aqlm", 8)
    assert t.kind == "aqlm"
    rel = (t.dequantize() - w).norm() / w.norm()
    assert rel < 0.6
    # more codebooks = better reconstruction
    from squish_b200.quant.aqlm import aqlm_quantize

    t1 = aqlm_quantize(w, n_codebooks=1, codebook_size=16, group_size=8)
    t3 = aqlm_quantize(w, n_codebooks=3, codebook_size=16, group_size=8)
    assert (t3.dequantize() - w).norm() < (t1.dequantize() - w).norm()


def test_df11_lossless_roundtrip_and_npy_dir(tmp_path):
    """DFloat11-style passthrough: bf16 values come back bit for bit, ~11 bits per value for
    normal-distributed weights; pickled blobs (the reference's writer) are refused."""
    import pickle

    import numpy as np
    import torch

    from squish_b200.io.entropy import df11_decode, df11_encode
    from squish_b200.io.npy_dir import read_tensor

    x = (torch.randn(64, 300) * 0.02).to(torch.bfloat16)
    blob = df11_encode(x)
    back = df11_decode(blob)
    assert torch.equal(torch.from_numpy(back).reshape(64, 300), x.float())
    assert len(blob) * 8 / x.numel() < 12.5
    td = tmp_path / "tensors"
    td.mkdir()
    np.save(td / "w__pt_df11.npy", np.frombuffer(blob, dtype=np.uint8))
    np.save(td / "w__shape.npy", np.array([64, 300], dtype=np.int64))
    t = read_tensor(td, "w")
    assert t.kind == "dense" and t.shape == (64, 300) and torch.equal(t.data.float(), x.float())
    np.save(td / "p__pt_df11.npy", np.frombuffer(pickle.dumps([1, 2], protocol=4), dtype=np.uint8))
    import pytest

    with pytest.raises(ValueError, match="pickle"):
        read_tensor(td, "p")


def test_vptq_files_decode(tmp_path):
    """The reference's VPTQ file set (squish/convert.py:362-420): codebooks with three trailing
    scalars, per-(row, group) indices, an optional residual stage and column scales."""
    import numpy as np
    import torch

    from squish_b200.io.npy_dir import read_tensor

    rng = np.random.default_rng(0)
    rows, cols, gs, ncb, nres = 6, 16, 4, 8, 4
    cb = rng.standard_normal((ncb, gs)).astype(np.float32)
    rcb = rng.standard_normal((nres, gs)).astype(np.float32) * 0.1
    idx = rng.integers(0, ncb, (rows, cols // gs))
    res = rng.integers(0, nres, (rows, cols // gs))
    cs = rng.uniform(0.5, 2.0, cols).astype(np.float32)
    td = tmp_path / "tensors"
    td.mkdir()
    np.save(td / "w__vq_idx.npy", idx.astype(np.int64))
    np.save(td / "w__vq_cb.npy", np.concatenate([cb.reshape(-1), [ncb, gs, 10]]).astype(np.float32))
    np.save(td / "w__vq_res.npy", res.astype(np.int64))
    np.save(td / "w__vq_rescb.npy", np.concatenate([rcb.reshape(-1), [nres, gs, 10]]).astype(np.float32))
    np.save(td / "w__vq_cols.npy", cs)
    np.save(td / "w__vq_meta.npy", np.array([rows, cols, gs, ncb, nres], dtype=np.int64))
    np.save(td / "w__shape.npy", np.array([rows, cols], dtype=np.int64))
    want = (cb[idx] + rcb[res]).reshape(rows, cols) * cs[None, :]
    t = read_tensor(td, "w")
    assert t.kind == "dense" and torch.allclose(t.data.float(), torch.from_numpy(want))
    # no residual stage: a one-element __vq_res
    np.save(td / "w__vq_res.npy", np.zeros(1, dtype=np.int64))
    np.save(td / "w__vq_cols.npy", np.array([], dtype=np.float32))
    t = read_tensor(td, "w")
    assert torch.allclose(t.data.float(), torch.from_numpy(cb[idx].reshape(rows, cols)))
