"""Convert-time quantization research methods and predictor helpers (csrc/quant_research.cpp,
quant/research.py) against plain numpy / torch restatements of their math: any4 Lloyd levels,
QuaRot group codes and rotated INT4 weights, AdaRound (the C++ gradient step against autograd
of the published objective, and the layer optimiser against round-to-nearest), FLUTE LUT codes,
QMoE block codebooks, BitDistiller / GGUF group codes, the GRU cell, cosine similarity and the
online logistic predictor."""
import numpy as np
import pytest
import torch

from squish_b200.quant import research as R


def _lloyd_np(v, c, iters):
    c = np.sort(c.copy())
    for _ in range(iters):
        a = np.abs(v[:, None] - c[None, :]).argmin(1)
        nc = np.array([v[a == j].mean() if (a == j).any() else c[j] for j in range(len(c))])
        nc = np.sort(nc)
        if np.array_equal(nc, c):
            break
        c = nc
    return c


def test_any4_lloyd_matches_numpy():
    rng = np.random.default_rng(0)
    v = rng.standard_normal(5000).astype(np.float32)
    init = np.linspace(-2, 2, 16).astype(np.float32)
    got = R.any4_lloyd(torch.from_numpy(v), torch.from_numpy(init), 50).numpy()
    want = _lloyd_np(v.astype(np.float64), init.astype(np.float64), 50)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)
    assert np.all(np.diff(got) > 0)


def test_any4_beats_nf4_on_non_normal_weights():
    from squish_b200.quant.codecs import quantize

    g = torch.Generator().manual_seed(1)
    w = torch.rand(64, 256, generator=g) ** 3 - 0.2  # skewed, far from a normal distribution
    t4 = quantize(w, "any4", 64)
    tn = quantize(w, "nf4", 64)
    assert t4.kind == "nf4" and t4.extra["levels"].shape == (16,)
    e4 = (t4.dequantize() - w).pow(2).mean().item()
    en = (tn.dequantize() - w).pow(2).mean().item()
    assert e4 < 0.8 * en, (e4, en)
    # the codes index the table: decoding by hand gives the same weights
    p = t4.packed
    codes = torch.stack([p & 0xF, p >> 4], -1).reshape(64, 256).long()
    lv = t4.extra["levels"].to(torch.bfloat16).float()
    want = lv[codes] * t4.scales.repeat_interleave(64, 1)
    torch.testing.assert_close(t4.dequantize(), want)


def test_quarot_group_quant_roundtrip():
    rng = np.random.default_rng(2)
    w = rng.standard_normal((8, 40)).astype(np.float32)
    for sym in (True, False):
        q, s, z = R.quarot_group_quant(torch.from_numpy(w), 16, 7.0, sym)
        q, s, z = q.numpy(), s.numpy(), z.numpy()
        for g in range(3):
            blk = w[:, g * 16:(g + 1) * 16]
            if sym:
                assert s[g] == pytest.approx(np.abs(blk).max() / 7.0, rel=1e-6)
                assert np.array_equal(q[:, g * 16:(g + 1) * 16], np.clip(np.round(blk / s[g]), -7, 7))
            else:
                sc = (blk.max() - blk.min()) / 14.0
                assert s[g] == pytest.approx(sc, rel=1e-6) and z[g] == pytest.approx(-blk.min() / sc, rel=1e-5)
        back = R.quarot_group_dequant(torch.from_numpy(q), torch.from_numpy(s), torch.from_numpy(z), 16, sym).numpy()
        assert np.abs(back - w).max() <= (s.max() * 0.5 + 1e-5) * (1 if sym else 1.0001)


def test_quarot_rotated_int4_weight():
    from squish_b200.quant.sqint2 import rotate

    g = torch.Generator().manual_seed(3)
    w = torch.randn(32, 256, generator=g)
    w[:, 5] *= 40  # an outlier column: the rotation spreads it over its block
    t = R.quarot_quantize(w, 64, bits=4, block=128, seed=7)
    assert t.kind == "q4a" and t.extra["rot_block"] == 128
    err_rot = (t.dequantize() - w).pow(2).mean().item()
    from squish_b200.quant.codecs import quantize

    err_plain = (quantize(w, "q4a", 64).dequantize() - w).pow(2).mean().item()
    assert err_rot < err_plain, (err_rot, err_plain)
    # the GEMM multiplies the stored codes (W R^T) by the rotated input: (W R^T)(R x) == W x
    x = torch.randn(4, 256, generator=g)
    stored = rotate(t.dequantize(), t.extra["rot_signs"], 128)  # rows of W R^T
    y = rotate(x, t.extra["rot_signs"], 128) @ stored.T
    assert torch.allclose(y, x @ t.dequantize().T, atol=1e-3)


def test_adaround_step_matches_autograd():
    g = torch.Generator().manual_seed(4)
    n = 1000
    v = torch.randn(n, generator=g)
    w = torch.randn(n, generator=g)
    s = torch.rand(n, generator=g) * 0.1 + 0.05
    f = torch.floor(w / s)
    lr, beta, lam = 0.1, 4.0, 0.3
    vv = v.clone().requires_grad_(True)
    h = torch.clamp(torch.sigmoid(vv) * 1.2 - 0.1, 0, 1)
    loss = (0.5 * (s * (f + h) - w) ** 2 + lam * (1 - (2 * h - 1).abs() ** beta)).sum()
    loss.backward()
    want = v - lr * vv.grad
    got = R.adaround_step(v, w, f, s, lr, beta, lam)
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5)


def test_adaround_layer_beats_round_to_nearest():
    from squish_b200.quant.codecs import quantize

    g = torch.Generator().manual_seed(5)
    w = torch.randn(24, 128, generator=g) * 0.05
    x = torch.randn(256, 128, generator=g)
    x[:, :8] *= 6  # a few dominant input channels make rounding decisions matter
    t = R.adaround_q4a(w, x, 64, iters=300)
    rtn = quantize(w, "q4a", 64)
    y = x @ w.T
    e_ada = (x @ t.dequantize().T - y).pow(2).mean().item()
    e_rtn = (x @ rtn.dequantize().T - y).pow(2).mean().item()
    assert e_ada < e_rtn, (e_ada, e_rtn)


def test_flute_lut_codes():
    rng = np.random.default_rng(6)
    w = rng.standard_normal((5, 24)).astype(np.float32)
    cb = np.sort(rng.standard_normal((3, 8)).astype(np.float32), axis=1)
    codes = R.flute_lut_encode(torch.from_numpy(w), torch.from_numpy(cb), 8).numpy()
    for c in range(24):
        want = np.abs(w[:, c:c + 1] - cb[c // 8][None, :]).argmin(1)
        assert np.array_equal(codes[:, c], want)
    back = R.flute_lut_decode(torch.from_numpy(codes), torch.from_numpy(cb), 8).numpy()
    assert np.array_equal(back, np.stack([cb[c // 8][codes[:, c]] for c in range(24)], 1))


def test_qmoe_codebook_matches_numpy_kmeans():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((300, 4)).astype(np.float32)
    k = 6
    cb, a = R.qmoe_compress(torch.from_numpy(x), k, 25)
    c = np.stack([x[min(299, i * 300 // k)] for i in range(k)]).astype(np.float64)
    asg = None
    for _ in range(25):
        na = ((x[:, None, :] - c[None]) ** 2).sum(-1).argmin(1)
        if asg is not None and np.array_equal(na, asg):
            break
        asg = na
        c = np.stack([x[asg == j].mean(0) if (asg == j).any() else c[j] for j in range(k)])
    assert np.array_equal(a.numpy(), asg)
    np.testing.assert_allclose(cb.numpy(), c, rtol=1e-4, atol=1e-5)


def test_bit_distiller_and_gguf_codes():
    rng = np.random.default_rng(8)
    w = rng.standard_normal((6, 64)).astype(np.float32)
    for bits in (2, 4, 8):
        q, s, z = R.bit_distiller_quant(torch.from_numpy(w), bits, 32)
        L = 2 ** bits - 1
        blk = w.reshape(6, 2, 32)
        mn, mx = blk.min(-1), blk.max(-1)
        np.testing.assert_allclose(s.numpy(), (mx - mn) / L, rtol=1e-6)
        want = np.clip(np.round((blk - mn[..., None]) / (mx - mn)[..., None] * L), 0, L).reshape(6, 64)
        assert np.array_equal(q.numpy().astype(np.int64), want.astype(np.int64))
        q2, s2, m2, sup = R.gguf_mixed_quant(torch.from_numpy(w), bits, 32)
        np.testing.assert_allclose(m2.numpy(), mn.reshape(-1), rtol=1e-5, atol=1e-6)
        sv = s2.numpy()
        np.testing.assert_allclose(sup.numpy(), [sv[i:i + 8].mean() for i in range(0, len(sv), 8)], rtol=1e-5)
        deq = q2.numpy().reshape(6, 2, 32) * s2.numpy().reshape(6, 2, 1) + m2.numpy().reshape(6, 2, 1)
        assert np.abs(deq.reshape(6, 64) - w).max() <= s2.numpy().max() * 0.5 + 1e-5


def test_gru_cell_and_cosine():
    g = torch.Generator().manual_seed(9)
    cell = torch.nn.GRUCell(16, 12)
    x, h = torch.randn(16, generator=g), torch.randn(12, generator=g)
    with torch.no_grad():
        gx = cell.weight_ih @ x + cell.bias_ih
        gh = cell.weight_hh @ h + cell.bias_hh
        want = cell(x[None], h[None])[0]
    torch.testing.assert_close(R.gru_step(gx, gh, h), want, rtol=1e-5, atol=1e-6)
    a, b = torch.randn(5, 32, generator=g), torch.randn(7, 32, generator=g)
    b[3] = 0
    want = torch.nn.functional.cosine_similarity(a[:, None], b[None], dim=-1)
    want[:, 3] = 0
    torch.testing.assert_close(R.batched_cosine_similarity(a, b), want, rtol=1e-5, atol=1e-6)


def test_online_logistic_learns_a_separable_rule():
    rng = np.random.default_rng(10)
    m = R.OnlineLogistic(3, lr=0.5)
    for _ in range(2000):
        x = np.array([rng.uniform(-1, 1), rng.uniform(-1, 1), 1.0], dtype=np.float32)
        m.update(x, float(x[0] + 0.5 * x[1] > 0))
    assert m.predict([0.9, 0.5, 1.0]) > 0.9 and m.predict([-0.9, -0.5, 1.0]) < 0.1


def test_any4_and_quarot_survive_npy_dir_and_compress(tmp_path):
    """Learned level tables and QuaRot rotations are written and read back with their codes
    (npy-dir __lv_nf4 / __rot_signs + __rot_meta), and ``compress --format any4 | quarot``
    produces them."""
    from squish_b200.io import convert, npy_dir
    from squish_b200.models.config import get_preset
    from squish_b200.models.weights import random_checkpoint
    from squish_b200.quant.codecs import quantize

    cfg, q = get_preset("tiny-llama")
    ck = random_checkpoint(cfg, q, seed=0)
    a = "model.layers.0.mlp.down_proj.weight"
    b = "model.layers.1.self_attn.o_proj.weight"
    ck.tensors[a] = quantize(ck[a].dequantize(), "any4", 32)
    ck.tensors[b] = quantize(ck[b].dequantize(), "quarot", 64)
    npy_dir.write_npy_dir(tmp_path / "m", ck)
    back, _ = convert.load_checkpoint(str(tmp_path / "m"))
    assert back[a].extra and torch.equal(back[a].extra["levels"], ck[a].extra["levels"])
    assert back[b].extra["rot_block"] == ck[b].extra["rot_block"]
    for n in (a, b):
        torch.testing.assert_close(back[n].dequantize(), ck[n].dequantize(), atol=0, rtol=0)
    for fmt, kind, key in (("any4", "nf4", "levels"), ("quarot", "q4a", "rot_signs")):
        out = tmp_path / fmt
        convert.compress(None, str(out), kind=fmt, random_preset="tiny-llama", group_size=32, device="cpu")
        c2, _ = convert.load_checkpoint(str(out))
        t = c2["model.layers.0.self_attn.q_proj.weight"]
        assert t.kind == kind and key in t.extra


def test_lowrank_residual_weights_fuse_exactly():
    """MiLo INT3 compensators and SQINT2 residuals survive the fused qkv (row concatenation) and
    gate/up (64-row interleave) layouts as block-diagonal factor pairs: the fused weight
    dequantizes to the fused dequantized parts."""
    from squish_b200.models.decoder import _cat_rows, _interleave_gate_up, _same_kind, gemm_extra_ok
    from squish_b200.quant.sqint2 import SQINT2Config, compress_weight

    g = torch.Generator().manual_seed(11)
    a = R.milo_int3(torch.randn(96, 128, generator=g) * 0.05, 32, 4)
    b = R.milo_int3(torch.randn(64, 128, generator=g) * 0.05, 32, 2)
    c = R.quantize_any4(torch.randn(64, 128, generator=g), 32)  # (a different kind)
    assert gemm_extra_ok(a) and _same_kind([a, b], 32) == [a, b]
    assert all(t.kind == "q4a" for t in _same_kind([a, c], 32))
    fused = _cat_rows([a, b])
    torch.testing.assert_close(fused.dequantize(), torch.cat([a.dequantize(), b.dequantize()]), rtol=0, atol=1e-5)
    gu = _interleave_gate_up(a, R.milo_int3(torch.randn(96, 128, generator=g) * 0.05, 32, 3))
    ga, ua = a.dequantize(), gu.dequantize()
    torch.testing.assert_close(ua[0:64], ga[0:64], rtol=0, atol=1e-5)  # first 64 gate rows lead
    torch.testing.assert_close(ua[128:160], ga[64:96], rtol=0, atol=1e-5)
    # SQINT2 with a rank-4 residual in the rotated frame
    s1 = compress_weight(torch.randn(64, 128, generator=g) * 0.05, SQINT2Config(group_size=32, residual_rank=4))
    s2 = compress_weight(torch.randn(32, 128, generator=g) * 0.05, SQINT2Config(group_size=32, residual_rank=4))
    assert "sq_L" in s1.extra and gemm_extra_ok(s1)
    if _same_kind([s1, s2], 32) == [s1, s2]:  # same rotation (same seed and block)
        f2 = _cat_rows([s1, s2])
        torch.testing.assert_close(f2.dequantize(), torch.cat([s1.dequantize(), s2.dequantize()]), rtol=0,
                                   atol=1e-4)


def test_milo_compensator_reduces_error():
    g = torch.Generator().manual_seed(12)
    w = torch.randn(128, 256, generator=g) * 0.05
    w += torch.randn(128, 4, generator=g) @ torch.randn(4, 256, generator=g) * 0.05  # a low-rank component
    from squish_b200.quant.codecs import quantize

    plain = (quantize(w, "q3", 32).dequantize() - w).pow(2).mean().item()
    comp = (R.milo_int3(w, 32, 8).dequantize() - w).pow(2).mean().item()
    assert comp < 0.8 * plain, (comp, plain)


def test_pq_cache_fit_is_a_lloyd_fixed_point():
    g = torch.Generator().manual_seed(13)
    x = torch.cat([torch.randn(100, 4, generator=g) + 5 * i for i in range(4)])
    cb = R.C().pq_cache_fit(x, 4, 50, 3)
    a = torch.cdist(x, cb).argmin(1)
    for j in range(4):
        if (a == j).any():
            torch.testing.assert_close(cb[j], x[a == j].mean(0), rtol=1e-4, atol=1e-4)


def test_bit_distiller_refine_lowers_teacher_weighted_error():
    g = torch.Generator().manual_seed(14)
    w = torch.randn(16, 128, generator=g)
    w[:, ::17] *= 6  # outliers stretch the min / max grid
    teacher = torch.randn(16, 128, generator=g)
    s, z = R.C().bit_distiller_refine(w, teacher, 4, 64, 16, 0.5)
    q0, s0, z0 = R.bit_distiller_quant(w, 4, 64)

    def err(scale, zero):
        sc = scale.repeat_interleave(64, 1)
        ze = zero.repeat_interleave(64, 1)
        q = torch.clamp(torch.round(w / sc + ze), 0, 15)
        p = torch.softmax(teacher.view(16, 2, 64) / 0.5, -1).view(16, 128)
        return (p * ((q - ze) * sc - w) ** 2).sum().item()

    assert err(s, z) <= err(s0, z0) + 1e-6


def test_randomized_svd_matches_exact_on_low_rank_plus_noise():
    g = torch.Generator().manual_seed(15)
    a = torch.randn(200, 6, generator=g) @ torch.randn(6, 150, generator=g) + 1e-3 * torch.randn(200, 150, generator=g)
    U, S, Vh = R.randomized_svd(a, 6, seed=1)
    torch.testing.assert_close(S, torch.linalg.svdvals(a)[:6], rtol=1e-3, atol=1e-3)
    assert ((U * S) @ Vh - a).abs().max().item() < 0.02
