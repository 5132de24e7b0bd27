"""KV budget / scoring research kernels (csrc/kv_research.cpp) against plain torch
restatements: CAKE entropy, GreenKV window scores, SVDq spectra, ShadowKV low-rank keys,
ClusterKV sums, PyramidKV budgets and the MagicPIG sampling estimator."""
import math

import torch

from squish_b200._ext import native


def C():
    return native().cpu


def test_cake_entropy_matches_torch():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(4, 3, 16, generator=g)  # [W, H, D]
    k = torch.randn(50, 3, 16, generator=g)  # [T, H, D]
    got = C().cake_entropy(q, k, 0.7)
    s = torch.einsum("whd,thd->hwt", q, k) / (math.sqrt(16) * 0.7)
    p = torch.softmax(s, -1)
    ent = -(p * p.clamp_min(1e-30).log()).sum(-1) / math.log(50)
    torch.testing.assert_close(got, ent.mean(-1), rtol=1e-4, atol=1e-5)
    assert (got > 0).all() and (got <= 1).all()


def test_green_kv_scores_are_window_mean_attention():
    g = torch.Generator().manual_seed(1)
    q = torch.randn(2, 5, 8, generator=g)
    k = torch.randn(2, 30, 8, generator=g)
    got = C().green_kv_score(q, k)
    want = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(8), -1).mean(1)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(got.sum(-1), torch.ones(2))


def test_svd_spectrum_and_shadow_kv_low_rank():
    g = torch.Generator().manual_seed(2)
    keys = torch.randn(2, 3, 40, 16, generator=g)
    torch.testing.assert_close(C().svd_head_spectrum(keys), torch.linalg.svdvals(keys), rtol=1e-4, atol=1e-4)
    # rank-4 keys plus noise: the fitted basis captures them
    base = torch.randn(3, 40, 4, generator=g) @ torch.randn(3, 4, 16, generator=g)
    kk = base + 0.01 * torch.randn(3, 40, 16, generator=g)
    V = C().shadow_kv_fit(kk, 4)
    assert V.shape == (3, 4, 16)
    torch.testing.assert_close(V @ V.transpose(1, 2), torch.eye(4).expand(3, 4, 4), rtol=1e-4, atol=1e-4)
    proj = C().shadow_kv_project(kk, V)
    rec = proj @ V
    sv = torch.linalg.svdvals(kk)
    err = (rec - kk).pow(2).sum((1, 2)).sqrt()
    torch.testing.assert_close(err, sv[:, 4:].pow(2).sum(-1).sqrt(), rtol=1e-3, atol=1e-4)


def test_cluster_sums_and_pyramid_budgets():
    a = torch.tensor([0, 2, 2, 1, 0, 2], dtype=torch.int32)
    w = torch.tensor([0.1, 0.2, 0.3, 0.05, 0.15, 0.2])
    torch.testing.assert_close(C().cluster_kv_score(a, w, 4), torch.tensor([0.25, 0.05, 0.7, 0.0]))
    b = C().pyramid_kv_budget(1000, 0.8, 5, 250)
    assert b.tolist() == [1000, 800, 600, 400, 250]
    assert C().pyramid_kv_budget(64, 0.5, 1, 1).tolist() == [64]


def test_magic_pig_estimate_approaches_exact_attention():
    g = torch.Generator().manual_seed(3)
    H, Tq, S, D = 2, 4, 256, 32
    q = torch.randn(H, Tq, D, generator=g)
    k = torch.randn(H, S, D, generator=g)
    v = torch.randn(H, S, D, generator=g)
    exact = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(D), -1) @ v
    # many short tables: nearly every key is sampled, the estimate is close to exact
    out, frac = C().magic_pig_attention(q, k, v, 64, 2, 0)
    assert (frac > 0.9).all()
    assert (out - exact).abs().max().item() < 0.05
    # long codes: few collisions; whatever is sampled, outputs stay convex combinations of v
    out2, frac2 = C().magic_pig_attention(q, k, v, 2, 16, 1)
    assert (frac2 < 0.5).all()
    assert (out2.abs().amax(-1) <= v.abs().amax((1, 2))[:, None] + 1e-5).all()
