"""Linear-recurrence scans and sparse GEMVs (csrc/recurrent.cpp) against plain torch loops of
the same recurrences: Mamba-2, Hawk RG-LRU, DeltaNet, ternary and activation-sparse GEMV."""
import torch

from squish_b200._ext import native


def C():
    return native().cpu


def test_mamba2_scan():
    g = torch.Generator().manual_seed(0)
    T, N = 40, 8
    a = -torch.rand(T, generator=g)
    B, Cm = torch.randn(T, N, generator=g), torch.randn(T, N, generator=g)
    x, h0 = torch.randn(T, generator=g), torch.randn(N, generator=g)
    y, hT = C().mamba2_scan(a, B, Cm, x, h0)
    h, ys = h0.clone(), []
    for t in range(T):
        h = torch.exp(a[t]) * h + B[t] * x[t]
        ys.append((Cm[t] * h).sum())
    torch.testing.assert_close(y, torch.stack(ys), rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(hT, h, rtol=1e-4, atol=1e-5)


def test_hawk_scan():
    g = torch.Generator().manual_seed(1)
    T, N = 30, 16
    x, dt = torch.randn(T, N, generator=g), torch.randn(T, N, generator=g)
    lam, h0 = torch.randn(N, generator=g) * 0.5, torch.randn(N, generator=g)
    out, hT = C().hawk_scan(x, dt, lam, h0)
    h, hs = h0.clone(), []
    for t in range(T):
        f = torch.exp(-torch.exp(lam) * torch.nn.functional.softplus(dt[t]))
        h = f * h + torch.sqrt(1 - f * f) * x[t]
        hs.append(h)
    torch.testing.assert_close(out, torch.stack(hs), rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(hT, h, rtol=1e-4, atol=1e-5)


def test_delta_net_scan():
    g = torch.Generator().manual_seed(2)
    T, H, D = 12, 2, 8
    q, k, v = (torch.randn(T, H, D, generator=g) for _ in range(3))
    beta = torch.rand(T, H, generator=g)
    y = C().delta_net_scan(q, k, v, beta)
    want = torch.zeros(T, H, D)
    for h in range(H):
        S = torch.zeros(D, D)
        for t in range(T):
            kh = k[t, h] / k[t, h].norm()
            S = S + beta[t, h] * torch.outer(v[t, h] - S @ kh, kh)
            want[t, h] = S @ q[t, h]
    torch.testing.assert_close(y, want, rtol=1e-4, atol=1e-4)


def test_ternary_and_sparse_gemv():
    g = torch.Generator().manual_seed(3)
    w = torch.randint(-1, 2, (20, 64), generator=g).to(torch.int8)
    x = torch.randn(64, generator=g)
    torch.testing.assert_close(C().ternary_gemv(w, x, 0.3), 0.3 * (w.float() @ x), rtol=1e-5, atol=1e-5)
    wf = torch.randn(20, 64, generator=g)
    xs = x * (x.abs() > 0.8)
    torch.testing.assert_close(C().sparse_act_gemv(wf, x, 0.8), wf @ xs, rtol=1e-5, atol=1e-5)


def test_mamba2_step_is_one_scan_step():
    g = torch.Generator().manual_seed(4)
    B, Cm, h = (torch.randn(8, generator=g) for _ in range(3))
    y, h1 = C().mamba2_step(-0.3, B, Cm, 0.7, h)
    ys, hs = C().mamba2_scan(torch.tensor([-0.3]), B[None], Cm[None], torch.tensor([0.7]), h)
    assert abs(y - float(ys[0])) < 1e-5
    torch.testing.assert_close(h1, hs)
