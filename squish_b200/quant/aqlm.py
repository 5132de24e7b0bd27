"""AQLM additive-codebook weight quantization (the npy-dir ``__aqlm_idx`` / ``__aqlm_cb`` pair).

Encoding follows the reference's iterative residual scheme (squish/quant/aqlm.py:284-456):
normalise the matrix by its RMS (``scale``), then for each of K codebooks fit k-means on the
residual groups of ``group_size`` input features, assign each group its nearest codeword
and subtract it. Decoding: W[i, g*gs:(g+1)*gs] = scale * sum_k CB_k[idx[i, g, k]].

k-means runs in PyTorch (on the GPU when the weight is on one): k-means++-style seeding by
sampling, then Lloyd iterations with chunked nearest-centroid search.
Serialised codebook: float32 [scale, codebook_size, group_size, CB_0 ..., CB_{K-1} ...].
"""
from __future__ import annotations

import torch

from ..models.weights import QTensor


def _nearest(x: torch.Tensor, c: torch.Tensor, chunk: int = 65536) -> torch.Tensor:
    out = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    cn = (c * c).sum(1)
    for i in range(0, x.shape[0], chunk):
        xb = x[i:i + chunk]
        d = cn[None, :] - 2.0 * xb @ c.T
        out[i:i + chunk] = d.argmin(1)
    return out


def kmeans(x: torch.Tensor, k: int, iters: int = 20, seed: int = 42) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device="cpu").manual_seed(seed)
    n = x.shape[0]
    k = min(k, n)
    c = x[torch.randperm(n, generator=g)[:k].to(x.device)].clone()
    assign = _nearest(x, c)
    for _ in range(iters):
        sums = torch.zeros_like(c).index_add_(0, assign, x)
        cnt = torch.bincount(assign, minlength=k).float().clamp_min(1)[:, None]
        c = torch.where(cnt > 0, sums / cnt, c)
        new = _nearest(x, c)
        if torch.equal(new, assign):
            break
        assign = new
    return c, assign


def aqlm_quantize(w: torch.Tensor, n_codebooks: int = 2, codebook_size: int = 256, group_size: int = 8,
                  iters: int = 20, seed: int = 42) -> QTensor:
    out_f, in_f = w.shape
    if in_f % group_size:
        raise ValueError(f"in_features {in_f} not divisible by AQLM group size {group_size}")
    wf = w.float()
    scale = float(wf.pow(2).mean().sqrt().clamp_min(1e-12))
    resid = (wf / scale).reshape(-1, group_size)
    idx = torch.empty(resid.shape[0], n_codebooks, dtype=torch.int64, device=w.device)
    cbs = []
    for k in range(n_codebooks):
        c, a = kmeans(resid, codebook_size, iters, seed + k)
        if c.shape[0] < codebook_size:
            c = torch.cat([c, torch.zeros(codebook_size - c.shape[0], group_size, device=c.device)])
        idx[:, k] = a
        resid = resid - c[a]
        cbs.append(c)
    flat = torch.cat([torch.tensor([scale, float(codebook_size), float(group_size)], device=w.device)] +
                     [c.reshape(-1) for c in cbs]).float().cpu()
    groups = in_f // group_size
    return QTensor("aqlm", (out_f, in_f), packed=idx.reshape(out_f, groups, n_codebooks).to(torch.int32).cpu(),
                   scales=flat, group=group_size)


def aqlm_dequantize(t: QTensor) -> torch.Tensor:
    cb = t.scales.float()
    scale, size, gs = float(cb[0]), int(cb[1]), int(cb[2])
    idx = t.packed.long()
    out_f, groups, K = idx.shape
    books = cb[3:].reshape(K, size, gs)
    acc = torch.zeros(out_f, groups, gs)
    for k in range(K):
        acc += books[k][idx[:, :, k]]
    return (acc * scale).reshape(out_f, groups * gs)
