"""AQLM additive-codebook weight quantization (the npy-dir ``__aqlm_idx`` / ``__aqlm_cb`` pair).

Encoding follows the reference's iterative residual scheme (squish/quant/aqlm.py:284-456):
normalise the matrix by its RMS (``scale``), then for each of K codebooks fit k-means on the
residual groups of ``group_size`` input features, assign each group its nearest codeword
and subtract it. Decoding: W[i, g*gs:(g+1)*gs] = scale * sum_k CB_k[idx[i, g, k]].

k-means is quant/pq.py: k-means++ seeding, then Lloyd iterations in the CUDA kernels of
csrc/kmeans.cu when the weight is on the GPU (torch on the CPU).
Serialised codebook: float32 [scale, codebook_size, group_size, CB_0 ..., CB_{K-1} ...].
"""
from __future__ import annotations

import torch

from ..models.weights import QTensor


from .pq import kmeans  # noqa: E402  (GPU kernels for CUDA tensors, torch otherwise)


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
