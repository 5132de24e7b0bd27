"""Vector quantization at convert time: k-means, product quantization (PQ) and asymmetric
distance computation (ADC).

The reference's Rayon versions are pq_kmeans_fit / pq_encode_batch / pq_adc_search
(squish_quant_rs/src/lib.rs:1836-1960) and the vector k-means used by VPTQ / AQLM
(2249-2383, 4858). CUDA tensors run the kernels of ``csrc/kmeans.cu`` (``_C.kmeans_fit``,
``_C.kmeans_assign``, ``_C.pq_adc``); CPU tensors run the same algorithm in torch, which is
also the oracle of the GPU tests. Vectors whose width is not 1/2/4/8/16/32/64 are zero-padded
for the kernels (padding changes no distance).

Seeding is k-means++ (D^2 sampling) from a seeded CPU generator, so a fit is reproducible.
"""
from __future__ import annotations

import torch

from .._ext import native

_WIDTHS = (1, 2, 4, 8, 16, 32, 64)


def _pad(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[1]
    w = next((v for v in _WIDTHS if v >= d), None)
    if w is None:
        raise ValueError(f"vector width {d} > 64 is not supported by the k-means kernels")
    return x if w == d else torch.nn.functional.pad(x, (0, w - d))


def _sqdist_min(x: torch.Tensor, c: torch.Tensor, chunk: int = 65536) -> tuple[torch.Tensor, torch.Tensor]:
    """(nearest index int64, squared distance) in torch; lowest index on ties."""
    idx = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    dist = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    for i in range(0, x.shape[0], chunk):
        d = ((x[i:i + chunk, None, :] - c[None, :, :]) ** 2).sum(-1) if c.shape[0] * x.shape[1] <= 4096 else \
            (x[i:i + chunk] * x[i:i + chunk]).sum(1, keepdim=True) - 2 * x[i:i + chunk] @ c.T + (c * c).sum(1)[None]
        v, j = d.min(1)
        idx[i:i + chunk], dist[i:i + chunk] = j, v.clamp_min(0)
    return idx, dist


def assign(x: torch.Tensor, c: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Nearest centroid of every row of ``x`` [n, d] among ``c`` [k, d]: (index int64, sq. distance)."""
    if x.is_cuda:
        a, d = native().kmeans_assign(_pad(x.float().contiguous()), _pad(c.float().contiguous()))
        return a.long(), d
    return _sqdist_min(x.float(), c.float())


def kmeans_pp_init(x: torch.Tensor, k: int, seed: int = 0, sample: int = 65536) -> torch.Tensor:
    """k-means++ seeds drawn from a seeded subsample of at most ``sample`` rows."""
    g = torch.Generator().manual_seed(seed)
    if x.shape[0] > sample:
        x = x[torch.randperm(x.shape[0], generator=g)[:sample].to(x.device)]
    n = x.shape[0]
    first = int(torch.randint(0, n, (1,), generator=g))
    cent = [x[first]]
    dmin = ((x - x[first]) ** 2).sum(1)
    for _ in range(1, k):
        w = dmin.double().cpu()
        j = int(torch.multinomial(w / w.sum(), 1, generator=g)) if float(w.sum()) > 0 else \
            int(torch.randint(0, n, (1,), generator=g))
        cent.append(x[j])
        dmin = torch.minimum(dmin, ((x - x[j]) ** 2).sum(1))
    return torch.stack(cent).clone()


def kmeans(x: torch.Tensor, k: int, iters: int = 20, seed: int = 42, init="kmeans++"
           ) -> tuple[torch.Tensor, torch.Tensor]:
    """Lloyd k-means of the rows of ``x``: (centroids [k, d] float32, assignment int64 [n]).
    ``init``: "kmeans++", "random" (k distinct rows) or a [k, d] tensor of starting centroids."""
    x = x.float().contiguous()
    n, d = x.shape
    k = min(k, n)
    if isinstance(init, torch.Tensor):
        c = init.float().to(x.device).clone()
        k = c.shape[0]
    elif init == "kmeans++":
        c = kmeans_pp_init(x, k, seed)
    else:
        g = torch.Generator().manual_seed(seed)
        c = x[torch.randperm(n, generator=g)[:k].to(x.device)].clone()
    if x.is_cuda:
        xp, cp = _pad(x), _pad(c).contiguous()
        a, _ = native().kmeans_fit(xp, cp, iters)
        return cp[:, :d].contiguous(), a.long()
    a, _ = _sqdist_min(x, c)
    for _ in range(iters):
        sums = torch.zeros_like(c).index_add_(0, a, x)
        cnt = torch.bincount(a, minlength=k).float()[:, None]
        c = torch.where(cnt > 0, sums / cnt.clamp_min(1), c)
        new, _ = _sqdist_min(x, c)
        if torch.equal(new, a):
            break
        a = new
    return c, a


def pq_fit(x: torch.Tensor, m: int, k: int = 256, iters: int = 20, seed: int = 0) -> torch.Tensor:
    """Codebooks [m, k, d/m] of a product quantizer over the rows of ``x`` [n, d]."""
    n, d = x.shape
    if d % m:
        raise ValueError(f"dimension {d} does not split into {m} subspaces")
    ds = d // m
    return torch.stack([kmeans(x[:, j * ds:(j + 1) * ds], k, iters, seed + j)[0] for j in range(m)])


def pq_encode(x: torch.Tensor, books: torch.Tensor) -> torch.Tensor:
    """uint8 codes [n, m] (k <= 256) of the rows of ``x`` under codebooks [m, k, d/m]."""
    m, k, ds = books.shape
    if k > 256:
        raise ValueError("PQ codes are bytes: at most 256 centroids per subspace")
    return torch.stack([assign(x[:, j * ds:(j + 1) * ds], books[j])[0] for j in range(m)], 1).to(torch.uint8)


def pq_lut(query: torch.Tensor, books: torch.Tensor) -> torch.Tensor:
    """[m, k] squared distances from the query's m subvectors to every centroid."""
    m, k, ds = books.shape
    q = query.float().reshape(m, 1, ds).to(books.device)
    return ((books.float() - q) ** 2).sum(-1)


def pq_adc_search(codes: torch.Tensor, lut: torch.Tensor) -> torch.Tensor:
    """Approximate squared distance of every encoded vector: sum_j lut[j, codes[:, j]]."""
    if codes.is_cuda:
        return native().pq_adc(codes.contiguous(), lut.float().contiguous())
    return lut.float().gather(1, codes.long().T).sum(0)


def pq_search(query: torch.Tensor, books: torch.Tensor, codes: torch.Tensor, topk: int = 10):
    """(distances, indices) of the ``topk`` nearest encoded vectors to ``query``."""
    d = pq_adc_search(codes, pq_lut(query, books).to(codes.device))
    v, i = torch.topk(d, min(topk, d.numel()), largest=False)
    return v, i
