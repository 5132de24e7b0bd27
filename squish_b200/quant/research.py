"""Convert-time quantization research methods and predictor helpers, on the C++ kernels of
csrc/quant_research.cpp (``native().cpu``).

  * any4 (learned 4-bit numerics): group absmax scaling as NF4, but the 16 levels are learned
    per tensor by Lloyd iterations over the normalised weights; the result is an NF4-format
    tensor with its own level table, which the W4A16 GEMM reads in place of the NormalFloat
    levels (reference kernel: squish_quant_rs/src/lib.rs:4470 ``any4_lloyd_step_f32``).
  * QuaRot: randomized block-Hadamard rotation of the weight's input dimension (the same
    rotation as SQINT2, undone online on the activations) and group quantization
    (lib.rs:2870-2932).
  * AdaRound: learned up / down rounding of INT4 asymmetric codes against a layer's
    calibration inputs (Nagel et al. 2020) -- rectified-sigmoid rounding variables, the
    annealed regulariser, output reconstruction loss; the weight-space gradient step alone is
    ``adaround_step`` (lib.rs:3421).
  * FLUTE lookup-table codes, QMoE block codebooks, BitDistiller and GGUF-style group codes
    (lib.rs:3764-3827, 4696, 4969, 5137).
  * GRU step, batched cosine similarity, logistic / SGD steps (lib.rs:1977-2013, 2765-2786):
    the numeric pieces of recurrent drafters and online acceptance predictors.
"""
from __future__ import annotations

import torch

from .._ext import native
from ..models.weights import QTensor


def C():
    return native().cpu


# ----------------------------------------------------------------------------- any4
def any4_lloyd(values: torch.Tensor, init: torch.Tensor, n_iter: int = 100, seed: int = 0) -> torch.Tensor:
    """1-D Lloyd k-means of ``values`` started at ``init`` (centroids returned ascending)."""
    return C().any4_lloyd(values.float().cpu(), init.float().cpu(), int(n_iter), int(seed))


def quantize_any4(w: torch.Tensor, group: int, n_iter: int = 30, seed: int = 0) -> QTensor:
    """any4 weight: NF4 layout (two codes per byte, low nibble first; absmax per group) with the
    tensor's learned 16-level table in ``extra['levels']``."""
    wf = w.detach().float().cpu().contiguous()
    codes, scales, levels = C().any4_quantize(wf, int(group), int(n_iter), int(seed))
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    return QTensor("nf4", tuple(wf.shape), packed=packed, scales=scales, group=int(group),
                   extra={"levels": levels})


# ----------------------------------------------------------------------------- QuaRot
def quarot_quantize(w: torch.Tensor, group: int, bits: int = 4, block: int = 128, seed: int = 0) -> QTensor:
    """QuaRot INT4 / INT2 weight: W R^T with R = blockdiag(H_b / sqrt(b)) diag(signs) over the
    input dimension (outliers spread over each block), then per-row group asymmetric codes.
    The runner rotates activations with the same R before the GEMM (csrc/hadamard.cu), so
    (W R^T)(R x) = W x. Returns a q4a / q2 tensor carrying the rotation."""
    from .codecs import quantize
    from .sqint2 import rotate, rotation_signs

    if bits not in (2, 4):
        raise ValueError("QuaRot weights here are INT4 or INT2")
    wf = w.detach().float().cpu()
    K = wf.shape[1]
    if K % block or block & (block - 1):
        raise ValueError("the rotation block must be a power of two dividing the input dimension")
    signs = rotation_signs(K, seed)
    t = quantize(rotate(wf, signs, block), "q4a" if bits == 4 else "q2", group)  # rows of W R^T
    t.extra = {"rot_signs": signs, "rot_block": block, "seed": seed}
    return t


def quarot_group_quant(w: torch.Tensor, group: int, q_max: float, symmetric: bool):
    """(codes int32 [R, C], scales [G], zeros [G]): one grid per column group over all rows."""
    return C().quarot_group_quant(w.float().cpu(), int(group), float(q_max), bool(symmetric))


def quarot_group_dequant(codes, scales, zeros, group: int, symmetric: bool) -> torch.Tensor:
    return C().quarot_group_dequant(codes, scales, zeros, int(group), bool(symmetric))


# ----------------------------------------------------------------------------- AdaRound
def adaround_step(v, w, w_floor, scale, lr: float, beta: float, lambda_reg: float, zeta: float = 1.1,
                  gamma: float = -0.1) -> torch.Tensor:
    return C().adaround_step(v, w, w_floor, scale, float(lr), float(beta), float(lambda_reg), float(zeta),
                             float(gamma))


def _rect_sigmoid(v: torch.Tensor, zeta: float = 1.1, gamma: float = -0.1) -> torch.Tensor:
    return torch.clamp(torch.sigmoid(v) * (zeta - gamma) + gamma, 0.0, 1.0)


def adaround_q4a(w: torch.Tensor, x: torch.Tensor, group: int, iters: int = 500, lr: float = 1e-2,
                 lambda_reg: float = 0.01, beta_range: tuple[float, float] = (20.0, 2.0),
                 warmup: float = 0.2) -> QTensor:
    """INT4 asymmetric weight whose per-element rounding (floor or ceil) is learned so that the
    layer's outputs on calibration inputs ``x`` [n, K] match the fp32 layer: minimise
    ||x W^T - x W~^T||^2 / n + lambda sum(1 - |2 h(V) - 1|^beta) over V, with the annealed beta
    (no regulariser during the warm-up fraction), then round by h(V) >= 0.5. The (scale, zero)
    grid is the plain min / max grid of each group."""
    from ..models.weights import QTensor as QT

    wf = w.detach().float()
    xf = x.detach().float().to(wf.device)
    N, K = wf.shape
    if K % group:
        raise ValueError("group must divide the input dimension")
    G = K // group
    wg = wf.view(N, G, group)
    mn, mx = wg.amin(-1, keepdim=True), wg.amax(-1, keepdim=True)
    scale = torch.clamp((mx - mn) / 15.0, min=1e-8)
    zero = torch.round(-mn / scale).clamp(0, 15)
    base = torch.floor(wg / scale)
    rest = wg / scale - base
    # start at round-to-nearest: h(V0) = rest
    r0 = rest.clamp(0.01, 0.99)
    v = torch.log((r0 - (-0.1)) / (1.1 - r0)).detach().requires_grad_(True)
    opt = torch.optim.Adam([v], lr=lr)
    y_ref = xf @ wf.T
    lo, hi = -zero, 15 - zero  # code range around the grid's zero
    for it in range(iters):
        h = _rect_sigmoid(v)
        q = torch.clamp(base + h, lo, hi)
        w_soft = (q * scale).view(N, K)
        rec = ((xf @ w_soft.T - y_ref) ** 2).mean()
        frac = it / max(iters - 1, 1)
        if frac < warmup:
            loss = rec
        else:
            t = (frac - warmup) / max(1 - warmup, 1e-9)
            beta = beta_range[0] + (beta_range[1] - beta_range[0]) * t
            loss = rec + lambda_reg * (1 - (2 * h - 1).abs().pow(beta)).sum() / wf.numel()
        opt.zero_grad()
        loss.backward()
        opt.step()
    with torch.no_grad():
        up = (_rect_sigmoid(v) >= 0.5).float()
        codes = torch.clamp(base + up + zero, 0, 15).to(torch.uint8).view(N, K).cpu()
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    # q4a stores offsets as the dequantisation bias: w = code * scale + offset
    return QT("q4a", (N, K), packed=packed, scales=scale.view(N, G).cpu().contiguous(),
              offsets=(-zero * scale).view(N, G).cpu().contiguous(), group=group)


# ----------------------------------------------------------------------------- other codecs
def flute_lut_encode(w, codebook, group: int) -> torch.Tensor:
    return C().flute_lut_encode(w.float().cpu(), codebook.float().cpu(), int(group))


def flute_lut_decode(codes, codebook, group: int) -> torch.Tensor:
    return C().flute_lut_decode(codes, codebook.float().cpu(), int(group))


def qmoe_compress(blocks, k: int, n_iter: int = 20):
    """(codebook [k, block], assignments [N]) of an expert's weight blocks."""
    return C().qmoe_compress(blocks.float().cpu(), int(k), int(n_iter))


def bit_distiller_quant(w, bits: int, group: int):
    return C().bit_distiller_quant(w.float().cpu(), int(bits), int(group))


def gguf_mixed_quant(w, bits: int, group: int):
    return C().gguf_mixed_quant(w.float().cpu(), int(bits), int(group))


# ----------------------------------------------------------------------------- predictors
def gru_step(gates_x, gates_h, h) -> torch.Tensor:
    return C().gru_step(gates_x, gates_h, h)


def batched_cosine_similarity(a, b) -> torch.Tensor:
    return C().batched_cosine_similarity(a, b)


class OnlineLogistic:
    """Online logistic regression (one SGD step per observation) on the C++ steps: used as an
    acceptance predictor (features of a request's recent drafting -> probability that the next
    draft gets at least one token accepted)."""

    def __init__(self, n_features: int, lr: float = 0.05):
        self.w = torch.zeros(n_features)
        self.lr = lr

    def predict(self, x) -> float:
        return C().logistic_step(self.w, torch.as_tensor(x, dtype=torch.float32), 0.0)[0]

    def update(self, x, y: float) -> float:
        x = torch.as_tensor(x, dtype=torch.float32)
        yh, err = C().logistic_step(self.w, x, float(y))
        self.w = C().sgd_weight_update(self.w, x, err, self.lr)
        return yh



# ----------------------------------------------------------------------------- MiLo
def milo_int3(w: torch.Tensor, group: int, rank: int) -> QTensor:
    """INT3 weight with a MiLo-style low-rank compensator: the rank-``rank`` truncated SVD of
    the INT3 quantization residual, W ~ deq(Q) + A B (npy-dir ``__lra`` / ``__lrb``; the runner
    adds (x B^T) A^T after the INT3 GEMM)."""
    from .codecs import quantize

    wf = w.detach().float().cpu()
    t = quantize(wf, "q3", group)
    U, S, Vh = torch.linalg.svd(wf - t.dequantize().float(), full_matrices=False)
    t.extra = {"lra": (U[:, :rank] * S[:rank]).contiguous(), "lrb": Vh[:rank].contiguous()}
    return t


# ----------------------------------------------------------------------------- randomized SVD
def randomized_svd(a: torch.Tensor, rank: int, oversample: int = 8, n_iter: int = 2, seed: int = 0):
    """Rank-``rank`` truncated SVD by random projection (Halko, Martinsson and Tropp 2011):
    Y = A G (G Gaussian, rank + oversample columns), ``n_iter`` power iterations with QR
    re-orthonormalisation, Q = qr(Y), then the exact SVD of the small Q^T A. Returns (U, S, Vh)
    with U [m, rank], S [rank], Vh [rank, n]; runs on the tensor's device."""
    af = a.float()
    m, n = af.shape
    k = min(rank + oversample, m, n)
    g = torch.Generator(device="cpu").manual_seed(seed)
    omega = torch.randn(n, k, generator=g).to(af.device)
    q, _ = torch.linalg.qr(af @ omega)
    for _ in range(n_iter):
        q, _ = torch.linalg.qr(af.T @ q)
        q, _ = torch.linalg.qr(af @ q)
    ub, s, vh = torch.linalg.svd(q.T @ af, full_matrices=False)
    return (q @ ub)[:, :rank], s[:rank], vh[:rank]

