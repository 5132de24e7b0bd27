"""GPTQ (Frantar et al., arXiv:2210.17323): INT4 rounding that compensates each column's error
on the columns not yet quantized, weighted by the calibration inputs' second moments.

The reference lists a ``gptq_column_solve_f32`` kernel among its convert-time research kernels
(squish_quant_rs/src/lib.rs:2819). Here: H = 2 X^T X / n per projection input (collected on the
fp32 model through ``ReferenceModel.tap``, on the GPU when present), dampened by 1% of its mean
diagonal; the upper Cholesky factor of H^-1 drives the column-by-column update in blocks of 128
columns, the published algorithm. Groups take their INT4-asymmetric grid (scale = (max - min) /
15, offset = min) from the error-updated weights when the group starts, so the result is an
ordinary ``q4a`` tensor that the tcgen05 GEMM runs unchanged.
"""
from __future__ import annotations

import torch

from ..models.weights import QTensor

# projection -> the tap whose activations are its input
_TAP_OF = {"self_attn.q_proj": "input_layernorm", "self_attn.k_proj": "input_layernorm",
           "self_attn.v_proj": "input_layernorm", "self_attn.o_proj": "self_attn.o_proj",
           "mlp.gate_proj": "post_attention_layernorm", "mlp.up_proj": "post_attention_layernorm",
           "mlp.down_proj": "mlp.down_proj"}


class HessianStats:
    def __init__(self):
        self.h: dict[str, torch.Tensor] = {}
        self.n: dict[str, int] = {}

    def __call__(self, name: str, x: torch.Tensor) -> None:
        x2 = x.reshape(-1, x.shape[-1]).float()
        h = self.h.get(name)
        if h is None:
            h = self.h[name] = torch.zeros(x2.shape[1], x2.shape[1], dtype=torch.float32, device=x2.device)
            self.n[name] = 0
        h.addmm_(x2.T, x2, alpha=2.0)
        self.n[name] += x2.shape[0]

    def hessian(self, name: str) -> torch.Tensor:
        return self.h[name] / max(1, self.n[name])


def collect_hessians(ck, tokens: list[list[int]], device=None) -> dict[str, torch.Tensor]:
    """weight name -> H for every dense-MLP / attention projection of the checkpoint."""
    from ..models.reference import ReferenceModel

    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    model = ReferenceModel(ck, device=dev)
    st = HessianStats()
    model.tap = st
    for seq in tokens:
        if seq:
            model.forward(seq, model.new_cache(), 0)
    out = {}
    for i in range(ck.config.num_layers):
        p = f"model.layers.{i}."
        for proj, tap in _TAP_OF.items():
            if p + tap in st.h and p + proj + ".weight" in ck.tensors:
                out[p + proj + ".weight"] = st.hessian(p + tap)
    return out


def _grid(w: torch.Tensor, qmax: float) -> tuple[torch.Tensor, torch.Tensor]:
    lo, hi = w.amin(1), w.amax(1)
    scale = torch.where(hi > lo, (hi - lo) / qmax, torch.ones_like(lo))
    return scale, lo


def gptq_quantize(w: torch.Tensor, H: torch.Tensor, group: int = 64, bits: int = 4, block: int = 128,
                  damp: float = 0.01) -> QTensor:
    """INT4-asymmetric (``bits`` = 4) GPTQ of ``w`` [N, K] with input second moments ``H`` [K, K]."""
    if bits != 4:
        raise ValueError("GPTQ here produces INT4-asymmetric tensors (bits = 4)")
    W = w.detach().float().clone()
    n, k = W.shape
    if k % group:
        raise ValueError(f"width {k} is not a multiple of the group size {group}")
    H = H.to(W.device).float().clone()
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    H += damp * torch.mean(torch.diag(H)) * torch.eye(k, device=W.device)
    Hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
    qmax = float(2 ** bits - 1)
    codes = torch.zeros(n, k, dtype=torch.uint8, device=W.device)
    scales = torch.zeros(n, k // group, device=W.device)
    offsets = torch.zeros(n, k // group, device=W.device)
    for i1 in range(0, k, block):
        i2 = min(i1 + block, k)
        W1 = W[:, i1:i2].clone()
        E1 = torch.zeros_like(W1)
        Hi = Hinv[i1:i2, i1:i2]
        for i in range(i2 - i1):
            col = i1 + i
            if col % group == 0:  # the group's grid from the weights as updated so far
                g = col // group
                span = W1[:, i:i + group] if i + group <= i2 - i1 else torch.cat(
                    [W1[:, i:], W[:, i2:col + group]], 1)
                scales[:, g], offsets[:, g] = _grid(span, qmax)
            g = col // group
            wcol = W1[:, i]
            q = torch.clamp(torch.round((wcol - offsets[:, g]) / scales[:, g]), 0, qmax)
            codes[:, col] = q.to(torch.uint8)
            deq = offsets[:, g] + q * scales[:, g]
            err = (wcol - deq) / Hi[i, i]
            W1[:, i:] -= err[:, None] * Hi[i, i:][None, :]
            E1[:, i] = err
        W[:, i2:] -= E1 @ Hinv[i1:i2, i2:]
    c = codes.to(torch.int64)
    packed = (c[:, 0::2] | (c[:, 1::2] << 4)).to(torch.uint8).cpu()
    return QTensor("q4a", (n, k), packed=packed, scales=scales.cpu(), offsets=offsets.cpu(), group=group)
