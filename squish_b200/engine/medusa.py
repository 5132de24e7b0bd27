"""Medusa heads: extra decoding heads on the target model's final hidden state that guess the
tokens after the next one, verified as a draft tree in the next step.

Head i (0-based) reads the final-norm hidden state h of the position whose logits produced the
pending token and proposes the token i + 1 positions after it:

    r = h;  r = r + SiLU(r W_j^T + b_j)   for each residual block j   (H x H)
    logits_i = r U_i^T (+ c_i)                                         (vocab x H)

The residual-block form and the tensor names follow the published Medusa checkpoints
(``medusa_head.{i}.{j}.linear.weight|bias`` for the blocks, ``medusa_head.{i}.{n}.weight`` for
the vocabulary projection); a head with no residual block and a bias is the reference's plain
linear head (squish/speculative/speculative.py:1859-1909, ``MedusaHead``). The draft tree is
the reference's Cartesian product of the heads' top-k tokens (``MedusaTreeDraft``,
speculative.py:1911-1964), ordered here by summed rank so the likeliest paths come first and a
node cap keeps a prefix of them; verification is the engine's on-device tree verifier (greedy
and temperature sampling are lossless).

On a GPU the vocabulary projections are INT4 weights run by the W4A16 GEMM (the same codes as
the model's own layers), the residual blocks bf16; the heads run once per step over the rows
that produced each request's newest token.
"""
from __future__ import annotations

import functools
import itertools
from pathlib import Path

import numpy as np
import torch


class MedusaHeads:
    def __init__(self, blocks: list[list[tuple[torch.Tensor, torch.Tensor]]], out: list[torch.Tensor],
                 out_bias: list[torch.Tensor | None], device="cpu", quantize: bool | None = None):
        if not out or len(blocks) != len(out) or len(out_bias) != len(out):
            raise ValueError("one list of residual blocks, one projection and one bias entry per head")
        dev = torch.device(device)
        self.device = dev
        self.num_heads = len(out)
        self.vocab, self.hidden = out[0].shape
        cuda = dev.type == "cuda"
        dt = self.dtype = torch.bfloat16 if cuda else torch.float32
        self.blocks = [[(w.to(dev, dt).contiguous(), b.to(dev, dt)) for w, b in hb] for hb in blocks]
        self.out_bias = [None if c is None else c.to(dev, torch.float32) for c in out_bias]
        self.quantized = bool(cuda if quantize is None else quantize) and cuda
        if self.quantized:
            from .. import ops
            from .._ext import native

            self.out = []
            for u in out:
                p, s, z = native().cpu.quantize_int4_asym(u.float().cpu().contiguous(), 64)
                self.out.append(ops.prepare_int4_weight(p, s, z, u.shape[1], 64, dev))
        else:
            self.out = [u.to(dev, dt).contiguous() for u in out]

    # ------------------------------------------------------------------ construction
    @classmethod
    def random(cls, hidden: int, vocab: int, num_heads: int = 3, num_layers: int = 1, seed: int = 0,
               device="cpu", quantize: bool | None = None) -> "MedusaHeads":
        """Randomly initialised heads (tests and benchmarks; the residual blocks start near the
        identity as in Medusa training)."""
        g = torch.Generator().manual_seed(seed)
        blocks = [[(torch.randn(hidden, hidden, generator=g) * 0.02 / hidden ** 0.5, torch.zeros(hidden))
                   for _ in range(num_layers)] for _ in range(num_heads)]
        out = [torch.randn(vocab, hidden, generator=g) * (2.0 / hidden) ** 0.5 for _ in range(num_heads)]
        return cls(blocks, out, [None] * num_heads, device, quantize)

    @classmethod
    def from_state_dict(cls, sd: dict, device="cpu", quantize: bool | None = None) -> "MedusaHeads":
        heads = sorted({int(k.split(".")[1]) for k in sd if k.startswith("medusa_head.")})
        if not heads or heads != list(range(len(heads))):
            raise ValueError("no medusa_head.{i}.* tensors (or the head indices are not 0..n-1)")
        blocks, out, bias = [], [], []
        for i in heads:
            pre = f"medusa_head.{i}."
            n = 0
            hb = []
            while f"{pre}{n}.linear.weight" in sd:
                hb.append((sd[f"{pre}{n}.linear.weight"].float(), sd[f"{pre}{n}.linear.bias"].float()))
                n += 1
            if f"{pre}{n}.weight" not in sd:
                raise ValueError(f"head {i}: missing the vocabulary projection {pre}{n}.weight")
            blocks.append(hb)
            out.append(sd[f"{pre}{n}.weight"].float())
            bias.append(sd[f"{pre}{n}.bias"].float() if f"{pre}{n}.bias" in sd else None)
        return cls(blocks, out, bias, device, quantize)

    @classmethod
    def load(cls, path: str | Path, device="cpu", quantize: bool | None = None) -> "MedusaHeads":
        """Heads from a ``.safetensors`` file, a tensor-only torch file or an ``.npz``."""
        p = Path(path)
        if p.is_dir():
            cands = sorted(p.glob("medusa*.safetensors")) or sorted(p.glob("*.safetensors")) or \
                sorted(p.glob("medusa*.pt")) + sorted(p.glob("medusa*.bin"))
            if not cands:
                raise FileNotFoundError(f"no Medusa head file in {p}")
            p = cands[0]
        if p.suffix == ".safetensors":
            from safetensors.torch import load_file

            sd = load_file(str(p))
        elif p.suffix == ".npz":
            with np.load(p) as z:
                sd = {k: torch.from_numpy(z[k]) for k in z.files}
        else:
            sd = torch.load(p, map_location="cpu", weights_only=True)
        return cls.from_state_dict(sd, device, quantize)

    def state_dict(self) -> dict:
        """The published tensor names (heads kept in floating point only)."""
        if self.quantized:
            raise ValueError("INT4 vocabulary projections keep no floating-point copy")
        sd = {}
        for i in range(self.num_heads):
            for j, (w, b) in enumerate(self.blocks[i]):
                sd[f"medusa_head.{i}.{j}.linear.weight"] = w.float().cpu()
                sd[f"medusa_head.{i}.{j}.linear.bias"] = b.float().cpu()
            n = len(self.blocks[i])
            sd[f"medusa_head.{i}.{n}.weight"] = self.out[i].float().cpu()
            if self.out_bias[i] is not None:
                sd[f"medusa_head.{i}.{n}.bias"] = self.out_bias[i].cpu()
        return sd

    # ------------------------------------------------------------------ compute
    def logits(self, hidden: torch.Tensor) -> list[torch.Tensor]:
        """[n, H] final-norm hidden rows -> per head [n, vocab] float logits."""
        from .. import ops

        x = hidden.to(self.device, self.dtype)
        outs = []
        for i in range(self.num_heads):
            r = x
            for w, b in self.blocks[i]:
                r = r + torch.nn.functional.silu(r @ w.T + b)
            if self.quantized:
                lg = ops.w4a16_linear(r.to(torch.bfloat16).contiguous(), self.out[i]).float()
            else:
                lg = (r @ self.out[i].T).float()
            if self.out_bias[i] is not None:
                lg = lg + self.out_bias[i]
            outs.append(lg)
        return outs

    def topk(self, hidden: torch.Tensor, k: int) -> np.ndarray:
        """[n, H] -> [n, heads, k] int32 token ids, best first per head."""
        if hidden.shape[0] == 0:
            return np.zeros((0, self.num_heads, k), dtype=np.int32)
        ids = torch.stack([lg.topk(k, dim=-1).indices for lg in self.logits(hidden)], 1)
        return ids.to(torch.int32).cpu().numpy()


@functools.lru_cache(maxsize=16)
def rank_paths(num_heads: int, k: int, limit: int) -> list[tuple[int, ...]]:
    """Rank tuples of the Cartesian product (one rank per head), ordered by rank sum, then
    lexicographically; at most ``limit``."""
    paths = sorted(itertools.product(range(k), repeat=num_heads), key=lambda p: (sum(p), p))
    return paths[:limit]
