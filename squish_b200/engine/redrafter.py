"""Recurrent drafter (ReDrafter-style): a GRU over the draft tokens, started from the target's
feature, proposes a greedy chain with no cache of its own.

Per draft step, for the feature f (the final-norm hidden row that produced the pending token)
and the recurrent state s (s_0 = f):

    s <- GRU(embed(token), s)                         (PyTorch gate order r, z, n)
    o  = f + SiLU(P [s ; f] + p)                      (2H -> H)
    draft token = argmax lm_head(norm(o))             (the target's final norm and LM head)

Tensor names: ``gru.weight_ih`` / ``gru.weight_hh`` [3H, H], ``gru.bias_ih`` / ``gru.bias_hh``
[3H], ``proj.weight`` [H, 2H], ``proj.bias`` [H]. The reference drives an injected ReDrafter
head from its speculative generator (squish/speculative/speculative.py:1249-1330) and ships the
GRU cell as a kernel (squish_quant_rs/src/lib.rs:1977); this module is the head itself, torch on
the target's device (the CPU path runs the GRU cell through the C++ kernel,
``_C.cpu.gru_step``). Drafts are verified by the engine, so greedy output is unchanged.
"""
from __future__ import annotations

import math
from pathlib import Path

import torch

from ..models.config import ModelConfig
from ..models.reference import _rms

_NAMES = ("gru.weight_ih", "gru.weight_hh", "gru.bias_ih", "gru.bias_hh", "proj.weight", "proj.bias")


class ReDrafterHead:
    def __init__(self, cfg: ModelConfig, tensors: dict, embed, lm_head, final_norm, device="cpu"):
        dev = torch.device(device)
        missing = [n for n in _NAMES if n not in tensors]
        if missing:
            raise ValueError(f"ReDrafter head lacks {missing}")
        self.cfg, self.device = cfg, dev
        self.t = {k: tensors[k].to(dev, torch.float32).contiguous() for k in _NAMES}
        self.embed = embed.to(dev, torch.float32)
        self.lm_head = lm_head.to(dev, torch.float32)
        self.norm = final_norm.to(dev, torch.float32)

    @classmethod
    def random(cls, cfg: ModelConfig, embed, lm_head, final_norm, seed: int = 0, device="cpu") -> "ReDrafterHead":
        g = torch.Generator().manual_seed(seed)
        H = cfg.hidden_size
        r = 1 / math.sqrt(H)
        t = {"gru.weight_ih": torch.randn(3 * H, H, generator=g) * r, "gru.weight_hh": torch.randn(3 * H, H, generator=g) * r,
             "gru.bias_ih": torch.zeros(3 * H), "gru.bias_hh": torch.zeros(3 * H),
             "proj.weight": torch.randn(H, 2 * H, generator=g) * r / math.sqrt(2), "proj.bias": torch.zeros(H)}
        return cls(cfg, t, embed, lm_head, final_norm, device)

    @classmethod
    def load(cls, path: str | Path, cfg: ModelConfig, embed, lm_head, final_norm, device="cpu") -> "ReDrafterHead":
        p = Path(path)
        if p.is_dir():
            cands = sorted(p.glob("*.safetensors")) or sorted(p.glob("*.pt"))
            if not cands:
                raise FileNotFoundError(f"no ReDrafter head file in {p}")
            p = cands[0]
        if p.suffix == ".safetensors":
            from safetensors.torch import load_file

            sd = load_file(str(p))
        else:
            sd = torch.load(p, map_location="cpu", weights_only=True)
        return cls(cfg, sd, embed, lm_head, final_norm, device)

    def state_dict(self) -> dict:
        return {k: v.cpu() for k, v in self.t.items()}

    def gru(self, e: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
        """GRU cell over a batch: e, s [n, H] -> s' [n, H]."""
        t = self.t
        gx = e @ t["gru.weight_ih"].T + t["gru.bias_ih"]
        gh = s @ t["gru.weight_hh"].T + t["gru.bias_hh"]
        if self.device.type == "cpu":
            from .._ext import native

            return torch.stack([native().cpu.gru_step(gx[i], gh[i], s[i]) for i in range(s.shape[0])])
        H = s.shape[1]
        r = torch.sigmoid(gx[:, :H] + gh[:, :H])
        z = torch.sigmoid(gx[:, H:2 * H] + gh[:, H:2 * H])
        n = torch.tanh(gx[:, 2 * H:] + r * gh[:, 2 * H:])
        return (1 - z) * n + z * s

    def draft(self, feats: torch.Tensor, toks: list[int], k: int) -> list[list[int]]:
        """k greedy tokens per row from features [n, H] and pending tokens."""
        f = feats.to(self.device, torch.float32)
        s = f.clone()
        cur = torch.as_tensor(toks, device=self.device)
        out = [[] for _ in toks]
        for _ in range(k):
            s = self.gru(self.embed[cur], s)
            o = f + torch.nn.functional.silu(torch.cat([s, f], 1) @ self.t["proj.weight"].T + self.t["proj.bias"])
            cur = (_rms(o, self.norm, self.cfg.rms_eps) @ self.lm_head.T).argmax(-1)
            for i, tk in enumerate(cur.tolist()):
                out[i].append(int(tk))
        return out
