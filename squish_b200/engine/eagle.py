"""EAGLE draft head: a one-layer draft model that runs on the target's features.

EAGLE (Li et al. 2024) predicts the target's next feature rather than the next token directly.
At each draft step the head reads the pair (feature f_t, embedding of token t+1):

    z = fc([f_t ; e_{t+1}])                          (2H -> H, with bias)
    h = one Llama decoder layer over the head's own sequence of z (causal self-attention with
        RoPE over the positions the head has seen, then the SwiGLU MLP)
    draft token = argmax lm_head(norm(h))             (the target's own LM head and final norm)

and feeds (h, draft token) back for the next step. The head's attention history holds one z per
target step: the engine hands the proposer, after every step, the final-norm hidden row that
produced each request's newest token (the feature) together with that token; draft steps extend
the history temporarily and are dropped again, so only features the target computed stay. The
tensor names follow the published EAGLE checkpoints (``fc.weight``, ``fc.bias``,
``layers.0.self_attn.{q,k,v,o}_proj.weight``, ``layers.0.mlp.{gate,up,down}_proj.weight``,
``layers.0.post_attention_layernorm.weight``; the first layer's input norm is optional). The
reference's ``EagleDraftHead`` (squish/speculative/speculative.py:416-580) wraps an MLX model;
here the head is plain torch on the target's device. Drafts are verified by the engine's tree
verifier, so greedy output is unchanged whatever the head proposes.
"""
from __future__ import annotations

import math
from pathlib import Path

import torch

from ..models.config import ModelConfig
from ..models.reference import _rms, _rope, rope_table


class EagleHead:
    def __init__(self, cfg: ModelConfig, tensors: dict, embed: torch.Tensor, lm_head: torch.Tensor,
                 final_norm: torch.Tensor, device="cpu"):
        dev = torch.device(device)
        self.cfg, self.device = cfg, dev
        dt = torch.float32
        self.t = {k: v.to(dev, dt).contiguous() for k, v in tensors.items()}
        need = ["fc.weight"] + [f"layers.0.self_attn.{n}_proj.weight" for n in "qkvo"] + \
               [f"layers.0.mlp.{n}_proj.weight" for n in ("gate", "up", "down")] + \
               ["layers.0.post_attention_layernorm.weight"]
        missing = [n for n in need if n not in self.t]
        if missing:
            raise ValueError(f"EAGLE head lacks {missing}")
        self.embed = embed.to(dev, dt)
        self.lm_head = lm_head.to(dev, dt)
        self.norm = final_norm.to(dev, dt)
        self.rope = rope_table(cfg, 1 << 14).to(dev)

    # ------------------------------------------------------------------ construction
    @classmethod
    def random(cls, cfg: ModelConfig, embed, lm_head, final_norm, seed: int = 0, device="cpu") -> "EagleHead":
        g = torch.Generator().manual_seed(seed)
        H, d, F = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size or 4 * cfg.hidden_size

        def w(*shape):
            return torch.randn(*shape, generator=g) / math.sqrt(shape[-1])

        t = {"fc.weight": w(H, 2 * H), "fc.bias": torch.zeros(H),
             "layers.0.self_attn.q_proj.weight": w(cfg.num_heads * d, H),
             "layers.0.self_attn.k_proj.weight": w(cfg.num_kv_heads * d, H),
             "layers.0.self_attn.v_proj.weight": w(cfg.num_kv_heads * d, H),
             "layers.0.self_attn.o_proj.weight": w(H, cfg.num_heads * d),
             "layers.0.mlp.gate_proj.weight": w(F, H), "layers.0.mlp.up_proj.weight": w(F, H),
             "layers.0.mlp.down_proj.weight": w(H, F),
             "layers.0.post_attention_layernorm.weight": torch.ones(H)}
        return cls(cfg, t, embed, lm_head, final_norm, device)

    @classmethod
    def load(cls, path: str | Path, cfg: ModelConfig, embed, lm_head, final_norm, device="cpu") -> "EagleHead":
        """A head from a ``.safetensors`` file (or a directory holding one) or a tensor-only torch
        file with the published names."""
        p = Path(path)
        if p.is_dir():
            cands = sorted(p.glob("*.safetensors")) or sorted(p.glob("*.bin")) + sorted(p.glob("*.pt"))
            if not cands:
                raise FileNotFoundError(f"no EAGLE head file in {p}")
            p = cands[0]
        if p.suffix == ".safetensors":
            from safetensors.torch import load_file

            sd = load_file(str(p))
        else:
            sd = torch.load(p, map_location="cpu", weights_only=True)
        sd = {k[len("model."):] if k.startswith("model.") else k: v for k, v in sd.items()}
        return cls(cfg, sd, embed, lm_head, final_norm, device)

    def state_dict(self) -> dict:
        return {k: v.cpu() for k, v in self.t.items()}

    # ------------------------------------------------------------------ compute
    def new_state(self) -> dict:
        """Per-sequence attention history of the head (post-RoPE keys and values)."""
        cfg = self.cfg
        e = torch.empty(0, cfg.num_kv_heads, cfg.head_dim, device=self.device)
        return {"k": e, "v": e.clone()}

    def step(self, states: list, feats: torch.Tensor, toks: list[int], commit: bool):
        """One draft position for a batch of sequences: the dense parts run batched, attention
        per sequence over its own history. Returns (h [n, H], logits [n, V]); ``commit`` keeps
        each new key / value in its sequence's history."""
        cfg, t = self.cfg, self.t
        hq, hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        n = len(states)
        x = torch.cat([feats.to(self.device, torch.float32).reshape(n, -1),
                       self.embed[torch.as_tensor(toks, device=self.device)]], dim=1)
        z = x @ t["fc.weight"].T
        if "fc.bias" in t:
            z = z + t["fc.bias"]
        a_in = _rms(z, t["layers.0.input_layernorm.weight"], cfg.rms_eps) \
            if "layers.0.input_layernorm.weight" in t else z
        q = (a_in @ t["layers.0.self_attn.q_proj.weight"].T).view(n, hq, d)
        k = (a_in @ t["layers.0.self_attn.k_proj.weight"].T).view(n, hkv, d)
        v = (a_in @ t["layers.0.self_attn.v_proj.weight"].T).view(n, hkv, d)
        rep = hq // hkv
        outs = []
        for i, st in enumerate(states):
            pos = st["k"].shape[0]
            cs = self.rope[pos:pos + 1]
            qi, ki = _rope(q[i:i + 1], cs), _rope(k[i:i + 1], cs)
            K, V = torch.cat([st["k"], ki]), torch.cat([st["v"], v[i:i + 1]])
            sc = torch.einsum("hd,thd->ht", qi[0], K.repeat_interleave(rep, dim=1)) / math.sqrt(d)
            outs.append(torch.einsum("ht,thd->hd", torch.softmax(sc, -1), V.repeat_interleave(rep, dim=1)).reshape(-1))
            if commit:
                st["k"], st["v"] = K, V
        h = z + torch.stack(outs) @ t["layers.0.self_attn.o_proj.weight"].T
        m_in = _rms(h, t["layers.0.post_attention_layernorm.weight"], cfg.rms_eps)
        g = m_in @ t["layers.0.mlp.gate_proj.weight"].T
        u = m_in @ t["layers.0.mlp.up_proj.weight"].T
        h = h + (torch.nn.functional.silu(g) * u) @ t["layers.0.mlp.down_proj.weight"].T
        return h, _rms(h, self.norm, cfg.rms_eps) @ self.lm_head.T

    def draft(self, states: list, h: torch.Tensor, logits: torch.Tensor, k: int) -> list[list[int]]:
        """k greedy draft tokens per sequence from a committed position's (h, logits); the draft
        positions extend the histories only while drafting."""
        saved = [dict(st) for st in states]
        out = [[] for _ in states]
        for j in range(k):
            toks = logits.argmax(-1).tolist()
            for i, tk in enumerate(toks):
                out[i].append(int(tk))
            if j + 1 < k:
                h, logits = self.step(states, h, toks, commit=True)
        for st, sv in zip(states, saved):
            st.update(sv)
        return out
