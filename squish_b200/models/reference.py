"""Pure-PyTorch fp32 decoder: the end-to-end oracle for the CUDA model.

It runs the same architecture with the dequantized weights (offset + q * scale in
fp32) and stores K/V through the same quantize -> dequantize codec as the device's
paged cache (the C++ CPU restatement of csrc/kv_write.cu), so CUDA logits can be
compared against it step by step. With ``bf16_storage`` every tensor the device keeps in
bf16 between kernels (normalised rows, q/k/v, attention output, SwiGLU activation,
residual stream, logits) is rounded to bf16 at that point while all arithmetic stays fp32:
the same op as the device, so code flips of the quantized KV cache that would come only from
fp32-vs-bf16 inputs to the codec do not mask kernel errors. It has no batching and no paging: one sequence,
dense per-layer caches. The reference framework has no model code of its own (the
forward pass lives in mlx_lm / HF transformers, squish/backend.py:222-390).
"""
from __future__ import annotations

import math

import torch

from .._ext import native
from ..ops.kernels import KV_FORMATS
from .config import ModelConfig, QuantConfig
from .weights import Checkpoint


def rope_table(cfg: ModelConfig, max_pos: int | None = None) -> torch.Tensor:
    """[max_pos, head_dim] fp32 table: cos (D/2) | sin (D/2), computed in float64."""
    d = cfg.head_dim
    n = max_pos or cfg.max_position
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    sc = cfg.rope_scaling or {}
    if sc.get("rope_type", sc.get("type")) == "llama3":
        # Llama-3 frequency smoothing (wavelength-dependent scaling)
        factor = sc.get("factor", 8.0)
        lo, hi = sc.get("low_freq_factor", 1.0), sc.get("high_freq_factor", 4.0)
        old = sc.get("original_max_position_embeddings", 8192)
        wl = 2 * math.pi / inv
        smooth = (old / wl - lo) / (hi - lo)
        scaled = torch.where(wl > old / lo, inv / factor, inv)
        mid = (wl <= old / lo) & (wl >= old / hi)
        inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
    t = torch.arange(n, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], dim=1).float()


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1]
    c, s = cs[:, None, : d // 2], cs[:, None, d // 2:]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


class ReferenceModel:
    """``device`` places the fp32 weights (CPU by default; a GPU runs calibration forwards).
    ``tap(name, x)``, when set, sees the input of every projection group, x of shape [T, width]:
    ``model.layers.{i}.input_layernorm`` (q/k/v), ``...post_attention_layernorm`` (gate/up, or
    the router and experts of a MoE layer), ``...self_attn.o_proj`` and ``...mlp.down_proj``
    (dense MLP layers)."""

    tap = None
    # optional attention restriction: kv_visible(qpos [t, 1], kpos [1, n]) -> bool [t, n]
    # (e.g. the serving engine's sink + recent-window eviction); causality is always applied
    kv_visible = None
    # optional KV override: kv_source(layer, start_pos, t) -> (K, V) [t, Hkv, D] fp32 to append
    # instead of this model's own codec output (e.g. the device's cache pages, read back), or None
    kv_source = None

    def __init__(self, ck: Checkpoint, device: str | torch.device = "cpu", bf16_storage: bool = False):
        self.bf16_storage = bf16_storage
        self.cfg: ModelConfig = ck.config
        self.q: QuantConfig = ck.quant
        cfg = self.cfg
        self.device = torch.device(device)
        self.w = {k: v.dequantize().float().to(self.device) for k, v in ck.tensors.items()}
        self.cos_sin = rope_table(cfg, min(cfg.max_position, 8192)).to(self.device)
        self.fk, self.fv = KV_FORMATS[self.q.kv_dtype]
        self.had = None
        if getattr(self.q, "kv_hadamard", False):
            from ..ops.kernels import kv_hadamard_signs, sylvester

            sk, sv = kv_hadamard_signs(cfg.head_dim)
            self.had = (sk.to(self.device), sv.to(self.device), sylvester(cfg.head_dim).float().to(self.device))

    def _kv_roundtrip(self, x: torch.Tensor, fmt: int) -> torch.Tensor:
        """[T, Hkv, D] -> through the KV page codec and back."""
        if fmt == 0:
            return x.to(torch.bfloat16).float()
        t, h, d = x.shape
        codes, scales = native().cpu.kv_quantize(x.reshape(t * h, d).cpu().contiguous(), fmt, self.q.kv_group)
        return native().cpu.kv_dequantize(codes, scales, fmt, self.q.kv_group, d).reshape(t, h, d).to(x.device)

    def rotate_kv(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """Hadamard-rotated KV: q, k -> H (s_k * x), v -> s_v * (H v) (identity when off)."""
        if self.had is None:
            return q, k, v
        sk, sv, H = self.had
        return (q * sk) @ H, (k * sk) @ H, (v @ H) * sv

    def unrotate_out(self, a: torch.Tensor) -> torch.Tensor:
        """Attention output over rotated values [.., D] -> H (s_v * a)."""
        if self.had is None:
            return a
        sk, sv, H = self.had
        return (a * sv) @ H

    def _st(self, x: torch.Tensor) -> torch.Tensor:
        """A tensor the device stores in bf16 (identity in the plain fp32 mode)."""
        return x.to(torch.bfloat16).float() if self.bf16_storage else x

    def new_cache(self):
        z = lambda: torch.zeros(0, self.cfg.num_kv_heads, self.cfg.head_dim, device=self.device)  # noqa: E731
        return [{"k": z(), "v": z()} for _ in range(self.cfg.num_layers)]

    # tensor-parallel hooks (set by the CPU tensor-parallel runner): row-parallel matmul
    # with an all-reduce, and the vocab-parallel LM head with a gather
    rp_hook = None
    head_hook = None
    reduce_hook = None  # expert parallelism: all-reduce of the local experts' partial output
    moe_hook = None     # expert parallelism with an all-to-all: callable(prefix, x) -> MoE(x)

    def _rp(self, x: torch.Tensor, wt: torch.Tensor) -> torch.Tensor:
        return x @ wt.T if self.rp_hook is None else self.rp_hook(x, wt)

    def _head(self, x: torch.Tensor, wt: torch.Tensor) -> torch.Tensor:
        return x @ wt.T if self.head_hook is None else self.head_hook(x, wt)

    def _mlp(self, p: str, x: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        if not cfg.is_moe:
            g = x @ w[p + "mlp.gate_proj.weight"].T
            u = x @ w[p + "mlp.up_proj.weight"].T
            act = self._st(torch.nn.functional.silu(g) * u)
            if self.tap is not None:
                self.tap(p + "mlp.down_proj", act)
            return self._rp(act, w[p + "mlp.down_proj.weight"])
        if self.moe_hook is not None:
            return self.moe_hook(p, x)
        logits = x @ w[p + "mlp.gate.weight"].T
        probs = torch.softmax(logits, dim=-1)
        topv, topi = probs.topk(cfg.num_experts_per_tok, dim=-1)
        if cfg.norm_topk_prob:
            topv = topv / topv.sum(-1, keepdim=True)
        out = torch.zeros_like(x)
        e0 = cfg.expert_offset
        e1 = e0 + (cfg.num_local_experts or cfg.num_experts)
        for t in range(x.shape[0]):
            for j in range(topi.shape[1]):
                e = int(topi[t, j])
                if not e0 <= e < e1:
                    continue
                out[t] += topv[t, j] * self.expert(p, e, x[t])
        return out if self.reduce_hook is None else self.reduce_hook(out)

    def route(self, p: str, x: torch.Tensor):
        """(weights, global expert ids) [T, K] of the router of MoE layer ``p``."""
        cfg = self.cfg
        probs = torch.softmax(x @ self.w[p + "mlp.gate.weight"].T, dim=-1)
        topv, topi = probs.topk(cfg.num_experts_per_tok, dim=-1)
        if cfg.norm_topk_prob:
            topv = topv / topv.sum(-1, keepdim=True)
        return topv, topi

    def expert(self, p: str, e: int, xr: torch.Tensor) -> torch.Tensor:
        """Expert ``e`` (global id) of MoE layer ``p`` on one row."""
        w = self.w
        q = p + f"mlp.experts.{e}."
        g = xr @ w[q + "gate_proj.weight"].T
        u = xr @ w[q + "up_proj.weight"].T
        return (torch.nn.functional.silu(g) * u) @ w[q + "down_proj.weight"].T

    @torch.no_grad()
    def forward(self, tokens: list[int], cache, start_pos: int) -> torch.Tensor:
        """Run ``tokens`` at positions start_pos.. (appending to ``cache``); return logits [T, V]."""
        cfg, w = self.cfg, self.w
        t = len(tokens)
        dev = self.device
        pos = torch.arange(start_pos, start_pos + t, device=dev)
        cs = self.cos_sin[pos]
        h = w["model.embed_tokens.weight"][torch.tensor(tokens, device=dev)]
        d, hq, hkv = cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            x = self._st(_rms(h, w[p + "input_layernorm.weight"], cfg.rms_eps))
            if self.tap is not None:
                self.tap(p + "input_layernorm", x)
            q = x @ w[p + "self_attn.q_proj.weight"].T
            k = x @ w[p + "self_attn.k_proj.weight"].T
            v = x @ w[p + "self_attn.v_proj.weight"].T
            if cfg.qkv_bias:
                q = q + w[p + "self_attn.q_proj.bias"]
                k = k + w[p + "self_attn.k_proj.bias"]
                v = v + w[p + "self_attn.v_proj.bias"]
            q, k, v = self._st(q).view(t, hq, d), self._st(k).view(t, hkv, d), self._st(v).view(t, hkv, d)
            if cfg.qk_norm:
                q = _rms(q, w[p + "self_attn.q_norm.weight"], cfg.rms_eps)
                k = _rms(k, w[p + "self_attn.k_norm.weight"], cfg.rms_eps)
            q, k, v = self.rotate_kv(_rope(q, cs), _rope(k, cs), v)
            q = self._st(q)
            c = cache[i]
            src = None if self.kv_source is None else self.kv_source(i, start_pos, t)
            kq, vq = src if src is not None else (self._kv_roundtrip(k, self.fk), self._kv_roundtrip(v, self.fv))
            c["k"] = torch.cat([c["k"], kq.to(dev)])
            c["v"] = torch.cat([c["v"], vq.to(dev)])
            kk = c["k"].repeat_interleave(hq // hkv, dim=1)
            vv = c["v"].repeat_interleave(hq // hkv, dim=1)
            s = torch.einsum("qhd,khd->hqk", q, kk) / math.sqrt(d)
            kpos = torch.arange(kk.shape[0], device=dev)
            s = s.masked_fill(kpos[None, None, :] > pos[None, :, None], float("-inf"))
            if self.kv_visible is not None:
                s = s.masked_fill(~self.kv_visible(pos[:, None], kpos[None, :])[None], float("-inf"))
            a = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vv)
            if self.had is not None:
                a = self.unrotate_out(self._st(a))
            a = self._st(a.reshape(t, hq * d))
            if self.tap is not None:
                self.tap(p + "self_attn.o_proj", a)
            h = self._st(h + a @ w[p + "self_attn.o_proj.weight"].T)
            x = self._st(_rms(h, w[p + "post_attention_layernorm.weight"], cfg.rms_eps))
            if self.tap is not None:
                self.tap(p + "post_attention_layernorm", x)
            h = self._st(h + self._mlp(p, x))
        x = self._st(_rms(h, w["model.norm.weight"], cfg.rms_eps))
        return self._st(x @ w["lm_head.weight"].T)

    def greedy(self, prompt: list[int], max_new: int) -> tuple[list[int], list[torch.Tensor]]:
        cache = self.new_cache()
        logits = self.forward(prompt, cache, 0)[-1]
        out, all_logits = [], []
        pos = len(prompt)
        for _ in range(max_new):
            all_logits.append(logits)
            tok = int(logits.argmax())
            out.append(tok)
            logits = self.forward([tok], cache, pos)[-1]
            pos += 1
        return out, all_logits
