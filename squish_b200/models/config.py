"""Model architecture descriptions and the named presets.

The reference has no model code of its own (it delegates to mlx_lm / HF transformers,
squish/backend.py:222-390); this module describes the decoder families the framework
implements itself: Llama, Qwen2 (q/k/v biases), Qwen3 (q/k RMSNorm) and Qwen3-MoE
(softmax router, top-k renormalised experts). Presets mirror the shapes of the
benchmark workloads; ``from_hf_config`` reads a HF ``config.json``.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field


@dataclass
class ModelConfig:
    name: str
    arch: str  # "llama" | "qwen2" | "qwen3" | "qwen3_moe"
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0
    tie_embeddings: bool = False
    qkv_bias: bool = False
    qk_norm: bool = False
    max_position: int = 32768
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    expert_offset: int = 0       # expert parallelism: this rank holds experts
    num_local_experts: int = 0   # [expert_offset, expert_offset + num_local_experts) (0 = all)
    rope_scaling: dict | None = None
    bos_token_id: int = 1
    eos_token_id: int = 2

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def num_params(self) -> int:
        h, l = self.hidden_size, self.num_layers
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        if self.is_moe:
            ffn = self.num_experts * 3 * h * self.moe_intermediate_size + h * self.num_experts
        else:
            ffn = 3 * h * self.intermediate_size
        emb = self.vocab_size * h * (1 if self.tie_embeddings else 2)
        return l * (attn + ffn + 2 * h) + emb + h

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    @staticmethod
    def from_dict(d: dict) -> "ModelConfig":
        names = {f.name for f in dataclasses.fields(ModelConfig)}
        return ModelConfig(**{k: v for k, v in d.items() if k in names})


@dataclass
class QuantConfig:
    """How weights and KV are stored on the device."""

    weight_bits: int = 4  # 4 (INT4 asym) | 16 (bf16)
    group_size: int = 64
    quantize_lm_head: bool = True
    kv_dtype: str = "int4"  # bf16 | int8 | int4 | int2 | k8v4
    kv_group: int = 32
    page_size: int = 16
    mse_clip: bool = False
    kv_hadamard: bool = False  # KV stored Hadamard-rotated (ops.kernels.kv_hadamard_signs)


PRESETS: dict[str, tuple[ModelConfig, QuantConfig]] = {}


def _register(cfg: ModelConfig, q: QuantConfig) -> None:
    PRESETS[cfg.name] = (cfg, q)


# Tiny Llama-style decoder (CPU fp32 end-to-end oracle): INT4 g32 weights, INT4 g32 KV, 16-token pages.
_register(ModelConfig("tiny-llama", "llama", 32000, 256, 4, 8, 2, 32, 688, 1e-6, 10000.0, tie_embeddings=True,
                      max_position=2048),
          QuantConfig(4, 32, True, "int4", 32, 16))
# Tiny Qwen3-MoE (tests): 16 experts, top-4, expert FFN 128.
_register(ModelConfig("tiny-moe", "qwen3_moe", 1024, 256, 2, 8, 2, 64, 512, 1e-6, 1e6, qk_norm=True, num_experts=16,
                      num_experts_per_tok=4, moe_intermediate_size=128, max_position=2048),
          QuantConfig(4, 64, True, "int4", 32, 16))
# Qwen2.5-7B shape: INT4 g64 weights (bf16 scales), INT4 KV in 16-token pages.
_register(ModelConfig("qwen2.5-7b", "qwen2", 152064, 3584, 28, 28, 4, 128, 18944, 1e-6, 1e6, qkv_bias=True,
                      max_position=32768, bos_token_id=151643, eos_token_id=151645),
          QuantConfig(4, 64, True, "int4", 32, 16))
# Qwen2.5-0.5B shape (speculative draft): INT4 g64.
_register(ModelConfig("qwen2.5-0.5b", "qwen2", 151936, 896, 24, 14, 2, 64, 4864, 1e-6, 1e6, qkv_bias=True,
                      tie_embeddings=True, max_position=32768, bos_token_id=151643, eos_token_id=151645),
          QuantConfig(4, 64, True, "int4", 32, 16))
# Qwen2.5-1.5B shape.
_register(ModelConfig("qwen2.5-1.5b", "qwen2", 151936, 1536, 28, 12, 2, 128, 8960, 1e-6, 1e6, qkv_bias=True,
                      tie_embeddings=True, max_position=32768, bos_token_id=151643, eos_token_id=151645),
          QuantConfig(4, 64, True, "int4", 32, 16))
# Llama-3-70B shape: INT4 g128 weights, k8v4 KV (8-bit keys, 4-bit values, group 64).
_register(ModelConfig("llama-3-70b", "llama", 128256, 8192, 80, 64, 8, 128, 28672, 1e-5, 5e5, max_position=131072,
                      bos_token_id=128000, eos_token_id=128009),
          QuantConfig(4, 128, True, "k8v4", 64, 16))
# Qwen3-30B-A3B shape MoE: 128 experts, top-8 renormalised, INT4 g64 experts, INT4 KV.
_register(ModelConfig("qwen3-30b-a3b", "qwen3_moe", 151936, 2048, 48, 32, 4, 128, 6144, 1e-6, 1e6, qk_norm=True,
                      num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768, max_position=40960,
                      bos_token_id=151643, eos_token_id=151645),
          QuantConfig(4, 64, True, "int4", 32, 16))


# Qwen3-8B shape: dense, q/k norms, INT4 g64 weights, INT4 KV.
_register(ModelConfig("qwen3-8b", "qwen3", 151936, 4096, 36, 32, 8, 128, 12288, 1e-6, 1e6, qk_norm=True,
                      max_position=40960, bos_token_id=151643, eos_token_id=151645),
          QuantConfig(4, 64, True, "int4", 32, 16))
# Llama-3.1-8B shape: Llama-3 RoPE frequency scaling, INT4 g64 weights, INT4 KV.
_register(ModelConfig("llama-3.1-8b", "llama", 128256, 4096, 32, 32, 8, 128, 14336, 1e-5, 5e5, max_position=131072,
                      rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                    "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
                      bos_token_id=128000, eos_token_id=128009),
          QuantConfig(4, 64, True, "int4", 32, 16))


def get_preset(name: str) -> tuple[ModelConfig, QuantConfig]:
    key = name.lower()
    if key not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    c, q = PRESETS[key]
    return dataclasses.replace(c), dataclasses.replace(q)


def from_hf_config(path: str) -> ModelConfig:
    """Read a HF transformers ``config.json`` (Llama / Qwen2 / Qwen3 / Qwen3-MoE)."""
    p = os.path.join(path, "config.json") if os.path.isdir(path) else path
    with open(p) as f:
        d = json.load(f)
    mt = d.get("model_type", "llama")
    arch = {"llama": "llama", "mistral": "llama", "qwen2": "qwen2", "qwen3": "qwen3", "qwen3_moe": "qwen3_moe"}.get(mt)
    if arch is None:
        raise ValueError(f"unsupported model_type {mt!r}")
    nh = d["num_attention_heads"]
    hd = d.get("head_dim") or d["hidden_size"] // nh
    eos = d.get("eos_token_id", 2)
    if isinstance(eos, list):
        eos = eos[0]
    return ModelConfig(
        name=d.get("_name_or_path", os.path.basename(os.path.dirname(p))) or mt,
        arch=arch,
        vocab_size=d["vocab_size"],
        hidden_size=d["hidden_size"],
        num_layers=d["num_hidden_layers"],
        num_heads=nh,
        num_kv_heads=d.get("num_key_value_heads", nh),
        head_dim=hd,
        intermediate_size=d.get("intermediate_size", 0),
        rms_eps=d.get("rms_norm_eps", 1e-6),
        rope_theta=d.get("rope_theta", 10000.0),
        tie_embeddings=d.get("tie_word_embeddings", False),
        qkv_bias=(arch == "qwen2") or bool(d.get("attention_bias", False)),
        qk_norm=arch in ("qwen3", "qwen3_moe"),
        max_position=d.get("max_position_embeddings", 32768),
        num_experts=d.get("num_experts", 0) or 0,
        num_experts_per_tok=d.get("num_experts_per_tok", 0) or 0,
        moe_intermediate_size=d.get("moe_intermediate_size", 0) or 0,
        norm_topk_prob=d.get("norm_topk_prob", True),
        rope_scaling=d.get("rope_scaling"),
        bos_token_id=d.get("bos_token_id", 1) or 1,
        eos_token_id=eos,
    )


def to_hf_config(cfg: ModelConfig) -> dict:
    """A HF-style config dict for this architecture (used when writing checkpoints)."""
    mt = {"llama": "llama", "qwen2": "qwen2", "qwen3": "qwen3", "qwen3_moe": "qwen3_moe"}[cfg.arch]
    d = {
        "model_type": mt,
        "architectures": [{"llama": "LlamaForCausalLM", "qwen2": "Qwen2ForCausalLM", "qwen3": "Qwen3ForCausalLM",
                           "qwen3_moe": "Qwen3MoeForCausalLM"}[cfg.arch]],
        "vocab_size": cfg.vocab_size,
        "hidden_size": cfg.hidden_size,
        "num_hidden_layers": cfg.num_layers,
        "num_attention_heads": cfg.num_heads,
        "num_key_value_heads": cfg.num_kv_heads,
        "head_dim": cfg.head_dim,
        "intermediate_size": cfg.intermediate_size,
        "rms_norm_eps": cfg.rms_eps,
        "rope_theta": cfg.rope_theta,
        "tie_word_embeddings": cfg.tie_embeddings,
        "max_position_embeddings": cfg.max_position,
        "bos_token_id": cfg.bos_token_id,
        "eos_token_id": cfg.eos_token_id,
        "hidden_act": "silu",
        "torch_dtype": "bfloat16",
    }
    if cfg.is_moe:
        d.update(num_experts=cfg.num_experts, num_experts_per_tok=cfg.num_experts_per_tok,
                 moe_intermediate_size=cfg.moe_intermediate_size, norm_topk_prob=cfg.norm_topk_prob,
                 decoder_sparse_step=1, mlp_only_layers=[])
    if cfg.rope_scaling:
        d["rope_scaling"] = cfg.rope_scaling
    return d


__all__ = ["ModelConfig", "QuantConfig", "PRESETS", "get_preset", "from_hf_config", "to_hf_config", "field"]
