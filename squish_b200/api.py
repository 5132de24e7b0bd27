"""Public Python API: load a model (checkpoint path or architecture preset) into an engine,
and an offline ``LLM.generate`` over it.

``model`` is either a checkpoint (npy-dir, MLX squish_4bit directory, HF safetensors
directory, ``.gguf`` or ``.squizd`` file) or the name of an architecture preset, which is
instantiated with random N(0, 0.02) weights (there are no downloads).
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from pathlib import Path

import torch

from .engine.engine import EngineConfig, LLMEngine
from .engine.sampling import SamplingParams
from .models.config import PRESETS, get_preset
from .models.weights import random_checkpoint
from .serving.tokenizer import load_tokenizer


@dataclass
class Loaded:
    engine: LLMEngine
    tokenizer: object
    name: str
    load_s: float


def default_device() -> str:
    return "cuda" if torch.cuda.is_available() else "cpu"


def load_engine(model: str, device: str | None = None, seed: int = 0, kv_dtype: str | None = None,
                ecfg: EngineConfig | None = None, page_size: int | None = None, **engine_kw) -> Loaded:
    from .utils.startup import StartupPhase, StartupTimer

    t0 = time.time()
    dev = torch.device(device or default_device())
    with StartupTimer(StartupPhase.CHECKPOINT_READ, model):
        if model.lower() in PRESETS:
            cfg, q = get_preset(model)
            if kv_dtype:
                q.kv_dtype = kv_dtype
            ck = random_checkpoint(cfg, q, seed=seed, device=dev)
            tok_dir = None
        else:
            if not Path(model).exists():
                raise FileNotFoundError(f"{model!r} is neither a checkpoint path nor a preset "
                                        f"({', '.join(sorted(PRESETS))})")
            from .io.convert import load_checkpoint

            ck, tok_dir = load_checkpoint(model, str(dev))
            if kv_dtype:
                ck.quant.kv_dtype = kv_dtype
    if page_size:
        if page_size % 16 or page_size <= 0:
            raise ValueError(f"page size {page_size} is not a positive multiple of 16")
        ck.quant.page_size = int(page_size)
    with StartupTimer(StartupPhase.WEIGHT_UPLOAD, "engine (weights, KV pool, graphs)"):
        eng = LLMEngine.from_checkpoint(ck, dev, ecfg, **engine_kw)
    with StartupTimer(StartupPhase.TOKENIZER):
        tok = load_tokenizer(tok_dir, vocab_size=ck.config.vocab_size, eos_token_id=ck.config.eos_token_id)
    return Loaded(eng, tok, ck.config.name, time.time() - t0)


class LLM:
    """Offline batch generation: ``LLM("qwen2.5-7b").generate(["hi"], SamplingParams(max_tokens=8))``."""

    def __init__(self, model: str, device: str | None = None, **kw):
        self.loaded = load_engine(model, device, **kw)
        self.engine = self.loaded.engine
        self.tokenizer = self.loaded.tokenizer

    def generate(self, prompts, params: SamplingParams | None = None) -> list[dict]:
        params = params or SamplingParams()
        rids = []
        for p in prompts:
            ids = p if isinstance(p, (list, tuple)) else self.tokenizer.encode(p)
            rids.append(self.engine.add_request(list(ids), params))
        outs = {r: [] for r in rids}
        while self.engine.has_unfinished():
            for o in self.engine.step():
                if o.rid in outs:
                    outs[o.rid].extend(o.new_tokens)
        res = []
        for r in rids:
            req = self.engine.requests[r]
            res.append({"token_ids": outs[r], "text": self.tokenizer.decode(outs[r]),
                        "finish_reason": req.finish_reason})
        return res
