"""``squish compress``: HF safetensors (or random init) -> npy-dir, shard by shard, resumable.

Per shard: load tensors (on the GPU when one is present, where the INT4 quantizer runs as a
CUDA kernel), quantize every 2-D projection weight, pass embeddings, norms, biases and MoE
routers through as fp16, write the tensor files, then commit ``manifest.json`` and
``_compress_progress.json`` (completed shards) before moving on — the reference's
streaming converter contract (squish/convert.py:610-935). Re-running after an interruption
skips completed shards. ``delete_source`` removes a raw shard only after its output and
progress are on disk.
"""
from __future__ import annotations

import json
import os
import shutil
import time
from pathlib import Path

import numpy as np
import torch

from ..models.config import QuantConfig, from_hf_config, get_preset, to_hf_config
from ..models.weights import QTensor, random_checkpoint
from ..quant.codecs import quantize
from .npy_dir import safe_key, tensor_files

PASSTHROUGH_PATTERNS = ("embed_tokens", "norm", "mlp.gate.weight", ".bias")


def should_quantize(name: str, shape: tuple, patterns=PASSTHROUGH_PATTERNS) -> bool:
    if len(shape) != 2:
        return False
    if any(p in name for p in patterns) and not name.endswith("lm_head.weight"):
        return False
    return True


def _write_tensor(td: Path, name: str, t: QTensor, df11: bool = False) -> int:
    n = 0
    for key, a in tensor_files(name, t, df11=df11).items():
        p = td / f"{key}.npy"
        np.save(str(p), a)
        n += p.stat().st_size
    return n


def _awq_ops(cfg, q, names, ck_loader, tokenizer_dir, out: Path, dev, awq_scales: str | None, alpha: float,
             samples: int, seq_len: int, seed: int, log) -> dict:
    """Per-tensor AWQ operations: from a scales directory, or calibrated here on the fp32 model
    (``ck_loader()`` builds it) and saved under ``out/awq``."""
    from ..quant.awq import (calibration_tokens, collect_activation_scales, load_awq_scales,
                             prepare_awq_application, save_awq_scales)

    if awq_scales:
        scales = load_awq_scales(awq_scales)
        if not scales:
            raise FileNotFoundError(f"no AWQ scales in {awq_scales}")
    else:
        tok = None
        if tokenizer_dir is not None and ((Path(tokenizer_dir) / "tokenizer.json").exists()):
            from ..serving.tokenizer import load_tokenizer

            tok = load_tokenizer(str(tokenizer_dir), cfg.vocab_size)
        toks = calibration_tokens(cfg.vocab_size, samples, seq_len, tokenizer=tok, seed=seed)
        t0 = time.time()
        scales = collect_activation_scales(ck_loader(), toks, alpha=alpha, device=dev)
        save_awq_scales(scales, out / "awq")
        log(f"  AWQ calibration: {len(toks)} sequences, {len(scales)} layers, {time.time() - t0:.1f}s")
    ops = prepare_awq_application(scales, names)
    log(f"  AWQ: scaling {sum(1 for o in ops.values() if o[0] == 'mul')} weights under "
        f"{sum(1 for o in ops.values() if o[0] == 'div')} norms")
    return ops


def compress(model_dir: str | None, out_dir: str, kind: str = "q4a", group_size: int = 64, mse_clip: bool = False,
             device: str | None = None, delete_source: bool = False, random_preset: str | None = None,
             seed: int = 0, kv_dtype: str = "int4", log=print, hqq: bool = False, awq: bool = False,
             awq_scales: str | None = None, awq_alpha: float = 0.5, awq_samples: int = 16,
             awq_seq_len: int = 256, super_weights: bool = True, gptq: bool = False, df11: bool = False) -> dict:
    """``hqq``: half-quadratic refinement of INT4 / INT2 grids. ``awq`` (or ``awq_scales``, a
    directory of saved scales): activation-aware scaling of norm-fed projections before
    quantization; calibration needs the whole fp32 model in memory once. ``super_weights``
    (with ``mse_clip``): rows holding a super weight skip the clip search; the coordinates found
    are written to ``super_weights.json``. ``df11``: passthrough (unquantized) tensors are
    stored losslessly as DFloat11-style ``__pt_df11`` (bf16 with entropy-coded exponents)."""
    from ..quant.super_weights import SuperWeightCalibrator, protect, save_coords

    if gptq and (awq or awq_scales or kind != "q4a" or hqq):
        raise ValueError("GPTQ produces INT4 (q4a) tensors and is not combined with AWQ or HQQ here")
    hess: dict = {}

    def calibrate_gptq(ck_loader, tokenizer_dir):
        from ..quant.awq import calibration_tokens
        from ..quant.gptq import collect_hessians

        tok = None
        if tokenizer_dir is not None and (Path(tokenizer_dir) / "tokenizer.json").exists():
            from ..serving.tokenizer import load_tokenizer

            tok = load_tokenizer(str(tokenizer_dir), cfg.vocab_size)
        t0 = time.time()
        hess.update(collect_hessians(ck_loader(), calibration_tokens(cfg.vocab_size, awq_samples, awq_seq_len,
                                                                     tokenizer=tok, seed=seed), dev))
        log(f"  GPTQ calibration: {len(hess)} projections, {time.time() - t0:.1f}s")

    def gptq_or(name, w, fallback):
        if name in hess:
            from ..models.weights import pick_group
            from ..quant.gptq import gptq_quantize

            return gptq_quantize(w.to(dev), hess[name], pick_group(w.shape[1], group_size))
        return fallback()
    sw_cal = SuperWeightCalibrator() if (super_weights and mse_clip and kind == "q4a") else None
    sw_found = []

    def q4(name, w, t):
        """the MSE-clipped tensor with super-weight rows re-quantized unclipped"""
        if sw_cal is None or t.kind != "q4a":
            return t
        hits = sw_cal.scan_tensor(name, w)
        sw_found.extend(hits)
        return protect(t, w, {h.row for h in hits})
    out = Path(out_dir)
    td = out / "tensors"
    td.mkdir(parents=True, exist_ok=True)
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    progress_path = out / "_compress_progress.json"
    man_path = out / "manifest.json"
    manifest = json.loads(man_path.read_text()) if man_path.exists() else {}
    done = json.loads(progress_path.read_text())["completed_shards"] if progress_path.exists() else []
    stats = {"n_quantized": 0, "n_passthrough": 0, "bytes": 0, "shards": 0, "skipped_shards": len(done)}
    t0 = time.time()

    if random_preset:
        cfg, q = get_preset(random_preset)
        q.group_size, q.mse_clip, q.kv_dtype = group_size, mse_clip, kv_dtype
        if "random-init" not in done:
            ck = random_checkpoint(cfg, q, seed=seed, device=dev)
            ops = {}
            if awq or awq_scales:
                ops = _awq_ops(cfg, q, list(ck.tensors), lambda: ck, None, out, dev, awq_scales, awq_alpha,
                               awq_samples, awq_seq_len, seed, log)
            if gptq:
                calibrate_gptq(lambda: ck, None)
            router = None
            if kind == "mixed":
                from ..quant.mixed import MixedPrecisionRouter

                router = MixedPrecisionRouter(cfg.num_layers)
            for name, t in ck.tensors.items():
                if name == "lm_head.weight" and cfg.tie_embeddings:
                    continue
                tkind = router.kind_for(name) if router is not None else kind
                if name in ops:
                    from ..quant.awq import apply_op

                    w = apply_op(t.dequantize(), ops[name])
                    t = (QTensor("dense", t.shape, data=w.cpu()) if t.kind == "dense"
                         else quantize(w, tkind, group_size, mse_clip, hqq=hqq))
                elif name in hess:
                    t = gptq_or(name, t.dequantize(), None)
                elif t.kind != "dense" and (tkind != "q4a" or hqq):
                    t = quantize(t.dequantize(), tkind, group_size, mse_clip, hqq=hqq)
                stats["bytes"] += _write_tensor(td, name, t, df11)
                stats["n_quantized" if t.kind != "dense" else "n_passthrough"] += 1
                manifest[name] = safe_key(name)
            done.append("random-init")
        shards = []
    else:
        from safetensors import safe_open

        src = Path(model_dir)
        cfg = from_hf_config(str(src))
        q = QuantConfig(weight_bits=16 if kind == "dense" else 4, group_size=group_size, mse_clip=mse_clip,
                        kv_dtype=kv_dtype)
        shards = sorted(p for p in src.glob("*.safetensors"))
        if not shards:
            raise FileNotFoundError(f"no *.safetensors in {src}")
        ops = {}
        if awq or awq_scales:
            names = []
            for shard in shards:
                with safe_open(str(shard), "pt", device="cpu") as f:
                    names += list(f.keys())

            def load_dense():
                from ..models.weights import Checkpoint

                ckd = Checkpoint(cfg, q)
                for shard in shards:
                    with safe_open(str(shard), "pt", device="cpu") as f:
                        for n in f.keys():
                            ckd.tensors[n] = QTensor("dense", tuple(f.get_slice(n).get_shape()), data=f.get_tensor(n))
                if "lm_head.weight" not in ckd.tensors and cfg.tie_embeddings:
                    ckd.tensors["lm_head.weight"] = ckd.tensors["model.embed_tokens.weight"]
                return ckd

            ops = _awq_ops(cfg, q, names, load_dense, src, out, dev, awq_scales, awq_alpha, awq_samples,
                           awq_seq_len, seed, log)
        if gptq:
            def load_dense_g():
                from ..models.weights import Checkpoint

                ckd = Checkpoint(cfg, q)
                for shard in shards:
                    with safe_open(str(shard), "pt", device="cpu") as f:
                        for n in f.keys():
                            ckd.tensors[n] = QTensor("dense", tuple(f.get_slice(n).get_shape()), data=f.get_tensor(n))
                if "lm_head.weight" not in ckd.tensors and cfg.tie_embeddings:
                    ckd.tensors["lm_head.weight"] = ckd.tensors["model.embed_tokens.weight"]
                return ckd

            calibrate_gptq(load_dense_g, src)
        router = None
        if kind == "mixed":
            from ..quant.mixed import MixedPrecisionRouter

            router = MixedPrecisionRouter(cfg.num_layers)
        for i, shard in enumerate(shards):
            if shard.name in done:
                continue
            with safe_open(str(shard), "pt", device=str(dev) if dev.type == "cuda" else "cpu") as f:
                for name in f.keys():
                    w = f.get_tensor(name)
                    if name in ops:
                        from ..quant.awq import apply_op

                        w = apply_op(w, ops[name])
                    if should_quantize(name, tuple(w.shape)):
                        tkind = router.kind_for(name) if router is not None else kind
                        wq = w if dev.type == "cuda" else w.float()
                        t = gptq_or(name, wq, lambda: quantize(wq, tkind, group_size, mse_clip, hqq=hqq))
                        t = q4(name, wq, t)
                        stats["n_quantized"] += 1
                    else:
                        t = QTensor("dense", tuple(w.shape), data=w.float().cpu())
                        stats["n_passthrough"] += 1
                    stats["bytes"] += _write_tensor(td, name, t, df11)
                    manifest[name] = safe_key(name)
                    del w
            man_path.write_text(json.dumps(manifest, indent=2))
            done.append(shard.name)
            progress_path.write_text(json.dumps({"completed_shards": done, "total_shards": len(shards),
                                                 "delete_source": delete_source}, indent=2))
            stats["shards"] += 1
            log(f"  shard {i + 1}/{len(shards)} {shard.name} done")
            if delete_source:
                shard.unlink()
        for extra in ("tokenizer.json", "tokenizer_config.json", "tokenizer.model", "special_tokens_map.json",
                      "generation_config.json", "vocab.json", "merges.txt"):
            if (src / extra).exists():
                shutil.copy2(src / extra, out / extra)
    if sw_cal is not None:
        save_coords(sw_found, out / "super_weights.json")
        stats["super_weights"] = len(sw_found)
    man_path.write_text(json.dumps(manifest, indent=2))
    progress_path.write_text(json.dumps({"completed_shards": done, "total_shards": max(len(shards), 1),
                                         "delete_source": delete_source}, indent=2))
    (out / "config.json").write_text(json.dumps(to_hf_config(cfg), indent=2))
    q.weight_bits = 16 if kind == "dense" else 4
    (out / "squish_quant.json").write_text(json.dumps(dict(q.__dict__, weight_kind=kind, hqq=hqq,
                                                           awq=bool(awq or awq_scales), gptq=gptq), indent=2))
    (td / ".manifest_ready").touch()
    stats["seconds"] = round(time.time() - t0, 2)
    return stats


def load_checkpoint(path: str, device: str | None = None):
    """Any supported checkpoint -> (Checkpoint, tokenizer directory or None)."""
    from .npy_dir import detect_format, read_npy_dir, read_squish_4bit

    fmt = detect_format(path)
    p = Path(path)
    if os.environ.get("SQUISH_ALLOW_UNSAFE") != "1":
        from ..serving.model_scanner import scan_before_load

        scan = scan_before_load(p)
        if scan.status == "unsafe":
            raise RuntimeError(f"refusing to load {p}: " + "; ".join(scan.findings[:3]) +
                               " (set SQUISH_ALLOW_UNSAFE=1 to override)")
    if fmt == "gguf":
        from .gguf import read_gguf

        return read_gguf(path), None
    if fmt == "squizd":
        from .squizd import read_squizd

        return read_squizd(path), None
    cfg = from_hf_config(str(p))
    qpath = p / "squish_quant.json"
    q = QuantConfig()
    if qpath.exists():
        d = json.loads(qpath.read_text())
        q = QuantConfig(**{k: v for k, v in d.items() if k in QuantConfig.__dataclass_fields__})
    if fmt == "npy-dir":
        return read_npy_dir(p, cfg, q), str(p)
    if fmt == "squish_4bit":
        return read_squish_4bit(p, cfg, q), str(p)
    if fmt == "hf":
        from safetensors.torch import load_file

        from ..models.weights import Checkpoint

        ck = Checkpoint(cfg, q)
        for f in sorted(p.glob("*.safetensors")):
            for name, w in load_file(str(f)).items():
                if should_quantize(name, tuple(w.shape)):
                    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
                    ck.tensors[name] = quantize(w.to(dev), "q4a", q.group_size, q.mse_clip)
                else:
                    ck.tensors[name] = QTensor("dense", tuple(w.shape), data=w.float())
        if "lm_head.weight" not in ck.tensors:
            ck.tensors["lm_head.weight"] = quantize(ck.tensors["model.embed_tokens.weight"].data, "q4a",
                                                    q.group_size)
        return ck, str(p)
    raise ValueError(fmt)
