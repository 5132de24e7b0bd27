"""The npy-dir checkpoint format (read and write), and the MLX ``squish_4bit`` directory.

npy-dir layout (the reference's convert.write_npy_dir, squish/convert.py:936-970):

    {dir}/manifest.json                 original tensor name -> safe key ("." -> "__")
    {dir}/tensors/{key}__{suffix}.npy   one array per file (mmap-able)
    {dir}/tensors/.manifest_ready       completion sentinel
    {dir}/_compress_progress.json       per-shard progress while converting

Suffix sets, in the reference loader's dispatch priority (squish/io/loader_utils.py:223-401):
    __nf4 + __s_nf4                     NF4 (16-level NormalFloat LUT), absmax per group
    __q4a + __s4a + __z4a               INT4 asymmetric: x = z + q * s (primary weight format)
    __q4 + __s4                         INT4 symmetric legacy: x = (q - 7) * s
    __q3 + __s3 (+ __z3, __lra, __lrb)  INT3 (8 values per 3 bytes) with optional low-rank term
    __q2 + __s2 + __z2                  INT2 asymmetric, 4 per byte
    __aqlm_idx + __aqlm_cb              AQLM additive codebooks
    __q + __s                           INT8 symmetric (per row or per group)
    __f8 + __sf8                        FP8 E4M3 codes + per-group scales (this package's extension)
    __nf4 + __s_nf4 + __lv_nf4          any4: NF4 codes with a learned 16-level table (extension)
    __q4a + ... + __rot_signs (+ __rot_meta) QuaRot: INT4 asymmetric codes of W R^T, R the block
                                        Hadamard over these input signs (extension)
    __sqint2_idx/_scales/_zp/_meta(+_L/_R) SQINT2 (Hadamard-rotated NF2 INT2, quant/sqint2.py)
    __pt_df11                           lossless bf16 passthrough, DFloat11-style (io/entropy.py df11_*)
    __vq_idx + __vq_cb (+ __vq_res, __vq_rescb, __vq_cols) + __vq_meta
                                        VPTQ vector quantization (squish/convert.py:362-420 layout)
    __pt                                float16 passthrough
plus __shape (the original shape) for every tensor. ``.npy.sqe`` files (rANS / Huffman coded,
io/entropy.py) are always readable; ``.npy.zst`` files when ``zstandard`` is importable.

``squish_4bit`` (squish/quant/compressed_loader.py:1109-1240): MLX affine 4-bit, one
safetensors file; ``weight`` uint32 words of 8 nibbles (lowest nibble = lowest column),
``scales``/``biases`` fp16 per group: x = bias + q * scale, i.e. exactly INT4 asymmetric.
"""
from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np
import torch

from ..models.weights import Checkpoint, QTensor

SUFFIXES = ("__pt_df11", "__vq_idx", "__vq_cb", "__vq_res", "__vq_rescb", "__vq_cols", "__vq_meta", "__lv_nf4", "__nf4",
            "__s_nf4", "__rot_signs", "__rot_meta", "__q4a", "__s4a", "__z4a", "__q4", "__s4", "__q3", "__s3", "__z3", "__lra",
            "__lrb", "__q2", "__s2", "__z2", "__aqlm_idx", "__aqlm_cb", "__f8", "__sf8", "__q", "__s", "__pt", "__shape")


def safe_key(name: str) -> str:
    return name.replace(".", "__")


def _load(path: Path) -> np.ndarray:
    if path.exists():
        return np.load(str(path), mmap_mode="r")
    sqe = Path(str(path) + ".sqe")
    if sqe.exists():  # rANS / Huffman coded copy (io/entropy.py)
        from .entropy import load_npy_sqe

        return load_npy_sqe(sqe)
    zst = Path(str(path) + ".zst")
    if zst.exists():
        try:
            import io

            import zstandard
        except ImportError as exc:
            raise RuntimeError(f"{zst} is zstd-compressed and the 'zstandard' module is not installed") from exc
        with open(zst, "rb") as f:
            raw = zstandard.ZstdDecompressor().decompress(f.read())
        return np.load(io.BytesIO(raw))
    raise FileNotFoundError(path)


def _exists(td: Path, key: str, suf: str) -> bool:
    p = td / f"{key}{suf}.npy"
    return p.exists() or Path(str(p) + ".zst").exists() or Path(str(p) + ".sqe").exists()


def tensor_dir(path: str | Path) -> Path:
    p = Path(path)
    return p / "tensors" if (p / "tensors").is_dir() else p


def read_tensor(td: Path, key: str) -> QTensor:
    """One npy-dir tensor as a QTensor (quantized kinds stay quantized)."""
    shape = tuple(int(x) for x in _load(td / f"{key}__shape.npy").tolist()) if _exists(td, key, "__shape") else None

    def arr(suf, dt=None):
        a = np.asarray(_load(td / f"{key}{suf}.npy"))
        return torch.from_numpy(np.array(a, dtype=dt or a.dtype, order="C", copy=True))

    if _exists(td, key, "__pt_df11"):  # (the reference checks this suffix first)
        from .entropy import df11_decode

        d = torch.from_numpy(df11_decode(np.asarray(_load(td / f"{key}__pt_df11.npy")).tobytes()).copy())
        return QTensor("dense", shape or tuple(d.shape), data=d.reshape(shape) if shape else d)
    if _exists(td, key, "__nf4") and _exists(td, key, "__s_nf4"):
        p, s = arr("__nf4", np.uint8), arr("__s_nf4", np.float32)
        t = QTensor("nf4", shape or (p.shape[0], p.shape[1] * 2), packed=p, scales=s,
                    group=(p.shape[1] * 2) // s.shape[1])
        if _exists(td, key, "__lv_nf4"):
            t.extra = {"levels": arr("__lv_nf4", np.float32)}
        return t
    if _exists(td, key, "__vq_idx"):
        d = torch.from_numpy(read_vptq(lambda suf: np.asarray(_load(td / f"{key}{suf}.npy")),
                                       lambda suf: _exists(td, key, suf)))
        return QTensor("dense", shape or tuple(d.shape), data=d.reshape(shape) if shape else d)
    if _exists(td, key, "__q4a"):
        p, s, z = arr("__q4a", np.uint8), arr("__s4a", np.float32), arr("__z4a", np.float32)
        t = QTensor("q4a", shape or (p.shape[0], p.shape[1] * 2), packed=p, scales=s, offsets=z,
                    group=(p.shape[1] * 2) // s.shape[1])
        if _exists(td, key, "__rot_signs"):
            meta = arr("__rot_meta", np.int64)
            t.extra = {"rot_signs": arr("__rot_signs", np.float32), "rot_block": int(meta[0]), "seed": int(meta[1])}
        return t
    if _exists(td, key, "__q4"):
        p, s = arr("__q4", np.uint8), arr("__s4", np.float32)
        if s.dim() == 1:
            s = s[:, None]
        # x = (q - 7) * s  ==  (-7 s) + q * s : the INT4 asymmetric form, exactly
        return QTensor("q4a", shape or (p.shape[0], p.shape[1] * 2), packed=p, scales=s, offsets=-7.0 * s,
                       group=(p.shape[1] * 2) // s.shape[1])
    if _exists(td, key, "__q3"):
        p, s = arr("__q3", np.uint8), arr("__s3", np.float32)
        extra = {}
        if _exists(td, key, "__lra"):
            extra = {"lra": arr("__lra", np.float32), "lrb": arr("__lrb", np.float32)}
        z = arr("__z3", np.float32) if _exists(td, key, "__z3") else None
        cols = shape[-1] if shape else (p.shape[1] * 8) // 3
        t = QTensor("q3", shape or (p.shape[0], cols), packed=p, scales=s, offsets=z, group=cols // s.shape[1])
        t.extra = extra
        return t
    if _exists(td, key, "__q2"):
        p, s, z = arr("__q2", np.uint8), arr("__s2", np.float32), arr("__z2", np.float32)
        return QTensor("q2", shape or (p.shape[0], p.shape[1] * 4), packed=p, scales=s, offsets=z,
                       group=(p.shape[1] * 4) // s.shape[1])
    if _exists(td, key, "__aqlm_idx"):
        idx, cb = arr("__aqlm_idx", np.int32), arr("__aqlm_cb", np.float32)
        t = QTensor("aqlm", shape, packed=idx, scales=cb, group=int(cb[2].item()))
        return t
    if _exists(td, key, "__sqint2_meta"):
        from ..quant.sqint2 import read_files

        return read_files(lambda suf: _load(td / f"{key}{suf}.npy"), key, shape)
    if _exists(td, key, "__f8"):
        q, s = arr("__f8", np.uint8), arr("__sf8", np.float32)
        return QTensor("fp8", shape or tuple(q.shape), packed=q, scales=s, group=q.shape[1] // s.shape[1])
    if _exists(td, key, "__q"):
        q, s = arr("__q", np.int8), arr("__s", np.float32)
        if s.dim() == 1:
            s = s[:, None]
        return QTensor("q8", shape or tuple(q.shape), packed=q, scales=s, group=q.shape[1] // s.shape[1])
    if _exists(td, key, "__pt"):
        d = arr("__pt")
        return QTensor("dense", shape or tuple(d.shape), data=d.reshape(shape) if shape else d)
    raise FileNotFoundError(f"no npy-dir files for tensor key {key!r} in {td}")


def read_vptq(load, exists) -> np.ndarray:
    """Dense fp32 weight of a VPTQ tensor in the reference's file layout (squish/convert.py
    :362-420): ``__vq_meta`` = [rows, cols, group, primary entries, residual entries];
    ``__vq_cb`` / ``__vq_rescb`` = codebook vectors (entries x group, flattened) followed by
    three trailing scalars (entries, group, fit iterations); ``__vq_idx`` / ``__vq_res`` =
    one codebook index per (row, group of ``group`` consecutive columns), row-major (a
    one-element ``__vq_res`` means no residual stage); ``__vq_cols`` = per-column scales
    (empty when absent). W[r, g*group:(g+1)*group] = cb[idx] (+ rescb[res]), times the
    column scales. The reference's own VPTQ module is not in its release, so the decoding
    follows this serialized layout."""
    meta = load("__vq_meta").astype(np.int64).reshape(-1)
    rows, cols, gs, n_cb, n_res = (int(v) for v in meta[:5])
    if gs <= 0 or cols % gs:
        raise ValueError(f"VPTQ group {gs} does not divide {cols} columns")
    ng = cols // gs
    cb = load("__vq_cb").astype(np.float32).reshape(-1)[:-3].reshape(-1, gs)
    idx = load("__vq_idx").astype(np.int64).reshape(rows, ng)
    if idx.min(initial=0) < 0 or idx.max(initial=0) >= cb.shape[0]:
        raise ValueError("VPTQ index outside its codebook")
    w = cb[idx]  # rows, ng, gs
    if n_res > 0 and exists("__vq_res"):
        res = load("__vq_res").astype(np.int64).reshape(-1)
        if res.size == rows * ng:
            rcb = load("__vq_rescb").astype(np.float32).reshape(-1)[:-3].reshape(-1, gs)
            res = res.reshape(rows, ng)
            if res.min(initial=0) < 0 or res.max(initial=0) >= rcb.shape[0]:
                raise ValueError("VPTQ residual index outside its codebook")
            w = w + rcb[res]
    w = w.reshape(rows, cols)
    if exists("__vq_cols"):
        cs = load("__vq_cols").astype(np.float32).reshape(-1)
        if cs.size == cols:
            w = w * cs[None, :]
    return np.ascontiguousarray(w, dtype=np.float32)


def read_npy_dir(path: str | Path, config, quant) -> Checkpoint:
    root = Path(path)
    td = tensor_dir(root)
    man_path = root / "manifest.json" if (root / "manifest.json").exists() else td.parent / "manifest.json"
    with open(man_path) as f:
        manifest = json.load(f)
    ck = Checkpoint(config, quant)
    for name, key in manifest.items():
        ck.tensors[name] = read_tensor(td, key)
    if "lm_head.weight" not in ck.tensors and config.tie_embeddings and "model.embed_tokens.weight" in ck.tensors:
        ck.tensors["lm_head.weight"] = ck.tensors["model.embed_tokens.weight"]
    return ck


def tensor_files(name: str, t: QTensor, df11: bool = False) -> dict[str, np.ndarray]:
    """The npy-dir files of one tensor (suffix -> array); ``df11`` stores dense tensors as
    lossless bf16 ``__pt_df11`` instead of float16 ``__pt``."""
    k = safe_key(name)
    out = {f"{k}__shape": np.asarray(t.shape, dtype=np.int64)}

    def np_(x, dt=None):
        a = x.detach().cpu().numpy() if isinstance(x, torch.Tensor) else np.asarray(x)
        return a.astype(dt) if dt is not None else a

    if t.kind == "q4a":
        out.update({f"{k}__q4a": np_(t.packed, np.uint8), f"{k}__s4a": np_(t.scales, np.float32),
                    f"{k}__z4a": np_(t.offsets, np.float32)})
        if t.extra and "rot_signs" in t.extra:
            out[f"{k}__rot_signs"] = np_(t.extra["rot_signs"], np.float32)
            out[f"{k}__rot_meta"] = np.asarray([int(t.extra["rot_block"]), int(t.extra.get("seed", 0))],
                                               dtype=np.int64)
    elif t.kind == "nf4":
        out.update({f"{k}__nf4": np_(t.packed, np.uint8), f"{k}__s_nf4": np_(t.scales, np.float32)})
        if t.extra and "levels" in t.extra:
            out[f"{k}__lv_nf4"] = np_(t.extra["levels"], np.float32)
    elif t.kind == "q8":
        out.update({f"{k}__q": np_(t.packed, np.int8), f"{k}__s": np_(t.scales, np.float32)})
    elif t.kind == "fp8":
        out.update({f"{k}__f8": np_(t.packed, np.uint8), f"{k}__sf8": np_(t.scales, np.float32)})
    elif t.kind == "q2" and t.extra and "rot_signs" in t.extra:
        from ..quant.sqint2 import write_files

        out.update(write_files(k, t))
    elif t.kind == "q2":
        out.update({f"{k}__q2": np_(t.packed, np.uint8), f"{k}__s2": np_(t.scales, np.float32),
                    f"{k}__z2": np_(t.offsets, np.float32)})
    elif t.kind == "q3":
        out.update({f"{k}__q3": np_(t.packed, np.uint8), f"{k}__s3": np_(t.scales, np.float32)})
        if t.offsets is not None:
            out[f"{k}__z3"] = np_(t.offsets, np.float32)
        for kk, v in (getattr(t, "extra", None) or {}).items():
            out[f"{k}__{kk}"] = np_(v, np.float32)
    elif t.kind == "aqlm":
        out.update({f"{k}__aqlm_idx": np_(t.packed, np.uint16), f"{k}__aqlm_cb": np_(t.scales, np.float32)})
    elif t.kind == "dense" and df11:
        from .entropy import df11_encode

        out[f"{k}__pt_df11"] = np.frombuffer(df11_encode(t.data), dtype=np.uint8).copy()
    elif t.kind == "dense":
        out[f"{k}__pt"] = np_(t.data.float(), np.float16)
    else:
        raise ValueError(f"cannot write tensor kind {t.kind!r}")
    return out


def write_npy_dir(path: str | Path, ck: Checkpoint, write_config: bool = True) -> int:
    """Write a whole checkpoint; returns bytes written."""
    root = Path(path)
    td = root / "tensors"
    td.mkdir(parents=True, exist_ok=True)
    manifest, total = {}, 0
    for name, t in ck.tensors.items():
        if name == "lm_head.weight" and ck.config.tie_embeddings and t is ck.tensors.get("model.embed_tokens.weight"):
            continue
        manifest[name] = safe_key(name)
        for key, a in tensor_files(name, t).items():
            p = td / f"{key}.npy"
            np.save(str(p), a)
            total += p.stat().st_size
    with open(root / "manifest.json", "w") as f:
        json.dump(manifest, f, indent=2)
    if write_config:
        from ..models.config import to_hf_config

        with open(root / "config.json", "w") as f:
            json.dump(to_hf_config(ck.config), f, indent=2)
        with open(root / "squish_quant.json", "w") as f:
            json.dump(ck.quant.__dict__, f, indent=2)
    (td / ".manifest_ready").touch()
    return total


# ----------------------------------------------------------------------------- MLX squish_4bit
def unpack_mlx_uint32(words: np.ndarray) -> np.ndarray:
    """uint32 words of 8 nibbles (lowest nibble = lowest column) -> uint8 codes."""
    w = words.astype(np.uint32)
    cols = [(w >> (4 * i)) & 0xF for i in range(8)]
    return np.stack(cols, axis=-1).reshape(w.shape[0], -1).astype(np.uint8)


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """(N, K) codes 0..15 -> (N, K/2) bytes, low nibble = even column."""
    c = codes.astype(np.uint8)
    return (c[:, 0::2] & 0xF) | ((c[:, 1::2] & 0xF) << 4)


def read_squish_4bit(path: str | Path, config, quant) -> Checkpoint:
    """An MLX affine 4-bit directory (``*.safetensors`` with weight/scales/biases triples)."""
    from safetensors.numpy import load_file

    root = Path(path)
    files = sorted(root.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors in {root}")
    raw: dict[str, np.ndarray] = {}
    for f in files:
        raw.update(load_file(str(f)))
    ck = Checkpoint(config, quant)
    for name, arr in raw.items():
        if name.endswith(".scales") or name.endswith(".biases"):
            continue
        base = name[: -len(".weight")] if name.endswith(".weight") else name
        if name.endswith(".weight") and f"{base}.scales" in raw:
            codes = unpack_mlx_uint32(arr)
            s = raw[f"{base}.scales"].astype(np.float32)
            b = raw[f"{base}.biases"].astype(np.float32)
            g = codes.shape[1] // s.shape[1]
            ck.tensors[name] = QTensor("q4a", (codes.shape[0], codes.shape[1]),
                                       packed=torch.from_numpy(pack_nibbles(codes)),
                                       scales=torch.from_numpy(s), offsets=torch.from_numpy(b), group=g)
        else:
            ck.tensors[name] = QTensor("dense", tuple(arr.shape), data=torch.from_numpy(arr.astype(np.float32)))
    if "lm_head.weight" not in ck.tensors and config.tie_embeddings and "model.embed_tokens.weight" in ck.tensors:
        ck.tensors["lm_head.weight"] = ck.tensors["model.embed_tokens.weight"]
    return ck


def detect_format(path: str | Path) -> str:
    p = Path(path)
    if p.is_file() and p.suffix == ".squizd":
        return "squizd"
    if p.is_file() and p.suffix == ".gguf":
        return "gguf"
    if (p / "manifest.json").exists() or (p / "tensors" / ".manifest_ready").exists():
        return "npy-dir"
    if p.is_dir() and any(str(f).endswith(".safetensors") for f in os.listdir(p)):
        from safetensors import safe_open

        f0 = sorted(x for x in os.listdir(p) if x.endswith(".safetensors"))[0]
        with safe_open(str(p / f0), "np") as f:
            if any(k.endswith(".scales") for k in f.keys()):
                return "squish_4bit"
        return "hf"
    raise ValueError(f"unrecognised checkpoint at {p}")
