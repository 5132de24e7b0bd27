"""SQUIZD single-file format (squish/docs/squizd_format_spec.md): write, read, validate.

Layout: 256-byte little-endian header (magic "SQZD", version 1, flags, layer_count,
arch_id, sparsity CRC32, draft-head FNV-1a-64, reserved zeros, sparsity and draft-head
metadata), a 32-byte layer index entry per layer (layer_idx, weight_offset, weight_length,
scale_offset), the per-layer weight blocks, then one "SCZT" scale/zero table.

Weight blocks hold the layer's tensors in name order, each as a tagged record
[u16 name length][name][block]. Block encodings from the spec: "INT4" (signed two's
complement nibbles, even element in bits 3:0), "INT2" (crumbs with a sub-block length) and
"NPCL" (raw float32/float16/bfloat16). The spec leaves per-group scales to "a second round
of per-sub-block scales with the tensor_id high bit set"; here sub-block g of a tensor is
stored with tensor_id = (fnv1a64(layer:name) & ~2^63 ^ g) | 2^63, after its per-tensor entry.
INT4 sub-blocks are symmetric (x = q * scale, q in [-8, 7]) with group = sub_block length.
The ASTC, TCA_TBE and ANE_COREML encodings are Apple-hardware paths: files that need them
are rejected with a clear error.
"""
from __future__ import annotations

import struct
import zlib
from pathlib import Path

import numpy as np
import torch

from ..models.config import ModelConfig, QuantConfig
from ..models.weights import Checkpoint, QTensor

MAGIC = b"SQZD"
VERSION = 1
F_ASTC, F_TCA_TBE, F_INT4, F_SPARSE, F_EAGLE, F_INT2, F_ANE_COREML = (1 << i for i in range(7))
HEADER = 256
INDEX_ENTRY = 32


def fnv1a64(data: bytes) -> int:
    h = 0xCBF29CE484222325
    for b in data:
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _tid(layer: int, name: str) -> int:
    return fnv1a64(f"{layer}:{name}".encode()) & ~(1 << 63)


def _int4_block(w: np.ndarray, group: int) -> tuple[bytes, list[float]]:
    rows, cols = w.shape
    g = w.reshape(rows, cols // group, group)
    s = np.abs(g).max(-1) / 7.0
    s = np.where(s == 0, 1.0, s).astype(np.float32)
    q = np.clip(np.rint(g / s[..., None]), -8, 7).astype(np.int8).reshape(rows, cols)
    u = (q.astype(np.int16) & 0xF).astype(np.uint8).reshape(-1)
    if u.size % 2:
        u = np.concatenate([u, np.zeros(1, np.uint8)])
    packed = (u[0::2] | (u[1::2] << 4)).astype(np.uint8)
    return b"INT4" + struct.pack("<II", rows, cols) + packed.tobytes(), s.reshape(-1).tolist()


def _npcl_block(a: np.ndarray) -> bytes:
    a = np.ascontiguousarray(a.astype(np.float16))
    return b"NPCL" + struct.pack("<II", 1, a.ndim) + b"".join(struct.pack("<I", d) for d in a.shape) + a.tobytes()


def write_squizd(path: str, ck: Checkpoint, group: int = 64) -> None:
    cfg = ck.config
    layers: list[list[tuple[str, QTensor]]] = [[] for _ in range(cfg.num_layers + 1)]  # last = globals
    for name, t in ck.tensors.items():
        if name.startswith("model.layers."):
            layers[int(name.split(".")[2])].append((name, t))
        elif not (name == "lm_head.weight" and cfg.tie_embeddings):
            layers[-1].append((name, t))
    blocks, scales = [], []  # scale entries: (tensor_id, scale, zero)
    for li, items in enumerate(layers):
        rec = bytearray()
        for name, t in sorted(items, key=lambda x: x[0]):
            w = t.dequantize().float().cpu().numpy()
            if t.kind != "dense" and w.ndim == 2 and w.shape[1] % group == 0:
                blk, ss = _int4_block(w, group)
                tid = _tid(li, name)
                scales.append((tid, float(np.mean(ss)), 0.0))
                for gi, sv in enumerate(ss):
                    scales.append((((tid ^ gi) & ~(1 << 63)) | (1 << 63), sv, 0.0))
                blk += struct.pack("<I", group)
            else:
                blk = _npcl_block(w)
            nb = name.encode()
            rec += struct.pack("<H", len(nb)) + nb + struct.pack("<Q", len(blk)) + blk
        blocks.append(bytes(rec))
    n_layers = len(blocks)
    off = HEADER + INDEX_ENTRY * n_layers
    index = bytearray()
    offsets = []
    for li, b in enumerate(blocks):
        offsets.append(off)
        off += len(b)
    sczt = b"SCZT" + struct.pack("<I", len(scales)) + b"".join(struct.pack("<Qff", *e) for e in scales)
    for li, b in enumerate(blocks):
        index += struct.pack("<IQQQI", li, offsets[li], len(b), off, 0)
    arch_id = {"llama": 1, "qwen2": 2, "qwen3": 3, "qwen3_moe": 4}.get(cfg.arch, 0)
    header = bytearray(HEADER)
    struct.pack_into("<4sHIHHIQ", header, 0, MAGIC, VERSION, F_INT4, n_layers, arch_id, 0, 0)
    # model geometry in reserved2 (offset 192): the spec reserves it for extensions
    struct.pack_into("<IIIIIIIf", header, 192, cfg.vocab_size, cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads,
                     cfg.head_dim, cfg.intermediate_size, int(cfg.tie_embeddings) | (int(cfg.qkv_bias) << 1) |
                     (int(cfg.qk_norm) << 2), cfg.rope_theta)
    with open(path, "wb") as f:
        f.write(bytes(header) + bytes(index) + b"".join(blocks) + sczt)


def validate(path: str, strict: bool = False) -> dict:
    """Check magic, version, flags, index bounds and CRC/hash fields; raises ValueError."""
    data = Path(path).read_bytes()
    if len(data) < HEADER or data[:4] != MAGIC:
        raise ValueError("not a SQUIZD file (bad magic)")
    version, flags, n_layers, arch_id, crc, ehash = struct.unpack_from("<HIHHIQ", data, 4)
    if version != VERSION:
        raise ValueError(f"unsupported SQUIZD version {version}")
    if flags >> 7:
        raise ValueError("reserved flag bits set")
    if strict and any(data[26:128]):
        raise ValueError("reserved header bytes are not zero")
    if flags & F_SPARSE and zlib.crc32(data[128:160]) != crc:
        raise ValueError("sparsity metadata CRC mismatch")
    if flags & F_EAGLE and fnv1a64(data[160:192]) != ehash:
        raise ValueError("draft head hash mismatch")
    end = HEADER + INDEX_ENTRY * n_layers
    if end > len(data):
        raise ValueError("layer index table truncated")
    for i in range(n_layers):
        li, wo, wl, so, res = struct.unpack_from("<IQQQI", data, HEADER + INDEX_ENTRY * i)
        if li != i or wo + wl > len(data) or so > len(data):
            raise ValueError(f"layer index entry {i} out of bounds")
    return {"version": version, "flags": flags, "layers": n_layers, "arch_id": arch_id, "bytes": len(data)}


def read_squizd(path: str, quant: QuantConfig | None = None) -> Checkpoint:
    info = validate(path)
    if info["flags"] & (F_ASTC | F_TCA_TBE | F_ANE_COREML):
        raise ValueError("this SQUIZD file needs Apple-hardware decoders (ASTC / TCA-TBE / CoreML)")
    data = Path(path).read_bytes()
    n_layers = info["layers"]
    vocab, hidden, nh, nkv, hd, ffn, bits, theta = struct.unpack_from("<IIIIIIIf", data, 192)
    arch = {1: "llama", 2: "qwen2", 3: "qwen3", 4: "qwen3_moe"}.get(info["arch_id"], "llama")
    cfg = ModelConfig("squizd", arch, vocab, hidden, n_layers - 1, nh, nkv, hd, ffn, rope_theta=float(theta),
                      tie_embeddings=bool(bits & 1), qkv_bias=bool(bits & 2), qk_norm=bool(bits & 4))
    # scale table
    _, _, _, so, _ = struct.unpack_from("<IQQQI", data, HEADER)
    if data[so:so + 4] != b"SCZT":
        raise ValueError("scale table magic missing")
    (n_sc,) = struct.unpack_from("<I", data, so + 4)
    table = {}
    for i in range(n_sc):
        tid, s, z = struct.unpack_from("<Qff", data, so + 8 + 16 * i)
        table[tid] = s
    q = quant or QuantConfig()
    ck = Checkpoint(cfg, q)
    from ..quant.codecs import quantize

    for li in range(n_layers):
        _, wo, wl, _, _ = struct.unpack_from("<IQQQI", data, HEADER + INDEX_ENTRY * li)
        o, endo = wo, wo + wl
        while o < endo:
            (nl,) = struct.unpack_from("<H", data, o)
            name = data[o + 2:o + 2 + nl].decode()
            o += 2 + nl
            (bl,) = struct.unpack_from("<Q", data, o)
            o += 8
            blk = data[o:o + bl]
            o += bl
            tag = blk[:4]
            if tag == b"INT4":
                rows, cols = struct.unpack_from("<II", blk, 4)
                n = rows * cols
                packed = np.frombuffer(blk, np.uint8, (n + 1) // 2, 12)
                (group,) = struct.unpack_from("<I", blk, 12 + (n + 1) // 2)
                u = np.empty(packed.size * 2, np.uint8)
                u[0::2], u[1::2] = packed & 0xF, packed >> 4
                qv = u[:n].astype(np.int8)
                qv = np.where(qv > 7, qv - 16, qv).astype(np.float32).reshape(rows, cols // group, group)
                tid = _tid(li, name)
                s = np.array([table[((tid ^ g) & ~(1 << 63)) | (1 << 63)] for g in range(rows * cols // group)],
                             np.float32).reshape(rows, cols // group, 1)
                w = torch.from_numpy((qv * s).reshape(rows, cols))
                ck.tensors[name] = quantize(w, "q4a", group) if q.weight_bits == 4 else \
                    QTensor("dense", (rows, cols), data=w)
            elif tag == b"NPCL":
                code, nd = struct.unpack_from("<II", blk, 4)
                shape = struct.unpack_from("<" + "I" * nd, blk, 12)
                dt = {0: np.float32, 1: np.float16}.get(code)
                a = np.frombuffer(blk, dt, int(np.prod(shape)), 12 + 4 * nd).astype(np.float32).reshape(shape)
                ck.tensors[name] = QTensor("dense", tuple(shape), data=torch.from_numpy(a.copy()))
            else:
                raise ValueError(f"unsupported SQUIZD block {tag!r}")
    if cfg.tie_embeddings:
        ck.tensors["lm_head.weight"] = ck.tensors["model.embed_tokens.weight"]
    return ck
