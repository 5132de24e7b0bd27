"""GGUF import (llama.cpp checkpoints) into a Checkpoint.

Parses the GGUF v2/v3 container (header, typed metadata, tensor infos, aligned data) and
maps llama.cpp tensor names to HF names. Block formats are converted without loss where
an equivalent exists: Q4_0 (x = (q - 8) d) and Q4_1 (x = q d + m), blocks of 32, become
INT4 asymmetric group-32; Q8_0 becomes INT8 symmetric group-32; F32/F16/BF16 pass through.
llama-architecture Q/K rows are un-permuted from llama.cpp's rotary layout back to HF's.
K-quant block types are rejected with a clear error. The reference's GGUF loader
(squish/io/gguf_loader.py) dequantizes to float; here quantized blocks stay quantized.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np
import torch

from ..models.config import ModelConfig, QuantConfig
from ..models.weights import Checkpoint, QTensor
from .npy_dir import pack_nibbles

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q8_0, GGML_BF16 = 0, 1, 2, 3, 8, 30
_VT = {0: ("B", 1), 1: ("b", 1), 2: ("H", 2), 3: ("h", 2), 4: ("I", 4), 5: ("i", 4), 6: ("f", 4), 7: ("?", 1),
       10: ("Q", 8), 11: ("q", 8), 12: ("d", 8)}


class _Reader:
    def __init__(self, buf: bytes):
        self.b = buf
        self.o = 0

    def take(self, fmt: str):
        v = struct.unpack_from("<" + fmt, self.b, self.o)
        self.o += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string(self) -> str:
        n = self.take("Q")
        s = self.b[self.o:self.o + n].decode("utf-8", errors="replace")
        self.o += n
        return s

    def value(self, vt: int):
        if vt in _VT:
            return self.take(_VT[vt][0])
        if vt == 8:
            return self.string()
        if vt == 9:
            et = self.take("I")
            n = self.take("Q")
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"unknown GGUF value type {vt}")


def parse_gguf(path: str) -> tuple[dict, list[dict], bytes, int]:
    buf = Path(path).read_bytes()
    r = _Reader(buf)
    if buf[:4] != b"GGUF":
        raise ValueError(f"{path} is not a GGUF file")
    r.o = 4
    version = r.take("I")
    if version not in (2, 3):
        raise ValueError(f"unsupported GGUF version {version}")
    n_tensors, n_kv = r.take("Q"), r.take("Q")
    meta = {}
    for _ in range(n_kv):
        k = r.string()
        meta[k] = r.value(r.take("I"))
    infos = []
    for _ in range(n_tensors):
        name = r.string()
        nd = r.take("I")
        dims = [r.take("Q") for _ in range(nd)]
        typ = r.take("I")
        off = r.take("Q")
        infos.append({"name": name, "dims": dims, "type": typ, "offset": off})
    align = int(meta.get("general.alignment", 32))
    data_start = (r.o + align - 1) // align * align
    return meta, infos, buf, data_start


def _name_map(n: str) -> str:
    if n == "token_embd.weight":
        return "model.embed_tokens.weight"
    if n == "output.weight":
        return "lm_head.weight"
    if n == "output_norm.weight":
        return "model.norm.weight"
    parts = n.split(".")
    if parts[0] == "blk":
        i, rest = parts[1], ".".join(parts[2:])
        m = {"attn_q.weight": "self_attn.q_proj.weight", "attn_k.weight": "self_attn.k_proj.weight",
             "attn_v.weight": "self_attn.v_proj.weight", "attn_output.weight": "self_attn.o_proj.weight",
             "attn_q.bias": "self_attn.q_proj.bias", "attn_k.bias": "self_attn.k_proj.bias",
             "attn_v.bias": "self_attn.v_proj.bias", "attn_norm.weight": "input_layernorm.weight",
             "ffn_norm.weight": "post_attention_layernorm.weight", "ffn_gate.weight": "mlp.gate_proj.weight",
             "ffn_up.weight": "mlp.up_proj.weight", "ffn_down.weight": "mlp.down_proj.weight",
             "attn_q_norm.weight": "self_attn.q_norm.weight", "attn_k_norm.weight": "self_attn.k_norm.weight"}
        if rest in m:
            return f"model.layers.{i}.{m[rest]}"
    return n


def _unpermute_rows(a: np.ndarray, n_head: int) -> np.ndarray:
    rows = a.shape[0]
    return a.reshape(n_head, rows // n_head // 2, 2, *a.shape[1:]).swapaxes(1, 2).reshape(a.shape)


def _tensor(info: dict, buf: bytes, data_start: int, unpermute_heads: int | None) -> QTensor:
    dims = info["dims"]
    cols = dims[0]
    rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
    shape = (rows, cols) if len(dims) > 1 else (cols,)
    off = data_start + info["offset"]
    t = info["type"]
    n = rows * cols
    if t in (GGML_F32, GGML_F16, GGML_BF16):
        if t == GGML_BF16:
            raw = np.frombuffer(buf, dtype=np.uint16, count=n, offset=off).astype(np.uint32) << 16
            a = raw.view(np.float32)
        else:
            a = np.frombuffer(buf, dtype=np.float32 if t == GGML_F32 else np.float16, count=n, offset=off)
        a = a.astype(np.float32).reshape(shape)
        if unpermute_heads:
            a = _unpermute_rows(a, unpermute_heads)
        return QTensor("dense", shape, data=torch.from_numpy(np.ascontiguousarray(a)))
    if cols % 32:
        raise ValueError(f"{info['name']}: row length {cols} is not a multiple of the 32-value block")
    nb = n // 32
    if t == GGML_Q8_0:
        blk = np.frombuffer(buf, dtype=np.uint8, count=nb * 34, offset=off).reshape(nb, 34)
        d = blk[:, :2].copy().view(np.float16).astype(np.float32).reshape(rows, cols // 32)
        q = blk[:, 2:].copy().view(np.int8).reshape(rows, cols)
        if unpermute_heads:
            q, d = _unpermute_rows(q, unpermute_heads), _unpermute_rows(d, unpermute_heads)
        return QTensor("q8", shape, packed=torch.from_numpy(np.ascontiguousarray(q)),
                       scales=torch.from_numpy(np.ascontiguousarray(d)), group=32)
    if t in (GGML_Q4_0, GGML_Q4_1):
        bs = 18 if t == GGML_Q4_0 else 20
        blk = np.frombuffer(buf, dtype=np.uint8, count=nb * bs, offset=off).reshape(nb, bs)
        d = blk[:, :2].copy().view(np.float16).astype(np.float32)[:, 0]
        if t == GGML_Q4_0:
            m = -8.0 * d
            qs = blk[:, 2:]
        else:
            m = blk[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
            qs = blk[:, 4:]
        codes = np.concatenate([qs & 0xF, qs >> 4], axis=1).reshape(rows, cols)  # element j and j+16
        s = d.reshape(rows, cols // 32)
        z = m.reshape(rows, cols // 32)
        if unpermute_heads:
            codes = _unpermute_rows(codes, unpermute_heads)
            s, z = _unpermute_rows(s, unpermute_heads), _unpermute_rows(z, unpermute_heads)
        return QTensor("q4a", shape, packed=torch.from_numpy(pack_nibbles(codes)),
                       scales=torch.from_numpy(np.ascontiguousarray(s)),
                       offsets=torch.from_numpy(np.ascontiguousarray(z)), group=32)
    raise ValueError(f"{info['name']}: GGML type {t} is not supported (use F16/F32/BF16/Q4_0/Q4_1/Q8_0)")


def read_gguf(path: str) -> Checkpoint:
    meta, infos, buf, data_start = parse_gguf(path)
    arch = meta.get("general.architecture", "llama")
    g = lambda k, d=None: meta.get(f"{arch}.{k}", d)  # noqa: E731
    n_head = int(g("attention.head_count"))
    n_kv = int(g("attention.head_count_kv", n_head))
    hidden = int(g("embedding_length"))
    vocab = len(meta.get("tokenizer.ggml.tokens", [])) or int(g("vocab_size", 32000))
    names = {i["name"] for i in infos}
    cfg = ModelConfig(
        name=str(meta.get("general.name", Path(path).stem)), arch={"qwen2": "qwen2", "qwen3": "qwen3"}.get(arch, "llama"),
        vocab_size=vocab, hidden_size=hidden, num_layers=int(g("block_count")), num_heads=n_head, num_kv_heads=n_kv,
        head_dim=int(g("attention.key_length", hidden // n_head)), intermediate_size=int(g("feed_forward_length")),
        rms_eps=float(g("attention.layer_norm_rms_epsilon", 1e-6)), rope_theta=float(g("rope.freq_base", 10000.0)),
        tie_embeddings="output.weight" not in names, qkv_bias=any(n.endswith("attn_q.bias") for n in names),
        qk_norm=any(n.endswith("attn_q_norm.weight") for n in names),
        max_position=int(g("context_length", 4096)),
        bos_token_id=int(meta.get("tokenizer.ggml.bos_token_id", 1)),
        eos_token_id=int(meta.get("tokenizer.ggml.eos_token_id", 2)))
    ck = Checkpoint(cfg, QuantConfig(group_size=32))
    for info in infos:
        hf = _name_map(info["name"])
        heads = None
        if cfg.arch == "llama" and hf.endswith("q_proj.weight"):
            heads = n_head
        elif cfg.arch == "llama" and hf.endswith("k_proj.weight"):
            heads = n_kv
        ck.tensors[hf] = _tensor(info, buf, data_start, heads)
    if cfg.tie_embeddings:
        ck.tensors["lm_head.weight"] = ck.tensors["model.embed_tokens.weight"]
    return ck


def write_gguf_minimal(path: str, meta: dict, tensors: dict[str, tuple[int, np.ndarray, tuple]]) -> None:
    """Write a small GGUF v3 file (tests and fixtures): tensors = name -> (ggml type, raw data
    array, GGUF dims with the row length first)."""
    def s(x: str) -> bytes:
        e = x.encode()
        return struct.pack("<Q", len(e)) + e

    out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for k, v in meta.items():
        out += s(k)
        if isinstance(v, str):
            out += struct.pack("<I", 8) + s(v)
        elif isinstance(v, float):
            out += struct.pack("<If", 6, v)
        elif isinstance(v, list):
            out += struct.pack("<IIQ", 9, 8, len(v)) + b"".join(s(x) for x in v)
        else:
            out += struct.pack("<II", 4, int(v))
    offs, data = {}, bytearray()
    for name, (typ, arr, dims) in tensors.items():
        while len(data) % 32:
            data += b"\0"
        offs[name] = len(data)
        data += arr.tobytes()
    for name, (typ, arr, dims) in tensors.items():
        out += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", typ, offs[name])
    while len(out) % 32:
        out += b"\0"
    Path(path).write_bytes(bytes(out) + bytes(data))
