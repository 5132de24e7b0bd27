"""Entropy coding of checkpoint bytes: rANS and Huffman codecs (C++, ``_C.cpu``) and a small
self-describing container for ``.npy`` files.

The codecs are the counterparts of the reference's ``rans_encode`` / ``rans_decode`` /
``huffman_encode`` / ``huffman_decode`` (squish_quant_rs/src/lib.rs:1637-1830) with the same
arguments (uint8 symbols, 256-entry tables). The reference's npy-dir entropy layer stores
INT8 ``.npy`` files as zstd streams (squish/io/entropy.py); zstd is not available here, so the
same role is played by ``.npy.sqe`` files: a rANS (or Huffman) coded copy of the ``.npy``
bytes, decoded at load time by the npy-dir reader.

Container (little-endian)::

    b"SQE1" | codec u8 (0 = rANS, 1 = Huffman) | n_bytes u64 | table | payload
    rANS table:    256 x u32 symbol frequencies
    Huffman table: 256 x u32 code words, 256 x u8 code lengths
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np
import torch

from .._ext import native

MAGIC = b"SQE1"
RANS, HUFFMAN = 0, 1


def _u8(x) -> torch.Tensor:
    a = np.ascontiguousarray(np.frombuffer(x, dtype=np.uint8) if isinstance(x, (bytes, bytearray, memoryview))
                             else np.asarray(x, dtype=np.uint8).reshape(-1))
    return torch.from_numpy(a.copy())


def histogram(data) -> np.ndarray:
    return np.bincount(_u8(data).numpy(), minlength=256).astype(np.uint32)


def rans_encode(symbols, freqs) -> np.ndarray:
    return native().cpu.rans_encode(_u8(symbols), torch.as_tensor(np.asarray(freqs, dtype=np.int64))).numpy()


def rans_decode(data, freqs, n_symbols: int) -> np.ndarray:
    return native().cpu.rans_decode(_u8(data), torch.as_tensor(np.asarray(freqs, dtype=np.int64)),
                                    int(n_symbols)).numpy()


def huffman_build(freqs) -> tuple[np.ndarray, np.ndarray]:
    w, ln = native().cpu.huffman_build(torch.as_tensor(np.asarray(freqs, dtype=np.int64)))
    return w.numpy().astype(np.uint32), ln.numpy()


def huffman_encode(symbols, code_words, code_lens) -> np.ndarray:
    return native().cpu.huffman_encode(_u8(symbols), torch.as_tensor(np.asarray(code_words, dtype=np.int64)),
                                       torch.as_tensor(np.asarray(code_lens, dtype=np.int64))).numpy()


def huffman_decode(data, code_words, code_lens, n_symbols: int) -> np.ndarray:
    return native().cpu.huffman_decode(_u8(data), torch.as_tensor(np.asarray(code_words, dtype=np.int64)),
                                       torch.as_tensor(np.asarray(code_lens, dtype=np.int64)),
                                       int(n_symbols)).numpy()


def compress_bytes(data: bytes, codec: int = RANS) -> bytes:
    sym = _u8(data)
    n = sym.numel()
    if n == 0:
        return MAGIC + struct.pack("<BQ", codec, 0)
    freqs = histogram(data)
    if codec == RANS:
        return MAGIC + struct.pack("<BQ", RANS, n) + freqs.tobytes() + rans_encode(sym, freqs).tobytes()
    if codec == HUFFMAN:
        w, ln = huffman_build(freqs)
        return (MAGIC + struct.pack("<BQ", HUFFMAN, n) + w.astype("<u4").tobytes() + ln.astype(np.uint8).tobytes()
                + huffman_encode(sym, w, ln).tobytes())
    raise ValueError(f"unknown codec {codec}")


def decompress_bytes(blob: bytes) -> bytes:
    if blob[:4] != MAGIC:
        raise ValueError("not an SQE1 container")
    codec, n = struct.unpack_from("<BQ", blob, 4)
    off = 4 + 9
    if n == 0:
        return b""
    if codec == RANS:
        freqs = np.frombuffer(blob, dtype="<u4", count=256, offset=off)
        return rans_decode(blob[off + 1024:], freqs, n).tobytes()
    if codec == HUFFMAN:
        w = np.frombuffer(blob, dtype="<u4", count=256, offset=off)
        ln = np.frombuffer(blob, dtype=np.uint8, count=256, offset=off + 1024)
        return huffman_decode(blob[off + 1280:], w, ln, n).tobytes()
    raise ValueError(f"unknown codec {codec}")


def compress_npy(path: str | Path, codec: int = RANS, remove: bool = True) -> tuple[int, int]:
    """``x.npy`` -> ``x.npy.sqe``; returns (original bytes, compressed bytes)."""
    p = Path(path)
    raw = p.read_bytes()
    blob = compress_bytes(raw, codec)
    Path(str(p) + ".sqe").write_bytes(blob)
    if remove:
        p.unlink()
    return len(raw), len(blob)


def compress_npy_dir(tensor_dir: str | Path, codec: int = RANS, only_integer: bool = True) -> tuple[int, int]:
    """Entropy-code the (integer) ``.npy`` files of an npy-dir in place; returns total bytes
    before / after. Float passthrough tensors compress poorly and are left alone by default."""
    before = after = 0
    for f in sorted(Path(tensor_dir).glob("*.npy")):
        if only_integer:
            arr = np.load(str(f), mmap_mode="r")
            if arr.dtype.kind not in "iu":
                continue
        b, a = compress_npy(f, codec)
        before += b
        after += a
    return before, after


def load_npy_sqe(path: str | Path) -> np.ndarray:
    import io

    return np.load(io.BytesIO(decompress_bytes(Path(path).read_bytes())))


# ----------------------------------------------------------------------------- DFloat11
DF11_MAGIC = b"SQDF11\x01"


def df11_encode(x) -> bytes:
    """Lossless compression of bf16 values in the DFloat11 manner (Zhang et al., 2025): the
    8 exponent bits of each value are entropy-coded (rANS over their histogram; a trained
    model's exponents carry ~2.6 bits), the sign and 7 mantissa bits stay raw, so a tensor
    takes ~11 bits per value. Layout: magic, u64 count, 256 u32 exponent frequencies, u64
    coded length, coded exponents, then one byte (sign << 7 | mantissa) per value."""
    t = torch.as_tensor(x).detach().to(torch.bfloat16).contiguous().view(torch.int16).reshape(-1)
    u = t.numpy().view(np.uint16)
    exp = ((u >> 7) & 0xFF).astype(np.uint8)
    sm = (((u >> 8) & 0x80) | (u & 0x7F)).astype(np.uint8)
    freqs = histogram(exp)
    coded = rans_encode(exp, freqs).tobytes()
    return (DF11_MAGIC + struct.pack("<Q", u.size) + freqs.astype(np.uint32).tobytes() +
            struct.pack("<Q", len(coded)) + coded + sm.tobytes())


def df11_decode(blob: bytes) -> np.ndarray:
    """Inverse of ``df11_encode``: float32 values (exactly the bf16 inputs)."""
    if not blob.startswith(DF11_MAGIC):
        if blob[:1] == b"\x80":
            raise ValueError("this __pt_df11 blob is a Python pickle (written by a compressor module that is not "
                             "part of the reference release); pickles are never loaded here. Re-convert the "
                             "checkpoint with plain passthrough or `squish compress --df11`.")
        raise ValueError("not a DFloat11 blob")
    off = len(DF11_MAGIC)
    (n,) = struct.unpack_from("<Q", blob, off)
    off += 8
    freqs = np.frombuffer(blob, dtype=np.uint32, count=256, offset=off).astype(np.int64)
    off += 1024
    (clen,) = struct.unpack_from("<Q", blob, off)
    off += 8
    exp = rans_decode(np.frombuffer(blob, dtype=np.uint8, count=clen, offset=off), freqs, n).astype(np.uint16)
    off += clen
    sm = np.frombuffer(blob, dtype=np.uint8, count=n, offset=off).astype(np.uint16)
    u = ((sm & 0x80) << 8) | (exp << 7) | (sm & 0x7F)
    return (u.astype(np.uint32) << 16).view(np.float32)
