"""The host C++ libraries under AddressSanitizer + UndefinedBehaviorSanitizer with randomized and
malformed inputs: entropy decoders fed arbitrary bytes and truncated streams, the JSON /
JSON-schema matchers fed random token sequences and random schemas, the CPU codecs and the
research codec / KV score kernels fed odd shapes, extreme values and bad arguments, the n-gram
index and loop detector fed random token streams. Any
sanitizer report (out-of-bounds access, use after free, signed overflow, misaligned load ...)
ends the child process with a non-zero status and fails the test."""
import pytest

FUZZ = r'''
import numpy as np, torch
import squish_b200._ext as ext
import _C_host_asan as M
ext._C = M  # every wrapper below calls the sanitized module
from squish_b200.io import entropy as E
from squish_b200.serving import grammar as G
rng = np.random.default_rng(12345)
C = M.cpu

# ---- entropy codecs: round trips, then arbitrary and truncated streams
for n in [0, 1, 2, 17, 1000, 65536]:
    sym = rng.integers(0, rng.integers(1, 256), n).astype(np.uint8)
    for codec in (E.RANS, E.HUFFMAN):
        blob = E.compress_bytes(sym.tobytes(), codec)
        assert E.decompress_bytes(blob) == sym.tobytes()
        for cut in (len(blob) // 2, len(blob) - 1, 8):
            try:
                E.decompress_bytes(blob[:cut])
            except Exception:
                pass
for _ in range(300):
    freqs = rng.integers(0, 50, 256)
    data = rng.integers(0, 256, rng.integers(0, 200)).astype(np.uint8)
    n = int(rng.integers(0, 500))
    for f in (E.rans_decode, lambda d, fr, k: E.huffman_decode(d, *E.huffman_build(fr), k)):
        try:
            f(data, freqs, n)
        except Exception:
            pass
    try:
        E.decompress_bytes(bytes(data))
    except Exception:
        pass
x = (torch.randn(37, 41) * 0.02).to(torch.bfloat16)
assert np.array_equal(E.df11_decode(E.df11_encode(x)), x.float().numpy().reshape(-1))

# ---- JSON / JSON-schema matchers over a random byte vocabulary
toks = [bytes(rng.integers(32, 127, rng.integers(1, 5)).astype(np.uint8)) for _ in range(300)]
toks += [b"{", b"}", b"[", b"]", b'"', b":", b",", b" ", b"true", b"null", b"-1", b"0.5e3", b"\\", b'\\"', b"\xc3\xa9"]
index = M.grammar.VocabIndex(toks + [b""], len(toks))
schemas = [
    {"type": "object", "properties": {"a": {"type": "integer"}, "b": {"type": "array", "items": {"type": "string"}}},
     "required": ["a"]},
    {"anyOf": [{"type": "number"}, {"type": "object", "properties": {"z": {"enum": ["x", 1, None]}}}]},
    {"type": "array", "items": {"$ref": "#/$defs/n"}, "$defs": {"n": {"type": ["null", "boolean"]}}},
    {"type": "object", "properties": {"deep": {"type": "object", "properties": {"deeper": {"type": "array",
     "items": {"type": "object"}}}}}},
]
matchers = [lambda: M.grammar.JsonMatcher(index, True), lambda: M.grammar.JsonMatcher(index, False)]
for sc in schemas:
    compiled = G.compile_schema(sc)
    matchers.append(lambda c=compiled: M.grammar.SchemaMatcher(index, c))
for mk in matchers:
    for trial in range(40):
        m = mk()
        for step in range(60):
            mask = m.allowed_mask().numpy().view(np.uint32)
            bits = np.unpackbits(mask.view(np.uint8), bitorder="little")[: len(toks) + 1]
            allowed = np.flatnonzero(bits)
            pick = int(rng.choice(allowed)) if len(allowed) and rng.random() < 0.9 else int(rng.integers(0, len(toks) + 1))
            ok = m.advance(pick)
            if m.is_terminated():
                break
# ---- CPU codecs: odd shapes, zeros, huge values
for shape in [(1, 2), (3, 64), (5, 96), (2, 4096)]:
    for scale in (0.0, 1e-30, 1.0, 3e4):
        w = torch.randn(*shape) * scale
        if shape[1] % 2 == 0:
            for g in (2, shape[1]):
                try:
                    p, s, o = C.quantize_int4_asym(w, g)
                    C.dequantize_int4_asym(p, s, o, g)
                except Exception:
                    pass
        for g in (0, shape[1]):
            try:
                q, s = C.quantize_int8(w, g)
            except Exception:
                pass
        for fmt in (1, 2, 3, 4, 5):
            for grp in (shape[1], 2):
                try:
                    c, s = C.kv_quantize(w, fmt, grp)
                    C.kv_dequantize(c, s, fmt, grp, shape[1])
                except Exception:
                    pass
        n4 = (w.numel() // 4) * 4
        try:
            C.fp6_decode(C.fp6_encode(w.reshape(-1)[:n4].contiguous(), 3, 2), n4, 3, 2)
        except Exception:
            pass
# ---- research codecs and KV scores: odd shapes, degenerate values, bad arguments
for shape in [(1, 2), (3, 64), (4, 96)]:
    for scale in (0.0, 1.0, 3e4):
        w = torch.randn(*shape) * scale
        for call in (lambda: C.any4_quantize(w, 2, 3, 1), lambda: C.any4_quantize(w, 5, 3, 1),
                     lambda: C.quarot_group_quant(w, 7, 7.0, True), lambda: C.quarot_group_quant(w, 3, 1.0, False),
                     lambda: C.bit_distiller_quant(w, 8, 5), lambda: C.gguf_mixed_quant(w, 3, 64),
                     lambda: C.flute_lut_encode(w, torch.randn(shape[1], 4), 1),
                     lambda: C.flute_lut_decode(torch.full(shape, 9, dtype=torch.uint8), torch.randn(shape[1], 4), 1),
                     lambda: C.qmoe_compress(w, 3, 4), lambda: C.any4_lloyd(w.reshape(-1), torch.randn(16), 5, 2),
                     lambda: C.adaround_step(w, w, w, w, 0.1, 2.0, 0.01, 1.1, -0.1),
                     lambda: C.batched_cosine_similarity(w, w), lambda: C.gru_step(w.reshape(-1)[:3], w.reshape(-1)[:3],
                                                                                  w.reshape(-1)[:1]),
                     lambda: C.cluster_kv_score(torch.randint(0, 5, (shape[1],)), w[0], 4),
                     lambda: C.green_kv_score(w[None], w[None]), lambda: C.cake_entropy(w[None], w[None], 1.0),
                     lambda: C.magic_pig_attention(w[None], w[None], w[None], 3, 5, 0),
                     lambda: C.mamba2_scan(w[0], w.T, w.T, w[0], w[0, :1].repeat(shape[0])),
                     lambda: C.hawk_scan(w, w, w[0], w[0]), lambda: C.delta_net_scan(w[None], w[None], w[None], w[:1]),
                     lambda: C.ternary_gemv(torch.randint(-2, 3, shape, dtype=torch.int8), w[0], 1.0),
                     lambda: C.sparse_act_gemv(w, w[0], 0.5)):
            try:
                call()
            except Exception:
                pass
# ---- serving helpers: loop detector and n-gram index on random streams
for _ in range(100):
    t = rng.integers(0, 20, rng.integers(0, 400)).tolist()
    M.host.detect_token_loop(t)
    idx = M.host.NGramIndex(1, 4)
    idx.extend(t)
    idx.continuations(4, 3)
print("FUZZ-OK")
'''


@pytest.mark.slow
def test_host_libraries_under_address_and_ub_sanitizers():
    from squish_b200 import sanitize

    try:
        sanitize.compiler()
    except RuntimeError as exc:
        pytest.skip(str(exc))
    r = sanitize.run(FUZZ, timeout=1200)
    tail = (r.stdout[-3000:] + "\n" + r.stderr[-6000:])
    assert r.returncode == 0 and "FUZZ-OK" in r.stdout, tail
    assert "runtime error" not in r.stderr and "AddressSanitizer" not in r.stderr, tail
