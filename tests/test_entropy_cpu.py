"""Host entropy codecs (rANS, Huffman) and the .npy.sqe container: round trips, ratios, errors."""
import numpy as np
import pytest

from squish_b200.io import entropy as E


def _skewed(n, seed=0):
    rng = np.random.default_rng(seed)
    return np.clip(rng.geometric(0.25, n), 0, 255).astype(np.uint8)


@pytest.mark.parametrize("n", [1, 7, 1000, 100_000])
def test_rans_round_trip(n):
    x = _skewed(n, n)
    f = E.histogram(x)
    enc = E.rans_encode(x, f)
    assert np.array_equal(E.rans_decode(enc, f, n), x)


def test_rans_compresses_near_entropy():
    x = _skewed(200_000)
    f = E.histogram(x).astype(np.float64)
    p = f[f > 0] / f.sum()
    h_bytes = -(p * np.log2(p)).sum() * x.size / 8
    enc = E.rans_encode(x, E.histogram(x))
    assert enc.size < 1.02 * h_bytes + 64


def test_rans_uniform_and_single_symbol():
    rng = np.random.default_rng(3)
    x = rng.integers(0, 256, 50_000).astype(np.uint8)
    f = E.histogram(x)
    assert np.array_equal(E.rans_decode(E.rans_encode(x, f), f, x.size), x)
    y = np.full(5000, 42, np.uint8)
    fy = E.histogram(y)
    enc = E.rans_encode(y, fy)
    assert enc.size <= 16 and np.array_equal(E.rans_decode(enc, fy, y.size), y)


def test_rans_rejects_symbol_without_frequency():
    f = np.zeros(256, np.uint32)
    f[1] = 10
    with pytest.raises(ValueError):
        E.rans_encode(np.array([1, 2], np.uint8), f)


@pytest.mark.parametrize("n", [1, 999, 100_000])
def test_huffman_round_trip_and_canonical(n):
    x = _skewed(n, 7)
    w, ln = E.huffman_build(E.histogram(x))
    # Kraft equality for a complete code (more than one symbol present)
    present = ln > 0
    if present.sum() > 1:
        assert abs(np.sum(2.0 ** -ln[present].astype(np.float64)) - 1.0) < 1e-9
    enc = E.huffman_encode(x, w, ln)
    assert np.array_equal(E.huffman_decode(enc, w, ln, n), x)


def test_huffman_long_codes_use_trie():
    # Fibonacci-like histogram forces code lengths above 16 bits
    f = np.zeros(256, np.uint32)
    a, b = 1, 1
    for s in range(22):
        f[s] = a
        a, b = b, a + b
    w, ln = E.huffman_build(f)
    assert ln.max() > 16
    x = np.repeat(np.arange(22, dtype=np.uint8), 3)
    assert np.array_equal(E.huffman_decode(E.huffman_encode(x, w, ln), w, ln, x.size), x)


def test_huffman_rejects_non_prefix_code():
    w = np.zeros(256, np.uint32)
    ln = np.zeros(256, np.uint8)
    w[0], ln[0] = 0b1, 1
    w[1], ln[1] = 0b10, 2  # "1" is a prefix of "10"
    with pytest.raises(RuntimeError):
        E.huffman_decode(np.array([0xFF], np.uint8), w, ln, 1)


@pytest.mark.parametrize("codec", [E.RANS, E.HUFFMAN])
def test_container_and_npy_dir(tmp_path, codec):
    rng = np.random.default_rng(1)
    q = np.clip(np.round(rng.normal(0, 12, (64, 96))), -127, 127).astype(np.int8)
    s = rng.random((64, 3)).astype(np.float16)
    np.save(tmp_path / "w__q.npy", q)
    np.save(tmp_path / "w__s.npy", s)
    before, after = E.compress_npy_dir(tmp_path, codec)
    assert after < before  # the int8 codes shrink
    assert (tmp_path / "w__q.npy.sqe").exists() and (tmp_path / "w__s.npy").exists()
    from squish_b200.io.npy_dir import _load

    assert np.array_equal(_load(tmp_path / "w__q.npy"), q)
    assert E.decompress_bytes(E.compress_bytes(b"", codec)) == b""
