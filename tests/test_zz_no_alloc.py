"""The allocation-free decode-attention entry point, called through its exported C symbol.

Some callers of this library cannot allocate device memory (a plug-in that lives inside a
host application's memory budget, or a binding that can only hand over pointers), so
``sq_paged_decode_attention_noalloc`` keeps its split-K partials in a fixed device array.
This test calls it through ctypes, twice in a row on different inputs, and checks each
result against the regular entry point (which uses a caller-provided workspace). Both run
the same kernel on the same inputs with the same split plan, so the outputs must be equal
bit for bit. It lives in its own file, named to be collected last, and needs nothing from
the other test files.
"""
import ctypes
import math

import pytest
import torch

import squish_b200._C as _C
from squish_b200 import ops
from squish_b200._ext import native

pytestmark = pytest.mark.gpu

SQ_NOALLOC_TOO_LARGE = -1
SQ_NOALLOC_BAD_ARGUMENT = -2


def _lib():
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.sq_paged_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = ([ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 5 + [ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_int] + [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p])
    err = lib.sq_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _case(seed, lens, hq, hkv, d, group, kvfmt, dev):
    """Random INT4 (or k8v4) page pools written through the C++ codec, a page table, queries."""
    g = torch.Generator().manual_seed(seed)
    fk, fv = ops.KV_FORMATS[kvfmt]
    ps = 16
    pages = [math.ceil(n / ps) for n in lens]
    npg = sum(pages) + 1
    pools = []
    for fmt in (fk, fv):
        rows = npg * hkv * ps
        x = torch.randn(rows, d, generator=g)
        c, s = native().cpu.kv_quantize(x, fmt, group)
        pools += [c.reshape(npg, hkv, ps, -1).contiguous().to(dev),
                  s.to(torch.float16).reshape(npg, hkv, ps, -1).contiguous().to(dev)]
    perm = torch.randperm(npg, generator=g)
    bt = torch.zeros(len(lens), max(pages), dtype=torch.int32)
    o = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[o:o + n].to(torch.int32)
        o += n
    q = (torch.randn(len(lens), hq * d, generator=g)).to(torch.bfloat16).to(dev)
    return q, pools, bt.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev), fk, fv


def _run_noalloc(fn, q, pools, bt, lens, out, hq, hkv, d, group, fk, fv, splits, tps):
    kc, ks, vc, vs = pools
    stream = torch.cuda.current_stream().cuda_stream
    return fn(q.data_ptr(), q.stride(0), kc.data_ptr(), ks.data_ptr(), vc.data_ptr(), vs.data_ptr(), bt.data_ptr(),
              bt.stride(0), lens.data_ptr(), lens.shape[0], out.data_ptr(), out.stride(0), hq, hkv, d, 16, group, fk,
              fv, 1.0 / math.sqrt(d), splits, tps, stream)


def test_noalloc_decode_matches_workspace_entry_point(cuda):
    fn, err = _lib()
    cases = [(1, [300, 17, 1000], 28, 4, 128, 32, "int4"), (2, [2048, 64, 5, 129], 16, 2, 128, 64, "k8v4")]
    for seed, lens, hq, hkv, d, group, kvfmt in cases:  # two calls in a row on the shared scratch
        q, pools, bt, sl, fk, fv = _case(seed, lens, hq, hkv, d, group, kvfmt, cuda)
        splits, tps = ops.kernels.decode_splits(len(lens), hkv, max(lens))
        assert splits > 1, "the case must exercise the split-K partials"
        want = torch.empty_like(q)
        ops.paged_decode_attention(q, *pools, bt, sl, want, hq, hkv, d, 16, group, fk, fv, 1.0 / math.sqrt(d),
                                   max(lens), splits=(splits, tps))
        got = torch.full_like(q, float("nan"))
        rc = _run_noalloc(fn, q, pools, bt, sl, got, hq, hkv, d, group, fk, fv, splits, tps)
        assert rc == 0, err(rc)
        torch.cuda.synchronize()
        assert torch.equal(got, want)


def _call(fn, q, pools, bt, sl, out, B, hq, hkv, d, page, group, fk, fv, splits, tps, ld_q=None, ld_out=None):
    return fn(q.data_ptr(), q.stride(0) if ld_q is None else ld_q, pools[0].data_ptr(), pools[1].data_ptr(),
              pools[2].data_ptr(), pools[3].data_ptr(), bt.data_ptr(), bt.stride(0), sl.data_ptr(), B, out.data_ptr(),
              out.stride(0) if ld_out is None else ld_out, hq, hkv, d, page, group, fk, fv, 0.1, splits, tps,
              torch.cuda.current_stream().cuda_stream)


def test_noalloc_rejects_oversized_requests(cuda):
    fn, err = _lib()
    # one sequence, 8 query heads of 128 dims: every tensor is valid for the shapes passed,
    # but 1 * 8 * 1025 splits * 128 partial floats exceed the fixed scratch
    q, pools, bt, sl, fk, fv = _case(3, [64], 8, 2, 128, 32, "int4", cuda)
    out = torch.full_like(q, 7.0)
    rc = _call(fn, q, pools, bt, sl, out, 1, 8, 2, 128, 16, 32, fk, fv, 1025, 1)
    assert rc == SQ_NOALLOC_TOO_LARGE
    assert b"too large" in err(rc)
    torch.cuda.synchronize()
    assert bool((out == 7.0).all()), "nothing may be launched for a rejected request"


def test_noalloc_rejects_shapes_the_kernel_does_not_handle(cuda):
    fn, err = _lib()
    q, pools, bt, sl, fk, fv = _case(4, [40], 8, 2, 128, 32, "int4", cuda)
    out = torch.full_like(q, 7.0)
    good = dict(B=1, hq=8, hkv=2, d=128, page=16, group=32, fk=fk, fv=fv, splits=1, tps=4)
    bad = [dict(hkv=0), dict(hkv=3), dict(hq=8, hkv=0), dict(page=24), dict(page=0), dict(tps=0), dict(splits=0),
           dict(d=96), dict(group=16), dict(group=48), dict(fk=2, fv=5), dict(fk=9, fv=9)]
    for change in bad:
        args = {**good, **change}
        rc = _call(fn, q, pools, bt, sl, out, args["B"], args["hq"], args["hkv"], args["d"], args["page"],
                   args["group"], args["fk"], args["fv"], args["splits"], args["tps"])
        assert rc == SQ_NOALLOC_BAD_ARGUMENT, (change, rc)
        assert b"invalid argument" in err(rc)
    # more than 16 query heads per KV head (the kernel's per-warp row limit)
    q2, pools2, bt2, sl2, fk2, fv2 = _case(5, [40], 34, 2, 128, 32, "int4", cuda)
    out2 = torch.full_like(q2, 7.0)
    assert _call(fn, q2, pools2, bt2, sl2, out2, 1, 34, 2, 128, 16, 32, fk2, fv2, 1, 4) == SQ_NOALLOC_BAD_ARGUMENT
    # a row stride shorter than Hq * D
    assert _call(fn, q, pools, bt, sl, out, 1, 8, 2, 128, 16, 32, fk, fv, 1, 4, ld_q=512) == SQ_NOALLOC_BAD_ARGUMENT
    torch.cuda.synchronize()
    assert bool((out == 7.0).all()) and bool((out2 == 7.0).all()), "nothing may be launched for a rejected request"
    # the same buffers with the good arguments do run
    assert _call(fn, q, pools, bt, sl, out, **good) == 0
    torch.cuda.synchronize()
    assert bool(torch.isfinite(out.float()).all()) and not bool((out == 7.0).all())
