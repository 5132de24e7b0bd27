"""Device tile layout of the GEMM's weight formats (INT4, NF4, INT8, INT2): a host emulation
of the kernel's decode of every tile must give back the codec's dequantized weight."""
import numpy as np
import pytest
import torch

from squish_b200.ops import kernels as K
from squish_b200.quant.codecs import quantize

NF4 = torch.tensor([-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453, -0.28444138169288635,
                    -0.18477343022823334, -0.09105003625154495, 0.0, 0.07958029955625534, 0.16093020141124725,
                    0.24611230194568634, 0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
                    0.7229568362236023, 1.0])
CODE_WORDS = {K.WF_INT4: 1024, K.WF_NF4: 1024, K.WF_INT8: 2048, K.WF_INT2: 512, K.WF_INT3: 768, K.WF_AQLM: 512}


def _bf16(bits):
    return (bits.to(torch.int32) << 16).view(torch.float32).to(torch.bfloat16).float()


def emulate(wt, fmt, n, k, group, books=None):
    """What the kernel's dequant warps produce for every weight (bf16 rounding included)."""
    rb, kb, _ = wt.shape
    gpk = 1 if group >= 64 else 64 // group
    w = wt.to(torch.int64) & 0xFFFFFFFF
    nw = CODE_WORDS[fmt]
    codes = w[..., :nw].reshape(rb, kb, 2, 128, nw // 256)
    aux = w[..., nw:].reshape(rb, kb, gpk, 128)
    out = torch.zeros(rb * 128, kb * 64)
    for c in range(2):
        for ch in range(4):  # 8-value chunk within the 32 values of part c
            g = ((c * 4 + ch) * gpk) >> 3
            sw = aux[:, :, g, :]  # [rb, kb, 128]
            s = _bf16(sw & 0xFFFF)
            z = _bf16(sw >> 16)
            if fmt == K.WF_AQLM:  # chunk ch = one 8-column group; books[k][idx] summed, times scale
                word = codes[:, :, c, :, ch // 2]
                idx = (word >> (16 * (ch % 2))) & 0xFFFF
                acc = books[0][idx & 0xFF].float()
                if books.shape[0] > 1:
                    acc = (acc + books[1][(idx >> 8) & 0xFF].float()).to(torch.bfloat16).float()
                vals = (acc * s[..., None]).to(torch.bfloat16).float()  # [rb, kb, 128, 8]
                for j in range(8):
                    out.view(rb, 128, kb, 64)[:, :, :, c * 32 + ch * 8 + j] = vals[..., j].permute(0, 2, 1)
                continue
            for j in range(8):
                if fmt == K.WF_INT3:
                    p_ = ch * 4 + j // 2
                    if p_ < 15:
                        word = codes[:, :, c, :, p_ // 5]
                        q = (word >> ((j % 2) * 16 + 3 * (p_ % 5))) & 7
                    else:
                        q = sum(((codes[:, :, c, :, b] >> (15 + 16 * (j % 2))) & 1) << b for b in range(3))
                    q = q - 4
                elif fmt in (K.WF_INT4, K.WF_NF4):
                    word = codes[:, :, c, :, ch]
                    q = (word >> K._NIB_POS[j]) & 0xF
                elif fmt == K.WF_INT2:
                    word = codes[:, :, c, :, ch // 2]
                    jj = (ch % 2) * 8 + j
                    q = (word >> ((jj % 2) * 16 + (jj // 2) * 2)) & 3
                else:
                    word = codes[:, :, c, :, 2 * ch + j // 4]
                    q = (word >> (8 * (j % 4))) & 0xFF
                    q = torch.where(q >= 128, q - 256, q)
                if fmt == K.WF_NF4:
                    v = (NF4[q].to(torch.bfloat16).float() * s).to(torch.bfloat16).float()
                elif fmt == K.WF_INT8:
                    v = (q.float() * s).to(torch.bfloat16).float()
                else:
                    v = (q.float() * s + z).to(torch.bfloat16).float()
                col = c * 32 + ch * 8 + j
                out.view(rb, 128, kb, 64)[:, :, :, col] = v.permute(0, 2, 1)
    return out[:n, :k]


@pytest.mark.parametrize("kind,fmt,group", [("nf4", K.WF_NF4, 64), ("q8", K.WF_INT8, 64), ("q8", K.WF_INT8, 32),
                                            ("q2", K.WF_INT2, 64), ("q2", K.WF_INT2, 128), ("nf4", K.WF_NF4, 32)])
def test_tile_layout_round_trip(kind, fmt, group):
    g = torch.Generator().manual_seed(group)
    w = torch.randn(300, 384, generator=g) * 0.05
    t = quantize(w, kind, group)
    dw = K.prepare_weight(t, "cpu")
    assert dw.fmt == fmt and dw.wq.shape[-1] == CODE_WORDS[fmt] + (1 if t.group >= 64 else 64 // t.group) * 128
    got = emulate(dw.wq, fmt, 300, 384, t.group)
    want = t.dequantize().float().to(torch.bfloat16).float()
    # one bf16 rounding of the scale/zero/product separates the two
    torch.testing.assert_close(got, want, atol=2e-3, rtol=2e-2)


def test_int4_codes_layout_matches_emulation():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(256, 128, generator=g) * 0.05
    t = quantize(w, "q4a", 64)
    p = t.packed
    codes = torch.stack([p & 0xF, p >> 4], dim=-1).reshape(256, -1)
    wt = K.repack_codes(codes, t.scales, t.offsets, 128, 64, K.WF_INT4)
    got = emulate(wt, K.WF_INT4, 256, 128, 64)
    torch.testing.assert_close(got, t.dequantize().float(), atol=3e-3, rtol=2e-2)


def test_int3_tile_layout():
    g = torch.Generator().manual_seed(3)
    w = torch.randn(200, 256, generator=g) * 0.05
    t = quantize(w, "q3", 64)
    dw = K.prepare_weight(t, "cpu")
    assert dw.fmt == K.WF_INT3
    got = emulate(dw.wq, K.WF_INT3, 200, 256, 64)
    torch.testing.assert_close(got, t.dequantize().float(), atol=2e-3, rtol=2e-2)


def test_aqlm_tile_layout():
    from squish_b200.quant.aqlm import aqlm_quantize

    g = torch.Generator().manual_seed(4)
    w = torch.randn(130, 192, generator=g) * 0.05
    t = aqlm_quantize(w, n_codebooks=2, codebook_size=256, group_size=8, iters=3)
    dw = K.prepare_weight(t, "cpu")
    assert dw.fmt == K.WF_AQLM and dw.codebook.shape == (2, 256, 8)
    got = emulate(dw.wq, K.WF_AQLM, 130, 192, 64, books=dw.codebook)
    torch.testing.assert_close(got, t.dequantize().float(), atol=4e-3, rtol=3e-2)
