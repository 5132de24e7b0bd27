"""A quantized KV cache for Hugging Face transformers models (``past_key_values=SquishCache(...)``).

The reference's SquishCache (squish/integrations/hf.py:62-240) lets an HF model keep its KV cache
in squish's quantized formats. Here it is a ``transformers`` ``Cache`` whose layers are
``QuantizedLayer`` s (a recent window kept in the model's dtype, older tokens quantized) with
this package's KV codecs -- per-token, per-group INT8 / INT4 / INT2 / k8v4, the same page
formats the CUDA engine stores -- computed by the C++ library (``_C.cpu.kv_quantize``).
"""
from __future__ import annotations

import torch
from transformers.cache_utils import Cache, QuantizedLayer

from .._ext import native
from ..ops.kernels import KV_FORMATS


class SquishKVLayer(QuantizedLayer):
    def __init__(self, kv_dtype: str = "int4", group: int = 32, residual_length: int = 128):
        fk, fv = KV_FORMATS[kv_dtype]
        super().__init__(nbits=8, q_group_size=group, residual_length=residual_length)
        self.fmt_k, self.fmt_v = fk, fv
        self._next_is_key = True

    def _quantize(self, tensor: torch.Tensor, axis: int):
        # QuantizedLayer quantizes keys, then values, each time; the formats follow that order
        fmt = self.fmt_k if self._next_is_key else self.fmt_v
        self._next_is_key = not self._next_is_key
        d = tensor.shape[-1]
        x = tensor.detach().float().reshape(-1, d).cpu().contiguous()
        if fmt == 0:
            return (x.to(torch.bfloat16), None, fmt, tensor.shape, tensor.dtype, tensor.device)
        codes, scales = native().cpu.kv_quantize(x, fmt, self.q_group_size)
        return (codes, scales, fmt, tensor.shape, tensor.dtype, tensor.device)

    def _dequantize(self, q) -> torch.Tensor:
        codes, scales, fmt, shape, dtype, device = q
        if fmt == 0:
            x = codes.float()
        else:
            x = native().cpu.kv_dequantize(codes, scales, fmt, self.q_group_size, shape[-1])
        return x.reshape(shape).to(device=device, dtype=dtype)


class SquishCache(Cache):
    """``SquishCache(model.config, kv_dtype="int4")``: one quantized layer per decoder layer."""

    def __init__(self, config, kv_dtype: str = "int4", group: int = 32, residual_length: int = 128):
        if kv_dtype not in KV_FORMATS:
            raise ValueError(f"kv_dtype must be one of {sorted(KV_FORMATS)}")
        n = config.get_text_config(decoder=True).num_hidden_layers
        super().__init__(layers=[SquishKVLayer(kv_dtype, group, residual_length) for _ in range(n)])
