"""CUDA ops of squish_b200 (sm_100a kernels) and their host-side plumbing."""
from .kernels import (  # noqa: F401
    KV_FORMATS,
    Int4Weight,
    Workspace,
    bf16_linear,
    dequant_weight,
    gemm_plan,
    paged_decode_attention,
    paged_prefill_attention,
    prepare_int4_weight,
    rmsnorm,
    rope_kv_write,
    sample,
    w4a16_linear,
    workspace,
)
