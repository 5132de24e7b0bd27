"""Host-tier KV restore on the GPU runner: device pages evicted to host RAM come back
byte-exact (checked directly), and the engine's output stays on the fp32 oracle."""
import numpy as np
import pytest
import torch

from squish_b200.engine.engine import EngineConfig, LLMEngine
from squish_b200.engine.sampling import SamplingParams
from squish_b200.models.config import get_preset
from squish_b200.models.reference import ReferenceModel
from squish_b200.models.weights import random_checkpoint

from .test_engine_gpu import _teacher_forced_ok

pytestmark = pytest.mark.gpu


def test_gpu_host_tier_round_trip(cuda):
    cfg, q = get_preset("tiny-llama")
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0), cuda, EngineConfig(
        max_num_seqs=2, max_num_batched_tokens=128, max_model_len=256, num_pages=24, kv_host_bytes=64 << 20))
    io = eng.blocks.tier.io
    before = io.read(3)
    io.write(5, before)
    assert all(np.array_equal(a, b) for a, b in zip(before, io.read(5)))
    rng = np.random.default_rng(0)
    sp = SamplingParams(max_tokens=6, ignore_eos=True)
    shared = rng.integers(0, 32000, 96).tolist()
    eng.generate([shared + [1, 2]], sp)
    for _ in range(4):
        eng.generate([rng.integers(0, 32000, 150).tolist()], sp)
    prompt = shared + [7]
    out = eng.generate([prompt], sp)[0]
    assert eng.blocks.tier.stats["restored_host"] >= 6
    ok, worst = _teacher_forced_ok(ReferenceModel(random_checkpoint(cfg, q, seed=0)), prompt, out)
    assert ok, (worst, out)
    torch.cuda.synchronize()
