"""Host-RAM and disk tiers behind the device prefix cache (CPU engine).

A prompt's cached blocks are pushed out of a small device pool by other requests; when a
request with the same prefix arrives, its blocks come back from the host tier (or from the
disk tier, also in a new engine) and the output equals a fresh computation.
"""
import json

import numpy as np

from squish_b200.engine.engine import EngineConfig, LLMEngine
from squish_b200.engine.sampling import SamplingParams
from squish_b200.models.config import get_preset
from squish_b200.models.weights import random_checkpoint


def _eng(**kw):
    cfg, q = get_preset("tiny-llama")
    ck = random_checkpoint(cfg, q, seed=0)
    return LLMEngine.from_checkpoint(ck, "cpu", EngineConfig(max_num_seqs=2, max_num_batched_tokens=128,
                                                             max_model_len=256, num_pages=24, cuda_graphs=False,
                                                             **kw))


SP = SamplingParams(max_tokens=6, ignore_eos=True)


def _workload(eng, rng):
    shared = rng.integers(0, 32000, 96).tolist()  # 6 full blocks
    first = eng.generate([shared + [11, 12, 13]], SP)[0]
    for _ in range(4):  # fill the 24-page pool with unrelated prompts, evicting the shared blocks
        eng.generate([rng.integers(0, 32000, 150).tolist()], SP)
    return shared


def test_host_tier_restores_evicted_prefix():
    rng = np.random.default_rng(0)
    eng = _eng(kv_host_bytes=64 << 20)
    shared = _workload(eng, rng)
    assert eng.blocks.tier.stats["offloaded"] > 0
    prompt = shared + [21, 22]
    out = eng.generate([prompt], SP)[0]
    assert eng.blocks.tier_hits >= 6 and eng.blocks.tier.stats["restored_host"] >= 6
    fresh = _eng().generate([prompt], SP)[0]
    assert out == fresh


def test_disk_tier_persists_across_engines(tmp_path):
    rng = np.random.default_rng(1)
    d = tmp_path / "kv"
    eng = _eng(kv_host_bytes=1, kv_disk_dir=str(d))  # host tier of 1 byte: everything spills
    shared = _workload(eng, rng)
    eng.close()
    assert eng.blocks.tier.stats["spilled"] > 0 and list(d.glob("*.npz"))
    man = json.loads((d / "manifest.json").read_text())
    assert man["page_size"] == 16 and man["kv_dtype"] == "int4"
    eng2 = _eng(kv_host_bytes=1, kv_disk_dir=str(d))  # a restarted server
    prompt = shared + [5]
    out = eng2.generate([prompt], SP)[0]
    assert eng2.blocks.tier.stats["restored_disk"] >= 6
    assert out == _eng().generate([prompt], SP)[0]
    # a directory written for another layout is ignored, not misread
    man["page_size"] = 32
    (d / "manifest.json").write_text(json.dumps(man))
    eng3 = _eng(kv_host_bytes=1, kv_disk_dir=str(d))
    assert not eng3.blocks.tier.disk


def test_kv_mode_selection_and_memory_planning():
    import pytest

    from squish_b200.kv.paged import KVPools
    from squish_b200.kv.planning import (estimate_kv_memory, estimate_max_context, recommended_kv_mode,
                                         recommended_kv_mode_3tier)
    from squish_b200.models.config import QuantConfig, get_preset

    assert recommended_kv_mode(4096) == "int8" and recommended_kv_mode(16384) == "int2"
    assert [recommended_kv_mode_3tier(n) for n in (8192, 8193, 16384, 16385)] == ["int8", "int4", "int4", "int2"]
    with pytest.raises(ValueError):
        recommended_kv_mode(10, medium_mode="int4")
    cfg, q = get_preset("tiny-llama")
    for mode in ("bf16", "int8", "int4", "int2", "k8v4"):
        est = estimate_kv_memory(cfg, 1000, mode, sequences=3)
        qq = QuantConfig(**{**q.__dict__, "kv_dtype": mode})
        pools = KVPools(cfg, qq, est.pages, "cpu")
        assert pools.nbytes() == est.total_bytes, mode  # the estimate is the allocation
        n = estimate_max_context(cfg, est.total_bytes, mode, sequences=3)
        assert n >= 1000 and estimate_kv_memory(cfg, n, mode, 3).total_bytes <= est.total_bytes
    e8, e2 = estimate_kv_memory(cfg, 4096, "int8"), estimate_kv_memory(cfg, 4096, "int2")
    assert e2.total_bytes < e8.total_bytes / 2.5


def test_saved_session_restores_in_a_new_engine(tmp_path):
    """A conversation saved explicitly (no eviction needed) is restored from disk by a restarted
    engine: its blocks come back instead of being recomputed, and the continuation equals a
    fresh computation."""
    rng = np.random.default_rng(2)
    d = tmp_path / "kv"
    eng = _eng(kv_host_bytes=1 << 20, kv_disk_dir=str(d))
    prompt = rng.integers(0, 32000, 70).tolist()
    out = eng.generate([prompt], SP)[0]
    convo = prompt + out  # 76 tokens: 4 full blocks
    assert eng.save_session(convo) == 4
    assert eng.save_session(convo) == 0  # already saved
    assert len(list(d.glob("*.npz"))) >= 4
    eng2 = _eng(kv_host_bytes=1 << 20, kv_disk_dir=str(d))
    follow = convo + [7, 8, 9]
    got = eng2.generate([follow], SP)[0]
    assert eng2.blocks.tier.stats["restored_disk"] >= 4
    assert got == _eng().generate([follow], SP)[0]
