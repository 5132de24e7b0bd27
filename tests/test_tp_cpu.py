"""Tensor parallelism on CPU ranks (gloo, world size 2): the sharded engine must produce
the oracle's tokens. Each rank runs the same engine host logic (SPMD)."""
import dataclasses
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from squish_b200.engine.engine import EngineConfig, LLMEngine
from squish_b200.engine.sampling import SamplingParams
from squish_b200.models.config import get_preset
from squish_b200.models.reference import ReferenceModel
from squish_b200.models.weights import random_checkpoint


def _cfg(preset="tiny-llama"):
    cfg, q = get_preset(preset)
    if preset == "tiny-moe":
        return dataclasses.replace(cfg, tie_embeddings=False), q
    return dataclasses.replace(cfg, tie_embeddings=False, intermediate_size=512), q


def _prompts(vocab):
    rng = np.random.default_rng(7)
    return [rng.integers(0, vocab, 23).tolist(), rng.integers(0, vocab, 40).tolist()]


def _worker(rank, world, port, q, preset="tiny-llama", mode="nvlink"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, qc = _cfg(preset)
        ck = random_checkpoint(cfg, qc, seed=0)
        eng = LLMEngine.from_checkpoint(ck, "cpu", EngineConfig(max_num_seqs=4, max_num_batched_tokens=64,
                                                                max_model_len=256, num_pages=64, tp=world,
                                                                tp_mode=mode))
        outs = eng.generate(_prompts(cfg.vocab_size), SamplingParams(max_tokens=10, ignore_eos=True))
        sampled = eng.generate(_prompts(cfg.vocab_size)[:1], SamplingParams(max_tokens=6, temperature=0.9,
                                                                            ignore_eos=True))
        q.put((rank, outs, sampled))
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,preset,mode", [(2, "tiny-llama", "nvlink"), (2, "tiny-moe", "nvlink"),
                                               (2, "tiny-moe", "sp")])
def test_tp_engine_matches_single_process(world, preset, mode):
    """mode "sp" with a MoE model: the expert all-to-all layout (routing of owned rows, slots
    with local ids or -1, weighted sums returned to the owners) on gloo ranks."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, preset, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(world)])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every rank emitted the same tokens (replicated host logic)
    assert all(r[1] == res[0][1] and r[2] == res[0][2] for r in res)
    cfg, qc = _cfg(preset)
    ref = ReferenceModel(random_checkpoint(cfg, qc, seed=0))
    from .test_engine_gpu import _teacher_forced_ok

    for p, o in zip(_prompts(cfg.vocab_size), res[0][1]):
        ok, worst = _teacher_forced_ok(ref, p, o, tol=1e-4)
        assert ok, (worst, o)
