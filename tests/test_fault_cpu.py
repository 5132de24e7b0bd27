"""Failure detection without a GPU fault: host-side injected faults on gloo CPU ranks.

A rank that raises, exits or freezes must make the surviving rank fail with an error in
bounded time (a PeerFailure from the heartbeat/liveness monitor, or the process group's
short timeout), never hang. Also unit tests of the monitor, the fault parser and the
engine watchdog behind ``/health``.
"""
import dataclasses
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from squish_b200.utils.fault import FaultInjector, PeerFailure, PeerMonitor, Watchdog, parse_faults


class FakeStore:
    def __init__(self):
        self.d = {}

    def set(self, k, v):
        self.d[k] = v.encode() if isinstance(v, str) else v

    def get(self, k):
        return self.d[k]

    def check(self, keys):
        return all(k in self.d for k in keys)


def test_parse_faults():
    f = parse_faults("1:3:raise, 0:5:delay:250,2:1:hang")
    assert [(x.rank, x.step, x.kind, x.arg) for x in f] == [(1, 3, "raise", 0.0), (0, 5, "delay", 250.0),
                                                             (2, 1, "hang", 0.0)]
    with pytest.raises(ValueError):
        parse_faults("1:2:explode")


def test_monitor_detects_error_lag_and_tolerates_a_dropped_beat():
    st = FakeStore()
    inj1 = FaultInjector(1, "1:2:drop")
    m0 = PeerMonitor(st, 0, 2, timeout_s=0.2, max_lag=1)
    m1 = PeerMonitor(st, 1, 2, timeout_s=0.2, max_lag=1, injector=inj1)
    for step in range(1, 4):
        inj1.before_step(step)
        m1.beat(step)
        m0.beat(step)
        m0.check()  # a single dropped heartbeat is within max_lag
    # rank 1 stops beating: rank 0 goes on and notices after timeout_s
    for step in range(4, 8):
        m0.beat(step)
        try:
            m0.check()
        except PeerFailure as exc:
            assert "stalled" in str(exc)
            break
        time.sleep(0.15)
    else:
        pytest.fail("stall not detected")
    m1.announce_error("boom")
    with pytest.raises(PeerFailure, match="boom"):
        m0.check()


def test_watchdog_flags_stalled_engine():
    pending = [True]
    wd = Watchdog(lambda: pending[0], stall_s=0.1)
    assert not wd.poll()
    time.sleep(0.15)
    assert wd.poll() and "no engine step" in wd.reason
    wd.heartbeat()
    assert not wd.degraded
    pending[0] = False
    time.sleep(0.15)
    assert not wd.poll()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, fault, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), SQUISH_FAULT=fault)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.engine.sampling import SamplingParams
    from squish_b200.models.config import get_preset
    from squish_b200.models.weights import random_checkpoint

    cfg, qc = get_preset("tiny-llama")
    cfg = dataclasses.replace(cfg, tie_embeddings=False, intermediate_size=512, num_layers=2)
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, qc, seed=0), "cpu", EngineConfig(
        max_num_seqs=2, max_num_batched_tokens=64, max_model_len=256, num_pages=64, tp=world, peer_timeout_s=3.0))
    eng.add_request(np.arange(10).tolist(), SamplingParams(max_tokens=200, ignore_eos=True))
    t0 = time.time()
    try:
        while eng.has_unfinished():
            eng.step()
        q.put((rank, "finished", "", time.time() - t0))
    except Exception as exc:  # noqa: BLE001 - the outcome is the test's subject
        q.put((rank, type(exc).__name__, str(exc)[:200], time.time() - t0))
    q.close()
    q.join_thread()  # flush the result before leaving
    os._exit(0)  # do not wait on a group whose peer is gone


@pytest.mark.parametrize("kind", ["raise", "exit", "hang"])
def test_surviving_rank_fails_fast(kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    fault = f"1:4:{kind}"
    ps = [ctx.Process(target=_rank, args=(r, 2, port, fault, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    deadline = time.time() + 120
    while 0 not in res and time.time() < deadline:
        try:
            r = q.get(timeout=5)
            res[r[0]] = r
        except Exception:  # noqa: BLE001 - queue empty
            pass
    for p in ps:
        p.join(timeout=5)
        if p.is_alive():
            p.kill()
    assert 0 in res, "surviving rank never reported"
    _, outcome, msg, dt = res[0]
    assert outcome in ("PeerFailure", "RuntimeError", "DistBackendError", "DistError"), (outcome, msg)
    assert dt < 60, dt
