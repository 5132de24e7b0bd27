"""Serving on several GPUs: data-parallel replicas behind a request router, and a
tensor-parallel engine whose ranks run the same step loop.

The reference serves one model from one process (its only multi-device behaviour is HF
``device_map="auto"`` layer placement, squish/backend.py:295). Here:

* ``DPRouter`` — N independent engines (one per GPU, each owned by its own AsyncEngine
  thread) behind the AsyncEngine interface the HTTP server uses. A request goes to the
  replica with the fewest requests in flight (ties: the one that got a request least
  recently), so long and short requests spread evenly. Request ids carry the replica
  index (``"<i>:<id>"``) so aborts and embedding lookups reach the right engine.
* ``TPAsyncEngine`` / ``follow`` — tensor parallelism over ``torch.distributed`` ranks
  (one process per GPU). Every rank runs the same scheduling, so every rank must apply
  the same request operations before the same step: rank 0 (the HTTP process) drains its
  inbox and broadcasts the batch of operations over a gloo group before applying it, and
  the other ranks (``follow``) apply what they receive and step whenever there is work.
  Engine-side aborts (repetition guard, failed step) go through the same broadcast, one
  iteration later on every rank. An idle rank 0 still broadcasts an empty batch every
  50 ms, which doubles as the followers' liveness signal.
"""
from __future__ import annotations

import pickle
import threading
import time

from .async_engine import AsyncEngine, GenEvent, QueueFullError


# ----------------------------------------------------------------------------- data parallel
class _Hidden:
    def __init__(self, router):
        self.router = router

    def pop(self, rid, default=None):
        i, local = self.router._split(rid)
        return self.router.replicas[i].engine.hidden_states.pop(local, default)


class _AggBlocks:
    """Sum of the replicas' page-pool counters (for /v1/metrics)."""

    def __init__(self, engines):
        self.engines = engines

    def _sum(self, attr):
        return sum(getattr(e.blocks, attr) for e in self.engines)

    @property
    def num_pages(self):
        return self._sum("num_pages")

    def num_free(self):
        return sum(e.blocks.num_free() for e in self.engines)

    @property
    def hits(self):
        return self._sum("hits")

    @property
    def hit_tokens(self):
        return self._sum("hit_tokens")

    @property
    def page_size(self):
        return self.engines[0].blocks.page_size


class _AggStats:
    def __init__(self, engines):
        self.engines = engines

    def __getattr__(self, name):
        vals = [getattr(e.stats, name) for e in self.engines]
        if name == "step_counts":  # histogram bins: element-wise
            return [sum(c) for c in zip(*vals)]
        if isinstance(vals[0], tuple):  # bin bounds: the same on every replica
            return vals[0]
        if isinstance(vals[0], dict):
            return {k: sum(v[k] for v in vals) for k in vals[0]}
        if isinstance(vals[0], list):
            return [v for part in vals for v in part]
        return sum(vals)


class _EngineView:
    """The read-only engine surface the server touches (config, pool and step counters,
    hidden states of embedding requests), over every replica."""

    def __init__(self, router):
        engines = [r.engine for r in router.replicas]
        self.cfg = engines[0].cfg
        self.qcfg = engines[0].qcfg
        self.ecfg = engines[0].ecfg
        self.blocks = _AggBlocks(engines)
        self.stats = _AggStats(engines)
        self.hidden_states = _Hidden(router)
        self.replicas = engines


class DPRouter:
    def __init__(self, replicas: list[AsyncEngine], max_pending: int = 256):
        if not replicas:
            raise ValueError("DPRouter needs at least one replica")
        self.replicas = replicas
        self.max_pending = max_pending
        self.model_name = replicas[0].model_name
        self.tokenizer = replicas[0].tokenizer
        self._lock = threading.Lock()
        self._last = [0.0] * len(replicas)
        self.engine = _EngineView(self)
        self.quality = replicas[0].quality  # every replica records into one monitor
        for r in replicas[1:]:
            r.quality = self.quality

    # ---------------------------------------------------------------- lifecycle
    def start(self) -> "DPRouter":
        for r in self.replicas:
            r.start()
        return self

    def stop(self, timeout: float = 5.0) -> None:
        for r in self.replicas:
            r.stop(timeout)

    # ---------------------------------------------------------------- routing
    def pick(self) -> int:
        with self._lock:
            i = min(range(len(self.replicas)), key=lambda j: (self.replicas[j].inflight, self._last[j]))
            self._last[i] = time.monotonic()
            return i

    @staticmethod
    def _split(rid: str) -> tuple[int, str]:
        i, _, local = rid.partition(":")
        return int(i), local

    def submit(self, prompt_ids, params, loop=None):
        if self.inflight >= self.max_pending:
            raise QueueFullError(f"server is at capacity ({self.max_pending} requests in flight)")
        i = self.pick()
        rid, sink = self.replicas[i].submit(prompt_ids, params, loop)
        return f"{i}:{rid}", sink

    def abort(self, rid: str) -> None:
        i, local = self._split(rid)
        self.replicas[i].abort(local)

    async def stream(self, prompt_ids, params):
        import asyncio

        rid, sink = self.submit(prompt_ids, params, asyncio.get_running_loop())
        i, local = self._split(rid)
        try:
            while True:
                ev = await sink.aq.get()
                yield ev
                if ev.finished:
                    return
        finally:
            if local in self.replicas[i]._sinks:
                self.replicas[i].abort(local)

    def generate(self, prompt_ids, params, timeout: float | None = None) -> GenEvent:
        rid, sink = self.submit(prompt_ids, params)
        toks: list[int] = []
        while True:
            ev = sink.q.get(timeout=timeout)
            toks.extend(ev.token_ids)
            if ev.finished:
                return GenEvent(toks, True, ev.reason, ev.prompt_tokens, ev.completion_tokens)

    # ---------------------------------------------------------------- aggregated stats
    @property
    def inflight(self) -> int:
        return sum(r.inflight for r in self.replicas)

    @property
    def alive(self) -> bool:
        return all(r.alive for r in self.replicas)

    @property
    def requests_total(self) -> int:
        return sum(r.requests_total for r in self.replicas)

    @property
    def tokens_total(self) -> int:
        return sum(r.tokens_total for r in self.replicas)

    @property
    def errors_total(self) -> int:
        return sum(r.errors_total for r in self.replicas)

    @property
    def loops_stopped(self) -> int:
        return sum(r.loops_stopped for r in self.replicas)

    @property
    def heartbeat(self) -> float:
        return min(r.heartbeat for r in self.replicas)

    @property
    def started_at(self) -> float:
        return min(r.started_at for r in self.replicas)

    @property
    def last_error(self):
        return next((r.last_error for r in self.replicas if r.last_error), None)

    @property
    def recent(self):
        return [x for r in self.replicas for x in r.recent]

    @property
    def step_ms(self):
        return [x for r in self.replicas for x in r.step_ms]

    @property
    def watchdog(self):
        return self.replicas[0].watchdog

    @property
    def avg_tps(self) -> float:
        rec = self.recent
        return sum(x[0] for x in rec) / len(rec) if rec else 0.0

    @property
    def avg_ttft(self) -> float:
        rec = self.recent
        return sum(x[1] for x in rec) / len(rec) if rec else 0.0


# ----------------------------------------------------------------------------- tensor parallel
class TPControl:
    """Broadcast of per-iteration request operations from rank 0 over a gloo group (the
    NCCL group carries the tensor traffic; this one only small pickled lists)."""

    def __init__(self, group=None, timeout_s: float = 86400.0):
        import datetime

        import torch.distributed as dist

        self.dist = dist
        self.group = group if group is not None else dist.new_group(
            backend="gloo", timeout=datetime.timedelta(seconds=timeout_s))
        self.rank = dist.get_rank()

    def publish(self, ops) -> None:
        self.dist.broadcast_object_list([ops], src=0, group=self.group)

    def receive(self):
        buf = [None]
        self.dist.broadcast_object_list(buf, src=0, group=self.group)
        return buf[0]


class TPAsyncEngine(AsyncEngine):
    """Rank 0's engine thread: operations are broadcast to the other ranks before they are
    applied, so every rank's scheduler sees the same requests in the same order."""

    def __init__(self, engine, ctrl: TPControl, *args, **kw):
        super().__init__(engine, *args, **kw)
        self.ctrl = ctrl
        self._closed = False

    def _engine_abort(self, rid: str) -> None:
        self._inbox.put(("abort", rid, None, None))  # applied on every rank next iteration

    def _drain_inbox(self) -> None:
        import queue

        ops, send = [], []
        while True:
            try:
                ops.append(self._inbox.get_nowait())
            except queue.Empty:
                break
        for op in ops:
            try:
                pickle.dumps(op)
                send.append(op)
            except Exception:  # noqa: BLE001 - a request the other ranks cannot receive fails alone
                sink = self._sinks.pop(op[1], None)
                if sink is not None:
                    sink.put(GenEvent([], True, "error: request cannot be sent to the tensor-parallel ranks "
                                                "(structured-output matchers stay on one process)", 0, 0))
        self.ctrl.publish(send)
        self._apply_ops(send)

    def stop(self, timeout: float = 5.0) -> None:
        super().stop(timeout)
        if not self._closed:
            self._closed = True
            self.ctrl.publish(None)  # followers leave their loop


def follow(engine, ctrl: TPControl, idle_timeout_s: float | None = None) -> int:
    """Rank > 0 of a tensor-parallel server: mirror rank 0's operations and steps.
    Returns the number of steps run once rank 0 broadcasts None."""
    steps = 0
    while True:
        ops = ctrl.receive()
        if ops is None:
            return steps
        for op, rid, prompt, params in ops:
            if op == "add":
                try:
                    engine.add_request(prompt, params, rid=rid)
                except Exception:  # noqa: BLE001 - rank 0 reported the same failure to the caller
                    pass
            elif op == "abort":
                engine.abort(rid)
        if engine.has_unfinished():
            for o in engine.step():
                if o.finished:
                    engine.requests.pop(o.rid, None)
            steps += 1


__all__ = ["DPRouter", "TPAsyncEngine", "TPControl", "follow"]
