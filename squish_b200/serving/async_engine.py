"""Thread-owned engine front-end for the HTTP server and the daemon.

The LLMEngine is not thread-safe; one background thread owns it and runs ``step()``
whenever work is pending. Callers submit requests through a queue and receive token
events on a per-request sink (an asyncio queue for coroutines, a plain queue for threads).
This mirrors the reference's single pinned inference thread (squish/server.py:494-530)
but batches every in-flight request into each step.
"""
from __future__ import annotations

import asyncio
import collections
import logging
import queue
import threading
import time
from dataclasses import dataclass

from ..engine.sampling import SamplingParams

log = logging.getLogger("squish_b200.serving")


class QueueFullError(RuntimeError):
    """Too many pending requests (HTTP 429)."""


@dataclass
class GenEvent:
    token_ids: list
    finished: bool
    reason: str | None
    prompt_tokens: int
    completion_tokens: int


class _Sink:
    def __init__(self, loop: asyncio.AbstractEventLoop | None):
        self.loop = loop
        self.aq: asyncio.Queue | None = asyncio.Queue() if loop is not None else None
        self.q: queue.Queue | None = None if loop is not None else queue.Queue()

    def put(self, ev: GenEvent) -> None:
        if self.loop is not None:
            self.loop.call_soon_threadsafe(self.aq.put_nowait, ev)
        else:
            self.q.put(ev)


class AsyncEngine:
    def __init__(self, engine, tokenizer=None, max_pending: int = 256, model_name: str = "model",
                 loop_guard: bool = True):
        from .quality_monitor import QualityMonitor

        self.engine = engine
        self.tokenizer = tokenizer
        self.model_name = model_name
        self.max_pending = max_pending
        self._inbox: queue.Queue = queue.Queue()
        self._sinks: dict[str, _Sink] = {}
        self._wake = threading.Event()
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self._lock = threading.Lock()
        self._ids = 0
        # metrics
        self.requests_total = 0
        self.tokens_total = 0
        self.errors_total = 0
        self.started_at = time.time()
        self.heartbeat = time.time()
        self.recent = collections.deque(maxlen=20)  # (tps, ttft) of finished requests
        self._t_first: dict[str, float] = {}
        self._t_submit: dict[str, float] = {}
        self.last_error: str | None = None
        self.loop_guard = loop_guard
        self._guards: dict = {}
        self._unguarded: set = set()  # ignore_eos requests ask for exactly max_tokens: never cut
        self.loops_stopped = 0
        self.quality = QualityMonitor()
        self.step_ms: collections.deque = collections.deque(maxlen=4096)  # engine step wall times
        from ..utils.fault import Watchdog

        self.watchdog = Watchdog(lambda: bool(self._sinks))

    # ------------------------------------------------------------------ lifecycle
    def start(self) -> "AsyncEngine":
        if self._thread is None or not self._thread.is_alive():
            self._stop.clear()
            self._thread = threading.Thread(target=self._run, name="squish-engine", daemon=True)
            self._thread.start()
            self.watchdog.start()
        return self

    def stop(self, timeout: float = 5.0) -> None:
        self._stop.set()
        self._wake.set()
        self.watchdog.stop()
        if self._thread is not None:
            self._thread.join(timeout)

    @property
    def inflight(self) -> int:
        return len(self._sinks)

    @property
    def alive(self) -> bool:
        return self._thread is not None and self._thread.is_alive()

    # ------------------------------------------------------------------ submission
    def submit(self, prompt_ids: list[int], params: SamplingParams, loop=None) -> tuple[str, _Sink]:
        if self.inflight >= self.max_pending:
            raise QueueFullError(f"server is at capacity ({self.max_pending} requests in flight)")
        params.validate()
        with self._lock:
            self._ids += 1
            rid = f"r{self._ids}"
        sink = _Sink(loop)
        if params.ignore_eos:
            self._unguarded.add(rid)
        self._sinks[rid] = sink
        self._t_submit[rid] = time.perf_counter()
        self._inbox.put(("add", rid, list(prompt_ids), params))
        self._wake.set()
        return rid, sink

    def abort(self, rid: str) -> None:
        self._inbox.put(("abort", rid, None, None))
        self._wake.set()

    def call(self, fn, timeout: float = 30.0):
        """Run ``fn(engine)`` on the engine thread between steps (the engine is not thread
        safe) and return its result; its exception is raised here."""
        box: queue.Queue = queue.Queue(maxsize=1)
        self._inbox.put(("call", None, fn, box))
        self._wake.set()
        ok, val = box.get(timeout=timeout)
        if not ok:
            raise val
        return val

    async def stream(self, prompt_ids: list[int], params: SamplingParams):
        """Async generator of GenEvent for one request."""
        rid, sink = self.submit(prompt_ids, params, asyncio.get_running_loop())
        try:
            while True:
                ev = await sink.aq.get()
                yield ev
                if ev.finished:
                    return
        finally:
            if rid in self._sinks:
                self.abort(rid)

    def generate(self, prompt_ids: list[int], params: SamplingParams, timeout: float | None = None) -> GenEvent:
        """Blocking: run one request to completion; returns the aggregated event."""
        rid, sink = self.submit(prompt_ids, params)
        toks: list[int] = []
        while True:
            ev = sink.q.get(timeout=timeout)
            toks.extend(ev.token_ids)
            if ev.finished:
                return GenEvent(toks, True, ev.reason, ev.prompt_tokens, ev.completion_tokens)

    # ------------------------------------------------------------------ engine thread
    def _engine_abort(self, rid: str) -> None:
        """Abort a request from inside the engine thread (loop guard, failed step)."""
        self.engine.abort(rid)

    def _drain_inbox(self) -> None:
        ops = []
        while True:
            try:
                ops.append(self._inbox.get_nowait())
            except queue.Empty:
                break
        self._apply_ops(ops)

    def _apply_ops(self, ops) -> None:
        eng = self.engine
        for op, rid, prompt, params in ops:
            if op == "call":  # (prompt = the function, params = the reply box)
                try:
                    params.put((True, prompt(eng)))
                except Exception as exc:  # noqa: BLE001 - handed back to the caller
                    params.put((False, exc))
                continue
            if op == "add":
                try:
                    eng.add_request(prompt, params, rid=rid)
                    self.requests_total += 1
                except Exception as exc:  # noqa: BLE001 - reported to the caller as an error finish
                    sink = self._sinks.pop(rid, None)
                    if sink is not None:
                        sink.put(GenEvent([], True, f"error: {exc}", len(prompt), 0))
            elif op == "abort":
                eng.abort(rid)
                self._guards.pop(rid, None)
                self._unguarded.discard(rid)
                self._t_submit.pop(rid, None)
                self._t_first.pop(rid, None)
                sink = self._sinks.pop(rid, None)
                if sink is not None:
                    sink.put(GenEvent([], True, "abort", 0, 0))

    def _run(self) -> None:
        eng = self.engine
        while not self._stop.is_set():
            self._drain_inbox()
            self.heartbeat = time.time()
            if not eng.has_unfinished():
                self._wake.wait(0.05)
                self._wake.clear()
                continue
            try:
                ts = time.perf_counter()
                outs = eng.step()
                self.step_ms.append((time.perf_counter() - ts) * 1e3)
                self.watchdog.heartbeat()
            except Exception as exc:  # noqa: BLE001 - fail the in-flight requests, keep serving
                log.exception("engine step failed")
                self.errors_total += 1
                self.last_error = repr(exc)
                for rid in list(self._sinks):
                    self._engine_abort(rid)
                    self._sinks.pop(rid).put(GenEvent([], True, "error", 0, 0))
                    t0 = self._t_submit.pop(rid, time.perf_counter())
                    self._t_first.pop(rid, None)
                    self._guards.pop(rid, None)
                    self.quality.record_request(self.model_name, time.perf_counter() - t0, None, 0, False,
                                                type(exc).__name__)
                continue
            now = time.perf_counter()
            for o in outs:
                sink = self._sinks.get(o.rid)
                self.tokens_total += len(o.new_tokens)
                if o.rid not in self._t_first:
                    self._t_first[o.rid] = now
                if sink is None:
                    continue
                finished, reason = o.finished, o.finish_reason
                if self.loop_guard and not finished and o.rid not in self._unguarded:
                    g = self._guards.get(o.rid)
                    if g is None:
                        from .loop_guard import LoopGuard

                        g = self._guards[o.rid] = LoopGuard()
                    if g.feed(o.new_tokens):
                        self._engine_abort(o.rid)  # verbatim loop: stop with finish reason "repetition"
                        finished, reason = True, "repetition"
                        self.loops_stopped += 1
                sink.put(GenEvent(o.new_tokens, finished, reason, o.num_prompt_tokens, o.num_output_tokens))
                if finished:
                    self._sinks.pop(o.rid, None)
                    self._guards.pop(o.rid, None)
                    self._unguarded.discard(o.rid)
                    t0 = self._t_submit.pop(o.rid, now)
                    t1 = self._t_first.pop(o.rid, now)
                    dec = max(now - t1, 1e-6)
                    self.recent.append((max(o.num_output_tokens - 1, 0) / dec, t1 - t0))
                    self.quality.record_request(self.model_name, now - t0, t1 - t0, o.num_output_tokens)
                    eng.requests.pop(o.rid, None)

    # ------------------------------------------------------------------ stats
    @property
    def avg_tps(self) -> float:
        return sum(r[0] for r in self.recent) / len(self.recent) if self.recent else 0.0

    @property
    def avg_ttft(self) -> float:
        return sum(r[1] for r in self.recent) / len(self.recent) if self.recent else 0.0
