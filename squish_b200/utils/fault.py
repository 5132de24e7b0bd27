"""Failure detection for multi-process serving, and host-side fault injection to test it.

GPU kernels here never trap or spin forever: every cross-GPU wait is bounded and reports
through a device status word (``TPComm.check``). What can still go wrong is on the host:
a rank raises, exits, or stops taking part. This module catches that before the next
collective is launched, so surviving ranks fail fast instead of blocking inside NCCL or a
peer-flag wait:

* ``PeerMonitor`` — every rank publishes a heartbeat (step number, wall time) in the
  torch.distributed key-value store after each step; before each step a rank reads its
  peers' heartbeats and raises ``PeerFailure`` when one is missing for ``timeout_s``, has
  announced an error, or lags more than ``max_lag`` steps. Reads are batched and cheap.
* ``Watchdog`` — a thread per engine that marks the engine ``degraded`` when no step
  completed for ``stall_s`` while work was pending (``/health`` reports it).
* ``FaultInjector`` — ``SQUISH_FAULT="rank:step:kind"`` (several separated by ``,``)
  makes a rank, on the host, ``raise`` an exception, ``exit`` the process, ``hang``
  (stop stepping and stop heartbeats), ``delay:<ms>`` a step, or ``drop`` its next
  heartbeat. It never touches device memory or kernels.

The reference runs one process and has none of this (its failure handling is 429/503 and
per-feature fallbacks, squish/server.py:1966-1977, 458-490); the design is new.
"""
from __future__ import annotations

import json
import os
import threading
import time
from dataclasses import dataclass


class PeerFailure(RuntimeError):
    """A peer rank failed, left, or stopped making progress."""


@dataclass
class Fault:
    rank: int
    step: int
    kind: str
    arg: float = 0.0


def parse_faults(spec: str | None) -> list[Fault]:
    out = []
    for part in (spec or "").split(","):
        part = part.strip()
        if not part:
            continue
        bits = part.split(":")
        if len(bits) < 3:
            raise ValueError(f"bad fault spec {part!r}: want rank:step:kind[:arg]")
        arg = float(bits[3]) if len(bits) > 3 else 0.0
        kind = bits[2]
        if kind not in ("raise", "exit", "hang", "delay", "drop"):
            raise ValueError(f"unknown fault kind {kind!r}")
        out.append(Fault(int(bits[0]), int(bits[1]), kind, arg))
    return out


class InjectedFault(RuntimeError):
    """Raised by a ``raise`` fault."""


class FaultInjector:
    def __init__(self, rank: int, spec: str | None = None, hang_s: float = 3600.0):
        self.rank = rank
        self.faults = [f for f in parse_faults(spec if spec is not None else os.environ.get("SQUISH_FAULT"))
                       if f.rank == rank]
        self.hang_s = hang_s
        self.drop_next = False

    def before_step(self, step: int, on_hang=None) -> None:
        for f in self.faults:
            if f.step != step:
                continue
            if f.kind == "raise":
                raise InjectedFault(f"injected failure on rank {self.rank} at step {step}")
            if f.kind == "exit":
                os._exit(17)
            if f.kind == "delay":
                time.sleep(f.arg / 1000.0)
            if f.kind == "drop":
                self.drop_next = True
            if f.kind == "hang":
                if on_hang is not None:
                    on_hang()
                time.sleep(self.hang_s)

    def take_drop(self) -> bool:
        d, self.drop_next = self.drop_next, False
        return d


class PeerMonitor:
    """Store-based heartbeats among the ranks of one process group."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, max_lag: int = 2,
                 prefix: str = "squish/hb", injector: FaultInjector | None = None):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.max_lag, self.prefix = timeout_s, max_lag, prefix
        self.injector = injector
        self.step = -1
        self.first_seen: dict[int, float] = {}
        self._live_stop = threading.Event()
        self._live: threading.Thread | None = None
        self.beat(0)

    # liveness: a process that died (or froze) stops refreshing this key
    def start_liveness(self, interval_s: float = 0.5) -> "PeerMonitor":
        def loop():
            while not self._live_stop.is_set():
                try:
                    self.store.set(f"{self.prefix}/alive/{self.rank}", str(time.time()))
                except Exception:  # noqa: BLE001 - store gone: the group is shutting down
                    return
                self._live_stop.wait(interval_s)

        self._live = threading.Thread(target=loop, name="squish-liveness", daemon=True)
        self._live.start()
        return self

    def stop_liveness(self) -> None:
        self._live_stop.set()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: int, error: str | None = None) -> None:
        self.step = step
        if self.injector is not None and error is None and self.injector.take_drop():
            return
        self.store.set(self._key(self.rank), json.dumps({"step": step, "t": time.time(), "error": error}))

    def announce_error(self, msg: str) -> None:
        try:
            self.beat(self.step, error=msg)
        except Exception:  # noqa: BLE001 - the store may already be gone
            pass

    def check(self) -> None:
        """Raise PeerFailure if any peer failed or stalled; otherwise return quickly."""
        now = time.time()
        peers = [r for r in range(self.world) if r != self.rank]

        def present(key):  # non-blocking: a missing key must not block in the store
            try:
                return self.store.check([key])
            except Exception as exc:  # noqa: BLE001 - store down = the group is gone
                raise PeerFailure(f"heartbeat store unreachable: {exc}") from exc

        for r in peers:
            if self._live is not None and present(f"{self.prefix}/alive/{r}"):
                t = float(self.store.get(f"{self.prefix}/alive/{r}"))
                if now - t > self.timeout_s:
                    raise PeerFailure(f"rank {r} stopped refreshing its liveness key {now - t:.1f}s ago")
            if not present(self._key(r)):
                hb = {"step": -1, "error": None}
            else:
                v = self.store.get(self._key(r))
                hb = json.loads(v.decode() if isinstance(v, (bytes, bytearray)) else v)
            if hb.get("error"):
                raise PeerFailure(f"rank {r} reported an error: {hb['error']}")
            if hb["step"] >= self.step - self.max_lag:
                self.first_seen.pop(r, None)
                continue
            # behind: give it timeout_s from when this rank first noticed (clocks are not compared)
            t0 = self.first_seen.setdefault(r, now)
            if now - t0 > self.timeout_s:
                raise PeerFailure(f"rank {r} stalled at step {hb['step']} (this rank is at {self.step})")


class Watchdog:
    """Flags an engine as degraded when it stops completing steps while work is pending."""

    def __init__(self, has_work, stall_s: float = 30.0, interval_s: float = 1.0):
        self.has_work = has_work
        self.stall_s, self.interval_s = stall_s, interval_s
        self.last_step = time.time()
        self.degraded = False
        self.reason = ""
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    def heartbeat(self) -> None:
        self.last_step = time.time()
        if self.degraded:
            self.degraded, self.reason = False, ""

    def poll(self) -> bool:
        idle = time.time() - self.last_step
        if self.has_work() and idle > self.stall_s:
            self.degraded = True
            self.reason = f"no engine step for {idle:.1f}s with requests pending"
        return self.degraded

    def start(self) -> "Watchdog":
        def loop():
            while not self._stop.wait(self.interval_s):
                self.poll()

        self._thread = threading.Thread(target=loop, name="squish-watchdog", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2.0)
