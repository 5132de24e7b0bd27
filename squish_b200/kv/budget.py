"""KV token-budget arbitration among the cache policies of one engine.

Several policies reserve KV tokens per sequence (the attention sinks + recent window, the
heavy-hitter budget, ...). Each registers the tokens it wants; while the requests fit the
total they are granted in full, otherwise every grant is scaled down in proportion (at least
one token each), so the sum never exceeds the total. The reference keeps one process-wide
broker (squish/kv/kv_cache.py:3737-3884, ``KVBudgetBroker``); here each engine owns one, and
the engine sets the total from its page pool, registering each running sequence's
heavy-hitter budget, so budgets shrink under memory pressure instead of sequences being
preempted.
"""
from __future__ import annotations


class KVBudgetBroker:
    def __init__(self, total_tokens: int = 0):
        self._total = max(0, int(total_tokens))
        self._req: dict[str, int] = {}
        self._alloc: dict[str, int] = {}

    @property
    def total(self) -> int:
        return self._total

    def set_total(self, total_tokens: int) -> None:
        """0 = unconstrained (every request granted in full)."""
        self._total = max(0, int(total_tokens))
        self._rebalance()

    def register(self, name: str, requested: int) -> int:
        if requested < 0:
            raise ValueError("a budget request is >= 0 tokens")
        self._req[name] = int(requested)
        self._rebalance()
        return self._alloc[name]

    def unregister(self, name: str) -> None:
        self._req.pop(name, None)
        self._alloc.pop(name, None)
        self._rebalance()

    def names(self) -> list[str]:
        return list(self._req)

    def allocated(self, name: str) -> int:
        return self._alloc[name]

    def requested(self, name: str) -> int:
        return self._req[name]

    def snapshot(self) -> dict:
        return {"total": self._total, "requested": dict(self._req), "allocated": dict(self._alloc)}

    def _rebalance(self) -> None:
        want = sum(self._req.values())
        if self._total == 0 or want <= self._total:
            self._alloc = dict(self._req)
            return
        # proportional shares: floors first (at least one token for a non-zero request), then
        # the remainder by largest fraction
        names = list(self._req)
        exact = {n: self._req[n] * self._total / want for n in names}
        alloc = {n: max(1 if self._req[n] else 0, int(exact[n])) for n in names}
        left = self._total - sum(alloc.values())
        for n in sorted(names, key=lambda n: exact[n] - int(exact[n]), reverse=True):
            if left <= 0:
                break
            if alloc[n] < self._req[n]:
                alloc[n] += 1
                left -= 1
        self._alloc = alloc
