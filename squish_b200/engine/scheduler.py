"""Iteration-level continuous batching with chunked prefill and prefix-page reuse.

Every engine step schedules, under a token budget (``max_num_batched_tokens``) and a
sequence cap (``max_num_seqs``):

  1. every running request that has exactly one pending token (decode) — these go
     first and use the decode attention kernel;
  2. the remaining budget to running requests that are still prefilling (chunked);
  3. new requests from the FIFO queue: their prompt is first matched against the
     prefix cache (chained block hashes), so shared full pages are reused and only
     the remainder is computed.

If the page pool runs out, the most recently admitted running request is preempted:
its pages are released and it re-enters the queue to be recomputed (prompt and generated
tokens are prefilled again, reusing any still-cached prefix pages).

This replaces the reference's BatchScheduler (squish/serving/scheduler.py:205-800),
which coalesces requests for 20 ms and then runs one single-token forward per request
per step (MLX) or re-forwards the whole padded sequence each step without a KV cache
(torch path, :724-800). Here one batched forward serves all running sequences.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass

from ..kv.paged import BlockManager, OutOfPages
from .request import Request, Status


@dataclass
class ScheduledEntry:
    req: Request
    start: int     # first position computed this step
    n: int         # tokens computed this step
    sample: bool   # this chunk reaches the end of the known tokens -> sample a token
    tree: object = None  # speculative draft tree verified by this entry (n = tree size)


@dataclass
class Schedule:
    decode: list[ScheduledEntry]
    prefill: list[ScheduledEntry]
    preempted: list[Request]

    @property
    def empty(self) -> bool:
        return not self.decode and not self.prefill


class Scheduler:
    def __init__(self, blocks: BlockManager, max_num_seqs: int, max_num_batched_tokens: int, max_model_len: int,
                 chunk_align: int = 0):
        self.blocks = blocks
        self.max_num_seqs = max_num_seqs
        self.budget = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.page_size = blocks.page_size
        # chunk_align > 0: prefill chunk boundaries fall on multiples of this many tokens
        # (grid-aligned chunked prefill makes a reused prefix byte-identical to a fresh one)
        self.chunk_align = chunk_align
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []

    def add(self, req: Request) -> None:
        if len(req.prompt) + req.params.max_tokens > self.max_model_len:
            req.params.max_tokens = max(1, self.max_model_len - len(req.prompt))
        if len(req.prompt) >= self.max_model_len:
            raise ValueError(f"prompt of {len(req.prompt)} tokens exceeds max_model_len {self.max_model_len}")
        self.waiting.append(req)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    # ------------------------------------------------------------------ page helpers
    def _ensure_pages(self, req: Request, upto: int) -> bool:
        need = (upto + self.page_size - 1) // self.page_size - len(req.pages)
        if need <= 0:
            return True
        if not self.blocks.can_allocate(need):
            return False
        for _ in range(need):
            req.pages.append(self.blocks.allocate())
        return True

    def _preempt(self, victim: Request) -> None:
        self.blocks.release(victim.pages)
        victim.pages = []
        victim.num_computed = 0
        victim.evicted_tokens = victim.evict_from = victim.h2o_scored = 0
        victim.h2o_mass = None
        victim.evicted_at = {}
        victim.registered_blocks = 0
        victim.chain_hash = None
        victim.status = Status.WAITING
        victim.preemptions += 1
        # recompute on resume: prompt + generated tokens are prefilled again, then decoding continues
        self.running.remove(victim)
        self.waiting.appendleft(victim)

    def finish(self, req: Request, reason: str) -> None:
        req.status = Status.FINISHED
        req.finish_reason = reason
        self.blocks.release(req.pages)
        req.pages = []
        if req in self.running:
            self.running.remove(req)

    # ------------------------------------------------------------------ schedule
    def schedule(self) -> Schedule:
        budget = self.budget
        decode: list[ScheduledEntry] = []
        prefill: list[ScheduledEntry] = []
        preempted: list[Request] = []
        # 1. decodes (oldest first); preempt from the back on page exhaustion
        for req in list(self.running):
            if req.status is not Status.RUNNING:  # (preempted this step: status WAITING, off the list)
                continue
            pending = req.total_len - req.num_computed
            if pending != 1:
                continue
            while not self._ensure_pages(req, req.num_computed + 1):
                victim = self.running[-1]
                self._preempt(victim)
                preempted.append(victim)
                if victim is req:
                    break
            if req.status is not Status.RUNNING:
                continue
            decode.append(ScheduledEntry(req, req.num_computed, 1, True))
            budget -= 1
        decode = [e for e in decode if e.req.status is Status.RUNNING]
        # 2. running prefills
        for req in self.running:
            if budget <= 0:
                break
            pending = req.total_len - req.num_computed
            if pending <= 1 and req.num_computed > 0:
                continue
            e = self._chunk(req, budget)
            if e is None:
                break
            prefill.append(e)
            budget -= e.n
        # 3. admissions
        while self.waiting and budget > 0 and len(self.running) < self.max_num_seqs:
            req = self.waiting[0]
            if req.num_computed == 0 and not req.pages:
                hit = self.blocks.match_prefix(req.tokens)
                req.pages = list(hit.pages)
                req.num_computed = hit.tokens
                req.prefix_hit_tokens = hit.tokens
                req.registered_blocks = len(hit.pages)
                req.chain_hash = hit.last_hash
            e = self._chunk(req, budget)
            if e is None:
                # undo the prefix match, retry next step
                self.blocks.release(req.pages)
                req.pages = []
                req.num_computed = 0
                break
            self.waiting.popleft()
            req.status = Status.RUNNING
            self.running.append(req)
            if e.n == 1 and e.start > 0:
                decode.append(e)
            else:
                prefill.append(e)
            budget -= e.n
        return Schedule(decode, prefill, preempted)

    def _chunk(self, req: Request, budget: int) -> ScheduledEntry | None:
        pending = req.total_len - req.num_computed
        n = min(pending, budget)
        if self.chunk_align and n < pending:
            end = (req.num_computed + n) // self.chunk_align * self.chunk_align
            n = end - req.num_computed
            if n <= 0:
                return None
        if n <= 0:
            return None
        if not self._ensure_pages(req, req.num_computed + n):
            return None
        return ScheduledEntry(req, req.num_computed, n, req.num_computed + n == req.total_len)
