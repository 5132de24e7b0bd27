"""Request state tracked by the scheduler."""
from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field

from .sampling import SamplingParams


class Status(enum.Enum):
    WAITING = 0
    RUNNING = 1
    FINISHED = 2


@dataclass(eq=False)  # identity: requests are unique, and field-wise equality is O(prompt) per compare
class Request:
    rid: str
    prompt: list[int]
    params: SamplingParams
    arrival: float = field(default_factory=time.perf_counter)
    output: list[int] = field(default_factory=list)
    logprobs: list[float] = field(default_factory=list)
    pages: list[int] = field(default_factory=list)
    num_computed: int = 0           # tokens whose KV is in the cache
    status: Status = Status.WAITING
    finish_reason: str | None = None
    first_token_time: float | None = None
    finish_time: float | None = None
    registered_blocks: int = 0      # full blocks already published for prefix sharing
    chain_hash: bytes | None = None
    prefix_hit_tokens: int = 0
    preemptions: int = 0
    rng_step: int = 0
    prompt_key: bytes | None = None  # key of the prompt in the engine's prompt-logit cache
    # attention window (sink pages + recent window): pages given back are -1 in `pages`; the
    # attention kernels see only the kept pages, in order, so their token count is
    # total - evicted_tokens
    evicted_tokens: int = 0
    evict_from: int = 0  # first page index not yet checked for eviction
    # heavy-hitter eviction: accumulated attention mass per logical page, pages scored so far,
    # and when each evicted page went (num_computed at the time)
    h2o_mass: object = field(default=None, repr=False)
    h2o_scored: int = 0
    evicted_at: dict = field(default_factory=dict, repr=False)
    # cached int32 copy of `pages` for the step's block table (valid while `_bt_src is pages`
    # and the length matches: pages only ever grow by append or are replaced by a new list)
    _bt_src: list | None = field(default=None, repr=False)
    _bt_arr: object = field(default=None, repr=False)
    _bt_n: int = field(default=-1, repr=False)
    _bt_ev: int = field(default=0, repr=False)
    # per-request constants of the step inputs, computed on first use
    _rng_base: int | None = field(default=None, repr=False)
    _samp_row: tuple | None = field(default=None, repr=False)

    def page_array(self):
        """int32 array of the kept pages (the block table row the attention kernels read)."""
        import numpy as np

        if self._bt_src is not self.pages or self._bt_n != len(self.pages) or self._bt_ev != self.evicted_tokens:
            self._bt_src, self._bt_n, self._bt_ev = self.pages, len(self.pages), self.evicted_tokens
            arr = np.asarray(self.pages, dtype=np.int32)
            self._bt_arr = arr[arr >= 0] if self.evicted_tokens else arr
        return self._bt_arr

    def logical_pages(self):
        """int32 array of every page position (-1 where evicted): slot = pages[pos // ps]."""
        import numpy as np

        return np.asarray(self.pages, dtype=np.int32) if self.evicted_tokens else self.page_array()

    def token_at(self, i: int) -> int:
        P = len(self.prompt)
        return self.prompt[i] if i < P else self.output[i - P]

    @property
    def tokens(self) -> list[int]:
        return self.prompt + self.output if self.output else self.prompt

    def token_slice(self, start: int, n: int) -> list[int]:
        """tokens[start:start + n] without building the concatenated token list."""
        P = len(self.prompt)
        if start >= P:
            return self.output[start - P:start - P + n]
        if start + n <= P:
            return self.prompt[start:start + n]
        return self.prompt[start:] + self.output[:start + n - P]

    @property
    def total_len(self) -> int:
        return len(self.prompt) + len(self.output)

    @property
    def in_prefill(self) -> bool:
        return self.num_computed < self.total_len - (1 if self.output else 0)

    @property
    def ttft(self) -> float | None:
        return None if self.first_token_time is None else self.first_token_time - self.arrival


@dataclass
class RequestOutput:
    rid: str
    new_tokens: list[int]
    finished: bool
    finish_reason: str | None
    num_prompt_tokens: int
    num_output_tokens: int
