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
    # cached int32 copy of `pages` for the step's block table (valid while `_bt_src is pages`
    # and the length matches: pages only ever grow by append or are replaced by a new list)
    _bt_src: list | None = field(default=None, repr=False)
    _bt_arr: object = field(default=None, repr=False)

    def page_array(self):
        import numpy as np

        if self._bt_src is not self.pages or len(self._bt_arr) != len(self.pages):
            self._bt_src = self.pages
            self._bt_arr = np.asarray(self.pages, dtype=np.int32)
        return self._bt_arr

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
