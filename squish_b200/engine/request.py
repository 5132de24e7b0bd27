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


@dataclass
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

    @property
    def tokens(self) -> list[int]:
        return self.prompt + self.output if self.output else self.prompt

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
