"""Self-consistency (Wang et al., ICLR 2023): sample several reasoning chains and return the
answer most of them reach.

As the reference's SelfConsistencyVoter (squish/reasoning/self_consistency.py): each chain's
final answer is the first capture of ``answer_pattern`` (default: the last non-empty line, or a
trailing "answer is X" / "= X" form), optionally normalised (trimmed, lower-cased, whitespace
collapsed, trailing period dropped) before counting; ties go to the answer seen first. The
server exposes it as ``self_consistency: {"k": ...}`` on chat completions.
"""
from __future__ import annotations

import re
from collections import Counter
from dataclasses import dataclass, field

_DEFAULT = re.compile(r"(?:answer\s*(?:is|:)\s*|=\s*)([^\n]+?)\s*\.?\s*$", re.IGNORECASE)


@dataclass
class SelfConsistencyConfig:
    k: int = 5
    temperature: float = 0.7
    answer_pattern: str | None = None
    normalise_answers: bool = True


@dataclass
class SelfConsistencyResult:
    answer: str
    votes: int
    total: int
    distribution: dict = field(default_factory=dict)
    winner_index: int = 0  # the first chain that reached the answer

    @property
    def agreement(self) -> float:
        return self.votes / self.total if self.total else 0.0


class SelfConsistencyVoter:
    def __init__(self, config: SelfConsistencyConfig | None = None):
        self.config = config or SelfConsistencyConfig()
        self._rx = re.compile(self.config.answer_pattern, re.IGNORECASE | re.MULTILINE) \
            if self.config.answer_pattern else None

    def extract(self, chain: str) -> str:
        if self._rx is not None:
            m = self._rx.findall(chain)
            ans = (m[-1][0] if isinstance(m[-1], tuple) else m[-1]) if m else ""
        else:
            lines = [l for l in chain.strip().splitlines() if l.strip()]
            last = lines[-1] if lines else ""
            m = _DEFAULT.search(last)
            ans = m.group(1) if m else last
        if self.config.normalise_answers:
            ans = re.sub(r"\s+", " ", ans.strip().lower()).rstrip(".")
        return ans

    def vote(self, chains: list[str]) -> SelfConsistencyResult:
        if not chains:
            raise ValueError("no chains to vote over")
        answers = [self.extract(c) for c in chains]
        counts = Counter(a for a in answers if a)
        if not counts:
            return SelfConsistencyResult("", 0, len(chains), {}, 0)
        top = max(counts.values())
        winner = next(a for a in answers if counts.get(a) == top)
        return SelfConsistencyResult(winner, top, len(chains), dict(counts), answers.index(winner))
