"""Rule-based prompt classification and model-family routing.

Behaviour of the reference's PromptRouter (squish/serving/router.py): a prompt is classified
into a task category by prioritised regular-expression rules (first match wins, confidence 1.0),
else by keyword overlap (confidence = share of the category's keywords seen, capped below 1),
else the fallback category; each decision can carry a model hint. Custom rules outrank the
defaults. The rules below are this package's own.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from enum import Enum


class RouterCategory(str, Enum):
    CODE = "code"
    MATH = "math"
    CREATIVE = "creative"
    FACTUAL = "factual"
    CONVERSATION = "conversation"
    UNKNOWN = "unknown"


@dataclass(frozen=True)
class RouterRule:
    name: str
    category: RouterCategory
    pattern: re.Pattern
    priority: int = 50
    model_hint: str | None = None


@dataclass(frozen=True)
class RouterDecision:
    category: RouterCategory
    confidence: float
    model_hint: str | None
    rule: str | None
    reasoning: str


def _rx(p: str) -> re.Pattern:
    return re.compile(p, re.IGNORECASE | re.MULTILINE)


DEFAULT_RULES = [
    RouterRule("code-fence", RouterCategory.CODE, _rx(r"```|^\s*(def|class|fn|func|public|#include)\b"), 95, "coder"),
    RouterRule("code-ask", RouterCategory.CODE, _rx(
        r"\b(python|javascript|typescript|rust|golang|c\+\+|sql|bash|regex|compile|stack ?trace|"
        r"refactor|debug|unit tests?|function|api endpoint)\b"), 85, "coder"),
    RouterRule("math-symbols", RouterCategory.MATH, _rx(r"(\d\s*[\^*/]\s*\d|\\frac|\\int|∫|∑|√|=\s*\?)"), 80, "math"),
    RouterRule("math-ask", RouterCategory.MATH, _rx(
        r"\b(solve|prove|integral|derivative|equation|probability|matrix|eigen\w*|theorem|calculate)\b"), 75, "math"),
    RouterRule("creative", RouterCategory.CREATIVE, _rx(
        r"\b(write|compose|draft) (me )?(a |an )?(story|poem|song|haiku|limerick|novel|script|lyrics)\b"), 70),
    RouterRule("creative-ask", RouterCategory.CREATIVE, _rx(r"\b(imagine|once upon a time|fictional|roleplay)\b"), 65),
    RouterRule("factual-wh", RouterCategory.FACTUAL, _rx(r"^\s*(who|what|when|where|which|how many|how much)\b"), 60),
    RouterRule("factual-ask", RouterCategory.FACTUAL, _rx(r"\b(define|definition of|capital of|history of|explain)\b"), 55),
]

KEYWORDS = {
    RouterCategory.CODE: {"def", "class", "function", "import", "algorithm", "bug", "code"},
    RouterCategory.MATH: {"equation", "formula", "calculate", "integral", "matrix", "sum"},
    RouterCategory.CREATIVE: {"write", "story", "poem", "imagine", "creative"},
    RouterCategory.FACTUAL: {"what", "when", "who", "where", "why", "how"},
}


@dataclass
class RouterConfig:
    rules: list[RouterRule] = field(default_factory=list)  # custom rules, before the defaults
    use_defaults: bool = True
    fallback_category: RouterCategory = RouterCategory.CONVERSATION
    model_hints: dict[str, str] = field(default_factory=dict)  # category -> model name override


class PromptRouter:
    def __init__(self, config: RouterConfig | None = None):
        self.config = config or RouterConfig()
        rules = list(self.config.rules) + (DEFAULT_RULES if self.config.use_defaults else [])
        custom = {id(r) for r in self.config.rules}
        # custom rules first at equal priority
        self.rules = sorted(rules, key=lambda r: (-r.priority, 0 if id(r) in custom else 1))

    def _hint(self, cat: RouterCategory, default: str | None) -> str | None:
        return self.config.model_hints.get(cat.value, default)

    def route(self, prompt: str) -> RouterDecision:
        if not prompt or not prompt.strip():
            return RouterDecision(RouterCategory.UNKNOWN, 0.0, None, None, "empty prompt")
        for r in self.rules:
            if r.pattern.search(prompt):
                return RouterDecision(r.category, 1.0, self._hint(r.category, r.model_hint), r.name,
                                      f"rule {r.name!r} matched")
        words = set(re.findall(r"[a-z]+", prompt.lower()))
        best, score = None, 0.0
        for cat, kws in KEYWORDS.items():
            s = len(words & kws) / len(kws)
            if s > score:
                best, score = cat, s
        if best is not None:
            return RouterDecision(best, min(0.9, score), self._hint(best, None), None,
                                  f"keyword overlap {score:.2f}")
        fb = self.config.fallback_category
        return RouterDecision(fb, 0.5, self._hint(fb, None), None, "fallback")


_DEFAULT: PromptRouter | None = None


def get_default_router() -> PromptRouter:
    global _DEFAULT
    if _DEFAULT is None:
        _DEFAULT = PromptRouter()
    return _DEFAULT
