"""Request-field validation with the reference's defaults and bounds
(squish/api/validation.py:69-160): temperature in [0, 2] (default 0.7), top_p in (0, 1]
(default 0.9), max_tokens an integer >= 0, embedding input a non-empty string or list."""
from __future__ import annotations

import math
from typing import Any

from fastapi import HTTPException

MAX_TOKENS_CEILING = 131072


def _bad(param: str, msg: str) -> HTTPException:
    return HTTPException(status_code=400, detail=f"'{param}' {msg}")


def _num(v: Any, param: str, default: float) -> float:
    if v is None:
        return default
    if isinstance(v, bool) or not isinstance(v, (int, float, str)):
        raise _bad(param, "must be a number")
    try:
        f = float(v)
    except (TypeError, ValueError) as exc:
        raise _bad(param, "must be a number") from exc
    if not math.isfinite(f):
        raise _bad(param, "must be a finite number")
    return f


def parse_max_tokens(v: Any, default: int) -> int:
    if v is None:
        return default
    if isinstance(v, bool) or not isinstance(v, (int, float, str)):
        raise _bad("max_tokens", "must be an integer")
    try:
        i = int(v)
    except (TypeError, ValueError) as exc:
        raise _bad("max_tokens", "must be an integer") from exc
    if i < 0:
        raise _bad("max_tokens", "must be >= 0")
    if i > MAX_TOKENS_CEILING:
        raise _bad("max_tokens", f"must be <= {MAX_TOKENS_CEILING}")
    return i


def parse_temperature(v: Any, default: float = 0.7) -> float:
    f = _num(v, "temperature", default)
    if not 0.0 <= f <= 2.0:
        raise _bad("temperature", "must be between 0.0 and 2.0")
    return f


def parse_top_p(v: Any, default: float = 0.9) -> float:
    f = _num(v, "top_p", default)
    if not 0.0 < f <= 1.0:
        raise _bad("top_p", "must be > 0.0 and <= 1.0")
    return f


def parse_int(v: Any, param: str, default: int, lo: int = 0) -> int:
    if v is None:
        return default
    try:
        i = int(v)
    except (TypeError, ValueError) as exc:
        raise _bad(param, "must be an integer") from exc
    if i < lo:
        raise _bad(param, f"must be >= {lo}")
    return i


def parse_embedding_input(v: Any) -> list[str]:
    if isinstance(v, str):
        if not v:
            raise _bad("input", "must be a non-empty string or list of strings")
        return [v]
    if isinstance(v, list) and v and all(isinstance(s, str) and s for s in v):
        return list(v)
    raise _bad("input", "must be a non-empty string or list of non-empty strings")
