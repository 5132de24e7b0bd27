"""Logging setup for the ``squish_b200`` logger tree: plain text or one JSON object per line.

The counterpart of the reference's squish/logging_config.py:33-58 (``configure_logging`` with
a JSON formatter, ``--log-level`` on the server, squish/server.py:5009). JSON records carry
``ts``, ``level``, ``logger``, ``message``, ``exc`` when an exception is attached, and every
field a caller passes through ``extra=`` (for example ``rid`` or ``step_ms``).

    configure_logging("info", json_format=True)
    get_logger(__name__).info("model loaded", extra={"load_s": 2.1})
"""
from __future__ import annotations

import json
import logging
import sys

ROOT = "squish_b200"
LEVELS = ("debug", "info", "warning", "error", "critical")

# attributes every LogRecord has: anything else on a record came from ``extra=``
_RECORD_FIELDS = frozenset(logging.LogRecord("", 0, "", 0, "", (), None).__dict__) | {"message", "asctime"}


class JsonLineFormatter(logging.Formatter):
    def format(self, record: logging.LogRecord) -> str:
        out = {"ts": self.formatTime(record, "%Y-%m-%dT%H:%M:%S") + f".{int(record.msecs):03d}",
               "level": record.levelname, "logger": record.name, "message": record.getMessage()}
        if record.exc_info:
            out["exc"] = self.formatException(record.exc_info)
        for k, v in record.__dict__.items():
            if k not in _RECORD_FIELDS and not k.startswith("_"):
                out[k] = v
        return json.dumps(out, default=str)


def configure_logging(level: str = "warning", json_format: bool = False, stream=None,
                      log_file=None) -> logging.Logger:
    """(Re)configure the package's loggers; calling it again replaces the handlers, so
    repeated calls never duplicate lines. Unknown level names mean WARNING. ``log_file``
    adds a second handler appending to that file (its directory is created)."""
    root = logging.getLogger(ROOT)
    root.setLevel(getattr(logging, str(level).upper(), logging.WARNING))
    for h in list(root.handlers):
        root.removeHandler(h)
        h.close()
    fmt = (JsonLineFormatter() if json_format else
           logging.Formatter("%(asctime)s %(levelname)-8s %(name)s %(message)s"))
    handlers = [logging.StreamHandler(stream or sys.stderr)]
    if log_file is not None:
        import os

        os.makedirs(os.path.dirname(os.path.abspath(str(log_file))), exist_ok=True)
        handlers.append(logging.FileHandler(str(log_file), mode="a"))
    for h in handlers:
        h.setFormatter(fmt)
        root.addHandler(h)
    root.propagate = False
    return root


def get_logger(name: str) -> logging.Logger:
    return logging.getLogger(name if name.startswith(ROOT) else f"{ROOT}.{name}")


__all__ = ["configure_logging", "get_logger", "JsonLineFormatter", "LEVELS"]
