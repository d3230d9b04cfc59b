"""Structured logging: one JSON object per line for switches and iterations."""
from __future__ import annotations

import json
import logging
import sys
from typing import Any, Optional

_LOGGER: Optional[logging.Logger] = None


def get_logger() -> logging.Logger:
    global _LOGGER
    if _LOGGER is None:
        _LOGGER = logging.getLogger("elasticmegatron_b200")
        if not _LOGGER.handlers:
            h = logging.StreamHandler(sys.stdout)
            h.setFormatter(logging.Formatter("%(message)s"))
            _LOGGER.addHandler(h)
        _LOGGER.setLevel(logging.INFO)
        _LOGGER.propagate = False
    return _LOGGER


def log_json(event: str, logger: Optional[logging.Logger] = None, **fields: Any) -> str:
    rec = {"event": event}
    rec.update(fields)
    line = json.dumps(rec, default=str)
    (logger or get_logger()).info(line)
    return line
