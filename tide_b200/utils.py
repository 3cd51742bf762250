"""Logging helper: the reference's "TIDE" logger format (python/TIDE/utils.py:14-21)."""
from __future__ import annotations

import logging


def setup_logging(level: str = "INFO") -> logging.Logger:
    logger = logging.getLogger("TIDE")
    if not logger.handlers:
        h = logging.StreamHandler()
        h.setFormatter(logging.Formatter("[TIDE %(levelname)s] %(message)s"))
        logger.addHandler(h)
    logger.setLevel(getattr(logging, level.upper()))
    return logger
