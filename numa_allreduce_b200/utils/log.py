"""Library logger (plain :mod:`logging`; the reference used vLLM's logger,
src/numa_all_reduce.py:36-40)."""

from __future__ import annotations

import logging
import os

_CONFIGURED = False


def get_logger(name: str) -> logging.Logger:
    global _CONFIGURED
    root = logging.getLogger("numa_allreduce_b200")
    if not _CONFIGURED:
        level = os.environ.get("NAB_LOG_LEVEL", "WARNING").upper()
        root.setLevel(getattr(logging, level, logging.WARNING))
        if not root.handlers:
            h = logging.StreamHandler()
            h.setFormatter(logging.Formatter("%(levelname)s %(name)s: %(message)s"))
            root.addHandler(h)
        _CONFIGURED = True
    return root.getChild(name.split(".")[-1]) if not name.startswith("numa_allreduce_b200") else logging.getLogger(name)
