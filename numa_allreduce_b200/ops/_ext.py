"""Loads the native library (``_C.so``) that registers ``torch.ops.nab``.

The library is built in-tree by :mod:`numa_allreduce_b200.native_build`; the
build is incremental, so calling it on every first import costs only a few
file hashes when nothing changed. On a machine with a GPU a missing or broken
library is an error: there is no silent PyTorch fallback for the kernels.
Set ``NAB_NO_BUILD=1`` to skip the build step and use whatever is on disk.
``NAB_DEBUG_BUILD=1`` loads ``_C_debug.so`` instead: the same library with the
device-side bounds checks compiled in (slower; for tests and debugging).
"""

from __future__ import annotations

import os
import threading
from pathlib import Path

import torch

_LOCK = threading.Lock()
_LOADED: str | None = None


def _debug() -> bool:
    return os.environ.get("NAB_DEBUG_BUILD", "0") == "1"


def library_path() -> Path:
    name = "_C_debug.so" if _debug() else "_C.so"
    return Path(__file__).resolve().parent.parent / name


def plain_library_path() -> Path:
    return Path(__file__).resolve().parent.parent / "libnab.so"


def load():
    """Returns ``torch.ops.nab`` after making sure the native library is loaded."""
    global _LOADED
    if _LOADED is not None:
        return torch.ops.nab
    with _LOCK:
        if _LOADED is not None:
            return torch.ops.nab
        path = library_path()
        if os.environ.get("NAB_NO_BUILD", "0") != "1":
            from .. import native_build

            native_build.build(debug=_debug())
        if not path.exists():
            raise RuntimeError(
                f"native library {path} is missing; run `python -m numa_allreduce_b200.native_build`")
        torch.ops.load_library(str(path))
        _LOADED = str(path)
    return torch.ops.nab


def loaded_path() -> str | None:
    return _LOADED
