"""Error reporting of the kernels that do not belong to a communicator.

The tcgen05 GEMM and the decode attention wait only on their own mbarriers
(TMA and tensor-core completions). Such a wait is bounded (``NAB_TIMEOUT_NS``,
default 5 s); one that runs out records where it gave up in a per-device
error record and the kernel returns with a partial output instead of hanging.
:func:`check_kernels` raises :class:`KernelError` when the record is set; with
``NAB_CHECK=1`` the op wrappers synchronise and check after every launch.
(The reference has no kernels of its own and unbounded spins:
src/numa_all_reduce.cu:177,202.)
"""

from __future__ import annotations

import os

import torch

from . import _ext

STAGES = {10: "GEMM + allreduce", 11: "GEMM", 12: "attention", 13: "bounds check"}


class KernelError(RuntimeError):
    """A bounded wait inside a GEMM or attention kernel gave up."""


def check_enabled() -> bool:
    return os.environ.get("NAB_CHECK", "0").strip().lower() in ("1", "true", "yes", "on")


def kernel_error_state() -> list[int]:
    """``[code, rank, peer, stage, block, epoch, observed, count]`` of the
    current device's record (synchronous)."""
    return [int(v) for v in _ext.load().kernel_error_state()]


def check_kernels(sync: bool = True) -> None:
    """Raises :class:`KernelError` if a GEMM or attention wait on the current
    device gave up since the last :func:`reset_kernels`."""
    ops = _ext.load()
    if sync:
        torch.cuda.current_stream().synchronize()
    if int(ops.kernel_error_code()) == 0:
        return
    code, _, _, stage, block, _, observed, count = kernel_error_state()
    raise KernelError(f"{STAGES.get(stage, stage)} kernel: a wait timed out (CTA {block}, step {observed}, "
                      f"{count} waits gave up); its output is incomplete. Call reset_kernels() to clear.")


def reset_kernels() -> None:
    """Clears the current device's record (synchronises the device)."""
    _ext.load().kernel_error_reset()


def after_launch() -> None:
    """Called by the op wrappers after a launch: checks under ``NAB_CHECK=1``."""
    if check_enabled() and not torch.cuda.is_current_stream_capturing():
        check_kernels(sync=True)
