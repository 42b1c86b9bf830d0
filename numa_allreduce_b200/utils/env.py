"""Environment-variable configuration.

Capability parity: the reference reads ``CUDA_VISIBLE_DEVICES`` and
``VLLM_SKIP_P2P_CHECK`` through ``vllm.envs`` (src/numa_all_reduce.py:155,241)
and documents ``VLLM_NUMA_AR_ENABLE``/``VLLM_NUMA_AR_DEBUG`` that the code never
reads. Every variable below is actually read:

=========================  ===================================================
``NAB_DISABLE``            ``1`` disables the custom path (callers fall back)
``NAB_ALGO``               force one protocol: ``oneshot``, ``twoshot``,
                           ``twoshot_pipe``, ``nvls_oneshot``, ``nvls_twoshot``,
                           ``hybrid``, ``hier``, ``pull``, ``nccl`` or ``auto``
                           (default)
``NAB_MAX_SIZE``           largest message (bytes) the custom path takes
``NAB_COLLECTIVE_MAX``     largest segment (bytes per rank) that
                           ``custom_reduce_scatter`` / ``custom_all_gather``
                           take (default 1 MiB); larger ones return None
``NAB_TIMEOUT_NS``         bound of every device-side wait (default 5 s)
``NAB_TUNING_FILE``        JSON table of protocol thresholds (see select.py)
``NAB_LOG_LEVEL``          logging level name (default WARNING)
``NAB_NVLS``               ``0`` turns off NVLink SHARP (multicast) protocols
``NAB_HIER_GROUPS``        explicit groups, e.g. ``0,1,2,3|4,5,6,7``
``NAB_SKIP_P2P_CHECK``     ``1`` trusts the driver for peer access
``NAB_CHECK``              ``1`` checks the device error word after every call
``NAB_NVTX``               ``1`` wraps calls in NVTX ranges
``NAB_PIPE_CTAS``          CTAs of the pipelined two-shot (default 128)
``NAB_PIPE_TILE``          bytes per ring slot of the pipelined two-shot
``NAB_HYBRID``             hybrid split ``permille,p2p_ctas,nvls_ctas``: the
                           P2P share of the message and each part's CTAs
``NAB_GEMM_PDL``           ``0`` launches the GEMMs without programmatic
                           dependent launch (read by the native code)
``NAB_GEMM_SPLIT_RULE``    split-K count: ``pow2`` (default, the largest
                           power of two that fits the CTA slots), ``waves``
                           (a wave-count model) or ``fill`` (every slot)
``NAB_NO_BUILD``           ``1``: never compile the extension on import
=========================  ===================================================
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field

ALGO_IDS = {
    "auto": 0,
    "oneshot": 1,
    "twoshot": 2,
    "nvls_oneshot": 3,
    "nvls_twoshot": 4,
    "hier": 5,
    "pull": 6,
    "copy": 7,
    "twoshot_pipe": 8,
    "hybrid": 9,
}
ALGO_NAMES = {v: k for k, v in ALGO_IDS.items()}
NCCL = "nccl"
NCCL_ID = 100  # selector result "use NCCL" (kAlgoNccl in the native library)


def _flag(name: str, default: bool = False) -> bool:
    v = os.environ.get(name)
    if v is None:
        return default
    return v.strip().lower() in ("1", "true", "yes", "on")


def _int(name: str, default: int | None) -> int | None:
    v = os.environ.get(name)
    if v is None or v.strip() == "":
        return default
    return int(v, 0)


def parse_groups(spec: str) -> list[list[int]]:
    """``"0,1,2,3|4,5,6,7"`` -> ``[[0, 1, 2, 3], [4, 5, 6, 7]]``."""
    groups = []
    for part in spec.split("|"):
        part = part.strip()
        if part:
            groups.append([int(x) for x in part.split(",") if x.strip() != ""])
    return groups


@dataclass
class EnvConfig:
    disable: bool = False
    algo: str = "auto"
    max_size: int | None = None
    collective_max: int = 1 << 20
    timeout_ns: int = 5_000_000_000
    tuning_file: str | None = None
    log_level: str = "WARNING"
    nvls: bool = True
    hier_groups: list[list[int]] | None = None
    skip_p2p_check: bool = False
    check: bool = False
    nvtx: bool = False
    pipe_ctas: int = 128
    pipe_tile: int = 256 << 10
    hybrid: tuple[int, int, int] | None = None
    extra: dict = field(default_factory=dict)


def read_env() -> EnvConfig:
    algo = os.environ.get("NAB_ALGO", "auto").strip().lower()
    if algo not in ALGO_IDS and algo != NCCL:
        raise ValueError(f"NAB_ALGO={algo!r} is not one of {sorted(ALGO_IDS) + [NCCL]}")
    groups = os.environ.get("NAB_HIER_GROUPS")
    return EnvConfig(
        disable=_flag("NAB_DISABLE"),
        algo=algo,
        max_size=_int("NAB_MAX_SIZE", None),
        collective_max=_int("NAB_COLLECTIVE_MAX", 1 << 20),
        timeout_ns=_int("NAB_TIMEOUT_NS", 5_000_000_000),
        tuning_file=os.environ.get("NAB_TUNING_FILE"),
        log_level=os.environ.get("NAB_LOG_LEVEL", "WARNING"),
        nvls=_flag("NAB_NVLS", True),
        hier_groups=parse_groups(groups) if groups else None,
        skip_p2p_check=_flag("NAB_SKIP_P2P_CHECK"),
        check=_flag("NAB_CHECK"),
        nvtx=_flag("NAB_NVTX"),
        pipe_ctas=_int("NAB_PIPE_CTAS", 128),
        pipe_tile=_int("NAB_PIPE_TILE", 256 << 10),
        hybrid=_triple("NAB_HYBRID"),
    )


def _triple(name: str) -> tuple[int, int, int] | None:
    v = os.environ.get(name)
    if v is None or v.strip() == "":
        return None
    parts = [int(x, 0) for x in v.split(",")]
    if len(parts) != 3:
        raise ValueError(f"{name} must be 'permille,p2p_ctas,nvls_ctas', got {v!r}")
    return parts[0], parts[1], parts[2]
