"""Loads the reference's NumaAwareAllReduce from baseline/_ref, unmodified.

The reference's module does not import as shipped against the installed vLLM
0.22 (three failures, all at import time). Instead of editing its source,
three import-time shims supply what it expects:

1. ``vllm.distributed.device_communicators.numa_utils``: the reference
   imports its own ``numa_utils`` under that vLLM path (src/numa_all_reduce.py:
   31-34); the shim registers the reference's module object there.
2. ``vllm.utils.torch_utils.cuda_device_count_stateless`` is not in vLLM 0.22
   (src/numa_all_reduce.py:38); the shim provides it from vLLM's CUDA platform.
3. ``Dict`` is used in annotations but never imported
   (src/numa_all_reduce.py:19,223); the shim adds ``typing.Dict`` to builtins.

Its data path is then the stock one: vLLM's compiled custom allreduce through
``vllm._custom_ops`` for messages within vLLM's sm_100 size cap, and ``None``
(caller uses NCCL) above it.
"""

from __future__ import annotations

import builtins
import sys
import typing
from pathlib import Path

REF_DIR = Path(__file__).resolve().parent / "_ref"


def load_reference_class():
    if not (REF_DIR / "numa_all_reduce.py").exists():
        raise RuntimeError("reference not installed in baseline/_ref (run sh baseline/install_ref.sh <dir>)")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import numa_utils  # the reference's own module

    sys.modules["vllm.distributed.device_communicators.numa_utils"] = numa_utils
    import vllm.utils.torch_utils as torch_utils

    if not hasattr(torch_utils, "cuda_device_count_stateless"):
        import vllm.envs as envs
        from vllm.platforms.cuda import _cuda_device_count_stateless

        torch_utils.cuda_device_count_stateless = lambda: _cuda_device_count_stateless(envs.CUDA_VISIBLE_DEVICES)
    if not hasattr(builtins, "Dict"):
        builtins.Dict = typing.Dict
    import numa_all_reduce

    if not numa_all_reduce.custom_ar:
        raise RuntimeError("vLLM custom allreduce ops are unavailable (vllm._C did not load)")
    return numa_all_reduce.NumaAwareAllReduce
