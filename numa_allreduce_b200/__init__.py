"""numa_allreduce_b200: a Blackwell-native intra-node allreduce library.

Public API (parity with the reference's ``src/__init__.py``, which exported
``NumaAwareAllReduce`` and ``NumaTopology``):

* :class:`NumaAwareAllReduce`: custom allreduce over NVLink 5 / NVSwitch with
  one-shot, two-shot, NVLink SHARP and hierarchical (NUMA-grouped) protocols,
  CUDA-graph buffer registration and bounded device waits, plus
  ``reduce_scatter`` / ``all_gather`` over contiguous rank segments;
* :class:`NumaTopology`, :class:`NumaNodeInfo`, :class:`GpuNumaInfo`,
  :func:`detect_numa_topology`: NUMA and GPU topology detection;
* :class:`HierSchedule` and :func:`emulate_allreduce`: the schedule and its
  gloo/CPU executor (:func:`emulate_reduce_scatter`, :func:`emulate_all_gather`
  for the segment collectives; :func:`reference_allreduce`,
  :func:`reference_reduce_scatter`, :func:`reference_all_gather`: exact CPU
  oracles);
* :func:`fused_allreduce_rmsnorm`, :func:`rmsnorm_residual`: the fused TP
  layer tail;
* :func:`gemm`, :func:`gemm_swiglu`, :func:`gemm_allreduce_rmsnorm`,
  :func:`pack_weight`, :func:`interleave_gate_up`: the tcgen05 GEMM and its
  fusions (SwiGLU epilogue; row-parallel GEMM -> allreduce -> residual ->
  RMSNorm);
* :class:`LlamaConfig`, :class:`LlamaTPDecoder`: the tensor-parallel decoder
  built on them (in ``numa_allreduce_b200.models``, imported lazily);
* :class:`PeerMonitor`, :class:`PeerLost`: host-side failure detection;
  :func:`check_kernels`, :class:`KernelError`: the error record of the GEMM
  and attention kernels' bounded waits.
"""

from .ops.errors import KernelError, check_kernels, reset_kernels
from .ops.fused import fused_allreduce_rmsnorm, rmsnorm_residual
from .ops.gemm import PackedWeight, gemm, gemm_allreduce_rmsnorm, gemm_swiglu, interleave_gate_up, pack_weight
from .parallel.comm import AllReduceError, NumaAwareAllReduce
from .parallel.emulate import emulate_all_gather, emulate_allreduce, emulate_reduce_scatter
from .parallel.health import PeerLost, PeerMonitor
from .parallel.schedule import HierSchedule, reference_all_gather, reference_allreduce, reference_reduce_scatter
from .parallel.select import AlgoSelector
from .utils.topology import GpuNumaInfo, NumaNodeInfo, NumaTopology, detect_numa_topology

__all__ = [
    "AlgoSelector",
    "AllReduceError",
    "GpuNumaInfo",
    "HierSchedule",
    "KernelError",
    "NumaAwareAllReduce",
    "NumaNodeInfo",
    "NumaTopology",
    "PackedWeight",
    "PeerLost",
    "PeerMonitor",
    "check_kernels",
    "detect_numa_topology",
    "emulate_all_gather",
    "emulate_allreduce",
    "emulate_reduce_scatter",
    "fused_allreduce_rmsnorm",
    "gemm",
    "gemm_allreduce_rmsnorm",
    "gemm_swiglu",
    "interleave_gate_up",
    "pack_weight",
    "reference_all_gather",
    "reference_allreduce",
    "reference_reduce_scatter",
    "reset_kernels",
    "rmsnorm_residual",
]

__version__ = "0.1.0"
