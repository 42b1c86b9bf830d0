"""NUMA and GPU topology detection.

Capability parity with the reference's ``numa_utils`` (src/numa_utils.py):
``NumaNodeInfo`` (:24), ``GpuNumaInfo`` (:39), ``NumaTopology`` with
``detect``, ``get_numa_node_for_gpu``, ``get_gpus_in_numa``, ``is_cross_numa``,
``get_nvlink_peers``, ``get_summary`` and ``print_topology`` (:54-303), and
``detect_numa_topology`` (:306).

Differences by design:

* A GPU's NUMA node is read from the exact PCI function of that GPU
  (``<root>/bus/pci/devices/DDDD:BB:DD.F/numa_node``) instead of the first
  sysfs entry whose bus number matches; a ``-1`` (no affinity reported) maps
  to node 0 instead of leaking out.
* ``gpu_info`` is keyed by physical GPU index (NVML order, which is what
  ``CUDA_VISIBLE_DEVICES`` numbers refer to on a B200 HGX board); each entry
  also records the CUDA ordinal this process sees, if any, so callers can map a
  ``torch.device`` to its NUMA node through the PCI address.
* ``p2p_accessible`` is filled (NVML P2P read status).
* The sysfs root and the GPU list are injectable, so the detection logic is
  tested against fake trees without a GPU.
"""

from __future__ import annotations

import os
import re
from dataclasses import dataclass, field

from .log import get_logger

logger = get_logger(__name__)


@dataclass
class NumaNodeInfo:
    """One NUMA node: its CPUs, the GPUs attached to it and its memory."""

    node_id: int
    cpu_cores: list[int] = field(default_factory=list)
    gpu_ids: list[int] = field(default_factory=list)
    total_memory: int = 0  # bytes
    free_memory: int = 0  # bytes

    def __repr__(self) -> str:
        return (f"NumaNodeInfo(node={self.node_id}, cpus={len(self.cpu_cores)}, gpus={self.gpu_ids}, "
                f"memory={self.total_memory / 2**30:.1f}GB)")


@dataclass
class GpuNumaInfo:
    """One GPU: its NUMA node, PCI address and direct peers."""

    gpu_id: int
    numa_node: int
    pci_bus_id: str  # "BB:DD.F"
    pci_domain: str = ""  # "DDDD"
    nvlink_peers: list[int] = field(default_factory=list)
    p2p_accessible: list[int] = field(default_factory=list)
    cuda_ordinal: int | None = None  # index in this process's torch.cuda, if visible
    name: str = ""

    @property
    def pci_address(self) -> str:
        return f"{self.pci_domain or '0000'}:{self.pci_bus_id}".lower()

    def __repr__(self) -> str:
        return (f"GpuNumaInfo(gpu={self.gpu_id}, numa={self.numa_node}, pci={self.pci_address}, "
                f"nvlink={self.nvlink_peers})")


@dataclass
class GpuProbe:
    """What topology detection needs to know about one GPU (injectable)."""

    index: int  # physical index
    pci_address: str  # "DDDD:BB:DD.F"
    nvlink_peers: list[int] = field(default_factory=list)
    p2p_accessible: list[int] = field(default_factory=list)
    cuda_ordinal: int | None = None
    name: str = ""


_PCI_RE = re.compile(r"^([0-9a-fA-F]{4,8}):([0-9a-fA-F]{2}):([0-9a-fA-F]{2})\.([0-7])$")


def normalize_pci(addr: str) -> str:
    """Canonical ``dddd:bb:dd.f`` (NVML reports an 8-digit domain)."""
    addr = addr.strip()
    m = _PCI_RE.match(addr)
    if not m:
        raise ValueError(f"not a PCI address: {addr!r}")
    dom, bus, dev, fn = m.groups()
    return f"{int(dom, 16):04x}:{bus.lower()}:{dev.lower()}.{fn}"


def parse_cpulist(text: str) -> list[int]:
    """``"0-3,5,7-9"`` -> ``[0, 1, 2, 3, 5, 7, 8, 9]`` (reference numa_utils.py:161-179)."""
    cores: list[int] = []
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        try:
            if "-" in part:
                lo, hi = part.split("-", 1)
                cores.extend(range(int(lo), int(hi) + 1))
            else:
                cores.append(int(part))
        except ValueError:
            continue
    return cores


def _probe_gpus_nvml() -> list[GpuProbe] | None:
    try:
        import pynvml
    except ImportError:
        return None
    try:
        pynvml.nvmlInit()
    except Exception:
        return None
    try:
        n = pynvml.nvmlDeviceGetCount()
        handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in range(n)]
        probes = []
        for i, h in enumerate(handles):
            pci = pynvml.nvmlDeviceGetPciInfo(h)
            bus_id = pci.busId.decode() if isinstance(pci.busId, bytes) else str(pci.busId)
            nv, p2p = [], []
            for j, hj in enumerate(handles):
                if i == j:
                    continue
                try:
                    if pynvml.nvmlDeviceGetP2PStatus(h, hj, pynvml.NVML_P2P_CAPS_INDEX_NVLINK) == \
                            pynvml.NVML_P2P_STATUS_OK:
                        nv.append(j)
                except Exception:
                    pass
                try:
                    if pynvml.nvmlDeviceGetP2PStatus(h, hj, pynvml.NVML_P2P_CAPS_INDEX_READ) == \
                            pynvml.NVML_P2P_STATUS_OK:
                        p2p.append(j)
                except Exception:
                    pass
            name = pynvml.nvmlDeviceGetName(h)
            probes.append(GpuProbe(index=i, pci_address=normalize_pci(bus_id), nvlink_peers=nv,
                                   p2p_accessible=p2p,
                                   name=name.decode() if isinstance(name, bytes) else str(name)))
        return probes
    except Exception as e:  # pragma: no cover - depends on the driver
        logger.warning("NVML GPU probe failed: %s", e)
        return None
    finally:
        try:
            pynvml.nvmlShutdown()
        except Exception:
            pass


def _torch_pci_addresses() -> list[str | None]:
    import torch

    if not torch.cuda.is_available():
        return []
    out = []
    for i in range(torch.cuda.device_count()):
        p = torch.cuda.get_device_properties(i)
        try:
            out.append(normalize_pci(f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"))
        except (AttributeError, ValueError):
            out.append(None)
    return out


def visible_physical_ids() -> list[int]:
    """Physical index of every CUDA device this process sees (CUDA_VISIBLE_DEVICES)."""
    import torch

    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    if cvd:
        ids = []
        for tok in cvd.split(","):
            tok = tok.strip()
            if tok.isdigit():
                ids.append(int(tok))
            else:  # UUIDs or MIG names: no index to map to, keep the ordinal
                return list(range(n))
        return ids[:n]
    return list(range(n))


def probe_gpus() -> list[GpuProbe]:
    """Probes the GPUs of this host: NVML for all of them when available,
    torch for the visible ones otherwise; the two are matched by PCI address."""
    torch_pci = _torch_pci_addresses()
    probes = _probe_gpus_nvml()
    if probes is None:
        phys = visible_physical_ids()
        probes = []
        for ordinal, addr in enumerate(torch_pci):
            idx = phys[ordinal] if ordinal < len(phys) else ordinal
            probes.append(GpuProbe(index=idx, pci_address=addr or f"0000:{idx:02x}:00.0",
                                   cuda_ordinal=ordinal))
        return probes
    by_pci = {p.pci_address: p for p in probes}
    for ordinal, addr in enumerate(torch_pci):
        if addr and addr in by_pci:
            by_pci[addr].cuda_ordinal = ordinal
    return probes


class NumaTopology:
    """NUMA nodes of the host and the NUMA node / peers of every GPU.

    ``sysfs_root`` and ``gpus`` may be given to detect a fake machine (tests);
    by default the live ``/sys`` tree and :func:`probe_gpus` are used.
    """

    def __init__(self, sysfs_root: str = "/sys", gpus: list[GpuProbe] | None = None,
                 probe: bool = True):
        self.sysfs_root = sysfs_root
        self.numa_nodes: dict[int, NumaNodeInfo] = {}
        self.gpu_info: dict[int, GpuNumaInfo] = {}
        self._detect_numa_nodes()
        if gpus is None and probe:
            try:
                gpus = probe_gpus()
            except Exception as e:  # pragma: no cover - depends on the host
                logger.warning("GPU probe failed: %s", e)
                gpus = []
        self._map_gpus(gpus or [])

    @classmethod
    def detect(cls, **kwargs) -> "NumaTopology":
        return cls(**kwargs)

    # ----------------------------------------------------------- detection --
    def _node_dir(self) -> str:
        return os.path.join(self.sysfs_root, "devices", "system", "node")

    def _detect_numa_nodes(self) -> None:
        base = self._node_dir()
        try:
            names = [d for d in os.listdir(base) if d.startswith("node") and d[4:].isdigit()]
        except OSError:
            names = []
        for d in sorted(names, key=lambda x: int(x[4:])):
            nid = int(d[4:])
            cpus: list[int] = []
            try:
                with open(os.path.join(base, d, "cpulist")) as f:
                    cpus = parse_cpulist(f.read())
            except OSError:
                pass
            total, free = self._read_meminfo(os.path.join(base, d, "meminfo"))
            self.numa_nodes[nid] = NumaNodeInfo(nid, cpus, [], total, free)
        if not self.numa_nodes:
            # not a NUMA machine (or no sysfs): one node with every CPU
            self.numa_nodes[0] = NumaNodeInfo(0, list(range(os.cpu_count() or 1)), [], 0, 0)

    @staticmethod
    def _read_meminfo(path: str) -> tuple[int, int]:
        total = free = 0
        try:
            with open(path) as f:
                for line in f:
                    m = re.search(r"(MemTotal|MemFree):\s+(\d+)\s*kB", line)
                    if m:
                        if m.group(1) == "MemTotal":
                            total = int(m.group(2)) * 1024
                        else:
                            free = int(m.group(2)) * 1024
        except OSError:
            pass
        return total, free

    def numa_node_of_pci(self, pci_address: str) -> int:
        path = os.path.join(self.sysfs_root, "bus", "pci", "devices", normalize_pci(pci_address),
                            "numa_node")
        try:
            with open(path) as f:
                node = int(f.read().strip())
        except (OSError, ValueError):
            return 0
        return node if node >= 0 else 0

    def _map_gpus(self, gpus: list[GpuProbe]) -> None:
        for g in gpus:
            addr = normalize_pci(g.pci_address)
            node = self.numa_node_of_pci(addr)
            dom, rest = addr.split(":", 1)
            self.gpu_info[g.index] = GpuNumaInfo(
                gpu_id=g.index, numa_node=node, pci_bus_id=rest, pci_domain=dom,
                nvlink_peers=list(g.nvlink_peers), p2p_accessible=list(g.p2p_accessible),
                cuda_ordinal=g.cuda_ordinal, name=g.name)
            if node not in self.numa_nodes:
                self.numa_nodes[node] = NumaNodeInfo(node)
            self.numa_nodes[node].gpu_ids.append(g.index)

    # ------------------------------------------------------------- queries --
    def get_numa_node_for_gpu(self, gpu_id: int) -> int:
        info = self.gpu_info.get(gpu_id)
        return info.numa_node if info else 0

    def get_numa_node_for_cuda_device(self, ordinal: int) -> int:
        for info in self.gpu_info.values():
            if info.cuda_ordinal == ordinal:
                return info.numa_node
        return 0

    def get_gpus_in_numa(self, numa_node: int) -> list[int]:
        node = self.numa_nodes.get(numa_node)
        return list(node.gpu_ids) if node else []

    def is_cross_numa(self, gpu1: int, gpu2: int) -> bool:
        return self.get_numa_node_for_gpu(gpu1) != self.get_numa_node_for_gpu(gpu2)

    def get_nvlink_peers(self, gpu_id: int) -> list[int]:
        info = self.gpu_info.get(gpu_id)
        return list(info.nvlink_peers) if info else []

    def get_p2p_peers(self, gpu_id: int) -> list[int]:
        info = self.gpu_info.get(gpu_id)
        return list(info.p2p_accessible) if info else []

    def is_fully_nvlink_connected(self, gpu_ids: list[int]) -> bool:
        for a in gpu_ids:
            peers = set(self.get_nvlink_peers(a))
            if any(b != a and b not in peers for b in gpu_ids):
                return False
        return len(gpu_ids) > 0

    def get_summary(self) -> str:
        lines = ["=" * 60, "NUMA Topology Summary", "=" * 60,
                 f"NUMA Nodes: {len(self.numa_nodes)}", f"GPUs: {len(self.gpu_info)}"]
        for nid in sorted(self.numa_nodes):
            n = self.numa_nodes[nid]
            lines += [f"\nNUMA Node {nid}:", f"  CPUs: {len(n.cpu_cores)} cores", f"  GPUs: {n.gpu_ids}",
                      f"  Memory: {n.total_memory / 2**30:.1f} GB"]
        lines.append("\nGPU Details:")
        for gid in sorted(self.gpu_info):
            g = self.gpu_info[gid]
            lines.append(f"  GPU {gid}: NUMA {g.numa_node}, PCI {g.pci_address}, "
                         f"NVLink peers {len(g.nvlink_peers)}")
        lines.append("=" * 60)
        return "\n".join(lines)

    def print_topology(self) -> None:
        print(self.get_summary())


def detect_numa_topology(**kwargs) -> NumaTopology:
    """Detects the topology of this host (see :class:`NumaTopology`)."""
    return NumaTopology.detect(**kwargs)
