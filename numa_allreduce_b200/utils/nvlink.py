"""NVLink traffic counters of a GPU, read through NVML (read-only queries).

``ncu`` cannot profile a multi-rank collective (each captured kernel is
replayed alone, and a kernel that waits on its peers cannot run alone), so
the NVLink bytes a collective moves are read here from the driver's link
counters around a timed loop instead: ``NvlinkCounters.read()`` before and
after, the difference divided by the number of calls gives bytes per call per
direction, which :func:`link_fraction` turns into a fraction of a link rate
(900 GB/s per direction nominal on B200, 770 GB/s measured peer copy).

Two counter families are tried, per link, summed over the active links:
the data-throughput counters (``NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX/RX``,
KiB, payload only) and the byte counters (``NVML_FI_DEV_NVLINK_COUNT_XMIT/
RCV_BYTES``). A family the driver does not report reads as None.
"""

from __future__ import annotations

NOMINAL_GBS_PER_DIR = 900.0
MEASURED_PEER_COPY_GBS = 770.0
MAX_LINKS = 18


class NvlinkCounters:
    def __init__(self, pci_bus_id: str | None = None, index: int | None = None):
        import pynvml

        self.nv = pynvml
        pynvml.nvmlInit()
        if pci_bus_id is not None:
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(pci_bus_id)
        else:
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index or 0)
        self.links = []
        self.diag: dict[str, object] = {}
        for link in range(MAX_LINKS):
            try:
                state = pynvml.nvmlDeviceGetNvLinkState(self.h, link)
            except pynvml.NVMLError as e:
                self.diag.setdefault("state_errors", []).append((link, str(e)))
                continue
            if state == pynvml.NVML_FEATURE_ENABLED:
                self.links.append(link)
        if not self.links:
            # no per-link state: query every possible link and keep the ones
            # whose counters answer
            self.links = list(range(MAX_LINKS))
        nv = pynvml
        self.families = {
            "data_kib": (getattr(nv, "NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX", None),
                         getattr(nv, "NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX", None), 1024),
            "bytes": (getattr(nv, "NVML_FI_DEV_NVLINK_COUNT_XMIT_BYTES", None),
                      getattr(nv, "NVML_FI_DEV_NVLINK_COUNT_RCV_BYTES", None), 1),
        }

    def read(self) -> dict[str, tuple[int, int] | None]:
        """Cumulative (tx_bytes, rx_bytes) per counter family, summed over the
        links whose counters answered."""
        out = {}
        for name, (tx_id, rx_id, unit) in self.families.items():
            if tx_id is None or rx_id is None:
                out[name] = None
                continue
            ids = [(tx_id, l) for l in self.links] + [(rx_id, l) for l in self.links]
            try:
                vals = self.nv.nvmlDeviceGetFieldValues(self.h, ids)
            except self.nv.NVMLError as e:
                self.diag[name] = str(e)
                out[name] = None
                continue
            tx = rx = 0
            answered = 0
            n = len(self.links)
            codes = []
            for i, v in enumerate(vals):
                codes.append(int(v.nvmlReturn))
                if v.nvmlReturn != 0:
                    continue
                answered += 1
                x = int(v.value.ullVal) * unit
                if i < n:
                    tx += x
                else:
                    rx += x
            self.diag[name + "_codes"] = sorted(set(codes))
            out[name] = (tx, rx) if answered else None
        return out

def delta(before: dict, after: dict, calls: int = 1) -> dict[str, tuple[float, float] | None]:
    """Bytes per call (tx, rx) between two reads."""
    out = {}
    for k in before:
        a, b = before[k], after.get(k)
        out[k] = None if a is None or b is None else ((b[0] - a[0]) / calls, (b[1] - a[1]) / calls)
    return out


def link_fraction(bytes_per_call: float, seconds_per_call: float, gbs: float = NOMINAL_GBS_PER_DIR) -> float:
    """Achieved link rate of one direction as a fraction of ``gbs``."""
    if seconds_per_call <= 0:
        return 0.0
    return bytes_per_call / seconds_per_call / 1e9 / gbs
