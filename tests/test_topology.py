"""Topology detection on fake sysfs trees and on the live host.

Parity with the reference's TestNumaTopologyDetection
(tests/test_numa_all_reduce.py:53-94), which read only the live machine;
here the fake trees cover 2-socket layouts, hex PCI domains, missing
affinity (-1) and machines without NUMA information.
"""

import os

import pytest

from numa_allreduce_b200.utils.topology import (GpuProbe, NumaTopology, detect_numa_topology,
                                                normalize_pci, parse_cpulist)


def _write(path, text):
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "w") as f:
        f.write(text)


def make_fake_sysfs(root, nodes, gpus):
    """nodes: {id: (cpulist, total_kb, free_kb)}; gpus: {pci: numa_node}."""
    for nid, (cpus, total, free) in nodes.items():
        d = os.path.join(root, "devices", "system", "node", f"node{nid}")
        _write(os.path.join(d, "cpulist"), cpus + "\n")
        _write(os.path.join(d, "meminfo"),
               f"Node {nid} MemTotal:       {total} kB\nNode {nid} MemFree:        {free} kB\n")
    # a non-node entry that must be ignored
    _write(os.path.join(root, "devices", "system", "node", "possible"), "0-1\n")
    for pci, node in gpus.items():
        _write(os.path.join(root, "bus", "pci", "devices", pci, "numa_node"), f"{node}\n")


HGX = {f"0000:{b:02x}:00.0": (0 if i < 4 else 1) for i, b in enumerate([0x18, 0x2a, 0x3a, 0x5d, 0x9a, 0xab, 0xba, 0xdb])}


def hgx_probes():
    addrs = list(HGX)
    return [GpuProbe(index=i, pci_address=a, nvlink_peers=[j for j in range(8) if j != i],
                     p2p_accessible=[j for j in range(8) if j != i], cuda_ordinal=i)
            for i, a in enumerate(addrs)]


def test_parse_cpulist():
    assert parse_cpulist("0-3,5,7-9") == [0, 1, 2, 3, 5, 7, 8, 9]
    assert parse_cpulist("") == []
    assert parse_cpulist("4, x, 6-7") == [4, 6, 7]


def test_normalize_pci():
    assert normalize_pci("00000000:1A:00.0") == "0000:1a:00.0"
    assert normalize_pci("000a:9a:00.1") == "000a:9a:00.1"
    with pytest.raises(ValueError):
        normalize_pci("1a:00.0")


def test_two_socket_hgx(tmp_path):
    make_fake_sysfs(str(tmp_path), {0: ("0-55,112-167", 1024 ** 2, 512 * 1024), 1: ("56-111,168-223", 2048, 1024)},
                    HGX)
    t = NumaTopology(sysfs_root=str(tmp_path), gpus=hgx_probes())
    assert sorted(t.numa_nodes) == [0, 1]
    assert len(t.numa_nodes[0].cpu_cores) == 112
    assert t.numa_nodes[0].total_memory == 1024 ** 3
    assert t.get_gpus_in_numa(0) == [0, 1, 2, 3]
    assert t.get_gpus_in_numa(1) == [4, 5, 6, 7]
    assert t.get_numa_node_for_gpu(5) == 1
    assert t.get_numa_node_for_cuda_device(2) == 0
    assert t.is_cross_numa(0, 4) and not t.is_cross_numa(0, 3)
    assert t.get_nvlink_peers(0) == [1, 2, 3, 4, 5, 6, 7]
    assert t.is_fully_nvlink_connected(list(range(8)))
    s = t.get_summary()
    assert "NUMA Topology" in s and "NUMA Nodes: 2" in s and "GPU 7: NUMA 1" in s


def test_unknown_affinity_maps_to_node0(tmp_path):
    make_fake_sysfs(str(tmp_path), {0: ("0-7", 100, 50)}, {"0000:1a:00.0": -1})
    t = NumaTopology(sysfs_root=str(tmp_path), gpus=[GpuProbe(0, "0000:1a:00.0")])
    assert t.get_numa_node_for_gpu(0) == 0
    assert t.get_numa_node_for_gpu(3) == 0  # unknown GPU -> 0, like the reference


def test_hex_domain_and_exact_function(tmp_path):
    # two functions on the same bus: the reference matched the first bus entry
    make_fake_sysfs(str(tmp_path), {0: ("0", 1, 1), 1: ("1", 1, 1)},
                    {"000a:9a:00.0": 0, "000a:9a:00.1": 1})
    t = NumaTopology(sysfs_root=str(tmp_path), gpus=[GpuProbe(0, "000a:9a:00.1")])
    assert t.get_numa_node_for_gpu(0) == 1
    assert t.gpu_info[0].pci_address == "000a:9a:00.1"


def test_no_numa_sysfs(tmp_path):
    t = NumaTopology(sysfs_root=str(tmp_path), gpus=[])
    assert list(t.numa_nodes) == [0]
    assert len(t.numa_nodes[0].cpu_cores) == (os.cpu_count() or 1)
    assert not t.is_fully_nvlink_connected([])


def test_live_host_detection_does_not_crash():
    t = detect_numa_topology()
    assert len(t.numa_nodes) >= 1
    for gid in t.gpu_info:
        assert t.get_numa_node_for_gpu(gid) >= 0
    assert "NUMA Nodes:" in t.get_summary()
