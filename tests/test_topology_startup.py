"""Topology discovery and production startup: the nvidia-smi topology matrix
(NVLink counts, ANSI-coloured headers, PCIe-only pairs), fabric capability
tokens, discovery failures, the startup relay policy (synthetic fixtures
refused, PCIe / fabric requirements, minimum relay count, target checks)
and the daemon it builds.  Behaviours follow unit/test_topology_provider.py
and the startup checks of the reference with independent fixtures."""

from __future__ import annotations

import pytest

from pcie_pool_b200.daemon.startup import (DaemonStartupConfig, DaemonStartupError, build_topology_provider,
                                           create_production_daemon, relay_candidates_for_policy)
from pcie_pool_b200.topology import StaticTopologyProvider, synthetic_inventory
from pcie_pool_b200.topology.cuda_nvml import (CudaNvmlTopologyProvider, TopologyDiscoveryError,
                                               fabric_capability, fabric_links_from_matrix)

ANSI_TOPO = [
    "\x1b[4mGPU0\tGPU1\tGPU2\tGPU3\tCPU Affinity\tNUMA Affinity\x1b[0m",
    "GPU0\t X \tNV18\tNV18\tSYS\t0-55\t0",
    "GPU1\tNV18\t X \tNV18\tSYS\t0-55\t0",
    "GPU2\tNV18\tNV18\t X \tSYS\t56-111\t1",
    "GPU3\tSYS\tSYS\tSYS\t X \t56-111\t1",
    "",
    "Legend:",
    "  X    = Self",
]


class Probe:
    def __init__(self, rows, matrix, fail=False):
        self.rows, self.matrix, self.fail = rows, matrix, fail

    def query_gpu_inventory(self):
        if self.fail:
            raise TopologyDiscoveryError("nvidia-smi not found")
        return self.rows

    def query_topology_matrix(self):
        return self.matrix


def rows(n):
    return [{"device_id": i, "pci_bus_id": f"00000000:{0x1b + i:02X}:00.0", "pcie_link_gen_current": 5,
             "pcie_link_width_current": 16, "name": "NVIDIA B200"} for i in range(n)]


def test_matrix_with_ansi_header_and_pcie_only_pairs():
    links = fabric_links_from_matrix({0, 1, 2, 3}, ANSI_TOPO)
    pairs = {(l.src_device_id, l.dst_device_id) for l in links}
    assert pairs == {(0, 1), (0, 2), (1, 2)}, "SYS pairs are not fabric links"
    assert all(l.link_count == 18 and l.fabric == "nvlink" for l in links)


def test_fabric_capability_tokens():
    assert fabric_capability("NV18")["link_count"] == 18
    assert fabric_capability("nv4")["fabric"] == "nvlink"
    assert fabric_capability("NVSW")["fabric"] == "nvswitch"
    for tok in ("PIX", "PXB", "PHB"):  # peer-to-peer through PCIe switches / the host bridge
        assert fabric_capability(tok)["capability"] == f"cuda_p2p_{tok.lower()}"
    for tok in ("SYS", "NODE", " X ", "", "N/A"):
        assert fabric_capability(tok) is None


def test_provider_reports_discovery_errors_and_invalidates():
    with pytest.raises(TopologyDiscoveryError):
        CudaNvmlTopologyProvider(Probe([], [], fail=True)).snapshot()
    now = [0.0]
    prov = CudaNvmlTopologyProvider(Probe(rows(2), ANSI_TOPO[:3]), sysfs_root="/nonexistent", now=lambda: now[0])
    a = prov.snapshot()
    prov.invalidate()
    b = prov.snapshot()
    assert b.version == a.version + 1, "invalidate forces a fresh discovery"
    assert {g.device_id for g in b.gpus} == {0, 1} and b.fabric_links


def _inventory(n=4, links=True, source="cuda-nvml"):
    prov = CudaNvmlTopologyProvider(Probe(rows(n), ANSI_TOPO if links else ANSI_TOPO[:1]), sysfs_root="/none")
    inv = prov.snapshot()
    return inv if source == "cuda-nvml" else synthetic_inventory(n, source=source)


def test_startup_refuses_synthetic_fixtures():
    inv = synthetic_inventory(4, source="test_fixture_static")
    with pytest.raises(DaemonStartupError, match="synthetic"):
        relay_candidates_for_policy(inv, DaemonStartupConfig())


def test_startup_policy_requirements():
    inv = _inventory()
    assert relay_candidates_for_policy(inv, DaemonStartupConfig()) == (0, 1, 2, 3)
    relays = relay_candidates_for_policy(inv, DaemonStartupConfig(target_gpu=0, min_relay_count=2))
    assert set(relays) == {1, 2}, "GPU3 has no NVLink to GPU0"
    with pytest.raises(DaemonStartupError, match="relay policy"):
        relay_candidates_for_policy(inv, DaemonStartupConfig(target_gpu=3, min_relay_count=1))
    with pytest.raises(DaemonStartupError, match="not discovered"):
        relay_candidates_for_policy(inv, DaemonStartupConfig(target_gpu=9))
    no_links = _inventory(links=False)
    with pytest.raises(DaemonStartupError, match="fabric"):
        relay_candidates_for_policy(no_links, DaemonStartupConfig())
    assert relay_candidates_for_policy(no_links, DaemonStartupConfig(require_fabric=False))
    with pytest.raises(ValueError):
        DaemonStartupConfig(min_relay_count=-1)
    with pytest.raises(DaemonStartupError, match="unsupported"):
        build_topology_provider("magic")


def test_create_production_daemon_with_a_fake_provider_and_executor():
    prov = CudaNvmlTopologyProvider(Probe(rows(4), ANSI_TOPO), sysfs_root="/none")
    made = []
    d = create_production_daemon(DaemonStartupConfig(target_gpu=0, execute=True), topology_provider=prov,
                                 executor_factory=lambda: made.append(1) or None)
    assert made == [1] and set(d.relay_gpus) == {1, 2}
    assert d.get_inventory().ok and d.discover_relays(0, [1, 2, 3]).ok
    with pytest.raises(DaemonStartupError):
        create_production_daemon(DaemonStartupConfig(), topology_provider=CudaNvmlTopologyProvider(
            Probe([], [], fail=True)))
    static = StaticTopologyProvider(gpu_count=2)
    with pytest.raises(DaemonStartupError, match="synthetic"):
        create_production_daemon(DaemonStartupConfig(), topology_provider=static)
