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


# ---- the CUDA/NVML provider: versions, cache, sysfs, explicit gaps -----------------------------------------

class Clock:
    def __init__(self, t=100.0):
        self.t = t

    def __call__(self):
        return self.t


class CountingProbe(Probe):
    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.queries = 0

    def query_gpu_inventory(self):
        self.queries += 1
        return super().query_gpu_inventory()


def test_provider_builds_versioned_snapshots_and_caches_them():
    clock = Clock()
    probe = CountingProbe(rows(4), ANSI_TOPO)
    prov = CudaNvmlTopologyProvider(probe, cache_max_age_seconds=30.0, now=clock, sysfs_root=None)
    a = prov.snapshot()
    assert (a.version, a.source, a.discovered_at) == (1, "cuda_nvml", 100.0)
    assert a.topology_snapshot_id() == "topology-cuda_nvml-v1-100.000000"
    snap = a.to_topology_snapshot()
    assert snap.snapshot_id == a.topology_snapshot_id() and len(snap.devices) == 4
    clock.t = 120.0
    assert prov.snapshot() is a and probe.queries == 1, "inside the cache age the snapshot is reused"
    clock.t = 131.0
    b = prov.snapshot()
    assert b.version == 2 and probe.queries == 2
    prov.invalidate()
    c = prov.snapshot()
    assert c.version == 3 and probe.queries == 3 and c.topology_snapshot_id() != b.topology_snapshot_id()
    uncached = CudaNvmlTopologyProvider(CountingProbe(rows(2), ANSI_TOPO), cache_max_age_seconds=0.0,
                                        now=clock, sysfs_root=None)
    assert uncached.snapshot().version == 1 and uncached.snapshot().version == 2


def test_missing_pcie_capabilities_stay_explicit():
    bare = [{"device_id": 0, "pci_bus_id": "00000000:1B:00.0"}, {"device_id": 1}]
    inv = CudaNvmlTopologyProvider(Probe(bare, ANSI_TOPO[:3]), sysfs_root=None).snapshot()
    p0, p1 = inv.pcie_paths
    assert (p0.link_generation, p0.link_width, p0.bandwidth_source) == (None, None, None)
    assert p0.bandwidth_gbps == 0.0 and p0.root_complex == "0000:1b" and p1.root_complex is None
    given = [{"device_id": 0, "pcie_link_gen_current": 5, "pcie_link_width_current": 16,
              "pcie_bandwidth_gbps": 55.0}]
    (p,) = CudaNvmlTopologyProvider(Probe(given, []), sysfs_root=None).snapshot().pcie_paths
    assert (p.bandwidth_gbps, p.bandwidth_source, p.negotiated_speed_gtps) == (55.0, "provider", 32.0)
    (e,) = CudaNvmlTopologyProvider(Probe(given[:1] and [{k: v for k, v in given[0].items()
                                                          if k != "pcie_bandwidth_gbps"}], []),
                                    sysfs_root=None).snapshot().pcie_paths
    assert e.bandwidth_source == "estimated_from_pcie_generation_width" and 60.0 < e.bandwidth_gbps < 64.0


def test_sysfs_fills_numa_link_and_switch_chain(tmp_path):
    from pcie_pool_b200.topology.cuda_nvml import pcie_tree

    chain = tmp_path / "devices" / "pci0000:15" / "0000:15:01.0" / "0000:16:00.0" / "0000:17:00.0"
    dev = chain / "0000:1b:00.0"
    dev.mkdir(parents=True)
    (dev / "numa_node").write_text("1\n")
    (dev / "current_link_speed").write_text("32.0 GT/s PCIe\n")
    (dev / "current_link_width").write_text("16\n")
    link = tmp_path / "bus" / "pci" / "devices"
    link.mkdir(parents=True)
    (link / "0000:1b:00.0").symlink_to(dev)
    t = pcie_tree("00000000:1B:00.0", tmp_path)
    assert t["numa_node"] == 1 and t["negotiated_speed_gtps"] == 32.0 and t["link_width"] == 16
    assert t["switch_hierarchy"] == ("0000:15:01.0", "0000:16:00.0", "0000:17:00.0")
    assert t["root_complex"] == "0000:15"
    (p,) = CudaNvmlTopologyProvider(Probe([{"device_id": 0, "pci_bus_id": "00000000:1B:00.0"}], []),
                                    sysfs_root=str(tmp_path)).snapshot().pcie_paths
    assert (p.link_generation, p.link_width, p.numa_node) == (5, 16, 1)
    assert p.switch_hierarchy == ("0000:15:01.0", "0000:16:00.0", "0000:17:00.0")
    assert pcie_tree("0000:99:00.0", tmp_path) == {}


def test_fabric_links_are_normalised_per_pair():
    links = fabric_links_from_matrix({0, 1, 2, 3}, ANSI_TOPO)
    pairs = {(l.src_device_id, l.dst_device_id) for l in links}
    assert pairs == {(0, 1), (0, 2), (1, 2)}, "one record per unordered pair, SYS pairs dropped"
    assert all(l.enabled and l.fabric == "nvlink" and l.link_count == 18 for l in links)
    pix = fabric_links_from_matrix({0, 1}, ["\tGPU0\tGPU1", "GPU0\t X \tPIX", "GPU1\tPIX\t X "])
    assert len(pix) == 1 and pix[0].fabric != "nvlink"
    assert fabric_links_from_matrix({0, 1}, []) == ()


def test_startup_reports_why_relays_were_filtered():
    inv = CudaNvmlTopologyProvider(Probe(rows(4), ANSI_TOPO), sysfs_root=None).snapshot()
    with pytest.raises(DaemonStartupError) as e:
        relay_candidates_for_policy(inv, DaemonStartupConfig(target_gpu=0, min_relay_count=3))
    msg = str(e.value)
    assert "eligible_relays=[1, 2]" in msg and "3:missing enabled fabric link" in msg


def test_daemon_cli_builds_the_startup_config():
    from pcie_pool_b200.daemon.__main__ import build_parser, startup_config_from_args

    a = build_parser().parse_args(["--target-gpu", "2", "--min-relays", "3", "--allow-missing-fabric",
                                   "--topology-provider", "cuda_nvml", "--max-inflight-chunks-per-relay", "64",
                                   "--execute", "--profile-store", "/tmp/p.json"])
    c = startup_config_from_args(a)
    assert (c.topology_provider, c.target_gpu, c.min_relay_count, c.require_fabric, c.require_pcie) == \
        ("cuda-nvml", 2, 3, False, True)
    assert (c.max_inflight_chunks_per_relay, c.execute, c.profile_store_path) == (64, True, "/tmp/p.json")
    with pytest.raises(SystemExit):
        build_parser().parse_args([])


def test_relays_spread_across_sockets_and_root_complexes():
    """Lanes into GPU0 take relays on the other socket first, then on root
    complexes (and switches) no chosen lane uses yet."""
    from pcie_pool_b200.topology import synthetic_inventory

    inv = synthetic_inventory(8)  # GPUs 0-3 on socket 0, 4-7 on socket 1, one root complex each
    assert inv.spread_relays(0, range(8), 1) == [4]
    assert inv.spread_relays(0, range(8), 3) == [4, 1, 5]
    assert sorted(inv.spread_relays(0, range(8), 7)) == [1, 2, 3, 4, 5, 6, 7]
    # two GPUs per switch, four per root complex: the switch partner of GPU0 comes last on its socket
    inv2 = synthetic_inventory(8, gpus_per_switch=2, gpus_per_root=4)
    assert inv2.spread_relays(0, range(8), 3) == [4, 2, 6]
    # only eligible candidates are chosen
    assert inv.spread_relays(0, [1, 2, 3], 2) == [1, 2]


def test_daemon_recommends_relays_spread_over_uplinks():
    from pcie_pool_b200.daemon import InProcessDaemonClient, TurboBusDaemon
    from pcie_pool_b200.topology import StaticTopologyProvider, synthetic_inventory

    d = TurboBusDaemon(range(1, 8), topology_provider=StaticTopologyProvider(synthetic_inventory(8)))
    r = InProcessDaemonClient(d).discover_relays(0)
    assert r.ok and r.payload["relay_discovery"]["recommended_relays"][:3] == [4, 1, 5]
    assert d.choose_relays(0, 3) == [4, 1, 5]
    assert d.choose_relays(0, 2, candidates=[1, 2, 3]) == [1, 2]


def test_contention_groups_from_measured_rates():
    """The rates of this pool's 8-GPU nodes: every link 55 GB/s alone, with
    all eight busy GPUs 0-3 get ~19 GB/s and GPUs 4-7 ~32 GB/s."""
    from pcie_pool_b200.topology.uplink_probe import contention_groups

    solo = {d: 55.0 + 0.3 * d for d in range(8)}
    conc = {d: (19.3 if d < 4 else 32.5) + 0.1 * d for d in range(8)}
    g = contention_groups(solo, conc)
    assert g[0] == g[1] == g[2] == g[3] != g[4] == g[5] == g[6] == g[7]
    # one level of concurrent rates: no structure to spread over
    assert contention_groups(solo, {d: 26.0 + 0.2 * d for d in range(8)}) == {}
    # a GPU that is slow on its own has a slow link, not a shared one
    assert contention_groups({**solo, 3: 30.0}, conc) == {}
    assert contention_groups({0: 55.0}, {0: 20.0}) == {}


def test_lane_set_spreads_over_measured_groups_before_topology():
    """Each GPU has its own root port in the topology (as NVML reports on
    these nodes); the measured groups still put the relays on the other
    group first: 4 lanes into GPU0 are 0, 4, 1, 5 rather than 0..3."""
    from pcie_pool_b200.topology import StaticTopologyProvider, synthetic_inventory
    from pcie_pool_b200.topology.cuda_nvml import cuda_lane_set

    from dataclasses import replace

    inv = synthetic_inventory(8, gpus_per_root=1)
    # as seen from the VM: one NUMA node, a root port per GPU
    inv = replace(inv, gpus=tuple(replace(g, numa_node=0) for g in inv.gpus),
                  pcie_paths=tuple(replace(p, numa_node=0) for p in inv.pcie_paths))
    bus = {i: _bus_of(inv, i) for i in range(8)}
    groups = {d: ("slow" if d < 4 else "fast") for d in range(8)}
    lanes, info = cuda_lane_set(4, 0, provider=StaticTopologyProvider(inv), bus_ids=bus, groups=groups)
    assert lanes == [0, 4, 1, 5] and info["groups"]["0"] == "slow"
    assert cuda_lane_set(2, 0, provider=StaticTopologyProvider(inv), bus_ids=bus, groups=groups)[0] == [0, 4]
    # without a measurement the topology sees nothing shared: index order
    plain, info = cuda_lane_set(4, 0, provider=StaticTopologyProvider(inv), bus_ids=bus)
    assert "groups" not in info and plain == [0, 1, 2, 3]

    class Broken:
        def snapshot(self):
            raise RuntimeError("no NVML here")

    lanes, info = cuda_lane_set(4, 0, provider=Broken(), bus_ids=bus, groups=groups)
    assert lanes == [0, 4, 1, 5] and "unavailable" in info["topology"]


def _bus_of(inv, i):
    from pcie_pool_b200.topology.cuda_nvml import _bdf

    return _bdf(next(g for g in inv.gpus if g.device_id == i).pci_bus_id)
