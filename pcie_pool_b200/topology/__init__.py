"""Topology inventory: GPUs, their PCIe paths (root complex, switch chain,
NUMA node, link bandwidth) and GPU<->GPU fabric links, plus relay eligibility.

Record names and fields match the reference (turbobus/topology/__init__.py:7-306)
because the daemon exports them on the wire (GET_INVENTORY, TopologySnapshot).
Relay eligibility drops, with a recorded reason, the target itself, unknown
GPUs, GPUs without a PCIe path and GPUs without an enabled fabric link to the
target.  ``uplink_groups`` is new: GPUs behind the same PCIe switch or root
port share one uplink and are planned against its concurrent capacity.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field
from collections.abc import Mapping
from typing import Iterable

from ..schema import as_bool, as_float, nonempty, nonneg_float, nonneg_int, opt


def _coerce(obj, table) -> None:
    for name, fn in table.items():
        object.__setattr__(obj, name, fn(getattr(obj, name), name))


@dataclass(frozen=True)
class GpuInventoryRecord:
    device_id: int
    backend: str = "unknown"
    vendor: str = "unknown"
    uuid: str | None = None
    pci_bus_id: str | None = None
    numa_node: int | None = None
    memory_bytes: int | None = None
    role: str = "general"
    visible: bool = True

    def __post_init__(self) -> None:
        _coerce(self, {"device_id": nonneg_int, "backend": nonempty, "vendor": nonempty,
                       "uuid": opt(lambda v, n: str(v)), "pci_bus_id": opt(lambda v, n: str(v)),
                       "numa_node": opt(nonneg_int), "memory_bytes": opt(nonneg_int),
                       "role": nonempty, "visible": as_bool})


@dataclass(frozen=True)
class PciePathRecord:
    device_id: int
    numa_node: int | None = None
    root_complex: str | None = None
    link_generation: int | None = None
    link_width: int | None = None
    bandwidth_gbps: float = 0.0
    negotiated_speed_gtps: float | None = None
    switch_hierarchy: tuple[str, ...] = field(default_factory=tuple)
    bandwidth_source: str | None = None

    def __post_init__(self) -> None:
        _coerce(self, {"device_id": nonneg_int, "numa_node": opt(nonneg_int),
                       "root_complex": opt(lambda v, n: str(v)),
                       "link_generation": opt(nonneg_int), "link_width": opt(nonneg_int),
                       "bandwidth_gbps": nonneg_float, "negotiated_speed_gtps": opt(nonneg_float),
                       "bandwidth_source": opt(lambda v, n: nonempty(str(v).strip(), n))})
        object.__setattr__(self, "switch_hierarchy",
                           tuple(str(s) for s in self.switch_hierarchy if str(s).strip()))

    @property
    def uplink(self) -> str | None:
        """Identity of the shared uplink: the top switch port below the root
        complex when one exists, else the root complex."""
        if self.switch_hierarchy:
            return self.switch_hierarchy[0]
        return self.root_complex


@dataclass(frozen=True)
class FabricLinkRecord:
    src_device_id: int
    dst_device_id: int
    fabric: str = "unknown"
    bandwidth_gbps: float = 0.0
    bidirectional: bool = True
    enabled: bool = False
    link_count: int | None = None
    capability: str | None = None
    raw_link_type: str | None = None

    def __post_init__(self) -> None:
        _coerce(self, {"src_device_id": nonneg_int, "dst_device_id": nonneg_int,
                       "fabric": nonempty, "bandwidth_gbps": nonneg_float,
                       "bidirectional": as_bool, "enabled": as_bool,
                       "link_count": opt(nonneg_int),
                       "capability": opt(lambda v, n: nonempty(str(v).strip(), n)),
                       "raw_link_type": opt(lambda v, n: nonempty(str(v).strip(), n))})
        if self.src_device_id == self.dst_device_id:
            raise ValueError("fabric link endpoints must be distinct")

    def connects(self, a: int, b: int) -> bool:
        if not self.enabled:
            return False
        if self.src_device_id == a and self.dst_device_id == b:
            return True
        return self.bidirectional and self.src_device_id == b and self.dst_device_id == a


@dataclass(frozen=True)
class DaemonResourceInventory:
    gpus: tuple[GpuInventoryRecord, ...] = field(default_factory=tuple)
    pcie_paths: tuple[PciePathRecord, ...] = field(default_factory=tuple)
    fabric_links: tuple[FabricLinkRecord, ...] = field(default_factory=tuple)
    source: str = "discovered"
    discovered_at: float = 0.0
    snapshot_id: str | None = None
    version: int = 0
    metadata: Mapping[str, object] = field(default_factory=dict)

    def __post_init__(self) -> None:
        _coerce(self, {"source": nonempty, "discovered_at": nonneg_float, "version": nonneg_int,
                       "snapshot_id": opt(nonempty)})
        object.__setattr__(self, "gpus", tuple(self.gpus))
        object.__setattr__(self, "pcie_paths", tuple(self.pcie_paths))
        object.__setattr__(self, "fabric_links", tuple(self.fabric_links))
        object.__setattr__(self, "metadata", dict(self.metadata))

    def as_dict(self) -> dict[str, object]:
        return asdict(self)

    def topology_snapshot_id(self) -> str:
        if self.snapshot_id is not None:
            return self.snapshot_id
        return f"topology-{self.source.replace(' ', '_')}-v{self.version}-{self.discovered_at:.6f}"

    def to_topology_snapshot(self):
        from ..schema import TopologySnapshot

        return TopologySnapshot(
            snapshot_id=self.topology_snapshot_id(), source=self.source,
            discovered_at=self.discovered_at, version=self.version,
            devices=tuple({"device_id": g.device_id, "kind": "gpu", "backend": g.backend,
                           "vendor": g.vendor, "uuid": g.uuid, "pci_bus_id": g.pci_bus_id,
                           "numa_node": g.numa_node, "memory_bytes": g.memory_bytes,
                           "role": g.role, "visible": g.visible} for g in self.gpus),
            pcie_links=tuple(asdict(p) for p in self.pcie_paths),
            fabric_links=tuple(asdict(l) for l in self.fabric_links),
            numa_nodes=tuple({"numa_node": n, "devices": [p.device_id for p in self.pcie_paths
                                                          if p.numa_node == n]}
                             for n in sorted({p.numa_node for p in self.pcie_paths
                                              if p.numa_node is not None})),
            metadata={**dict(self.metadata), "inventory_source": self.source,
                      "inventory_snapshot_id": self.topology_snapshot_id()})

    def pcie_path(self, device: int) -> PciePathRecord | None:
        for p in self.pcie_paths:
            if p.device_id == int(device):
                return p
        return None

    def has_fabric_link(self, a: int, b: int) -> bool:
        return any(l.connects(int(a), int(b)) for l in self.fabric_links)

    def uplink_groups(self) -> dict[int, int]:
        """device -> group id; devices behind the same uplink share an id."""
        ids: dict[str, int] = {}
        out: dict[int, int] = {}
        for p in self.pcie_paths:
            key = p.uplink
            if key is None:
                continue
            out[p.device_id] = ids.setdefault(key, len(ids))
        return out

    def uplink_keys(self, device: int) -> tuple[str | None, str | None, str | None]:
        """(socket, root complex, top switch) of a GPU's PCIe path, the three
        levels at which lanes share upstream bandwidth; None where unknown."""
        p = self.pcie_path(int(device))
        if p is None:
            return (None, None, None)
        sock = None if p.numa_node is None else f"numa{p.numa_node}"
        return (sock, p.root_complex, p.switch_hierarchy[0] if p.switch_hierarchy else None)

    def spread_relays(self, target_device: int, candidates: Iterable[int], count: int) -> list[int]:
        """Pick ``count`` relays from eligible ``candidates`` for lanes into
        ``target_device`` so the lane set (target included) shares as little
        upstream PCIe as possible: greedily the candidate whose socket, then
        root complex, then top switch carries the fewest lanes chosen so far
        (ties: lower index).  Lanes behind one root port or socket share its
        bandwidth, so spreading them raises the aggregate (on an 8-GPU node
        whose GPUs 0-3 share a socket, 4 lanes as {0, 4, 1, 5} rather than
        {0, 1, 2, 3}).  The reference picks relays by index and isolated
        per-link bandwidth (turbobus/scheduler/daemon.py:222-281)."""
        pool = list(self.eligible_relay_devices(int(target_device), candidates))
        return spread_by_keys(int(target_device), pool, count, self.uplink_keys)

    def eligible_relay_devices(self, target_device: int, requested_relays: Iterable[int]) -> tuple[int, ...]:
        return tuple(e["relay_gpu"] for e in
                     self.relay_eligibility(target_device, requested_relays)["eligible_relays"])

    def relay_eligibility(self, target_device: int, requested_relays: Iterable[int]) -> dict[str, object]:
        requested = sorted({int(g) for g in requested_relays})
        target = int(target_device)
        filtered: list[dict[str, object]] = []
        checks = [("target gpu cannot relay", lambda g: g != target)]
        if self.gpus:
            known = {g.device_id for g in self.gpus}
            checks.append(("unknown gpu", lambda g: g in known))
        if self.pcie_paths:
            has_path = {p.device_id for p in self.pcie_paths}
            checks.append(("missing pcie path", lambda g: g in has_path))
        if self.fabric_links:
            checks.append(("missing enabled fabric link", lambda g: self.has_fabric_link(g, target)))
        kept = list(requested)
        for reason, ok in checks:
            filtered.extend({"relay_gpu": g, "reason": reason} for g in kept if not ok(g))
            kept = [g for g in kept if ok(g)]
        return {"requested_relays": requested,
                "eligible_relays": [{"relay_gpu": g, "reason": "eligible"} for g in kept],
                "filtered_relays": filtered, "inventory_source": self.source,
                "inventory_discovered_at": self.discovered_at}


class TopologyProvider:
    def snapshot(self) -> DaemonResourceInventory:
        raise NotImplementedError

    def invalidate(self) -> None:
        raise NotImplementedError


class StaticTopologyProvider(TopologyProvider):
    """Fixed inventory (tests, simulations).  Its source is tagged
    ``test_fixture_static`` so production startup refuses it."""

    FIXTURE_SOURCE = "test_fixture_static"

    def __init__(self, inventory: DaemonResourceInventory | None = None, *, gpu_count: int = 4,
                 fabric: str = "nvswitch") -> None:
        self._inventory = inventory or synthetic_inventory(gpu_count, fabric=fabric,
                                                           source=self.FIXTURE_SOURCE)
        self.invalidations = 0

    def snapshot(self) -> DaemonResourceInventory:
        return self._inventory

    def invalidate(self) -> None:
        self.invalidations += 1


def spread_by_keys(target: int, pool: Iterable[int], count: int, keys_of) -> list[int]:
    """Greedy uplink spreading (see ``DaemonResourceInventory.spread_relays``)
    over any device numbering: ``keys_of(dev)`` gives its sharing keys, most
    significant first -- (socket, root complex, top switch), optionally led by
    a measured contention group."""
    pool = list(pool)
    levels = max([len(tuple(keys_of(int(target))))] + [len(tuple(keys_of(d))) for d in pool])
    load: list[dict[str, int]] = [{} for _ in range(levels)]

    def add(dev: int) -> None:
        for lvl, key in enumerate(keys_of(dev)):
            if key is not None:
                load[lvl][key] = load[lvl].get(key, 0) + 1

    def cost(dev: int):
        return tuple(load[lvl].get(k, 0) if k is not None else 0 for lvl, k in enumerate(keys_of(dev))) + (dev,)

    add(int(target))
    out: list[int] = []
    while pool and len(out) < max(0, int(count)):
        best = min(pool, key=cost)
        pool.remove(best)
        out.append(best)
        add(best)
    return out


def synthetic_inventory(gpu_count: int, *, fabric: str = "nvswitch", source: str = "synthetic",
                        gen: int = 5, width: int = 16, gpus_per_switch: int = 1,
                        gpus_per_root: int | None = None) -> DaemonResourceInventory:
    """An HGX-like node: every GPU on its own Gen5 x16 link (or
    ``gpus_per_switch`` GPUs per switch), all pairs joined by the fabric; the
    first half of the GPUs on socket (NUMA node) 0, the rest on 1, and
    ``gpus_per_root`` GPUs per root complex (default: one per switch)."""
    per_root = gpus_per_root or gpus_per_switch
    gpus = tuple(GpuInventoryRecord(i, backend="cuda", vendor="nvidia", uuid=f"GPU-synthetic-{i}",
                                    pci_bus_id=f"0000:{0x10 * (i + 1):02x}:00.0",
                                    numa_node=0 if i < max(1, gpu_count // 2) else 1,
                                    memory_bytes=183359 << 20) for i in range(gpu_count))
    paths = tuple(PciePathRecord(i, numa_node=g.numa_node,
                                 root_complex=f"0000:{0x10 * (i // per_root + 1):02x}",
                                 link_generation=gen, link_width=width,
                                 bandwidth_gbps=round(pcie_gbps(gen, width) or 0.0, 3),
                                 switch_hierarchy=(f"switch{i // gpus_per_switch}",),
                                 bandwidth_source="synthetic") for i, g in enumerate(gpus))
    links = tuple(FabricLinkRecord(a, b, fabric=fabric, enabled=True, link_count=18,
                                   capability=fabric, raw_link_type="NV18")
                  for a in range(gpu_count) for b in range(a + 1, gpu_count))
    return DaemonResourceInventory(gpus=gpus, pcie_paths=paths, fabric_links=links, source=source,
                                   discovered_at=1.0, version=1,
                                   metadata={"provider": source, "gpu_count": gpu_count})


# PCIe usable bandwidth per lane after encoding, GB/s (Gen3+ 128b/130b).
PCIE_GBPS_PER_LANE = {1: 0.25, 2: 0.5, 3: 0.985, 4: 1.969, 5: 3.938, 6: 7.877}
PCIE_GTPS = {1: 2.5, 2: 5.0, 3: 8.0, 4: 16.0, 5: 32.0, 6: 64.0}


def pcie_gbps(gen: int | None, width: int | None) -> float | None:
    if gen is None or width is None or int(width) <= 0:
        return None
    per = PCIE_GBPS_PER_LANE.get(int(gen))
    return None if per is None else round(per * int(width), 3)


__all__ = ["DaemonResourceInventory", "FabricLinkRecord", "GpuInventoryRecord", "PCIE_GBPS_PER_LANE",
           "PCIE_GTPS", "PciePathRecord", "StaticTopologyProvider", "TopologyProvider", "pcie_gbps",
           "spread_by_keys", "synthetic_inventory"]
