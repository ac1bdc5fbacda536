"""Topology discovery on a real node.

Three probes, tried in order, each returning the same row shape:
  * ``NvmlProbe``    - NVML through ctypes (index, UUID, bus id, memory, current
                       PCIe generation/width, NVLink state, P2P status);
  * ``NvidiaSmiProbe`` - ``nvidia-smi --query-gpu`` + ``nvidia-smi topo -m``
                       (the reference's only probe, topology/cuda_nvml.py:70-130);
  * sysfs (``pcie_tree``) - walks ``/sys/bus/pci/devices/<bdf>`` up to the root
                       port for the switch chain, NUMA node and link speed.
``CudaNvmlTopologyProvider`` merges them into a ``DaemonResourceInventory``
and caches it for ``cache_max_age_seconds`` (30 s by default).
"""

from __future__ import annotations

import csv
import ctypes
import os
import re
import subprocess
import time
from dataclasses import dataclass
from pathlib import Path
from collections.abc import Mapping
from typing import Callable, Protocol, Sequence

from . import (PCIE_GTPS, DaemonResourceInventory, FabricLinkRecord, GpuInventoryRecord,
               PciePathRecord, TopologyProvider, pcie_gbps)


class TopologyDiscoveryError(RuntimeError):
    pass


class CudaTopologyProbe(Protocol):
    def query_gpu_inventory(self) -> Sequence[Mapping[str, object]]:
        ...

    def query_topology_matrix(self) -> Sequence[str]:
        ...


# ---- nvidia-smi ------------------------------------------------------------------------

SMI_FIELD_SETS = (
    ("index", "uuid", "pci.bus_id", "memory.total", "pcie.link.gen.current",
     "pcie.link.width.current"),
    ("index", "uuid", "pci.bus_id", "memory.total"),
)
SMI_KEYS = {"index": "device_id", "uuid": "uuid", "pci.bus_id": "pci_bus_id",
            "memory.total": "memory_mib", "pcie.link.gen.current": "pcie_link_gen_current",
            "pcie.link.width.current": "pcie_link_width_current"}


@dataclass(frozen=True)
class NvidiaSmiProbe:
    executable: str = "nvidia-smi"
    timeout_seconds: float = 5.0

    def query_gpu_inventory(self) -> Sequence[Mapping[str, object]]:
        err: Exception | None = None
        for fields in SMI_FIELD_SETS:
            try:
                out = self._run([self.executable, "--query-gpu=" + ",".join(fields),
                                 "--format=csv,noheader,nounits"])
            except TopologyDiscoveryError as exc:
                err = exc
                continue
            rows = []
            ok = True
            for row in csv.reader(out.splitlines()):
                if not row:
                    continue
                if len(row) < len(fields):
                    ok = False
                    err = TopologyDiscoveryError("nvidia-smi gpu inventory output is missing fields")
                    break
                rows.append({SMI_KEYS[f]: v.strip() for f, v in zip(fields, row)})
            if ok:
                return rows
        if err:
            raise err
        return ()

    def query_topology_matrix(self) -> Sequence[str]:
        try:
            return self._run([self.executable, "topo", "-m"]).splitlines()
        except TopologyDiscoveryError:
            return ()

    def _run(self, cmd: Sequence[str]) -> str:
        try:
            done = subprocess.run(list(cmd), capture_output=True, text=True, check=False,
                                  timeout=float(self.timeout_seconds))
        except (OSError, subprocess.TimeoutExpired) as exc:
            raise TopologyDiscoveryError(f"failed to run {cmd[0]}: {exc}") from exc
        if done.returncode != 0:
            raise TopologyDiscoveryError(
                f"{cmd[0]} failed with exit code {done.returncode}: "
                f"{(done.stderr or done.stdout or '').strip()}")
        return done.stdout


# ---- NVML through ctypes -----------------------------------------------------------------

class _PciInfo(ctypes.Structure):
    _fields_ = [("busIdLegacy", ctypes.c_char * 16), ("domain", ctypes.c_uint),
                ("bus", ctypes.c_uint), ("device", ctypes.c_uint),
                ("pciDeviceId", ctypes.c_uint), ("pciSubSystemId", ctypes.c_uint),
                ("busId", ctypes.c_char * 32)]


class _Memory(ctypes.Structure):
    _fields_ = [("total", ctypes.c_ulonglong), ("free", ctypes.c_ulonglong),
                ("used", ctypes.c_ulonglong)]


NVML_P2P_CAPS_INDEX_READ = 0
NVML_P2P_STATUS_OK = 0
NVML_NVLINK_MAX_LINKS = 18


class NvmlProbe:
    """NVML probe.  ``lib`` may be injected (tests pass a fake with the same
    function names); otherwise ``libnvidia-ml.so.1`` is loaded."""

    def __init__(self, lib=None, devices: Sequence[int] | None = None) -> None:
        if lib is None:
            try:
                lib = ctypes.CDLL("libnvidia-ml.so.1")
            except OSError as exc:
                raise TopologyDiscoveryError(f"NVML unavailable: {exc}") from exc
        self._lib = lib
        # only these GPU indices are queried (None: every GPU of the node)
        self.devices = None if devices is None else tuple(int(d) for d in devices)
        rc = self._lib.nvmlInit_v2()
        if rc != 0:
            raise TopologyDiscoveryError(f"nvmlInit failed with {rc}")

    def _handle(self, i: int):
        h = ctypes.c_void_p()
        rc = self._lib.nvmlDeviceGetHandleByIndex_v2(ctypes.c_uint(i), ctypes.byref(h))
        if rc != 0:
            raise TopologyDiscoveryError(f"nvmlDeviceGetHandleByIndex({i}) failed with {rc}")
        return h

    def device_count(self) -> int:
        n = ctypes.c_uint()
        rc = self._lib.nvmlDeviceGetCount_v2(ctypes.byref(n))
        if rc != 0:
            raise TopologyDiscoveryError(f"nvmlDeviceGetCount failed with {rc}")
        return int(n.value)

    def query_gpu_inventory(self) -> Sequence[Mapping[str, object]]:
        rows = []
        n = self.device_count()
        for i in (range(n) if self.devices is None else [d for d in self.devices if 0 <= d < n]):
            h = self._handle(i)
            row: dict[str, object] = {"device_id": i}
            buf = ctypes.create_string_buffer(96)
            if self._lib.nvmlDeviceGetUUID(h, buf, ctypes.c_uint(96)) == 0:
                row["uuid"] = buf.value.decode()
            pci = _PciInfo()
            if self._lib.nvmlDeviceGetPciInfo_v3(h, ctypes.byref(pci)) == 0:
                row["pci_bus_id"] = pci.busId.decode()
            mem = _Memory()
            if self._lib.nvmlDeviceGetMemoryInfo(h, ctypes.byref(mem)) == 0:
                row["memory_bytes"] = int(mem.total)
            v = ctypes.c_uint()
            if self._lib.nvmlDeviceGetCurrPcieLinkGeneration(h, ctypes.byref(v)) == 0:
                row["pcie_link_gen_current"] = int(v.value)
            if self._lib.nvmlDeviceGetCurrPcieLinkWidth(h, ctypes.byref(v)) == 0:
                row["pcie_link_width_current"] = int(v.value)
            active = 0
            for link in range(NVML_NVLINK_MAX_LINKS):
                st = ctypes.c_int()
                if self._lib.nvmlDeviceGetNvLinkState(h, ctypes.c_uint(link), ctypes.byref(st)) == 0 \
                        and st.value == 1:
                    active += 1
            row["nvlink_active_links"] = active
            rows.append(row)
        return rows

    def p2p_read_ok(self, a: int, b: int) -> bool:
        st = ctypes.c_int(-1)
        rc = self._lib.nvmlDeviceGetP2PStatus(self._handle(a), self._handle(b),
                                              ctypes.c_int(NVML_P2P_CAPS_INDEX_READ), ctypes.byref(st))
        return rc == 0 and st.value == NVML_P2P_STATUS_OK

    def query_topology_matrix(self) -> Sequence[str]:
        return ()


# ---- sysfs ------------------------------------------------------------------------------

def pcie_tree(bus_id: str, root: str | os.PathLike = "/sys") -> dict[str, object]:
    """Walk a PCI function's sysfs path: numa node, current link, and the chain
    of bridges between the root complex and the device (top first)."""
    bdf = _norm_bdf(bus_id)
    dev = Path(root) / "bus" / "pci" / "devices" / bdf
    out: dict[str, object] = {}
    if not dev.exists():
        return out
    real = dev.resolve()
    parts = [p for p in real.parts if _looks_bdf(p)]
    # parts: [root port, switch up, switch down, ..., device]
    if parts:
        out["switch_hierarchy"] = tuple(parts[:-1])
        out["root_complex"] = ":".join(parts[0].split(":")[:2]) if parts else None
    numa = _read(dev / "numa_node")
    if numa is not None and numa.lstrip("-").isdigit() and int(numa) >= 0:
        out["numa_node"] = int(numa)
    speed = _read(dev / "current_link_speed")
    if speed:
        try:
            out["negotiated_speed_gtps"] = float(speed.split()[0])
        except ValueError:
            pass
    width = _read(dev / "current_link_width")
    if width and width.strip().isdigit():
        out["link_width"] = int(width)
    return out


def _read(p: Path) -> str | None:
    try:
        return p.read_text().strip()
    except OSError:
        return None


def _looks_bdf(s: str) -> bool:
    bits = s.split(":")
    return len(bits) == 3 and "." in bits[2]


def _norm_bdf(bus_id: str) -> str:
    text = str(bus_id).strip().lower()
    bits = text.split(":")
    if len(bits) == 3 and len(bits[0]) > 4:  # nvidia-smi prints an 8-digit domain
        bits[0] = bits[0][-4:]
    return ":".join(bits)


def _gen_from_gtps(gtps: float | None) -> int | None:
    if gtps is None:
        return None
    for gen, v in PCIE_GTPS.items():
        if abs(v - gtps) < 0.5:
            return gen
    return None


# ---- topology matrix parsing -------------------------------------------------------------

def fabric_capability(token: str) -> dict[str, object] | None:
    """Classify one ``nvidia-smi topo -m`` cell: NV# / NVSW -> NVLink /
    NVSwitch, PIX/PXB/PHB -> PCIe peer-to-peer, SYS/NODE/X -> no fabric."""
    t = str(token).strip().upper()
    if not t or t in {"X", "N/A", "SYS", "NODE"}:
        return None
    if t.startswith("NV"):
        fabric = "nvswitch" if t in {"NVSW", "NVS", "NVSWITCH"} else "nvlink"
        count = int(t[2:]) if t[2:].isdigit() else None
        return {"fabric": fabric, "capability": fabric, "link_count": count, "raw_link_type": t}
    if t in {"PIX", "PXB", "PHB"}:
        return {"fabric": "cuda_p2p", "capability": f"cuda_p2p_{t.lower()}", "link_count": None,
                "raw_link_type": t}
    return None


_ANSI = re.compile(r"\x1b\[[0-9;]*[A-Za-z]")


def fabric_links_from_matrix(gpu_ids: set[int], lines: Sequence[str]) -> tuple[FabricLinkRecord, ...]:
    # nvidia-smi underlines the header row with ANSI escapes; the header is the
    # first row whose first token is a GPU column name and whose second token
    # is another column name (data rows have a cell there instead)
    rows = [_ANSI.sub("", str(ln)).split() for ln in lines if str(ln).strip()]
    header = next((r for r in rows if len(r) > 1 and r[0].startswith("GPU") and r[1].startswith("GPU")), None)
    if not header:
        return ()

    def gid(s: str) -> int | None:
        s = s.strip()
        # tolerate escape sequences nvidia-smi puts around the header
        s = s[s.find("GPU"):] if "GPU" in s else s
        try:
            return int(s[3:]) if s.startswith("GPU") else None
        except ValueError:
            return None

    out = []
    for r in rows:
        src = gid(r[0]) if r else None
        if src is None or src not in gpu_ids or r is header:
            continue
        for col, name in enumerate(header):
            dst = gid(name)
            if dst is None or dst not in gpu_ids or dst <= src or col + 1 >= len(r):
                continue
            cap = fabric_capability(r[col + 1])
            if cap is None:
                continue
            out.append(FabricLinkRecord(src, dst, fabric=str(cap["fabric"]), bidirectional=True,
                                        enabled=True, link_count=cap["link_count"],
                                        capability=str(cap["capability"]),
                                        raw_link_type=str(cap["raw_link_type"])))
    return tuple(out)


# ---- provider ---------------------------------------------------------------------------

class CudaNvmlTopologyProvider(TopologyProvider):
    def __init__(self, probe: CudaTopologyProbe | None = None, *, cache_max_age_seconds: float = 30.0,
                 now: Callable[[], float] | None = None, sysfs_root: str | None = "/sys",
                 fabric_probe: CudaTopologyProbe | None = None,
                 devices: Sequence[int] | None = None) -> None:
        """``devices`` limits discovery to those GPU indices: a daemon that
        may only use part of a shared node queries nothing about the rest."""
        self._devices = None if devices is None else frozenset(int(d) for d in devices)
        if probe is None:
            try:
                probe = NvmlProbe(devices=devices)
            except TopologyDiscoveryError:
                probe = NvidiaSmiProbe()
        self._probe = probe
        self._fabric_probe = fabric_probe
        self._max_age = max(0.0, float(cache_max_age_seconds))
        self._now = now or time.time
        self._sysfs = sysfs_root
        self._cached: DaemonResourceInventory | None = None
        self._version = 0

    def snapshot(self) -> DaemonResourceInventory:
        now = float(self._now())
        if self._cached is not None and self._max_age > 0.0 \
                and now - self._cached.discovered_at <= self._max_age:
            return self._cached
        rows = list(self._probe.query_gpu_inventory())
        if self._devices is not None:
            rows = [r for r in rows if int(r.get("device_id", r.get("index", -1))) in self._devices]
        if not rows:
            raise TopologyDiscoveryError("cuda-nvml topology discovery found no GPUs")
        gpus = tuple(_gpu_record(r) for r in rows)
        paths = tuple(self._pcie_path(g, r) for g, r in zip(gpus, rows))
        matrix = list(self._probe.query_topology_matrix())
        if not matrix and self._fabric_probe is not None:
            matrix = list(self._fabric_probe.query_topology_matrix())
        links = fabric_links_from_matrix({g.device_id for g in gpus}, matrix)
        if not links and isinstance(self._probe, NvmlProbe):
            links = self._nvml_links(gpus)
        self._version += 1
        inv = DaemonResourceInventory(
            gpus=gpus, pcie_paths=paths, fabric_links=links, source="cuda_nvml",
            discovered_at=now, snapshot_id=f"topology-cuda_nvml-v{self._version}-{now:.6f}",
            version=self._version,
            metadata={"provider": "cuda-nvml", "probe": type(self._probe).__name__,
                      "gpu_count": len(gpus), "cache_max_age_seconds": self._max_age})
        self._cached = inv
        return inv

    def invalidate(self) -> None:
        self._cached = None

    def _pcie_path(self, gpu: GpuInventoryRecord, row: Mapping[str, object]) -> PciePathRecord:
        tree = pcie_tree(gpu.pci_bus_id, self._sysfs) if (gpu.pci_bus_id and self._sysfs) else {}
        gen = _first_int(row, ("pcie_link_gen_current", "link_generation"))
        width = _first_int(row, ("pcie_link_width_current", "link_width"))
        if gen is None:
            gen = _gen_from_gtps(tree.get("negotiated_speed_gtps"))  # type: ignore[arg-type]
        if width is None:
            width = tree.get("link_width")  # type: ignore[assignment]
        explicit = _first_float(row, ("pcie_bandwidth_gbps", "bandwidth_gbps"))
        est = pcie_gbps(gen, width)
        bw = explicit if explicit is not None else (est or 0.0)
        src = "provider" if explicit is not None else ("estimated_from_pcie_generation_width"
                                                       if est is not None else None)
        numa = _first_int(row, ("numa_node",))
        if numa is None:
            numa = tree.get("numa_node")  # type: ignore[assignment]
        root = _optional_str(row.get("root_complex")) or tree.get("root_complex") \
            or _root_complex(gpu.pci_bus_id)
        hier = row.get("switch_hierarchy") or tree.get("switch_hierarchy") or ()
        if isinstance(hier, str):
            hier = tuple(h.strip() for h in hier.replace(">", ",").split(",") if h.strip())
        gtps = tree.get("negotiated_speed_gtps") or (PCIE_GTPS.get(int(gen)) if gen else None)
        return PciePathRecord(gpu.device_id, numa_node=numa, root_complex=root,
                              link_generation=gen, link_width=width, bandwidth_gbps=bw,
                              negotiated_speed_gtps=gtps, switch_hierarchy=tuple(hier),
                              bandwidth_source=src)

    def _nvml_links(self, gpus) -> tuple[FabricLinkRecord, ...]:
        out = []
        ids = [g.device_id for g in gpus]
        for i, a in enumerate(ids):
            for b in ids[i + 1:]:
                try:
                    ok = self._probe.p2p_read_ok(a, b)  # type: ignore[attr-defined]
                except Exception:
                    ok = False
                if ok:
                    out.append(FabricLinkRecord(a, b, fabric="nvlink", enabled=True,
                                                capability="nvml_p2p_read", raw_link_type="NVML"))
        return tuple(out)


def _gpu_record(row: Mapping[str, object]) -> GpuInventoryRecord:
    mem = row.get("memory_bytes")
    if mem is None and row.get("memory_mib") not in (None, ""):
        mem = int(float(str(row["memory_mib"]))) * 1024 * 1024
    return GpuInventoryRecord(
        device_id=int(row.get("device_id", row.get("index", 0))), backend="cuda", vendor="nvidia",
        uuid=_optional_str(row.get("uuid")), pci_bus_id=_optional_str(row.get("pci_bus_id")),
        numa_node=_first_int(row, ("numa_node",)), memory_bytes=None if mem is None else int(mem),
        role=_optional_str(row.get("role")) or "general",
        visible=str(row.get("visible", True)).lower() not in ("0", "false", "no"))


def _optional_str(v) -> str | None:
    if v is None:
        return None
    t = str(v).strip()
    return None if not t or t.upper() in ("N/A", "[N/A]") else t


def _first_int(row: Mapping[str, object], keys) -> int | None:
    for k in keys:
        v = row.get(k)
        if v is None:
            continue
        t = str(v).strip()
        if not t or t.upper() in ("N/A", "[N/A]"):
            continue
        try:
            return int(float(t))
        except ValueError:
            continue
    return None


def _first_float(row: Mapping[str, object], keys) -> float | None:
    for k in keys:
        v = row.get(k)
        if v is None or not str(v).strip():
            continue
        try:
            return float(str(v).strip())
        except ValueError:
            continue
    return None


def _root_complex(bus_id: str | None) -> str | None:
    """``domain:bus`` of a bus id, in the sysfs spelling (4-digit lower-case
    domain) so it groups with root complexes read from sysfs."""
    if not bus_id:
        return None
    parts = _norm_bdf(bus_id).split(":")
    return ":".join(parts[:2]) if len(parts) >= 2 else str(bus_id)


__all__ = ["CudaNvmlTopologyProvider", "CudaTopologyProbe", "NvidiaSmiProbe", "NvmlProbe",
           "TopologyDiscoveryError", "fabric_capability", "fabric_links_from_matrix", "pcie_tree"]


def _bdf(s: str | None) -> tuple[int, int, int] | None:
    """(domain, bus, device) of a PCI address like ``00000000:18:00.0``."""
    if not s:
        return None
    try:
        dom, bus, rest = str(s).strip().lower().split(":")
        return int(dom, 16), int(bus, 16), int(rest.split(".")[0], 16)
    except ValueError:
        return None


def cuda_lane_set(n: int, target: int = 0, provider: "CudaNvmlTopologyProvider | None" = None,
                  bus_ids: dict[int, tuple[int, int, int]] | None = None,
                  groups: dict[int, str] | None = None) -> tuple[list[int], dict]:
    """CUDA device indices of ``target`` plus ``n - 1`` relays among the
    visible GPUs, spread over PCIe uplinks (socket, root complex, switch)
    with the daemon's rule.  Topology comes from NVML and sysfs and CUDA
    indices are matched to it by PCI address, so no CUDA context is created
    on any GPU.  ``groups`` (CUDA index -> measured contention group,
    ``uplink_probe.contention_groups``) leads the keys when given.  Falls
    back to ``target, 0, 1, ...`` when discovery fails."""
    from . import spread_by_keys

    groups = {int(k): v for k, v in (groups or {}).items()}
    info: dict = {"rule": "spread over measured contention group, socket, root complex, switch" if groups
                  else "spread over socket, root complex, switch"}
    if bus_ids is None:
        import torch

        bus_ids = {}
        for i in range(torch.cuda.device_count()):
            p = torch.cuda.get_device_properties(i)
            bus_ids[i] = (int(p.pci_domain_id), int(p.pci_bus_id), int(p.pci_device_id))
    cands = [i for i in sorted(bus_ids) if i != int(target)]
    fallback = [int(target)] + cands[:max(0, n - 1)]
    if n <= 1:
        return [int(target)], {**info, "reason": "single lane"}
    try:
        inv = (provider or CudaNvmlTopologyProvider()).snapshot()
    except Exception as exc:  # noqa: BLE001 - any discovery failure keeps the index order
        if groups:  # the measurement alone still spreads the lanes
            relays = spread_by_keys(int(target), cands, n - 1, lambda i: (groups.get(i),))
            return [int(target), *relays], {**info, "groups": groups, "topology": f"unavailable: {exc}"}
        return fallback, {**info, "fallback": f"topology unavailable: {exc}"}
    nvml_of = {}
    by_bdf = {_bdf(g.pci_bus_id): g.device_id for g in inv.gpus}
    for i, b in bus_ids.items():
        if b in by_bdf:
            nvml_of[i] = by_bdf[b]
    if int(target) not in nvml_of:
        return fallback, {**info, "fallback": "target GPU not found in the topology"}

    def keys(i: int):
        topo = inv.uplink_keys(nvml_of[i]) if i in nvml_of else (None, None, None)
        return (groups.get(i), *topo) if groups else topo

    relays = spread_by_keys(int(target), [c for c in cands if c in nvml_of], n - 1, keys)
    if len(relays) < n - 1:
        relays += [c for c in cands if c not in relays][:n - 1 - len(relays)]
    info["uplinks"] = {str(i): list(keys(i)) for i in [int(target), *relays]}
    if groups:
        info["groups"] = {str(k): v for k, v in sorted(groups.items())}
    return [int(target), *relays], info
