"""Production bootstrap of the daemon.

Discovers the node (NVML / nvidia-smi / sysfs), refuses synthetic test
topologies, applies the relay policy (minimum relay count, PCIe and fabric
requirements) and, unlike the reference (turbobus/daemon/startup.py:50-65,
which starts with an empty profile cache so every plan falls back to the
direct lane), can attach the GPU executor and measure link bandwidth at
startup so the first intent already pools lanes.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

from ..topology import DaemonResourceInventory, TopologyProvider
from ..topology.cuda_nvml import CudaNvmlTopologyProvider, TopologyDiscoveryError
from .server import TurboBusDaemon


class DaemonStartupError(RuntimeError):
    pass


@dataclass(frozen=True)
class DaemonStartupConfig:
    topology_provider: str = "cuda-nvml"
    target_gpu: int | None = None
    min_relay_count: int = 1
    require_fabric: bool = True
    require_pcie: bool = True
    max_sessions_per_relay: int = 1
    max_inflight_chunks_per_relay: int = 8
    session_timeout_seconds: float = 0.0
    profile_max_age_seconds: float = 0.0
    execute: bool = False            # attach the GPU executor (data plane in the daemon)
    profile_on_start: bool = False   # run the link probe and cache profiles at startup
    profile_store_path: str | None = None
    # GPUs the daemon may discover, lend and drive (None: every GPU of the
    # node); on a shared node the others are never queried or touched
    devices: tuple[int, ...] | None = None
    executor_workers: int = 4

    def __post_init__(self) -> None:
        if self.devices is not None:
            object.__setattr__(self, "devices", tuple(int(d) for d in self.devices))
            if self.target_gpu is not None and int(self.target_gpu) not in self.devices:
                raise ValueError("target_gpu must be one of the daemon's devices")
        if int(self.executor_workers) < 1:
            raise ValueError("executor_workers must be >= 1")
        if int(self.min_relay_count) < 0:
            raise ValueError("min_relay_count must be non-negative")
        if self.target_gpu is not None and int(self.target_gpu) < 0:
            raise ValueError("target_gpu must be non-negative")
        object.__setattr__(self, "topology_provider",
                           str(self.topology_provider).strip().lower().replace("_", "-"))
        object.__setattr__(self, "min_relay_count", int(self.min_relay_count))
        if self.target_gpu is not None:
            object.__setattr__(self, "target_gpu", int(self.target_gpu))


def build_topology_provider(name: str, devices=None) -> TopologyProvider:
    n = str(name).strip().lower().replace("_", "-")
    if n in ("cuda-nvml", "nvidia-smi", "nvml"):
        return CudaNvmlTopologyProvider(devices=devices)
    raise DaemonStartupError(f"unsupported topology provider: {name}")


def relay_candidates_for_policy(inventory: DaemonResourceInventory, config: DaemonStartupConfig) -> tuple[int, ...]:
    src = str(inventory.source).lower()
    if src.startswith("test_fixture") or "test fixture" in str(inventory.metadata.get("discovery", "")).lower():
        raise DaemonStartupError("production daemon startup cannot use synthetic topology fixtures")
    if not inventory.gpus:
        raise DaemonStartupError("topology discovery found no GPUs")
    if config.require_pcie and not inventory.pcie_paths:
        raise DaemonStartupError("topology discovery did not report PCIe paths")
    if config.require_fabric and not inventory.fabric_links:
        raise DaemonStartupError("topology discovery did not report GPU fabric links")
    visible = tuple(sorted(g.device_id for g in inventory.gpus if g.visible))
    if config.target_gpu is None:
        if len(visible) < config.min_relay_count:
            raise DaemonStartupError("topology discovery found fewer visible GPUs than min_relay_count")
        return visible
    target = int(config.target_gpu)
    if target not in {g.device_id for g in inventory.gpus}:
        raise DaemonStartupError(f"target GPU {target} was not discovered")
    e = inventory.relay_eligibility(target, visible)
    relays = tuple(x["relay_gpu"] for x in e["eligible_relays"])
    if len(relays) < config.min_relay_count:
        filtered = ", ".join(f"{x['relay_gpu']}:{x['reason']}" for x in e["filtered_relays"])
        raise DaemonStartupError(
            "topology discovery could not satisfy relay policy: "
            f"target_gpu={target} min_relay_count={config.min_relay_count} "
            f"eligible_relays={list(relays)} filtered_relays=[{filtered}]")
    return relays


def create_production_daemon(config: DaemonStartupConfig, *,
                             topology_provider: TopologyProvider | None = None,
                             executor_factory: Callable[[], object] | None = None) -> TurboBusDaemon:
    provider = topology_provider or build_topology_provider(config.topology_provider, config.devices)
    try:
        inventory = provider.snapshot()
    except TopologyDiscoveryError as exc:
        raise DaemonStartupError(str(exc)) from exc
    relays = relay_candidates_for_policy(inventory, config)
    executor = None
    if config.execute:
        if executor_factory is None:
            from .executor import EngineDataPlane, IntentExecutor

            executor = IntentExecutor(EngineDataPlane(devices=[g.device_id for g in inventory.gpus]),
                                      max_workers=int(config.executor_workers))
        else:
            executor = executor_factory()
    daemon = TurboBusDaemon(relays, max_sessions_per_relay=config.max_sessions_per_relay,
                            max_inflight_chunks_per_relay=config.max_inflight_chunks_per_relay,
                            session_timeout_seconds=config.session_timeout_seconds,
                            profile_max_age_seconds=config.profile_max_age_seconds,
                            topology_provider=provider, executor=executor,
                            profile_store_path=config.profile_store_path)
    if config.profile_on_start:
        from ..parallel.linkprobe import profile_daemon

        targets = [config.target_gpu] if config.target_gpu is not None else [g.device_id for g in inventory.gpus]
        profile_daemon(daemon, targets=targets, relays=relays)
    return daemon


__all__ = ["DaemonStartupConfig", "DaemonStartupError", "build_topology_provider", "create_production_daemon",
           "relay_candidates_for_policy"]
