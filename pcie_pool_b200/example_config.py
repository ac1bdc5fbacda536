"""Map physical GPU ids onto CUDA runtime ordinals for examples and tools:
with ``CUDA_VISIBLE_DEVICES`` unset, expose ``target,relays...`` and use
ordinals 0..n (behaviour of turbobus/example_config.py)."""

from __future__ import annotations

import os
from dataclasses import dataclass


@dataclass(frozen=True)
class CudaRuntimeMapping:
    physical_target_gpu: int
    physical_relay_gpus: tuple[int, ...]
    runtime_target_gpu: int
    runtime_relay_gpus: tuple[int, ...]
    cuda_visible_devices: str


def parse_gpu_list(value: str) -> list[int]:
    return [int(x) for x in str(value).split(",") if x.strip()]


def configure_cuda_runtime_mapping(target_gpu: int, relay_gpus: str, *,
                                   map_physical_gpus: bool = True) -> CudaRuntimeMapping:
    relays = tuple(parse_gpu_list(relay_gpus))
    if map_physical_gpus and not os.environ.get("CUDA_VISIBLE_DEVICES"):
        visible = ",".join(str(g) for g in (int(target_gpu), *relays))
        os.environ["CUDA_VISIBLE_DEVICES"] = visible
        return CudaRuntimeMapping(int(target_gpu), relays, 0, tuple(range(1, len(relays) + 1)), visible)
    return CudaRuntimeMapping(int(target_gpu), relays, int(target_gpu), relays,
                              os.environ.get("CUDA_VISIBLE_DEVICES", ""))


__all__ = ["CudaRuntimeMapping", "configure_cuda_runtime_mapping", "parse_gpu_list"]
