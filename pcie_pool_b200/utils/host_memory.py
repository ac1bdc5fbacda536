"""Page-locked host buffers with optional NUMA placement.

``PinnedHostBuffer`` maps anonymous (or shared) memory, optionally places its
pages on a NUMA node by first touch from a thread bound to that node's CPUs,
and registers it with CUDA as portable + mapped so every GPU context of the
process can DMA from it.  The reference registers POSIX shared memory with
``cudaHostRegister(..., Portable)`` (turbobus/client.py:224-231,
cpp/src/pybind.cpp:73-95); NUMA placement is new here, because relay lanes
on the far socket otherwise pull every byte across the socket link.
"""

from __future__ import annotations

import mmap
import os
import threading
from pathlib import Path

import numpy as np

from .._native import native


def numa_nodes() -> dict[int, list[int]]:
    """NUMA node -> CPU list, from sysfs (empty when unavailable)."""
    out: dict[int, list[int]] = {}
    base = Path("/sys/devices/system/node")
    if not base.exists():
        return out
    for d in sorted(base.glob("node[0-9]*")):
        try:
            cpus = parse_cpulist((d / "cpulist").read_text().strip())
        except OSError:
            continue
        out[int(d.name[4:])] = cpus
    return out


def parse_cpulist(text: str) -> list[int]:
    cpus: list[int] = []
    for part in text.split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.extend(range(int(a), int(b) + 1))
        else:
            cpus.append(int(part))
    return cpus


def _touch(view: np.ndarray, cpus: list[int] | None, value: int) -> None:
    if cpus:
        try:
            os.sched_setaffinity(0, cpus)
        except OSError:
            pass
    view[::4096] = value  # one write per page is enough for first touch
    view[:] = value


def first_touch(arr: np.ndarray, node: int | None, threads: int = 8, value: int = 0) -> None:
    """Fault in every page of ``arr`` from CPUs of ``node`` (None: any CPU)."""
    cpus = numa_nodes().get(node) if node is not None else None
    parts = np.array_split(arr, max(1, threads))
    ths = [threading.Thread(target=_touch, args=(p, cpus, value)) for p in parts if p.size]
    for t in ths:
        t.start()
    for t in ths:
        t.join()


class PinnedHostBuffer:
    """Anonymous host memory, optionally NUMA-placed, registered with CUDA."""

    def __init__(self, nbytes: int, numa_node: int | None = None, register: bool = True,
                 interleave: list[int] | None = None, fill: int | None = 0) -> None:
        if nbytes <= 0:
            raise ValueError("nbytes must be positive")
        self.nbytes = int(nbytes)
        self._map = mmap.mmap(-1, self.nbytes, flags=mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS)
        self._arr = np.frombuffer(self._map, dtype=np.uint8)
        if interleave:
            parts = np.array_split(self._arr, len(interleave))
            for node, part in zip(interleave, parts):
                first_touch(part, node, value=fill or 0)
        elif fill is not None:
            first_touch(self._arr, numa_node, value=fill)
        self.ptr = self._arr.ctypes.data
        self.registered = False
        if register:
            native().host_register(self.ptr, self.nbytes)
            self.registered = True

    def numpy(self) -> np.ndarray:
        return self._arr

    def torch(self, dtype=None):
        import torch

        t = torch.frombuffer(self._map, dtype=torch.uint8)
        return t if dtype is None else t.view(dtype)

    def release(self) -> None:
        if self.registered:
            native().host_unregister(self.ptr)
            self.registered = False
        if self._map is not None:
            self._arr = None
            try:
                self._map.close()
            except BufferError:
                pass  # live views keep the mapping; it goes with them
            self._map = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.release()
        except Exception:
            pass
