"""Lane planning for the data plane: split a transfer into chunks and assign
them to lanes with the native earliest-finish policy (or evenly when no
bandwidth profile is known)."""

from __future__ import annotations

from typing import Sequence

import numpy as np

from .engine import Lane


def chunk_offsets(total: int, chunk: int) -> tuple[np.ndarray, np.ndarray]:
    offs = np.arange(0, total, chunk, dtype=np.uint64)
    sizes = np.minimum(np.uint64(chunk), np.uint64(total) - offs).astype(np.uint64)
    return offs, sizes


def assign(sizes: np.ndarray, bw_gibps: Sequence[float], latency_s: Sequence[float] = (),
           policy: str = "earliest_finish") -> np.ndarray:
    """Lane index per chunk via the native planner core."""
    from .._native import native

    C = native()
    pol = C.POLICY_LEGACY if policy == "legacy" else C.POLICY_EARLIEST_FINISH
    return np.asarray(C.assign_chunks(np.ascontiguousarray(sizes, dtype=np.uint64),
                                      [float(b) for b in bw_gibps],
                                      [float(x) for x in latency_s], pol))


def plan_lanes(total: int, chunk: int, devices: Sequence[int], target: int,
               bw_gibps: Sequence[float] | None = None, latency_s: Sequence[float] = (),
               policy: str = "earliest_finish", src_start: int = 0,
               dst_start: int = 0) -> list[Lane]:
    """Chunk [0, total) and spread the chunks over the lanes of ``devices``
    (``target`` is the direct lane).  Without a profile every lane is assumed
    equally fast and chunks go round-robin, interleaved so every lane streams
    from across the whole buffer."""
    offs, sizes = chunk_offsets(total, chunk)
    devs = list(devices)
    if bw_gibps is None:
        idx = np.arange(offs.size) % len(devs)
    else:
        idx = assign(sizes, bw_gibps, latency_s, policy)
    lanes = []
    for li, dev in enumerate(devs):
        sel = idx == li
        if not np.any(sel):
            continue
        lanes.append(Lane(int(dev), offs[sel] + np.uint64(src_start),
                          offs[sel] + np.uint64(dst_start), sizes[sel].copy()))
    # direct lane first for readability of stats
    lanes.sort(key=lambda l: (l.device != target, l.device))
    return lanes
