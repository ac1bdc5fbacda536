"""Lane planning for the data plane: split a transfer into chunks and give
each lane a share proportional to its bandwidth.

Two layouts:
  * ``blocked`` (default) - each lane streams one contiguous span of the
    buffer, so plain direct-lane chunks merge into large copy-engine
    transfers;
  * ``interleaved`` - chunk i goes to the lane the assignment loop picks
    (round robin without a profile).
Chunk counts per lane come from the native earliest-finish assignment when a
bandwidth profile is given.
"""

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
               dst_start: int = 0, layout: str = "blocked") -> list[Lane]:
    """Chunk [0, total) and spread the chunks over the lanes of ``devices``
    (``target`` is the direct lane).  Without a profile every lane is assumed
    equally fast."""
    if layout not in ("blocked", "interleaved"):
        raise ValueError("layout must be 'blocked' or 'interleaved'")
    offs, sizes = chunk_offsets(total, chunk)
    devs = list(devices)
    if bw_gibps is None:
        idx = np.arange(offs.size) % len(devs)
    else:
        idx = assign(sizes, bw_gibps, latency_s, policy)
    if layout == "blocked":
        # same per-lane chunk counts, contiguous spans in lane order
        counts = np.bincount(idx, minlength=len(devs))
        idx = np.repeat(np.arange(len(devs)), counts)
    lanes = []
    for li, dev in enumerate(devs):
        sel = idx == li
        if not np.any(sel):
            continue
        lanes.append(Lane(int(dev), offs[sel] + np.uint64(src_start),
                          offs[sel] + np.uint64(dst_start), sizes[sel].copy()))
    lanes.sort(key=lambda l: (l.device != target, l.device))
    return lanes
