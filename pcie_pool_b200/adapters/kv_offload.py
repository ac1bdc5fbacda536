"""Paged-KV save / restore on the pooled data plane.

A request's KV prefix (every layer, K and V, ``n`` blocks) is saved to one
page-locked host region laid out ``[layer][lane][block index]`` -- per layer
exactly the reference connector's CPU slot order ``start + lane*n + index``
(turbobus/adapters/vllm_kv_connector.py:189-208).  Saving is ONE device->host
transfer whose push kernel gathers every block through the request's block
table; restoring is ONE host->device transfer whose landing kernel scatters
host-contiguous chunks into the (permuted) block table.  The reference moves
each 32 KiB block lane as a separate range and chunk (131,072 per 32k-token
request when the block table is permuted).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np

from .vllm import block_table_units, kv_layout


@dataclass
class KVTransferStats:
    bytes: int
    units: int
    cuda_ms: float
    gb_per_s: float
    lanes: list


def kv_segments(nunits: int, host_off: int, span_blocks: int | None, nblocks: int, unit_bytes: int):
    """(host offset, first unit, unit count) runs of a prefix.  With
    ``span_blocks`` larger than the request the host region keeps
    ``span_blocks`` slots per (layer, lane) and only the first ``nblocks`` of
    each move."""
    if span_blocks is None or span_blocks == nblocks:
        return [(host_off, 0, nunits)]
    if span_blocks < nblocks:
        raise ValueError("span_blocks must be >= the number of blocks moved")
    spans = nunits // max(1, nblocks)
    return [(host_off + s * span_blocks * unit_bytes, s * nblocks, nblocks) for s in range(spans)]


class PagedKVOffloader:
    """Save / restore vLLM-layout KV prefixes through a ``PoolEngine``."""

    def __init__(self, engine, kv_caches: Sequence, target: int, relays: Sequence[int] = (),
                 units_per_chunk: int = 128, checksum: bool = True, balancer=None, sync_stream: bool = True) -> None:
        self.engine = engine
        self.kv_caches = list(kv_caches)
        if not self.kv_caches:
            raise ValueError("at least one KV cache tensor is required")
        self.target = int(target)
        self.relays = [int(r) for r in relays if int(r) != int(target)]
        self.units_per_chunk = int(units_per_chunk)
        self.checksum = checksum
        self.balancer = balancer
        self.sync_stream = sync_stream
        lay = kv_layout(self.kv_caches[0])
        self.unit_bytes = lay.unit_bytes
        self.units_per_block = lay.lanes * len(self.kv_caches)

    def prefix_bytes(self, block_count: int) -> int:
        return int(block_count) * self.units_per_block * self.unit_bytes

    def _segments(self, nunits: int, host_off: int, span_blocks: int | None, nblocks: int):
        return kv_segments(nunits, host_off, span_blocks, nblocks, self.unit_bytes)

    def _lanes(self, segments, direction: str, h2d: bool):
        from ..parallel.engine import Lane

        devices = [self.target, *self.relays]
        hs, us, cs = [], [], []
        for hoff, u0, n in segments:
            st = np.arange(0, n, self.units_per_chunk, dtype=np.int64)
            hs.append(hoff + st * self.unit_bytes)
            us.append(u0 + st)
            cs.append(np.minimum(self.units_per_chunk, n - st))
        host_offs, starts, counts = np.concatenate(hs), np.concatenate(us), np.concatenate(cs)
        if len(devices) == 1:
            idx = np.zeros(starts.size, dtype=np.int64)
        else:
            w = None if self.balancer is None else self.balancer.weights(self.target, direction, devices)
            if w is None:
                idx = np.arange(starts.size) % len(devices)
            else:
                from ..parallel.planning import assign

                idx = assign((counts * self.unit_bytes).astype(np.uint64), w)
            # contiguous span per lane keeps each lane's host reads sequential
            n_per = np.bincount(idx, minlength=len(devices))
            idx = np.repeat(np.arange(len(devices)), n_per)
        lanes = []
        for li, dev in enumerate(devices):
            sel = idx == li
            if not np.any(sel):
                continue
            host = host_offs[sel].astype(np.uint64)
            nbytes = (counts[sel] * self.unit_bytes).astype(np.uint64)
            zeros = np.zeros(host.size, dtype=np.uint64)
            u0 = starts[sel].astype(np.uint32)
            lanes.append(Lane(dev, host, zeros, nbytes, unit0=u0) if h2d else Lane(dev, zeros, host, nbytes, unit0=u0))
        return lanes

    def _run(self, h2d: bool, block_ids: Sequence[int], host_ptr: int, host_bytes: int,
             host_off: int = 0, span_blocks: int | None = None) -> KVTransferStats:
        from .._native import native
        from ..parallel.engine import D2H, H2D

        C = native()
        addrs, unit = block_table_units(self.kv_caches, block_ids)
        nunits = int(addrs.size)
        nblocks = len(block_ids)
        segs = self._segments(nunits, host_off, span_blocks, nblocks)
        need = max(h + n * unit for h, _, n in segs)
        if need > host_bytes:
            raise ValueError("host backing is smaller than the KV prefix")
        direction = "h2d" if h2d else "d2h"
        lanes = self._lanes(segs, direction, h2d)
        kv0 = self.kv_caches[0]
        if self.sync_stream:
            # the engine runs on its own streams: work already queued on the
            # caller's stream (the forward that wrote these blocks, or reads
            # of the blocks about to be overwritten) must finish first
            import torch

            torch.cuda.current_stream(kv0.device).synchronize()
        r = self.engine.run(H2D if h2d else D2H, self.target, host_ptr, host_bytes, kv0.data_ptr(),
                            kv0.numel() * kv0.element_size(), lanes,
                            op=C.OP_SCATTER_UNITS if h2d else C.OP_GATHER_UNITS, checksum=self.checksum,
                            unit_bytes=unit, unit_addrs=addrs)
        r.raise_for_status()
        if self.balancer is not None:
            self.balancer.observe(self.target, direction, r)
        return KVTransferStats(bytes=r.bytes, units=nunits, cuda_ms=r.cuda_ms, gb_per_s=r.gb_per_s,
                               lanes=[(l.device, l.bytes, round(l.cuda_ms, 3)) for l in r.lanes])

    def save(self, block_ids: Sequence[int], host_ptr: int, host_bytes: int, host_off: int = 0) -> KVTransferStats:
        """GPU blocks -> host region (gather through the block table)."""
        return self._run(False, block_ids, host_ptr, host_bytes, host_off)

    def restore(self, block_ids: Sequence[int], host_ptr: int, host_bytes: int,
                host_off: int = 0, span_blocks: int | None = None) -> KVTransferStats:
        """Host region -> GPU blocks (scatter through the block table).  A
        region saved with ``span_blocks`` blocks restores its first
        ``len(block_ids)`` blocks when given ``span_blocks``."""
        return self._run(True, block_ids, host_ptr, host_bytes, host_off, span_blocks)


class DaemonKVOffloader:
    """Save / restore vLLM-layout KV prefixes as daemon intents.

    Each save or restore is ONE intent whose landing spec asks the data plane
    for the fused unit gather (save) or scatter (restore) through the
    request's block table, so the move runs under the daemon's plan, relay
    leases, fairness and isolation rules like any other transfer -- relays
    come only from leases -- and the bytes still cross PCIe once per lane and
    NVLink once.  The KV cache of every layer is registered with the daemon
    as a device buffer (CUDA IPC when the daemon is another process, the
    address when it runs in this process); host regions are registered on
    first use (shared page-locked memory for a daemon process).

    The reference moves the same prefix as one range per block lane through
    its slot adapter (turbobus/adapters/vllm_kv_connector.py:816-872)."""

    def __init__(self, client, daemon_client, *, session_id: str, job_id: str, kv_caches: Sequence,
                 units_per_chunk: int = 128, prefix: str = "kv", ctas_per_lane: int = 0,
                 timeout_s: float = 600.0, sync_stream: bool = True) -> None:
        from ..daemon.client import InProcessDaemonClient

        self.client = client
        self.dc = daemon_client
        self.session_id = str(session_id)
        self.job_id = str(job_id)
        self.kv_caches = list(kv_caches)
        if not self.kv_caches:
            raise ValueError("at least one KV cache tensor is required")
        lay = kv_layout(self.kv_caches[0])
        self.unit_bytes = lay.unit_bytes
        self.units_per_block = lay.lanes * len(self.kv_caches)
        self.units_per_chunk = int(units_per_chunk)
        self.prefix = str(prefix)
        self.ctas_per_lane = int(ctas_per_lane)
        self.timeout_s = float(timeout_s)
        self.sync_stream = sync_stream
        self.in_process = isinstance(daemon_client, InProcessDaemonClient)
        self._seq = 0
        self._spec = None
        self._host_ids: dict[int, str] = {}
        self._keep: list = []
        self.kv_buffer_ids = [f"{self.prefix}-layer{i}" for i in range(len(self.kv_caches))]
        for bid, kv in zip(self.kv_buffer_ids, self.kv_caches):
            self._register_device(bid, kv)

    # ---- registrations ------------------------------------------------------------
    def _check(self, r) -> None:
        if not r.ok:
            raise RuntimeError(r.error or "daemon request failed")

    def _register_device(self, bid: str, t) -> None:
        if self.in_process:
            dev = t.device.index if t.device.index is not None else 0
            self._check(self.dc.register_buffer(bid, self.job_id, "gpu", t.numel() * t.element_size(),
                                                device_index=int(dev), address=int(t.data_ptr())))
        else:
            from ..client import CudaIpcDeviceBuffer

            buf = CudaIpcDeviceBuffer.from_tensor(bid, self.job_id, t)
            self._check(buf.register_with_daemon(self.dc))
            self._keep.append(buf)

    def host_buffer_id(self, host) -> str:
        """Register a host region (a page-locked torch tensor for an
        in-process daemon, a ``SharedPinnedCpuBuffer`` for a daemon process)
        once and return its buffer id."""
        from ..client import SharedPinnedCpuBuffer

        key = id(host)
        if key in self._host_ids:
            return self._host_ids[key]
        bid = f"{self.prefix}-host{len(self._host_ids)}"
        if isinstance(host, SharedPinnedCpuBuffer):
            reg = host.buffer_registration()

            self._check(self.dc.register_buffer(bid, self.job_id, reg.kind, reg.size_bytes,
                                                handle_type=reg.handle_type, metadata=dict(reg.metadata),
                                                pinned=True))
        else:
            if not self.in_process:
                raise ValueError("a daemon process needs a SharedPinnedCpuBuffer host region")
            self._check(self.dc.register_buffer(bid, self.job_id, "cpu_pinned", host.numel() * host.element_size(),
                                                address=int(host.data_ptr()), pinned=True))
        self._host_ids[key] = bid
        self._keep.append(host)
        return bid

    # ---- transfers --------------------------------------------------------------------
    def prefix_bytes(self, block_count: int) -> int:
        return int(block_count) * self.units_per_block * self.unit_bytes

    def _run(self, h2d: bool, block_ids: Sequence[int], host, host_off: int, span_blocks: int | None):
        from .. import TransferIntent, TransferStatusState
        from ..daemon.landing import kv_spec
        from ..schema import WorkloadKind

        ids = [int(b) for b in block_ids]
        nunits = len(ids) * self.units_per_block
        u = self.unit_bytes
        segs = kv_segments(nunits, int(host_off), span_blocks, len(ids), u)
        hid = self.host_buffer_id(host)
        if h2d:
            ranges = tuple({"src_offset": h, "dst_offset": u0 * u, "bytes": n * u} for h, u0, n in segs)
            src, dst = hid, self.kv_buffer_ids[0]
        else:
            ranges = tuple({"src_offset": u0 * u, "dst_offset": h, "bytes": n * u} for h, u0, n in segs)
            src, dst = self.kv_buffer_ids[0], hid
        if self._spec is None:  # the layer layout is fixed: check it once
            self._spec = kv_spec(self.kv_caches, ids[:1], self.kv_buffer_ids, op="scatter_units",
                                 ctas_per_lane=self.ctas_per_lane)
        from dataclasses import replace

        spec = replace(self._spec, op="scatter_units" if h2d else "gather_units",
                       kv=replace(self._spec.kv, block_ids=tuple(ids)))
        self._seq += 1
        iid = f"{self.prefix}-{'restore' if h2d else 'save'}-{self._seq}"
        intent = TransferIntent(iid, self.job_id, self.session_id, src, dst, "h2d" if h2d else "d2h",
                                nunits * u, ranges, workload_kind=WorkloadKind.KV_CACHE,
                                metadata={"chunk_bytes": self.units_per_chunk * u, "landing": spec.to_metadata()})
        if self.sync_stream:
            # the daemon's data plane runs on its own streams: the forward
            # that wrote these blocks (or still reads them) must be done
            import torch

            torch.cuda.current_stream(self.kv_caches[0].device).synchronize()
        r = self.client.transfer(intent, timeout_seconds=self.timeout_s)
        if r.state is not TransferStatusState.COMPLETE:
            raise RuntimeError(f"kv {'restore' if h2d else 'save'} failed: {r.error}")
        meas = (r.metadata or {}).get("measured", {}) or {}
        cuda_ms = float(meas.get("cuda_ms", 0.0) or 0.0)
        nbytes = nunits * u
        return KVTransferStats(bytes=nbytes, units=nunits, cuda_ms=cuda_ms,
                               gb_per_s=nbytes / 1e9 / (cuda_ms / 1e3) if cuda_ms > 0 else 0.0,
                               lanes=[(p.get("relay_device"), p.get("bytes"), round(float(p.get("cuda_ms", 0.0)), 3))
                                      for p in (r.path_stats or ())])

    def save(self, block_ids: Sequence[int], host, host_off: int = 0) -> KVTransferStats:
        """GPU blocks -> host region (fused gather through the block table)."""
        return self._run(False, block_ids, host, host_off, None)

    def restore(self, block_ids: Sequence[int], host, host_off: int = 0,
                span_blocks: int | None = None) -> KVTransferStats:
        """Host region -> GPU blocks (fused scatter through the block table)."""
        return self._run(True, block_ids, host, host_off, span_blocks)


__all__ = ["DaemonKVOffloader", "KVTransferStats", "PagedKVOffloader", "kv_segments"]
