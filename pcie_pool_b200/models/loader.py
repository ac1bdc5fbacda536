"""Pooled weight loading: a packed host image of a model's weights goes into
one GPU over the direct lane plus relay lanes, landing either as bf16 (plain
copy) or as fp8 e4m3 with fp32 scales per 128x128 block, quantized inside
the landing kernel (no separate quantization pass, no bf16 copy on the
device).

Chunking: bf16 images are cut into ``chunk_bytes`` pieces of the packed
image; fp8 matrices are cut per tensor on 128-row tiles (a chunk holds
``k * 128`` whole rows, k chosen so the chunk fits the staging slot).  Chunks
are assigned to lanes by the native earliest-finish planner with the lanes'
concurrent rates (a ``LaneBalancer`` or a probed profile) and each lane's
chunks are then laid out host-contiguously.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from .llama import WeightManifest


@dataclass
class LoadStats:
    bytes: int
    cuda_ms: float
    wall_ms: float
    transfers: int
    lanes: list = field(default_factory=list)

    @property
    def gb_per_s(self) -> float:
        return self.bytes / 1e9 / (self.cuda_ms / 1e3) if self.cuda_ms > 0 else 0.0


@dataclass
class LoadedWeights:
    tensors: dict
    scales: dict
    stats: LoadStats
    storage: list = field(default_factory=list)


def _assign(sizes: np.ndarray, weights: Sequence[float] | None, nlanes: int) -> np.ndarray:
    if nlanes == 1:
        return np.zeros(sizes.size, dtype=np.int64)
    if weights is None:
        weights = [1.0] * nlanes
    from ..parallel.planning import assign

    idx = np.asarray(assign(sizes.astype(np.uint64), list(weights)), dtype=np.int64)
    return idx


def fp8_chunks(manifest: WeightManifest, chunk_bytes: int):
    """(src_off, rows_start, nbytes, tensor_index) of every fp8 chunk: each
    matrix cut on 128-row tiles into pieces of at most ``chunk_bytes``."""
    src, row0, nbytes, tidx = [], [], [], []
    for ti, t in enumerate(manifest.matrices()):
        rows, cols = t.shape
        rb = cols * 2
        step = max(1, int(chunk_bytes) // (128 * rb)) * 128
        for r in range(0, rows, step):
            n = min(step, rows - r)
            src.append(t.offset + r * rb)
            row0.append(r)
            nbytes.append(n * rb)
            tidx.append(ti)
    return (np.array(src, np.int64), np.array(row0, np.int64), np.array(nbytes, np.int64),
            np.array(tidx, np.int64))


class PooledWeightLoader:
    def __init__(self, engine, target: int, relays: Sequence[int] = (), *, chunk_bytes: int = 16 << 20,
                 balancer=None, lane_weights: Sequence[float] | None = None, checksum: bool = True,
                 fp8_ctas_per_lane: int = 12) -> None:
        # The fp8 landing does the quantization arithmetic (amax reduction and
        # an IEEE division per element) in the landing CTAs; 4 CTAs land
        # ~27 GB/s of bf16, so fp8 lanes get more CTAs to stay PCIe-bound.
        self.fp8_ctas_per_lane = int(fp8_ctas_per_lane)
        self.engine = engine
        self.target = int(target)
        self.relays = [int(r) for r in relays if int(r) != int(target)]
        self.chunk_bytes = int(min(chunk_bytes, engine.slot_bytes))
        self.balancer = balancer
        self.lane_weights = None if lane_weights is None else list(lane_weights)
        self.checksum = checksum

    @property
    def devices(self) -> list[int]:
        return [self.target, *self.relays]

    def _weights(self, direction: str = "h2d"):
        if self.lane_weights is not None:
            return self.lane_weights
        if self.balancer is not None:
            return self.balancer.weights(self.target, direction, self.devices)
        return None

    def _lanes(self, src: np.ndarray, dst: np.ndarray, nbytes: np.ndarray, unit0=None, tensor=None):
        from ..parallel.engine import Lane

        idx = _assign(nbytes, self._weights(), len(self.devices))
        lanes = []
        for li, dev in enumerate(self.devices):
            sel = np.flatnonzero(idx == li)
            if sel.size == 0:
                continue
            sel = sel[np.argsort(src[sel], kind="stable")]  # host-sequential per lane
            lanes.append(Lane(dev, src[sel].astype(np.uint64), dst[sel].astype(np.uint64),
                              nbytes[sel].astype(np.uint64),
                              unit0=None if unit0 is None else unit0[sel].astype(np.uint32),
                              tensor=None if tensor is None else tensor[sel].astype(np.uint32)))
        return lanes

    def _observe(self, r) -> None:
        if self.balancer is not None:
            self.balancer.observe(self.target, "h2d", r)

    # ---- bf16 -----------------------------------------------------------------------------
    def bf16_lanes(self, total: int):
        """Lanes of a plain copy of a ``total``-byte image (current lane weights)."""
        offs = np.arange(0, int(total), self.chunk_bytes, dtype=np.int64)
        sizes = np.minimum(self.chunk_bytes, int(total) - offs)
        return self._lanes(offs, offs, sizes)

    def load_bf16(self, host_ptr: int, host_bytes: int, manifest: WeightManifest, device_buffer=None) -> LoadedWeights:
        import time

        import torch

        from ..parallel.engine import H2D

        total = manifest.total_bytes
        if host_bytes < total:
            raise ValueError("host image is smaller than the manifest")
        dev = torch.device("cuda", self.target)
        buf = device_buffer if device_buffer is not None else torch.empty(total, dtype=torch.uint8, device=dev)
        lanes = self.bf16_lanes(total)
        t0 = time.perf_counter()
        r = self.engine.run(H2D, self.target, host_ptr, host_bytes, buf.data_ptr(), total, lanes,
                            checksum=self.checksum)
        wall = (time.perf_counter() - t0) * 1e3
        r.raise_for_status()
        self._observe(r)
        views = {}
        for t in manifest.tensors:
            views[t.name] = buf[t.offset:t.offset + t.nbytes].view(torch.bfloat16).view(*t.shape)
        return LoadedWeights(views, {}, LoadStats(r.bytes, r.cuda_ms, wall, 1,
                                                  [(l.device, l.bytes, round(l.cuda_ms, 3)) for l in r.lanes]),
                             storage=[buf])

    # ---- fp8 -----------------------------------------------------------------------------------
    def fp8_plan(self, manifest: WeightManifest):
        """(src_off, rows_start, nbytes, tensor_index) of every fp8 chunk."""
        return fp8_chunks(manifest, self.chunk_bytes)

    def load_fp8(self, host_ptr: int, host_bytes: int, manifest: WeightManifest) -> LoadedWeights:
        """Matrices land as e4m3 codes + fp32 scales [ceil(R/128), C/128];
        1-D weights land as bf16 (one small copy transfer)."""
        import time

        import torch

        from .._native import native
        from ..parallel.engine import H2D, Lane

        if self.chunk_bytes < 128 * 2 * max(t.shape[1] for t in manifest.matrices()):
            raise ValueError("chunk_bytes must hold at least one 128-row tile of the widest matrix")
        C = native()
        dev = torch.device("cuda", self.target)
        mats = manifest.matrices()
        q_total = sum(t.numel for t in mats)
        qbuf = torch.empty(q_total, dtype=torch.uint8, device=dev)
        qviews, sviews, table = {}, {}, []
        qoff = 0
        for t in mats:
            rows, cols = t.shape
            q = qbuf[qoff:qoff + t.numel].view(rows, cols)
            s = torch.empty(((rows + 127) // 128, cols // 128), dtype=torch.float32, device=dev)
            qviews[t.name], sviews[t.name] = q, s
            table.append((q.data_ptr(), s.data_ptr(), rows, cols))
            qoff += t.numel
        src, row0, nbytes, tidx = self.fp8_plan(manifest)
        lanes = self._lanes(src, np.zeros_like(src), nbytes, unit0=row0, tensor=tidx)
        vecs = manifest.vectors()
        vbytes = sum(t.nbytes for t in vecs)
        vbuf = torch.empty(max(vbytes, 16), dtype=torch.uint8, device=dev)
        vlane = None
        if vecs:
            vo, so, nb = [], [], []
            off = 0
            for t in vecs:
                so.append(t.offset)
                vo.append(off)
                nb.append(t.nbytes)
                qviews[t.name] = vbuf[off:off + t.nbytes].view(torch.bfloat16).view(*t.shape)
                off += t.nbytes
            vlane = Lane(self.target, np.array(so, np.uint64), np.array(vo, np.uint64), np.array(nb, np.uint64))
        t0 = time.perf_counter()
        r = self.engine.run(H2D, self.target, host_ptr, host_bytes, qbuf.data_ptr(), q_total, lanes,
                            op=C.OP_FP8_QUANT, checksum=self.checksum, tensors=table,
                            ctas_per_lane=self.fp8_ctas_per_lane)
        r.raise_for_status()
        cuda_ms, moved, lane_stats = r.cuda_ms, r.bytes, [(l.device, l.bytes, round(l.cuda_ms, 3)) for l in r.lanes]
        self._observe(r)
        transfers = 1
        if vlane is not None:
            rv = self.engine.run(H2D, self.target, host_ptr, host_bytes, vbuf.data_ptr(), vbuf.numel(), [vlane],
                                 checksum=self.checksum)
            rv.raise_for_status()
            cuda_ms += rv.cuda_ms
            moved += rv.bytes
            transfers += 1
        wall = (time.perf_counter() - t0) * 1e3
        return LoadedWeights(qviews, sviews, LoadStats(moved, cuda_ms, wall, transfers, lane_stats),
                             storage=[qbuf, vbuf])


class DaemonWeightLoader:
    """Pooled weight loading as daemon intents.

    The same two loads as ``PooledWeightLoader`` -- a packed bf16 image, or
    matrices landing as fp8 e4m3 + fp32 per-128x128-block scales quantised in
    the landing kernel -- but each is an intent to the node daemon, so the
    relays it uses come from the daemon's leases and fairness rules (the
    reference's ``ModelWeightLoader`` submits the same kind of intent,
    turbobus/adapters/model_loading.py).  The fp8 intent carries a landing
    spec (daemon/landing.py) naming every matrix's output inside ONE device
    buffer of codes and scales; its ranges are pre-cut on 128-row tiles.
    Host images are page-locked tensors (daemon in this process) or
    ``SharedPinnedCpuBuffer`` (daemon process); device buffers are registered
    by address or CUDA IPC accordingly."""

    def __init__(self, client, daemon_client, *, session_id: str, job_id: str, target: int,
                 chunk_bytes: int = 16 << 20, prefix: str = "weights", fp8_ctas_per_lane: int = 12,
                 timeout_s: float = 600.0) -> None:
        from ..daemon.client import InProcessDaemonClient

        self.client, self.dc = client, daemon_client
        self.session_id, self.job_id, self.target = str(session_id), str(job_id), int(target)
        self.chunk_bytes = int(chunk_bytes)
        self.prefix = str(prefix)
        self.fp8_ctas_per_lane = int(fp8_ctas_per_lane)
        self.timeout_s = float(timeout_s)
        self.in_process = isinstance(daemon_client, InProcessDaemonClient)
        self._n = 0
        self._keep: list = []

    def _ok(self, r) -> None:
        if not r.ok:
            raise RuntimeError(r.error or "daemon request failed")

    def _register_host(self, host) -> tuple[str, int]:
        from ..client import SharedPinnedCpuBuffer

        self._n += 1
        bid = f"{self.prefix}-host{self._n}"
        if isinstance(host, SharedPinnedCpuBuffer):
            reg = host.buffer_registration()
            self._ok(self.dc.register_buffer(bid, self.job_id, reg.kind, reg.size_bytes, handle_type=reg.handle_type,
                                             metadata=dict(reg.metadata), pinned=True))
            size = reg.size_bytes
        else:
            if not self.in_process:
                raise ValueError("a daemon process needs a SharedPinnedCpuBuffer host image")
            size = host.numel() * host.element_size()
            self._ok(self.dc.register_buffer(bid, self.job_id, "cpu_pinned", size, address=int(host.data_ptr()),
                                             pinned=True))
        self._keep.append(host)
        return bid, size

    def _register_device(self, t) -> str:
        self._n += 1
        bid = f"{self.prefix}-dev{self._n}"
        if self.in_process:
            self._ok(self.dc.register_buffer(bid, self.job_id, "gpu", t.numel() * t.element_size(),
                                             device_index=self.target, address=int(t.data_ptr())))
        else:
            from ..client import CudaIpcDeviceBuffer

            buf = CudaIpcDeviceBuffer.from_tensor(bid, self.job_id, t)
            self._ok(buf.register_with_daemon(self.dc))
            self._keep.append(buf)
        return bid

    def _transfer(self, src: str, dst: str, ranges, chunk: int, landing=None):
        from .. import TransferIntent, TransferStatusState

        self._n += 1
        meta = {"chunk_bytes": int(chunk)}
        if landing is not None:
            meta["landing"] = landing
        total = sum(int(r["bytes"]) for r in ranges)
        it = TransferIntent(f"{self.prefix}-load{self._n}", self.job_id, self.session_id, src, dst, "h2d", total,
                            tuple(ranges), workload_kind="model_weights", metadata=meta)
        r = self.client.transfer(it, timeout_seconds=self.timeout_s)
        if r.state is not TransferStatusState.COMPLETE:
            raise RuntimeError(f"weight load failed: {r.error}")
        meas = (r.metadata or {}).get("measured", {}) or {}
        return r, float(meas.get("cuda_ms", 0.0) or 0.0)

    def load_bf16(self, host, manifest: WeightManifest, device_buffer=None) -> LoadedWeights:
        import time

        import torch

        total = manifest.total_bytes
        hid, hsize = self._register_host(host)
        if hsize < total:
            raise ValueError("host image is smaller than the manifest")
        dev = torch.device("cuda", self.target)
        buf = device_buffer if device_buffer is not None else torch.empty(total, dtype=torch.uint8, device=dev)
        did = self._register_device(buf)
        t0 = time.perf_counter()
        r, cuda_ms = self._transfer(hid, did, ({"src_offset": 0, "dst_offset": 0, "bytes": total},), self.chunk_bytes)
        wall = (time.perf_counter() - t0) * 1e3
        views = {t.name: buf[t.offset:t.offset + t.nbytes].view(torch.bfloat16).view(*t.shape)
                 for t in manifest.tensors}
        lanes = [(p.get("relay_device"), p.get("bytes"), round(float(p.get("cuda_ms", 0.0)), 3))
                 for p in (r.path_stats or ())]
        return LoadedWeights(views, {}, LoadStats(total, cuda_ms, wall, 1, lanes), storage=[buf])

    def load_fp8(self, host, manifest: WeightManifest) -> LoadedWeights:
        import time

        import torch

        mats = manifest.matrices()
        if self.chunk_bytes < 128 * 2 * max(t.shape[1] for t in mats):
            raise ValueError("chunk_bytes must hold at least one 128-row tile of the widest matrix")
        hid, _ = self._register_host(host)
        dev = torch.device("cuda", self.target)
        q_total = sum(t.numel for t in mats)
        s_base = -(-q_total // 256) * 256
        s_total = sum(-(-t.shape[0] // 128) * (t.shape[1] // 128) * 4 for t in mats)
        out = torch.empty(s_base + s_total, dtype=torch.uint8, device=dev)
        table, qviews, sviews = [], {}, {}
        qo, so = 0, s_base
        for t in mats:
            rows, cols = t.shape
            ns = -(-rows // 128) * (cols // 128) * 4
            table.append({"host_offset": t.offset, "rows": rows, "cols": cols, "q_offset": qo, "scales_offset": so})
            qviews[t.name] = out[qo:qo + t.numel].view(rows, cols)
            sviews[t.name] = out[so:so + ns].view(torch.float32).view(-(-rows // 128), cols // 128)
            qo += t.numel
            so += ns
        did = self._register_device(out)
        src, _row0, nbytes, _tidx = fp8_chunks(manifest, self.chunk_bytes)
        ranges = [{"src_offset": int(a), "dst_offset": int(a), "bytes": int(n)} for a, n in zip(src, nbytes)]
        landing = {"op": "fp8_quant", "tensors": table, "ctas_per_lane": self.fp8_ctas_per_lane}
        t0 = time.perf_counter()
        r, cuda_ms = self._transfer(hid, did, ranges, int(nbytes.max()), landing)
        moved, transfers = int(nbytes.sum()), 1
        vecs = manifest.vectors()
        storage = [out]
        if vecs:
            vbuf = torch.empty(max(16, sum(t.nbytes for t in vecs)), dtype=torch.uint8, device=dev)
            vid = self._register_device(vbuf)
            vr, off = [], 0
            for t in vecs:
                vr.append({"src_offset": t.offset, "dst_offset": off, "bytes": t.nbytes})
                qviews[t.name] = vbuf[off:off + t.nbytes].view(torch.bfloat16).view(*t.shape)
                off += t.nbytes
            _rv, ms2 = self._transfer(hid, vid, vr, self.chunk_bytes)
            cuda_ms += ms2
            moved += off
            transfers += 1
            storage.append(vbuf)
        wall = (time.perf_counter() - t0) * 1e3
        lanes = [(p.get("relay_device"), p.get("bytes"), round(float(p.get("cuda_ms", 0.0)), 3))
                 for p in (r.path_stats or ())]
        return LoadedWeights(qviews, sviews, LoadStats(moved, cuda_ms, wall, transfers, lanes), storage=storage)


__all__ = ["DaemonWeightLoader", "LoadStats", "LoadedWeights", "PooledWeightLoader", "fp8_chunks"]
