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
        src, row0, nbytes, tidx = [], [], [], []
        for ti, t in enumerate(manifest.matrices()):
            rows, cols = t.shape
            rb = cols * 2
            tile = 128 * rb
            k = max(1, self.chunk_bytes // tile)
            step = k * 128
            for r in range(0, rows, step):
                n = min(step, rows - r)
                src.append(t.offset + r * rb)
                row0.append(r)
                nbytes.append(n * rb)
                tidx.append(ti)
        return (np.array(src, np.int64), np.array(row0, np.int64), np.array(nbytes, np.int64),
                np.array(tidx, np.int64))

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


__all__ = ["LoadStats", "LoadedWeights", "PooledWeightLoader"]
