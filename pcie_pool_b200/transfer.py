"""Transfer request model: byte ranges, chunk-count arithmetic and the
``PLAN_TRANSFER`` payload (same fields as turbobus/transfer.py:35-136)."""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field
from enum import Enum
from collections.abc import Mapping
from typing import Iterable

from .schema import TransferMode


class TransferDirection(str, Enum):
    H2D = "h2d"
    D2H = "d2h"


@dataclass(frozen=True)
class TransferRange:
    src_offset: int
    dst_offset: int
    bytes: int

    def __post_init__(self) -> None:
        for name in ("src_offset", "dst_offset", "bytes"):
            object.__setattr__(self, name, int(getattr(self, name)))
        if self.src_offset < 0 or self.dst_offset < 0:
            raise ValueError("range offsets must be non-negative")
        if self.bytes <= 0:
            raise ValueError("range bytes must be positive")

    def as_dict(self) -> dict[str, int]:
        return asdict(self)


def coerce_range(item) -> TransferRange:
    """TransferRange from a TransferRange, mapping, 3-sequence or attribute object."""
    if isinstance(item, TransferRange):
        return item
    if isinstance(item, Mapping):
        return TransferRange(item["src_offset"], item["dst_offset"], item["bytes"])
    if isinstance(item, (tuple, list)):
        if len(item) != 3:
            raise ValueError("range tuples must be (src_offset, dst_offset, bytes)")
        return TransferRange(*item)
    return TransferRange(item.src_offset, item.dst_offset, item.bytes)


def chunk_count(total_bytes: int, chunk_bytes: int, ranges: tuple[TransferRange, ...] = ()) -> int:
    if ranges:
        return sum(max(1, math.ceil(r.bytes / chunk_bytes)) for r in ranges)
    return max(1, math.ceil(total_bytes / chunk_bytes))


@dataclass(frozen=True)
class TransferRequest:
    total_bytes: int
    chunk_bytes: int
    direction: TransferDirection | str
    mode: TransferMode | str = TransferMode.POOL
    request_chunks: int | None = None
    ranges: tuple[TransferRange, ...] = field(default_factory=tuple)
    job_id: str | None = None
    metadata: Mapping[str, object] = field(default_factory=dict)

    def __post_init__(self) -> None:
        total, chunk = int(self.total_bytes), int(self.chunk_bytes)
        if total < 0:
            raise ValueError("total_bytes must be non-negative")
        if chunk <= 0:
            raise ValueError("chunk_bytes must be positive")
        ranges = tuple(coerce_range(r) for r in self.ranges)
        if ranges and sum(r.bytes for r in ranges) != total:
            raise ValueError("total_bytes must equal the sum of range bytes")
        computed = chunk_count(total, chunk, ranges)
        req = computed if self.request_chunks is None else int(self.request_chunks)
        if req <= 0:
            raise ValueError("request_chunks must be positive")
        if ranges and req < computed:
            raise ValueError("request_chunks cannot be smaller than range chunk count")
        object.__setattr__(self, "total_bytes", total)
        object.__setattr__(self, "chunk_bytes", chunk)
        object.__setattr__(self, "direction", TransferDirection(self.direction))
        object.__setattr__(self, "mode", TransferMode(self.mode))
        object.__setattr__(self, "request_chunks", req)
        object.__setattr__(self, "ranges", ranges)
        object.__setattr__(self, "metadata", dict(self.metadata or {}))

    @classmethod
    def from_ranges(cls, ranges: Iterable, *, chunk_bytes: int, direction: TransferDirection | str,
                    mode: TransferMode | str = TransferMode.POOL, job_id: str | None = None,
                    metadata: Mapping[str, object] | None = None) -> "TransferRequest":
        rs = tuple(coerce_range(r) for r in ranges)
        return cls(total_bytes=sum(r.bytes for r in rs), chunk_bytes=chunk_bytes,
                   direction=direction, mode=mode, ranges=rs, job_id=job_id,
                   metadata=dict(metadata or {}))

    def with_mode(self, mode: TransferMode | str) -> "TransferRequest":
        return TransferRequest(self.total_bytes, self.chunk_bytes, self.direction, mode,
                               self.request_chunks, self.ranges, self.job_id, self.metadata)

    def daemon_payload(self, mode: TransferMode | str | None = None) -> dict[str, object]:
        payload: dict[str, object] = {
            "total_bytes": self.total_bytes,
            "chunk_bytes": self.chunk_bytes,
            "mode": TransferMode(self.mode if mode is None else mode).value,
            "direction": self.direction.value,
            "request_chunks": self.request_chunks,
        }
        if self.job_id is not None:
            payload["job_id"] = self.job_id
        if self.ranges:
            payload["ranges"] = [r.as_dict() for r in self.ranges]
        if self.metadata.get("buffer_ids") is not None:
            payload["buffer_ids"] = [str(b) for b in self.metadata["buffer_ids"]]
        return payload

    def as_dict(self) -> dict[str, object]:
        data = self.daemon_payload()
        if self.metadata:
            data["metadata"] = dict(self.metadata)
        return data


__all__ = ["TransferDirection", "TransferRange", "TransferRequest", "chunk_count", "coerce_range"]
