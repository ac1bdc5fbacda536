"""Landing specs: fused data-plane ops carried by a transfer intent.

A plain intent moves bytes range by range.  An intent whose
``metadata["landing"]`` holds a spec asks the data plane to run a fused op
in the same pass, under the same plan, leases and ticket as any intent:

* ``scatter_units`` (H2D): the host stream is a sequence of fixed-size
  units that land at scattered device addresses -- a vLLM paged-KV prefix
  restored into a (permuted) block table;
* ``gather_units`` (D2H): the reverse -- a KV prefix saved from its blocks
  into one host-contiguous region;
* ``fp8_quant`` (H2D): bf16 matrices land as fp8 e4m3 codes plus one fp32
  scale per 128x128 block, quantised in the landing kernel;
* ``adamw`` (H2D round trip): the host range is fp32 optimizer state in
  24 KiB tiles ``[master | exp_avg | exp_avg_sq]`` x 2048 parameters; each
  tile is updated on the GPU with the bf16 gradients of a registered buffer,
  the intent's device buffer receives the bf16 parameters, and the tile
  returns to the host (adapters/streamed_optimizer.py);
* ``copy``: the plain op (the default without a spec).

The reference has no such path: its KV connector and model loader submit
one range per block or tensor and the daemon only plans them
(turbobus/adapters/vllm_kv_connector.py:578-595, 816-872;
turbobus/daemon/server.py:624-724).

Unit ops address the device through a KV layout instead of a raw address
table, so the spec stays small on the wire (block ids, not 131k addresses)
and the daemon can prove every unit lies inside a buffer the job registered::

    {"op": "scatter_units", "unit_bytes": U,
     "kv": {"buffers": [buffer_id per layer], "lanes": 2, "lane_stride": S,
            "block_stride": B, "num_blocks": NB, "block_ids": [...]},
     "ctas_per_lane": 0}

The unit stream is ordered ``[layer][lane][index]`` (the connector's CPU
slot order); the device side of every range is a stream position, so a chunk
starting at stream byte ``p`` begins at unit ``p // U``.  fp8 specs name the
matrices inside the intent's device buffer::

    {"op": "fp8_quant", "tensors": [{"host_offset", "rows", "cols",
                                      "q_offset", "scales_offset"}, ...]}

and a chunk starting at host byte ``h`` of tensor ``t`` begins at row
``(h - t.host_offset) / (2 * cols)``, which must be a multiple of 128.
"""

from __future__ import annotations

from bisect import bisect_right
from collections.abc import Mapping
from dataclasses import dataclass, field
from typing import Any, Sequence

OPS = ("copy", "scatter_units", "gather_units", "fp8_quant", "adamw")
_PARSED: dict[int, tuple] = {}  # id(landing object) -> (object, parsed spec)
TILE_ROWS = 128
ADAM_TILE_PARAMS = 2048
ADAM_TILE_BYTES = 3 * 4 * ADAM_TILE_PARAMS
ADAM_KEYS = ("lr", "beta1", "beta2", "eps", "weight_decay", "grad_scale", "step")


@dataclass(frozen=True)
class KVUnits:
    buffers: tuple[str, ...]
    lanes: int
    lane_stride: int
    block_stride: int
    num_blocks: int
    block_ids: tuple[int, ...]
    # the same ids as a read-only int64 array, kept by the parser so the
    # checks and the unit-address table need no second conversion
    ids_array: Any = field(default=None, compare=False, repr=False, hash=False)

    def ids(self):
        import numpy as np

        return self.ids_array if self.ids_array is not None else np.asarray(self.block_ids, dtype=np.int64)

    @property
    def units(self) -> int:
        return len(self.buffers) * self.lanes * len(self.block_ids)


@dataclass(frozen=True)
class Fp8Tensor:
    host_offset: int
    rows: int
    cols: int
    q_offset: int
    scales_offset: int

    @property
    def host_bytes(self) -> int:
        return self.rows * self.cols * 2

    @property
    def q_bytes(self) -> int:
        return self.rows * self.cols

    @property
    def scales_bytes(self) -> int:
        return -(-self.rows // TILE_ROWS) * (self.cols // 128) * 4


@dataclass(frozen=True)
class LandingSpec:
    op: str = "copy"
    unit_bytes: int = 0
    kv: KVUnits | None = None
    tensors: tuple[Fp8Tensor, ...] = field(default_factory=tuple)
    ctas_per_lane: int = 0
    # adamw: {"grads_buffer", "nparams", "lr", "beta1", "beta2", "eps",
    # "weight_decay", "grad_scale", "step"}
    adam: tuple[tuple[str, Any], ...] = ()

    # ---- wire form ------------------------------------------------------------------
    @classmethod
    def from_metadata(cls, meta: Any) -> "LandingSpec | None":
        """The spec in ``intent.metadata["landing"]`` (None when absent).
        An intent is parsed at submit, by the buffer lookup and by the
        executor: the parse of one landing object is remembered (by identity,
        the object kept alive with it) so its block table is read once."""
        if not isinstance(meta, Mapping) or meta.get("landing") is None:
            return None
        d = meta["landing"]
        hit = _PARSED.get(id(d))
        if hit is not None and hit[0] is d:
            return hit[1]
        spec = cls._parse(d)
        if len(_PARSED) >= 64:
            _PARSED.pop(next(iter(_PARSED)))
        _PARSED[id(d)] = (d, spec)
        return spec

    @classmethod
    def _parse(cls, d: Any) -> "LandingSpec":
        if not isinstance(d, Mapping):
            raise ValueError("landing spec must be an object")
        op = str(d.get("op", "copy")).lower()
        if op not in OPS:
            raise ValueError(f"landing op must be one of {', '.join(OPS)}")
        kv = None
        if d.get("kv") is not None:
            k = d["kv"]
            if not isinstance(k, Mapping):
                raise ValueError("landing kv layout must be an object")
            try:
                import numpy as np

                ids = np.asarray(k["block_ids"], dtype=np.int64)
                if ids.ndim != 1:
                    raise ValueError("block_ids must be a flat list")
                ids.setflags(write=False)
                kv = KVUnits(buffers=tuple(str(b) for b in k["buffers"]), lanes=int(k.get("lanes", 1)),
                             lane_stride=int(k.get("lane_stride", 0)), block_stride=int(k["block_stride"]),
                             num_blocks=int(k["num_blocks"]), block_ids=tuple(ids.tolist()), ids_array=ids)
            except (KeyError, TypeError, ValueError) as exc:
                raise ValueError(f"landing kv layout is incomplete: {exc}") from None
        tensors = []
        for t in d.get("tensors", ()) or ():
            try:
                tensors.append(Fp8Tensor(int(t["host_offset"]), int(t["rows"]), int(t["cols"]),
                                         int(t["q_offset"]), int(t["scales_offset"])))
            except (KeyError, TypeError, ValueError) as exc:
                raise ValueError(f"landing fp8 tensor is incomplete: {exc}") from None
        adam = ()
        if d.get("adam") is not None:
            a = d["adam"]
            if not isinstance(a, Mapping):
                raise ValueError("landing adam parameters must be an object")
            try:
                vals = {"grads_buffer": str(a["grads_buffer"]), "nparams": int(a["nparams"]),
                        "step": int(a.get("step", 1))}
                for k in ADAM_KEYS[:-1]:
                    vals[k] = float(a.get(k, {"lr": 1e-3, "beta1": 0.9, "beta2": 0.999, "eps": 1e-8,
                                              "weight_decay": 0.0, "grad_scale": 1.0}[k]))
            except (KeyError, TypeError, ValueError) as exc:
                raise ValueError(f"landing adam parameters are incomplete: {exc}") from None
            adam = tuple(sorted(vals.items()))
        return cls(op=op, unit_bytes=int(d.get("unit_bytes", 0) or 0), kv=kv, tensors=tuple(tensors),
                   ctas_per_lane=int(d.get("ctas_per_lane", 0) or 0), adam=adam)

    def to_metadata(self) -> dict[str, Any]:
        d: dict[str, Any] = {"op": self.op}
        if self.unit_bytes:
            d["unit_bytes"] = self.unit_bytes
        if self.kv is not None:
            k = self.kv
            d["kv"] = {"buffers": list(k.buffers), "lanes": k.lanes, "lane_stride": k.lane_stride,
                       "block_stride": k.block_stride, "num_blocks": k.num_blocks, "block_ids": list(k.block_ids)}
        if self.tensors:
            d["tensors"] = [{"host_offset": t.host_offset, "rows": t.rows, "cols": t.cols,
                             "q_offset": t.q_offset, "scales_offset": t.scales_offset} for t in self.tensors]
        if self.ctas_per_lane:
            d["ctas_per_lane"] = self.ctas_per_lane
        if self.adam:
            d["adam"] = dict(self.adam)
        return d

    @property
    def adam_params(self) -> dict[str, Any]:
        return dict(self.adam)

    @property
    def units_op(self) -> bool:
        return self.op in ("scatter_units", "gather_units")

    def buffer_ids(self) -> tuple[str, ...]:
        if self.op == "adamw" and self.adam:
            return (str(self.adam_params["grads_buffer"]),)
        return self.kv.buffers if self.kv is not None else ()


# ---- daemon-side validation -------------------------------------------------------------

def validate_landing(spec: LandingSpec, *, direction: str, job_id: str, device_buffer, host_buffer,
                     ranges: Sequence[Mapping[str, int]] | None, total_bytes: int, chunk_bytes: int,
                     buffers: Mapping[str, Any]) -> None:
    """Reject a spec the data plane could not run safely: wrong direction,
    unit or tensor addresses outside buffers the job registered, chunks that
    would split a unit or a 128-row tile.  Raises ValueError."""
    h2d = direction == "h2d"
    if spec.op in ("scatter_units", "fp8_quant") and not h2d:
        raise ValueError(f"landing op {spec.op} lands data: h2d only")
    if spec.op == "gather_units" and h2d:
        raise ValueError("landing op gather_units pushes data: d2h only")
    if spec.op == "adamw" and not h2d:
        raise ValueError("landing op adamw is an h2d round trip")
    if spec.ctas_per_lane < 0 or spec.ctas_per_lane > 64:
        raise ValueError("landing ctas_per_lane must be between 0 and 64")
    rs = list(ranges) if ranges is not None else [{"src_offset": 0, "dst_offset": 0, "bytes": int(total_bytes)}]
    if spec.units_op:
        _validate_units(spec, job_id=job_id, device_buffer=device_buffer, ranges=rs, h2d=h2d,
                        chunk_bytes=chunk_bytes, buffers=buffers)
    elif spec.op == "fp8_quant":
        _validate_fp8(spec, device_buffer=device_buffer, host_buffer=host_buffer, ranges=rs,
                      chunk_bytes=chunk_bytes)
    elif spec.op == "adamw":
        _validate_adam(spec, job_id=job_id, device_buffer=device_buffer, host_buffer=host_buffer, ranges=rs,
                       chunk_bytes=chunk_bytes, buffers=buffers)


def _validate_units(spec, *, job_id, device_buffer, ranges, h2d, chunk_bytes, buffers) -> None:
    k, u = spec.kv, int(spec.unit_bytes)
    if k is None:
        raise ValueError("unit landing ops need a kv layout")
    if u <= 0 or u % 16 != 0:
        raise ValueError("landing unit_bytes must be a positive multiple of 16")
    if chunk_bytes % u != 0:
        raise ValueError("chunk_bytes must be a whole number of units")
    if k.lanes < 1 or k.num_blocks < 1 or not k.buffers or not k.block_ids:
        raise ValueError("landing kv layout needs buffers, lanes, blocks and block ids")
    if device_buffer.buffer_id not in k.buffers:
        raise ValueError("the intent's device buffer must be one of the kv buffers")
    ids = k.ids()
    if int(ids.min()) < 0 or int(ids.max()) >= k.num_blocks:
        raise ValueError("landing block id outside the kv cache")
    if k.lane_stride < 0 or k.block_stride < u or k.block_stride % 16 or k.lane_stride % 16:
        raise ValueError("landing kv strides must be 16-byte aligned and hold a unit")
    extent = (k.lanes - 1) * k.lane_stride + (k.num_blocks - 1) * k.block_stride + u
    for bid in k.buffers:
        b = buffers.get(bid)
        if b is None:
            raise ValueError(f"landing kv buffer {bid} is not registered")
        if b.job_id != job_id:
            raise ValueError(f"landing kv buffer {bid} belongs to another job")
        if b.device_index != device_buffer.device_index or str(b.kind).lower() != str(device_buffer.kind).lower():
            raise ValueError(f"landing kv buffer {bid} is not on the intent's device")
        if extent > int(b.size_bytes):
            raise ValueError(f"landing kv layout exceeds buffer {bid}")
    stream = k.units * u
    for r in ranges:
        dev_off = int(r["dst_offset"] if h2d else r["src_offset"])
        n = int(r["bytes"])
        if dev_off % u or n % u or int(r["src_offset" if h2d else "dst_offset"]) % 16:
            raise ValueError("landing unit ranges must be whole, 16-byte aligned units")
        if dev_off + n > stream:
            raise ValueError("landing range exceeds the kv unit stream")


def _validate_fp8(spec, *, device_buffer, host_buffer, ranges, chunk_bytes) -> None:
    if not spec.tensors:
        raise ValueError("fp8 landing needs a tensor table")
    size = int(device_buffer.size_bytes)
    ts = sorted(spec.tensors, key=lambda t: t.host_offset)
    for a, b in zip(ts, ts[1:]):
        if a.host_offset + a.host_bytes > b.host_offset:
            raise ValueError("fp8 landing tensors overlap on the host")
    for t in ts:
        if t.rows <= 0 or t.cols <= 0 or t.cols % 128:
            raise ValueError("fp8 landing needs rows > 0 and cols % 128 == 0")
        if t.q_offset % 16 or t.scales_offset % 4 or t.host_offset % 16:
            raise ValueError("fp8 landing offsets must be aligned (q 16, scales 4, host 16 bytes)")
        if t.q_offset + t.q_bytes > size or t.scales_offset + t.scales_bytes > size:
            raise ValueError("fp8 landing outputs exceed the device buffer")
        if t.host_offset + t.host_bytes > int(host_buffer.size_bytes):
            raise ValueError("fp8 landing tensor exceeds the host buffer")
    starts = [t.host_offset for t in ts]
    for r in ranges:
        h, n = int(r["src_offset"]), int(r["bytes"])
        if n > chunk_bytes:
            raise ValueError("fp8 landing ranges must each fit one chunk (pre-cut on 128-row tiles)")
        i = bisect_right(starts, h) - 1
        if i < 0:
            raise ValueError("fp8 landing range starts outside every tensor")
        t = ts[i]
        rb = 2 * t.cols
        if (h - t.host_offset) % (rb * TILE_ROWS) or h + n > t.host_offset + t.host_bytes or n % rb:
            raise ValueError("fp8 landing ranges must be whole 128-row tiles of one tensor")


def _validate_adam(spec, *, job_id, device_buffer, host_buffer, ranges, chunk_bytes, buffers) -> None:
    a = spec.adam_params
    if not a:
        raise ValueError("adamw landing needs its adam parameters")
    n = int(a["nparams"])
    if n <= 0 or int(a["step"]) < 1:
        raise ValueError("adamw needs nparams > 0 and step >= 1")
    g = buffers.get(a["grads_buffer"])
    if g is None:
        raise ValueError(f"adamw grads buffer {a['grads_buffer']} is not registered")
    if g.job_id != job_id:
        raise ValueError("adamw grads buffer belongs to another job")
    if g.device_index != device_buffer.device_index or str(g.kind).lower() != str(device_buffer.kind).lower():
        raise ValueError("adamw grads buffer is not on the intent's device")
    if int(g.size_bytes) < 2 * n or int(device_buffer.size_bytes) < 2 * n:
        raise ValueError("adamw grads and params buffers must hold nparams bf16 values")
    tiles = -(-n // ADAM_TILE_PARAMS)
    if int(host_buffer.size_bytes) < tiles * ADAM_TILE_BYTES:
        raise ValueError("adamw host state is smaller than the tiled optimizer state")
    if chunk_bytes % ADAM_TILE_BYTES:
        raise ValueError("adamw chunk_bytes must be a whole number of 24 KiB state tiles")
    for r in ranges:
        s, d, b = int(r["src_offset"]), int(r["dst_offset"]), int(r["bytes"])
        if s != d or s % ADAM_TILE_BYTES or b % ADAM_TILE_BYTES or s + b > tiles * ADAM_TILE_BYTES:
            raise ValueError("adamw ranges must be whole state tiles with dst_offset == src_offset")


# ---- executor side ------------------------------------------------------------------------

def unit_addresses(spec: LandingSpec, base_of) -> "Any":
    """uint64 device address of every unit in stream order; ``base_of(id)``
    gives a kv buffer's device address."""
    import numpy as np

    k = spec.kv
    ids = k.ids().astype(np.uint64)
    # one row per (layer, lane) base address, one column per block: stream order
    per_buffer = np.array([int(base_of(bid)) for bid in k.buffers], dtype=np.uint64)
    bases = (per_buffer[:, None] + np.arange(k.lanes, dtype=np.uint64)[None, :] * np.uint64(k.lane_stride)).ravel()
    return (bases[:, None] + ids[None, :] * np.uint64(k.block_stride)).ravel()


def annotate_lanes(spec: LandingSpec, lanes, h2d: bool) -> None:
    """Per-chunk op fields on engine lanes: first unit (unit ops) or tensor
    index and first row (fp8)."""
    import numpy as np

    if spec.units_op:
        u = np.uint64(spec.unit_bytes)
        for L in lanes:
            pos = L.dst_off if h2d else L.src_off
            L.unit0 = (pos // u).astype(np.uint32)
    elif spec.op == "adamw":
        for L in lanes:
            L.unit0 = (L.src_off // np.uint64(ADAM_TILE_BYTES)).astype(np.uint32)
    elif spec.op == "fp8_quant":
        order = sorted(range(len(spec.tensors)), key=lambda i: spec.tensors[i].host_offset)
        starts = np.array([spec.tensors[i].host_offset for i in order], dtype=np.int64)
        for L in lanes:
            h = L.src_off.astype(np.int64)
            pos = np.searchsorted(starts, h, side="right") - 1
            idx = np.array(order, dtype=np.int64)[pos]
            rb = np.array([2 * spec.tensors[i].cols for i in order], dtype=np.int64)[pos]
            L.tensor = idx.astype(np.uint32)
            L.unit0 = ((h - starts[pos]) // rb).astype(np.uint32)


def fp8_table(spec: LandingSpec, dev_ptr: int) -> list[tuple[int, int, int, int]]:
    return [(dev_ptr + t.q_offset, dev_ptr + t.scales_offset, t.rows, t.cols) for t in spec.tensors]


# ---- spec builders for adapters ------------------------------------------------------------

def kv_spec(kv_caches, block_ids: Sequence[int], buffer_ids: Sequence[str], *, op: str,
            ctas_per_lane: int = 0) -> LandingSpec:
    """Spec for a vLLM KV prefix over per-layer cache tensors registered as
    ``buffer_ids`` (same order)."""
    from ..adapters.vllm import kv_layout

    lay = [kv_layout(kv) for kv in kv_caches]
    l0 = lay[0]
    for x in lay[1:]:
        if (x.lanes, x.lane_stride, x.block_stride, x.unit_bytes, x.num_blocks) != \
                (l0.lanes, l0.lane_stride, l0.block_stride, l0.unit_bytes, l0.num_blocks):
            raise ValueError("all kv layers must share one layout")
    import numpy as np

    return LandingSpec(op=op, unit_bytes=l0.unit_bytes,
                       kv=KVUnits(tuple(str(b) for b in buffer_ids), l0.lanes, l0.lane_stride, l0.block_stride,
                                  l0.num_blocks, tuple(np.asarray(block_ids, dtype=np.int64).tolist())),
                       ctas_per_lane=int(ctas_per_lane))


__all__ = ["Fp8Tensor", "KVUnits", "LandingSpec", "OPS", "annotate_lanes", "fp8_table", "kv_spec",
           "unit_addresses", "validate_landing"]
