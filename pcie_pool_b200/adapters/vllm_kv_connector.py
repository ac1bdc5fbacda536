"""vLLM KV-transfer connector (V1 API) for prefix save and restore.

Requests opt in through ``kv_transfer_params``:
``turbobus.do_save`` / ``turbobus.do_restore`` / ``turbobus.prefix_key`` /
``turbobus.matched_tokens`` / ``turbobus.save_blocks``.  Configuration comes
from ``kv_connector_extra_config`` (``turbobus.*`` keys) or ``TURBOBUS_*``
environment variables, as in the reference connector
(turbobus/adapters/vllm_kv_connector.py:240-307).  Every lifecycle step is
recorded as an event and printed as a ``turbobus_kv_connector_event key=value``
line (set ``TURBOBUS_CONNECTOR_EVENTS=0`` to silence the print).

Two data paths:

* ``engine`` (default when CUDA is usable): the prefix of ALL layers is one
  host region and moves as ONE pooled transfer -- the push kernel gathers the
  request's blocks on save (``wait_for_save``), the landing kernel scatters
  them into the newly allocated (permuted) blocks on restore
  (``start_load_kv``), over the direct lane plus ``turbobus.relay_gpus``;
* ``intent``: one daemon transfer intent per layer through the KV slot
  adapters (the reference's path), for deployments where the daemon's
  executor owns the data plane.
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import Any

from ..offload_store import AdapterTransferContext, TransferStats, summarize_transfer_handles
from ..schema import WorkloadKind
from .vllm import kv_layout, make_vllm_layer_range_refs_from_ids
from .vllm_integration import extract_vllm_block_ids, normalize_block_id_groups

try:  # pragma: no cover - depends on an installed vLLM build
    from vllm.distributed.kv_transfer.kv_connector.v1.base import (KVConnectorBase_V1, KVConnectorMetadata,
                                                                  KVConnectorRole)
    try:
        from vllm.distributed.kv_transfer.kv_connector.v1.base import SupportsHMA
    except ImportError:
        SupportsHMA = object
except Exception:  # noqa: BLE001 - importable without vLLM (tests, CPU tools)
    class KVConnectorMetadata:  # type: ignore[no-redef]
        pass

    class KVConnectorBase_V1:  # type: ignore[no-redef]
        def __init__(self, vllm_config, role, kv_cache_config=None):
            self._vllm_config = vllm_config
            self._role = role
            self._connector_metadata = None

        def bind_connector_metadata(self, metadata):
            self._connector_metadata = metadata

        def clear_connector_metadata(self):
            self._connector_metadata = None

        def has_connector_metadata(self):
            return self._connector_metadata is not None

    class KVConnectorRole:  # type: ignore[no-redef]
        SCHEDULER = "scheduler"
        WORKER = "worker"

    SupportsHMA = object


@dataclass
class TurboBusRequestMetadata:
    request_id: str
    prefix_key: str
    block_ids: tuple[int, ...]
    matched_tokens: int
    block_count: int
    cpu_slot_start: int = 0


@dataclass
class TurboBusSavedPrefix:
    key: str
    cpu_backings: list[Any]
    block_count: int
    matched_tokens: int
    session_id: str = "default"
    source_request_id: str = ""
    bytes: int = 0
    elapsed_ms: float = 0.0
    transfer_ms: float = 0.0
    total_ms: float = 0.0
    direct_chunks: int = 0
    relay_chunks: int = 0
    direct_bytes: int = 0
    relay_bytes: int = 0
    receipt_ids: str = ""
    fallback_reason: str = ""
    save_layer_count: int = 0
    save_layer_ranges: int = 0
    data_path: str = "engine"
    host: Any = None            # engine path: the single host region of all layers
    cuda_ms: float = 0.0


class TurboBusPrefixStore:
    """In-process saved prefixes keyed ``"{session}\\0{key}"``, oldest evicted
    first once ``max_prefixes`` (0 = unbounded) is exceeded."""

    def __init__(self, max_prefixes: int = 0) -> None:
        self._p: dict[str, TurboBusSavedPrefix] = {}
        self.max_prefixes = max(0, int(max_prefixes))

    @staticmethod
    def _key(key: str, session_id: str = "default") -> str:
        return f"{session_id}\0{key}"

    def put(self, prefix: TurboBusSavedPrefix) -> list[TurboBusSavedPrefix]:
        if not prefix.key:
            raise ValueError("prefix key must not be empty")
        k = self._key(prefix.key, prefix.session_id)
        evicted = [self._p.pop(k)] if k in self._p else []
        self._p[k] = prefix
        while self.max_prefixes and len(self._p) > self.max_prefixes:
            evicted.append(self._p.pop(next(iter(self._p))))
        return evicted

    def get(self, key: str, session_id: str = "default") -> TurboBusSavedPrefix | None:
        return self._p.get(self._key(key, session_id))

    def remove(self, key: str, session_id: str = "default") -> TurboBusSavedPrefix | None:
        return self._p.pop(self._key(key, session_id), None)

    def clear(self, session_id: str | None = None) -> None:
        if session_id is None:
            self._p.clear()
            return
        pre = f"{session_id}\0"
        for k in [k for k in self._p if k.startswith(pre)]:
            self._p.pop(k)

    def __len__(self) -> int:
        return len(self._p)


def _lanes_per_layer(kv) -> int:
    return kv_layout(kv).lanes


def _unit_bytes(kv) -> int:
    return kv_layout(kv).unit_bytes


def _signature(block_count: int, kv_caches: list[Any]) -> tuple:
    return (int(block_count),) + tuple((_lanes_per_layer(kv), _unit_bytes(kv)) for kv in kv_caches)


class TurboBusCPUBackingPool:
    """Reuses page-locked host backings by shape signature.  A backing is one
    pinned uint8 region of ``layers x lanes x blocks`` units; ``views`` are the
    per-layer slices (the reference's one-tensor-per-layer layout)."""

    def __init__(self, shared: bool = False) -> None:
        self._free: dict[tuple, list[Any]] = {}
        # shared: backings live in shared page-locked memory so a daemon
        # process can map them (its data plane moves the bytes)
        self.shared = bool(shared)

    def acquire(self, block_count: int, kv_caches: list[Any]) -> tuple[Any, bool]:
        sig = _signature(block_count, kv_caches)
        if self._free.get(sig):
            return self._free[sig].pop(), True
        return self._allocate(block_count, kv_caches, self.shared), False

    def release(self, block_count: int, kv_caches: list[Any], cpu_backings) -> None:
        self._free.setdefault(_signature(block_count, kv_caches), []).append(cpu_backings)

    def release_prefix(self, prefix: "TurboBusSavedPrefix", kv_caches: list[Any]) -> None:
        """Return a saved prefix's CPU backings to the pool."""
        self.release(prefix.block_count, kv_caches, prefix.cpu_backings)

    @staticmethod
    def _allocate(block_count: int, kv_caches: list[Any], shared: bool = False):
        import torch

        per = [max(1, block_count * _lanes_per_layer(kv)) * _unit_bytes(kv) for kv in kv_caches]
        shm = None
        if shared:
            from ..client import SharedPinnedCpuBuffer

            shm = SharedPinnedCpuBuffer.allocate(f"kv-backing-{id(per)}", "vllm-kv", sum(per))
            whole = torch.from_numpy(shm.numpy())
        else:
            whole = torch.empty(sum(per), dtype=torch.uint8, pin_memory=torch.cuda.is_available())
        views, off = [], 0
        for n in per:
            views.append(whole[off:off + n])
            off += n
        return {"tensor": whole, "views": views, "shm": shm}


class TurboBusConnectorMetadata(KVConnectorMetadata):
    def __init__(self) -> None:
        super().__init__()
        self.requests: list[TurboBusRequestMetadata] = []
        self.save_requests: list[TurboBusRequestMetadata] = []

    def add_request(self, request: TurboBusRequestMetadata) -> None:
        self.requests.append(request)

    def add_save_request(self, request: TurboBusRequestMetadata) -> None:
        self.save_requests.append(request)

    def __len__(self) -> int:
        return len(self.requests) + len(self.save_requests)


@dataclass
class TurboBusKVConnectorState:
    kv_caches: dict[str, Any] = field(default_factory=dict)
    pending_loads: dict[str, TurboBusRequestMetadata] = field(default_factory=dict)
    pending_saves: dict[str, TurboBusRequestMetadata] = field(default_factory=dict)
    save_params_by_request_id: dict[str, dict[str, Any]] = field(default_factory=dict)
    save_request_ids: set[str] = field(default_factory=set)
    saved_request_ids: set[str] = field(default_factory=set)
    finished_sending: set[str] = field(default_factory=set)
    finished_recving: set[str] = field(default_factory=set)
    events: list[dict[str, Any]] = field(default_factory=list)


def _extra(vllm_config, key: str, default):
    kv = getattr(vllm_config, "kv_transfer_config", None)
    get = getattr(kv, "get_from_extra_config", None)
    if callable(get):
        return get(key, default)
    extra = getattr(kv, "kv_connector_extra_config", None)
    if isinstance(extra, dict):
        return extra.get(key, default)
    return default


def _as_bool(v) -> bool:
    return v if isinstance(v, bool) else str(v).lower() in ("1", "true", "yes", "on")


@dataclass(frozen=True)
class TurboBusConnectorConfig:
    job_id: str
    session_id: str
    cpu_buffer_id: str
    gpu_buffer_id: str
    chunk_bytes: int
    daemon_socket_path: str
    wait_timeout_seconds: float | None
    restore_block_limit: int
    restore_enabled: bool
    max_saved_prefixes: int
    data_path: str = "engine"
    relay_gpus: tuple[int, ...] = ()
    load_async: bool = False

    @classmethod
    def from_vllm_config(cls, vllm_config) -> "TurboBusConnectorConfig":
        env = os.environ.get
        kv = getattr(vllm_config, "kv_transfer_config", None)
        engine_id = getattr(kv, "engine_id", None)
        session = str(_extra(vllm_config, "turbobus.session_id", str(engine_id) if engine_id else "default"))
        timeout = _extra(vllm_config, "turbobus.wait_timeout_seconds", env("TURBOBUS_WAIT_TIMEOUT_SECONDS", ""))
        relays = _extra(vllm_config, "turbobus.relay_gpus", env("TURBOBUS_RELAY_GPUS", ""))
        if isinstance(relays, str):
            relays = [int(x) for x in relays.split(",") if x.strip()]
        return cls(
            job_id=str(_extra(vllm_config, "turbobus.job_id", env("TURBOBUS_JOB_ID", session))),
            session_id=session,
            cpu_buffer_id=str(_extra(vllm_config, "turbobus.cpu_buffer_id",
                                     env("TURBOBUS_CPU_BUFFER_ID", "vllm-kv-cpu-buffer"))),
            gpu_buffer_id=str(_extra(vllm_config, "turbobus.gpu_buffer_id",
                                     env("TURBOBUS_GPU_BUFFER_ID", "vllm-kv-gpu-buffer"))),
            chunk_bytes=int(_extra(vllm_config, "turbobus.chunk_bytes", int(env("TURBOBUS_CHUNK_BYTES", 4 << 20)))),
            daemon_socket_path=str(_extra(vllm_config, "turbobus.daemon_socket_path",
                                          env("TURBOBUS_DAEMON_SOCKET_PATH", ""))),
            # unset means "wait until done": a prefix is registered only after its bytes landed
            wait_timeout_seconds=600.0 if timeout in (None, "") else float(timeout),
            restore_block_limit=int(_extra(vllm_config, "turbobus.restore_block_limit",
                                           int(env("TURBOBUS_RESTORE_BLOCK_LIMIT", "0") or 0))),
            restore_enabled=_as_bool(_extra(vllm_config, "turbobus.restore_enabled",
                                             env("TURBOBUS_RESTORE_ENABLED", "0") == "1")),
            max_saved_prefixes=int(_extra(vllm_config, "turbobus.max_saved_prefixes",
                                          int(env("TURBOBUS_MAX_SAVED_PREFIXES", "0") or 0))),
            data_path=str(_extra(vllm_config, "turbobus.data_path", env("TURBOBUS_DATA_PATH", "engine"))),
            load_async=_as_bool(_extra(vllm_config, "turbobus.load_async", env("TURBOBUS_LOAD_ASYNC", "0") == "1")),
            relay_gpus=tuple(int(x) for x in (relays or ())))


_PREFIX_STORE = TurboBusPrefixStore()
_CONNECTOR_EVENTS: list[dict[str, Any]] = []


def clear_saved_prefixes(session_id: str | None = None) -> None:
    _PREFIX_STORE.clear(session_id)


def get_saved_prefix(key: str, session_id: str = "default") -> TurboBusSavedPrefix | None:
    return _PREFIX_STORE.get(str(key), str(session_id))


def clear_connector_events() -> None:
    _CONNECTOR_EVENTS.clear()


def get_connector_events() -> list[dict[str, Any]]:
    return list(_CONNECTOR_EVENTS)


def _emit(event: str, **fields) -> dict[str, Any]:
    rec = {"event": event, **fields}
    _CONNECTOR_EVENTS.append(rec)
    if os.environ.get("TURBOBUS_CONNECTOR_EVENTS", "1") != "0":
        print("turbobus_kv_connector_event " + " ".join(f"{k}={v}" for k, v in rec.items()), flush=True)
    return rec


def _params(request) -> dict[str, Any]:
    for attr in ("kv_transfer_params",):
        p = getattr(request, attr, None)
        if isinstance(p, dict):
            return p
    sp = getattr(request, "sampling_params", None)
    p = getattr(sp, "extra_args", None) if sp is not None else None
    if isinstance(p, dict) and isinstance(p.get("kv_transfer_params"), dict):
        return p["kv_transfer_params"]
    return {}


def _prefix_key(params: dict[str, Any]) -> str:
    return str(params.get("turbobus.prefix_key", "default"))


def _flat(groups) -> tuple[int, ...]:
    seen: set[int] = set()
    out = []
    for g in groups:
        for b in g:
            if b not in seen:
                seen.add(b)
                out.append(int(b))
    return tuple(out)


def _blocks_for_tokens(tokens: int, block_size: int) -> int:
    return 0 if tokens <= 0 or block_size <= 0 else (int(tokens) + block_size - 1) // block_size


def _save_blocks(params: dict[str, Any], block_size: int) -> int:
    if params.get("turbobus.save_blocks") is not None:
        return int(params.get("turbobus.save_blocks") or 0)
    return _blocks_for_tokens(int(params.get("turbobus.matched_tokens", 0) or 0), block_size)


def _matched_for_save(params: dict[str, Any], block_size: int) -> int:
    m = int(params.get("turbobus.matched_tokens", 0) or 0)
    return m if m > 0 else _save_blocks(params, block_size) * block_size


class TurboBusConnector(KVConnectorBase_V1, SupportsHMA):
    """vLLM connector entry point (``kv_connector="TurboBusConnector"``,
    ``kv_connector_module_path="pcie_pool_b200.vllm_kv_connector"``)."""

    @classmethod
    def requires_piecewise_for_cudagraph(cls, extra_config: dict[str, Any]) -> bool:
        return True

    def __init__(self, vllm_config, role: "KVConnectorRole", kv_cache_config=None) -> None:
        try:
            super().__init__(vllm_config=vllm_config, role=role, kv_cache_config=kv_cache_config)
        except TypeError:
            super().__init__(vllm_config=vllm_config, role=role)
        self.state = TurboBusKVConnectorState()
        self.vllm_block_size = int(getattr(getattr(vllm_config, "cache_config", None), "block_size", 16) or 16)
        self.config = TurboBusConnectorConfig.from_vllm_config(vllm_config)
        self.restore_block_limit = self.config.restore_block_limit
        self.restore_enabled = self.config.restore_enabled
        self.session_id = self.config.session_id
        self.job_id = self.config.job_id
        self.max_saved_prefixes = self.config.max_saved_prefixes
        self._client = None
        self._offloader = None
        self._save_layers: dict[str, set[int]] = {}
        self._backing_pool = TurboBusCPUBackingPool()
        self._prefix_store = TurboBusPrefixStore(max_prefixes=self.max_saved_prefixes)
        _emit("init", role=str(role), job_id=self.job_id, session_id=self.session_id,
              restore_enabled=self.restore_enabled, restore_block_limit=self.restore_block_limit,
              max_saved_prefixes=self.max_saved_prefixes, data_path=self.config.data_path)

    # ---- clients / data path -------------------------------------------------------------
    @property
    def client(self):
        if self._client is None:
            from ..api import TurboBusClient

            self._client = TurboBusClient(socket_path=self.config.daemon_socket_path)
        return self._client

    @client.setter
    def client(self, value) -> None:
        self._client = value

    def _kv_list(self) -> list[Any]:
        return [kv for _, kv in self.state.kv_caches.items()]

    def _engine_offloader(self):
        """The fused KV data path, driven through the node daemon: each save
        or restore is one intent with a gather / scatter landing spec, so the
        relays it uses come from the daemon's leases.  With
        ``turbobus.daemon_socket_path`` the daemon is the node's daemon
        process (KV caches exported by CUDA IPC, backings in shared memory);
        without it the worker runs a daemon of its own over the target and
        ``turbobus.relay_gpus`` (same scheduler, leases and executor)."""
        if self._offloader is None:
            from .kv_offload import DaemonKVOffloader

            kvs = self._kv_list()
            target = int(kvs[0].device.index)
            relays = [r for r in self.config.relay_gpus if r != target]
            dc, client = self._node_daemon(target, relays)
            sess = dc.register_session(target, relays, max_inflight_chunks=1 << 16)
            if not sess.ok:
                raise RuntimeError(f"daemon session registration failed: {sess.error}")
            sid = sess.payload["session"]["session_id"]
            r = dc.register_job(self.job_id, session_id=sid)
            if not r.ok:
                raise RuntimeError(f"daemon job registration failed: {r.error}")
            upc = max(1, self.config.chunk_bytes // _unit_bytes(kvs[0]))
            self._offloader = DaemonKVOffloader(client, dc, session_id=sid, job_id=self.job_id, kv_caches=kvs,
                                                units_per_chunk=upc, prefix=f"{self.job_id}-kv")
        return self._offloader

    def _node_daemon(self, target: int, relays: list[int]):
        from ..api import TurboBusClient

        path = self.config.daemon_socket_path
        if path and os.path.exists(path):
            from ..daemon import TurboBusDaemonClient

            dc = TurboBusDaemonClient(path, persistent=True)
            self._backing_pool.shared = True
            return dc, TurboBusClient(daemon=dc)
        from ..e2e import build_inprocess_node, nominal_profile
        from ..parallel.engine import PoolEngine

        devs = [target, *relays]
        eng = PoolEngine(devs, slot_bytes=max(self.config.chunk_bytes, 1 << 20), slots=3)
        daemon, dc = build_inprocess_node(eng, devs, target, nominal_profile(target, relays) if relays else None)
        self._node = daemon
        return dc, TurboBusClient(daemon=dc)

    # ---- worker side: caches -----------------------------------------------------------------
    def register_kv_caches(self, kv_caches: dict[str, Any]) -> None:
        self.state.kv_caches = dict(kv_caches)
        self.state.events.append({"event": "register_kv_caches", "layers": len(self.state.kv_caches)})
        _emit("register_kv_caches", layers=len(self.state.kv_caches))

    # ---- scheduler side -------------------------------------------------------------------------
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int) -> tuple[int | None, bool]:
        p = _params(request)
        rid = str(getattr(request, "request_id", "unknown"))
        if not p.get("turbobus.do_restore"):
            return 0, False
        if not self.restore_enabled:
            self.state.events.append({"event": "match_skipped", "request_id": rid, "restore_enabled": False})
            _emit("match_skipped", request_id=rid, restore_enabled=False)
            return 0, False
        key = _prefix_key(p)
        saved = get_saved_prefix(key, self.session_id)
        if saved is None:
            self.state.events.append({"event": "match_miss", "request_id": rid, "prefix_key": key,
                                      "session_id": self.session_id})
            _emit("match_miss", request_id=rid, prefix_key=key, session_id=self.session_id)
            return 0, False
        matched = int(p.get("turbobus.matched_tokens", 0) or 0) or saved.matched_tokens
        matched = min(matched, saved.matched_tokens)
        if matched <= num_computed_tokens:
            return 0, False
        avail = matched - int(num_computed_tokens)
        # vLLM must compute at least the last prompt token itself
        if avail == matched and avail == int(getattr(request, "num_tokens", 0)):
            avail -= 1
        rec = {"event": "match", "request_id": rid, "prefix_key": key, "session_id": self.session_id,
               "matched_tokens": matched, "num_computed_tokens": int(num_computed_tokens),
               "available_tokens": max(0, avail)}
        self.state.events.append(rec)
        _emit(**rec)
        # The restore runs synchronously inside start_load_kv, before the
        # forward that reads the blocks, so the load is not asynchronous
        # unless turbobus.load_async asks for vLLM's async-load protocol.
        return max(0, avail), bool(self.config.load_async and avail > 0)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int) -> None:
        p = _params(request)
        if p.get("turbobus.do_save"):
            self._save_state_after_alloc(request, blocks, p)
        if num_external_tokens <= 0:
            return
        key = _prefix_key(p)
        rid = str(getattr(request, "request_id", "unknown"))
        saved = get_saved_prefix(key, self.session_id)
        if saved is None:
            _emit("alloc_miss", request_id=rid, prefix_key=key, session_id=self.session_id)
            return
        ids = _flat(extract_vllm_block_ids(blocks))
        if not ids:
            return
        n = _blocks_for_tokens(num_external_tokens, self.vllm_block_size)
        if self.restore_block_limit > 0:
            n = min(n, self.restore_block_limit)
        n = min(n, saved.block_count)
        meta = TurboBusRequestMetadata(rid, key, tuple(ids[:n]), int(num_external_tokens), len(ids[:n]))
        self.state.pending_loads[rid] = meta
        rec = {"event": "alloc", "request_id": rid, "prefix_key": key, "session_id": self.session_id,
               "matched_tokens": int(num_external_tokens), "block_count": meta.block_count}
        self.state.events.append(rec)
        _emit(**rec)

    def _save_state_after_alloc(self, request, blocks, p: dict[str, Any]) -> None:
        rid = str(getattr(request, "request_id", "unknown"))
        if rid in self.state.save_request_ids:
            return
        self.state.save_params_by_request_id[rid] = dict(p)
        ids = _flat(extract_vllm_block_ids(blocks))
        if not ids:
            return
        want = _save_blocks(p, self.vllm_block_size) or len(ids)
        if len(ids) < want:
            rec = {"event": "save_waiting", "request_id": rid, "available_blocks": len(ids), "requested_blocks": want}
            self.state.events.append(rec)
            _emit(**rec)
            return
        self._queue_save(rid, p, ids[:want])

    def _queue_save(self, rid: str, p: dict[str, Any], ids) -> None:
        self.state.pending_saves[rid] = TurboBusRequestMetadata(rid, _prefix_key(p), tuple(ids),
                                                                _matched_for_save(p, self.vllm_block_size), len(ids))
        self.state.save_request_ids.add(rid)
        self.state.save_params_by_request_id.pop(rid, None)

    def build_connector_meta(self, scheduler_output) -> TurboBusConnectorMetadata:
        self._collect_saves(scheduler_output)
        md = TurboBusConnectorMetadata()
        for rid in sorted(self.state.pending_loads):
            md.add_request(self.state.pending_loads[rid])
        for rid in sorted(self.state.pending_saves):
            md.add_save_request(self.state.pending_saves[rid])
        if len(md):
            _emit("build_connector_meta", requests=len(md), loads=len(md.requests), saves=len(md.save_requests))
        self.state.pending_loads.clear()
        self.state.pending_saves.clear()
        return md

    def _collect_saves(self, scheduler_output) -> None:
        """Requests waiting for more blocks become saves once scheduled with enough."""
        if scheduler_output is None or not self.state.save_params_by_request_id:
            return
        for req in _scheduled(scheduler_output):
            rid = str(getattr(req, "req_id", getattr(req, "request_id", "")))
            p = self.state.save_params_by_request_id.get(rid)
            if p is None:
                continue
            raw = getattr(req, "block_ids", None) or getattr(req, "new_block_ids", None)
            ids = _flat(normalize_block_id_groups(raw))
            want = _save_blocks(p, self.vllm_block_size) or len(ids)
            if ids and len(ids) >= want:
                self._queue_save(rid, p, ids[:want])

    # ---- worker side: load / save -------------------------------------------------------------
    def _meta(self):
        return getattr(self, "_connector_metadata", None)

    def start_load_kv(self, forward_context, **kwargs) -> None:
        md = self._meta()
        if not isinstance(md, TurboBusConnectorMetadata) or not md.requests:
            return
        t0 = time.perf_counter()
        for r in md.requests:
            if self.restore_enabled:
                self._restore(r)
            else:
                self.state.events.append({"event": "load_ready", "request_id": r.request_id,
                                          "block_count": len(r.block_ids), "restore_enabled": False})
                _emit("load_ready", request_id=r.request_id, block_count=len(r.block_ids), restore_enabled=False)
            if self.config.load_async:
                self.state.finished_recving.add(r.request_id)
        _emit("start_load_done", requests=len(md.requests), restore_enabled=self.restore_enabled,
              elapsed_ms=f"{(time.perf_counter() - t0) * 1e3:.3f}")

    def _restore(self, r: TurboBusRequestMetadata) -> None:
        saved = get_saved_prefix(r.prefix_key, self.session_id)
        if saved is None:
            raise RuntimeError(f"saved prefix {r.prefix_key} vanished before restore")
        t0 = time.perf_counter()
        n = min(len(r.block_ids), saved.block_count)
        ids = list(r.block_ids[:n])
        if saved.data_path == "engine":
            host = saved.host.get("shm") or saved.host["tensor"]
            stats = self._engine_offloader().restore(ids, host, span_blocks=saved.block_count)
            cuda_ms, nbytes = stats.cuda_ms, stats.bytes
        else:
            refs = make_vllm_layer_range_refs_from_ids(r.request_id, ids, self._kv_list())
            adapter = self._intent_adapter(saved.cpu_backings)
            handles = adapter.restore_prefix(refs)
            ts = summarize_transfer_handles(handles)
            cuda_ms, nbytes = 0.0, ts.bytes
        rec = {"event": "restore", "request_id": r.request_id, "prefix_key": r.prefix_key,
               "block_count": n, "bytes": nbytes, "cuda_ms": round(cuda_ms, 3),
               "transfer_ms": f"{(time.perf_counter() - t0) * 1e3:.3f}", "data_path": saved.data_path}
        self.state.events.append(rec)
        _emit(**rec)

    def wait_for_layer_load(self, layer_name: str) -> None:
        return None

    def save_kv_layer(self, layer_name: str, kv_layer, attn_metadata, **kwargs) -> None:
        md = self._meta()
        if not isinstance(md, TurboBusConnectorMetadata) or not md.save_requests:
            return None
        if not self.state.kv_caches:
            raise RuntimeError("vLLM did not register KV caches for the connector")
        names = list(self.state.kv_caches)
        idx = names.index(layer_name) if layer_name in names else next(
            (i for i, kv in enumerate(self.state.kv_caches.values()) if kv is kv_layer), len(names) - 1)
        for r in md.save_requests:
            self._save_layers.setdefault(r.request_id, set()).add(idx)
        return None

    def wait_for_save(self) -> None:
        md = self._meta()
        if not isinstance(md, TurboBusConnectorMetadata) or not md.save_requests:
            return None
        done = 0
        for r in md.save_requests:
            seen = self._save_layers.pop(r.request_id, None)
            if not seen:
                raise RuntimeError(f"vLLM did not call save_kv_layer before wait_for_save for request {r.request_id}")
            if len(seen) != len(self.state.kv_caches):
                raise RuntimeError(f"saved {len(seen)} of {len(self.state.kv_caches)} KV layers for request "
                                   f"{r.request_id}")
            self._save(r)
            done += 1
        self.state.events.append({"event": "wait_for_save_done", "requests": done})
        _emit("wait_for_save_done", requests=done)
        return None

    def _save(self, r: TurboBusRequestMetadata) -> None:
        t0 = time.perf_counter()
        kvs = self._kv_list()
        path = self.config.data_path
        # the data path first: a daemon process needs shared backings
        off = self._engine_offloader() if path == "engine" else None
        backing, reused = self._backing_pool.acquire(r.block_count, kvs)
        if off is not None:
            host = backing.get("shm") or backing["tensor"]
            st = off.save(list(r.block_ids), host)
            nbytes, cuda_ms, receipts, fallback = st.bytes, st.cuda_ms, "", ""
            ranges = st.units
        else:
            refs = make_vllm_layer_range_refs_from_ids(r.request_id, r.block_ids, kvs)
            handles = self._intent_adapter(backing["views"]).save_prefix(refs)
            ts: TransferStats = summarize_transfer_handles(handles)
            nbytes, cuda_ms = ts.bytes, 0.0
            receipts = ",".join(sorted({h.receipt.receipt_id for h in handles}))
            fallback = ",".join(sorted({str(h.receipt.metadata.get("fallback_reason")) for h in handles
                                        if h.receipt.metadata.get("fallback_reason")}))
            ranges = len(refs)
        total_ms = (time.perf_counter() - t0) * 1e3
        prefix = TurboBusSavedPrefix(key=r.prefix_key, cpu_backings=list(backing["views"]),
                                     block_count=r.block_count, matched_tokens=r.matched_tokens,
                                     session_id=self.session_id, source_request_id=r.request_id, bytes=nbytes,
                                     transfer_ms=total_ms, total_ms=total_ms, receipt_ids=receipts,
                                     fallback_reason=fallback, save_layer_count=len(kvs), save_layer_ranges=ranges,
                                     data_path=path, host=backing, cuda_ms=cuda_ms)
        for old in _PREFIX_STORE.put(prefix) + self._prefix_store.put(prefix):
            if old is not prefix and old.host is not None:
                self._backing_pool.release(old.block_count, kvs, old.host)
        self.state.saved_request_ids.add(r.request_id)
        rec = {"event": "save", "request_id": r.request_id, "prefix_key": r.prefix_key,
               "block_count": r.block_count, "bytes": nbytes, "reused_backing": reused,
               "cuda_ms": round(cuda_ms, 3), "total_ms": f"{total_ms:.3f}", "data_path": path}
        self.state.events.append(rec)
        _emit(**rec)

    def _intent_adapter(self, cpu_backings):
        from .vllm import VllmKVSlotAdapter, make_vllm_layer_groups_from_kv_caches

        ctx = AdapterTransferContext(job_id=self.job_id, session_id=self.session_id,
                                     cpu_buffer_id=self.config.cpu_buffer_id,
                                     gpu_buffer_id=self.config.gpu_buffer_id, workload_kind=WorkloadKind.KV_CACHE,
                                     metadata={"chunk_bytes": self.config.chunk_bytes},
                                     wait_timeout_seconds=self.config.wait_timeout_seconds)
        return VllmKVSlotAdapter(self.client, ctx, make_vllm_layer_groups_from_kv_caches(cpu_backings,
                                                                                         self._kv_list()))

    # ---- completion ----------------------------------------------------------------------------
    def get_finished(self, finished_req_ids: set[str]):
        # Saves complete inside wait_for_save and request_finished never
        # delays the free, so there is nothing "sending" to report (vLLM has
        # already dropped finished requests); only asynchronous loads report.
        if finished_req_ids:
            self.state.saved_request_ids -= set(finished_req_ids)
        recving, self.state.finished_recving = self.state.finished_recving, set()
        return None, recving or None

    def request_finished(self, request, block_ids: list[int]):
        p = _params(request)
        if not p.get("turbobus.do_save"):
            return False, None
        rid = str(getattr(request, "request_id", "unknown"))
        if rid not in self.state.save_request_ids:
            return False, None
        # The save already completed inside wait_for_save of the step that
        # computed the prefix, so the blocks can be freed at once.
        return False, {"turbobus.prefix_key": _prefix_key(p),
                      "turbobus.matched_tokens": _matched_for_save(p, self.vllm_block_size)}

    def request_finished_all_groups(self, request, block_ids: tuple[list[int], ...]):
        return self.request_finished(request, [b for g in block_ids for b in g])


def _scheduled(scheduler_output) -> list[Any]:
    out = []
    for attr in ("scheduled_new_reqs", "scheduled_cached_reqs"):
        v = getattr(scheduler_output, attr, None)
        if v is None:
            continue
        if isinstance(v, (list, tuple)):
            out.extend(v)
        else:
            ids = getattr(v, "req_ids", None) or []
            blocks = getattr(v, "new_block_ids", None) or [None] * len(ids)
            for rid, b in zip(ids, blocks):
                out.append(type("ScheduledReq", (), {"req_id": rid, "new_block_ids": b})())
    return out


__all__ = ["KVConnectorRole", "TurboBusCPUBackingPool", "TurboBusConnector", "TurboBusConnectorConfig", "TurboBusConnectorMetadata",
           "TurboBusKVConnectorState", "TurboBusPrefixStore", "TurboBusRequestMetadata", "TurboBusSavedPrefix",
           "clear_connector_events", "clear_saved_prefixes", "get_connector_events", "get_saved_prefix"]
