"""Worker-managed pooled transfers between a client's shared pinned host
buffer and its CUDA IPC device buffer.

Steps (turbobus/client_transfer.py:55-297): open a daemon session ->
register job and both buffers -> PLAN_TRANSFER -> check the relay leases
against the plan -> hand the authorization to the worker helper -> check
the completion envelope field by field -> confirm the daemon status.  A
plan without relay lanes runs locally under a daemon-issued direct ticket
(:370-576) on this process's persistent engine.  Every failure after
planning releases the planned relay leases.
"""

from __future__ import annotations

from .planner_types import assignment_has_chunks, assignment_spans

from dataclasses import asdict, dataclass, field
from collections.abc import Mapping
from typing import Iterable

from .client import CudaIpcDeviceBuffer, SharedPinnedCpuBuffer
from .schema import (BufferRegistration, DaemonResponse, ExecutionTicket, WorkerTransferAuthorizationRequest)
from .transfer import TransferRequest
from .worker.helper import TICKET_ISSUER, WorkerServiceRequestEnvelope, WorkerServiceResponseEnvelope

DEFAULT_CHUNK_BYTES = 16 << 20


def _require_ok(resp: DaemonResponse, what: str) -> DaemonResponse:
    if not isinstance(resp, DaemonResponse):
        raise TypeError(f"{what}: daemon returned {type(resp).__name__}")
    if not resp.ok:
        raise RuntimeError(f"{what}: {resp.error}")
    return resp


class _CompletionError(RuntimeError):
    pass


@dataclass(frozen=True)
class WorkerManagedTransferResult:
    transfer_id: str
    session_id: str
    job_id: str
    source_buffer_id: str
    target_buffer_id: str
    plan: Mapping[str, object]
    lease_token: Mapping[str, object] | None
    lease_tokens: tuple[Mapping[str, object], ...]
    authorization_request: WorkerTransferAuthorizationRequest | None
    worker_lifecycle: Mapping[str, object] | None
    worker_completion: Mapping[str, object] | None
    final_status: Mapping[str, object]
    path: str = "worker"
    measured: Mapping[str, object] = field(default_factory=dict)

    @property
    def bytes_completed(self) -> int:
        return int(self.final_status.get("bytes_completed", 0))

    @property
    def state(self) -> str:
        s = self.final_status.get("state", "unknown")
        return str(getattr(s, "value", s))


@dataclass
class WorkerManagedTransferClient:
    daemon_client: object
    worker_client: object
    target_gpu: int
    relay_gpus: Iterable[int]
    max_inflight_chunks: int = 8
    engine: object | None = None
    checksum: bool = True
    _session_id: str | None = field(default=None, init=False, repr=False)

    # -- session ----------------------------------------------------------------------------------
    def open_session(self) -> str:
        if self._session_id is None:
            r = _require_ok(self.daemon_client.register_session(int(self.target_gpu),
                                                                [int(g) for g in self.relay_gpus],
                                                                int(self.max_inflight_chunks)),
                            "daemon session registration failed")
            self._session_id = str(r.payload["session"]["session_id"])
        return self._session_id

    def close_session(self) -> DaemonResponse:
        if self._session_id is None:
            return DaemonResponse(ok=True, payload={"closed": False})
        r = self.daemon_client.close_session(self._session_id)
        if r.ok:
            self._session_id = None
        return r

    # -- public transfers ----------------------------------------------------------------------------
    def fetch_shared_cpu_to_cuda_ipc(self, source: SharedPinnedCpuBuffer, target: CudaIpcDeviceBuffer, *,
                                     ranges=None, chunk_bytes: int = DEFAULT_CHUNK_BYTES, mode: str = "relay",
                                     job_id: str | None = None, user_id: str | None = None) -> WorkerManagedTransferResult:
        if not isinstance(source, SharedPinnedCpuBuffer):
            raise TypeError("source must be a SharedPinnedCpuBuffer")
        if not isinstance(target, CudaIpcDeviceBuffer):
            raise TypeError("target must be a CudaIpcDeviceBuffer")
        return self._transfer(source, target, "h2d", ranges, chunk_bytes, mode, job_id, user_id)

    def offload_cuda_ipc_to_shared_cpu(self, source: CudaIpcDeviceBuffer, target: SharedPinnedCpuBuffer, *,
                                       ranges=None, chunk_bytes: int = DEFAULT_CHUNK_BYTES, mode: str = "relay",
                                       job_id: str | None = None,
                                       user_id: str | None = None) -> WorkerManagedTransferResult:
        if not isinstance(source, CudaIpcDeviceBuffer):
            raise TypeError("source must be a CudaIpcDeviceBuffer")
        if not isinstance(target, SharedPinnedCpuBuffer):
            raise TypeError("target must be a SharedPinnedCpuBuffer")
        return self._transfer(source, target, "d2h", ranges, chunk_bytes, mode, job_id, user_id)

    # -- flow ------------------------------------------------------------------------------------------
    def _transfer(self, source, target, direction, ranges, chunk_bytes, mode, job_id, user_id):
        job = str(job_id or source.job_id)
        if source.job_id != job or target.job_id != job:
            raise ValueError("source and target buffers must belong to the transfer job")
        sid = self.open_session()
        _require_ok(self.daemon_client.register_job(job_id=job, user_id=user_id, session_id=sid),
                    "daemon job registration failed")
        for reg in (source.buffer_registration(), target.buffer_registration()):
            _register(self.daemon_client, reg)
        req = TransferRequest.from_ranges(_ranges_or_full(ranges, source.size_bytes, target.size_bytes),
                                          chunk_bytes=int(chunk_bytes), direction=direction, mode=mode, job_id=job,
                                          metadata={"buffer_ids": (source.buffer_id, target.buffer_id)})
        planned = _require_ok(self.daemon_client.plan_transfer_request(sid, req, mode=mode),
                              "daemon transfer planning failed")
        p = planned.payload
        tid = str(p["transfer_id"])
        if is_direct_only_plan(p):
            return self._direct(req, p, sid, job, source, target)
        tokens = tuple(dict(t) for t in (p.get("lease_tokens") or ()))
        if not tokens:
            raise RuntimeError("worker-managed transfer requires relay leases")
        try:
            check_plan_matches_leases(p, tokens, direction)
        except Exception:
            _release_leases(self.daemon_client, tokens, "worker_plan_mismatch")
            raise
        primary = tokens[0]
        auth = WorkerTransferAuthorizationRequest(
            transfer_id=tid, lease_id=str(primary["lease_id"]), token=str(primary["token"]), session_id=sid,
            job_id=job, src_buffer_id=source.buffer_id, dst_buffer_id=target.buffer_id, direction=direction,
            ranges=(), relay_gpu=int(primary["relay_gpu"]))
        try:
            env = submit_worker_execution(self.worker_client, auth)
            completion = check_worker_completion(env, auth, expected_bytes=req.total_bytes)
        except _CompletionError:
            _release_leases(self.daemon_client, tokens, "worker_completion_invalid")
            raise
        except Exception:
            _release_leases(self.daemon_client, tokens, "worker_execution_exception")
            raise
        try:
            status = dict(_require_ok(self.daemon_client.transfer_status(tid),
                                      "daemon transfer status query failed").payload["status"])
        except Exception:
            _release_leases(self.daemon_client, tokens, "daemon_status_query_failed")
            raise
        if env.final_state != "complete":
            _release_leases(self.daemon_client, tokens, "worker_completion_not_complete")
            raise RuntimeError(env.error or status.get("error") or "worker-managed transfer did not complete")
        try:
            require_daemon_complete(status, req.total_bytes)
        except Exception:
            _release_leases(self.daemon_client, tokens, "daemon_completion_mismatch")
            raise
        res = (completion.get("worker_result") or {}).get("metadata") or {}
        return WorkerManagedTransferResult(
            transfer_id=tid, session_id=sid, job_id=job, source_buffer_id=source.buffer_id,
            target_buffer_id=target.buffer_id, plan=p, lease_token=primary, lease_tokens=tokens,
            authorization_request=auth, worker_lifecycle=completion, worker_completion=completion,
            final_status=status, path=str(res.get("path", "worker")),
            measured={k: res[k] for k in ("cuda_ms", "gb_per_s", "lanes") if k in res})

    def _direct(self, req: TransferRequest, p: Mapping[str, object], sid: str, job: str, source, target):
        tid = str(p["transfer_id"])
        try:
            ticket = direct_ticket(p, req, tid, job, source.buffer_id, target.buffer_id)
            measured = self._run_direct(req.direction.value, ticket, source, target)
            done = int(measured["bytes"])
            if done != ticket.total_bytes:
                raise RuntimeError(f"direct fallback completed {done} of {ticket.total_bytes} daemon-ticketed bytes")
        except Exception as exc:
            self.daemon_client.transfer_status(tid, state="failed", bytes_completed=0,
                                               error=str(exc) or type(exc).__name__)
            raise
        _require_ok(self.daemon_client.transfer_status(tid, state="complete", bytes_completed=done),
                    "daemon direct transfer completion update failed")
        status = dict(_require_ok(self.daemon_client.transfer_status(tid),
                                  "daemon transfer status query failed").payload["status"])
        require_daemon_complete(status, ticket.total_bytes)
        return WorkerManagedTransferResult(
            transfer_id=tid, session_id=sid, job_id=job, source_buffer_id=source.buffer_id,
            target_buffer_id=target.buffer_id, plan=p, lease_token=None, lease_tokens=(),
            authorization_request=None, worker_lifecycle=None, worker_completion=None, final_status=status,
            path=f"direct_{req.direction.value}", measured=measured)

    def _run_direct(self, direction: str, ticket: ExecutionTicket, source, target) -> dict[str, object]:
        host, dev = (source, target) if direction == "h2d" else (target, source)
        if not isinstance(host, SharedPinnedCpuBuffer) or not isinstance(dev, CudaIpcDeviceBuffer):
            raise TypeError(f"direct {direction} needs a SharedPinnedCpuBuffer and a CudaIpcDeviceBuffer")
        if not dev.device_ptr:
            raise ValueError("direct fallback requires a local CUDA device pointer")
        check_direct_plan(ticket.plan, int(dev.device_index), direction, host.size_bytes, dev.size_bytes)
        from .parallel.engine import D2H, H2D, PoolEngine, lanes_from_plan

        if self.engine is None:
            self.engine = PoolEngine([int(dev.device_index)])
        host.register_for_cuda()
        r = self.engine.run(H2D if direction == "h2d" else D2H, int(dev.device_index), host.address, host.size_bytes,
                            int(dev.device_ptr), dev.size_bytes, lanes_from_plan(dict(ticket.plan),
                                                                                 int(dev.device_index)),
                            checksum=self.checksum)
        r.raise_for_status()
        return {"bytes": r.bytes, "cuda_ms": r.cuda_ms, "gb_per_s": r.gb_per_s}


# ---- helpers ---------------------------------------------------------------------------------------

def _register(daemon_client, reg: BufferRegistration) -> None:
    _require_ok(daemon_client.register_buffer(buffer_id=reg.buffer_id, job_id=reg.job_id, kind=reg.kind,
                                              size_bytes=reg.size_bytes, device_index=reg.device_index,
                                              address=reg.address, pinned=reg.pinned, handle_type=reg.handle_type,
                                              metadata=dict(reg.metadata)),
                "daemon buffer registration failed")


def _ranges_or_full(ranges, src_bytes: int, dst_bytes: int):
    if ranges is not None:
        return list(ranges)
    n = min(int(src_bytes), int(dst_bytes))
    if n <= 0:
        raise ValueError("transfer buffers must be non-empty")
    return [{"src_offset": 0, "dst_offset": 0, "bytes": n}]


def is_direct_only_plan(payload: Mapping[str, object]) -> bool:
    if payload.get("lease_tokens") or payload.get("reservations"):
        return False
    plan = payload.get("plan")
    if not isinstance(plan, Mapping) or not plan.get("assignments"):
        return False
    for a in plan["assignments"]:
        p = a.get("path") if isinstance(a, Mapping) else None
        if not isinstance(p, Mapping) or str(p.get("kind", "")).lower() != "direct":
            return False
    return True


def direct_ticket(p: Mapping[str, object], req: TransferRequest, tid: str, job: str, src_id: str,
                  dst_id: str) -> ExecutionTicket:
    raw = p.get("ticket")
    if not isinstance(raw, Mapping):
        raise RuntimeError("daemon direct transfer did not include execution ticket")
    t = ExecutionTicket(**dict(raw))
    md = t.metadata
    checks = ((md.get("issuer") == TICKET_ISSUER, f"daemon direct ticket was not issued by {TICKET_ISSUER}"),
              (int(md.get("plan_generation", 0)) == int(p.get("plan_generation", 0)),
               "daemon direct ticket plan generation mismatch"),
              (str(md.get("transfer_id")) == tid, "daemon direct ticket transfer mismatch"),
              (t.job_id == job, "daemon direct ticket job mismatch"),
              (t.source_buffer_id == src_id, "daemon direct ticket source buffer mismatch"),
              (t.destination_buffer_id == dst_id, "daemon direct ticket destination buffer mismatch"),
              (t.direction == req.direction.value, "daemon direct ticket direction mismatch"),
              (t.total_bytes == req.total_bytes, "daemon direct ticket byte total mismatch"),
              (_covers(t.ranges, req), "daemon direct ticket ranges mismatch"),
              (dict(t.plan) == dict(p.get("plan") or {}), "daemon direct ticket plan mismatch"),
              (not t.lease_ids, "daemon direct ticket must not include relay leases"))
    for ok, msg in checks:
        if not ok:
            raise RuntimeError(msg)
    return t


def _covers(ticket_ranges, req: TransferRequest) -> bool:
    want = [r.as_dict() for r in req.ranges] if req.ranges else None
    if want is None:
        return True
    for tr in ticket_ranges:
        if not any(w["src_offset"] <= tr["src_offset"] and tr["src_offset"] + tr["bytes"] <= w["src_offset"] + w["bytes"]
                   and tr["dst_offset"] - w["dst_offset"] == tr["src_offset"] - w["src_offset"] for w in want):
            return False
    return True


def check_direct_plan(plan: Mapping[str, object], target: int, direction: str, host_bytes: int,
                      dev_bytes: int) -> None:
    asg = plan.get("assignments") or ()
    if not asg:
        raise RuntimeError("daemon direct plan has no assignments")
    src_size, dst_size = (host_bytes, dev_bytes) if direction == "h2d" else (dev_bytes, host_bytes)
    total = 0
    for a in asg:
        if not isinstance(a, Mapping) or not isinstance(a.get("path"), Mapping):
            raise RuntimeError("daemon direct plan assignment must be a mapping with a path")
        path = a["path"]
        if str(path.get("kind", "")).lower() != "direct":
            raise RuntimeError("daemon direct fallback requires direct paths")
        if str(path.get("direction", "")).lower() != direction:
            raise RuntimeError("daemon direct plan direction does not match request")
        if int(path.get("target_device", target)) != target:
            raise RuntimeError("daemon direct plan target does not match buffer device")
        if not bool(path.get("enabled", True)):
            raise RuntimeError("daemon direct plan path is disabled")
        for s, d, n in assignment_spans(a):
            if n <= 0:
                raise RuntimeError("daemon direct plan chunk bytes must be positive")
            if s < 0 or s + n > src_size:
                raise RuntimeError("daemon direct plan chunk exceeds source buffer")
            if d < 0 or d + n > dst_size:
                raise RuntimeError("daemon direct plan chunk exceeds destination buffer")
            total += n
    if total <= 0:
        raise RuntimeError("daemon direct plan has no chunk assignments")
    if int(plan.get("total_bytes", total)) != total:
        raise RuntimeError("daemon direct plan total bytes do not match chunks")


def check_plan_matches_leases(p: Mapping[str, object], tokens, direction: str) -> None:
    plan = p.get("plan")
    if not isinstance(plan, Mapping):
        raise RuntimeError("daemon response did not include a transfer plan")
    if not tokens:
        raise RuntimeError("worker-managed transfer requires relay leases")
    relays = set()
    for a in plan.get("assignments") or ():
        if not isinstance(a, Mapping) or not isinstance(a.get("path"), Mapping):
            raise RuntimeError("daemon transfer plan assignment must be a mapping with a path")
        path = a["path"]
        if str(path.get("direction", direction)).lower() != direction:
            raise RuntimeError("daemon transfer plan direction does not match request")
        if str(path.get("kind", "")).lower() == "relay" and assignment_has_chunks(a):
            relays.add(int(path.get("relay_device", -1)))
    if not relays:
        raise RuntimeError("daemon relay plan did not include worker chunks")
    if relays != {int(t["relay_gpu"]) for t in tokens}:
        raise RuntimeError("daemon relay leases do not match worker plan")


def _release_leases(daemon_client, tokens, reason: str) -> None:
    """Best-effort cleanup on an error path: a lease that cannot be cleaned
    here expires on the daemon; the failure is logged, not raised, so the
    original error reaches the caller."""
    from .utils.log import logger

    for t in tokens:
        lid = str(t["lease_id"])
        try:
            r = daemon_client.cleanup(target_kind="reservation", target_id=lid, reason=reason, force=True)
            if not getattr(r, "ok", True):
                logger("client").warning("lease_cleanup_refused", lease_id=lid, error=getattr(r, "error", ""))
        except Exception as exc:  # noqa: BLE001 - best effort on an error path
            logger("client").warning("lease_cleanup_failed", lease_id=lid, error=f"{type(exc).__name__}: {exc}")


def submit_worker_execution(worker_client, auth: WorkerTransferAuthorizationRequest) -> WorkerServiceResponseEnvelope:
    env = WorkerServiceRequestEnvelope(payload={"authorization": asdict(auth)})
    for name in ("submit", "handle_envelope"):
        fn = getattr(worker_client, name, None)
        if callable(fn):
            out = fn(env)
            if isinstance(out, Mapping):
                out = WorkerServiceResponseEnvelope(**dict(out))
            if not isinstance(out, WorkerServiceResponseEnvelope):
                raise TypeError("worker client returned an invalid response envelope")
            return out
    raise TypeError("worker_client must submit worker-managed transfers")


def check_worker_completion(env: WorkerServiceResponseEnvelope, auth: WorkerTransferAuthorizationRequest,
                            expected_bytes: int) -> dict[str, object]:
    if not env.ok:
        raise _CompletionError(env.error or "worker service returned an error")
    c = dict(env.completion or {})
    if not c.get("ok"):
        raise _CompletionError("worker completion was not ok")
    if not c.get("transfer_id"):
        raise _CompletionError("worker completion missing transfer id")
    if c["transfer_id"] != auth.transfer_id:
        raise _CompletionError("worker completion transfer mismatch")
    if not c.get("lease_id"):
        raise _CompletionError("worker completion missing lease id")
    if c["lease_id"] != auth.lease_id:
        raise _CompletionError("worker completion lease mismatch")
    if env.final_state != "complete":
        return c
    res = c.get("worker_result")
    if not isinstance(res, Mapping):
        raise _CompletionError("worker completion missing worker result")
    if res.get("state") != "complete":
        raise _CompletionError("worker result did not complete")
    if res.get("transfer_id") != auth.transfer_id:
        raise _CompletionError("worker result transfer mismatch")
    if int(res.get("bytes_completed", -1)) != int(expected_bytes):
        raise _CompletionError(f"worker result completed {res.get('bytes_completed')} of {expected_bytes} bytes")
    upd = c.get("daemon_status_update")
    if not isinstance(upd, Mapping) or upd.get("transfer_id") != auth.transfer_id or upd.get("state") != "complete":
        raise _CompletionError("worker daemon status update does not match the transfer")
    if int(upd.get("bytes_completed", -1)) != int(expected_bytes):
        raise _CompletionError("worker daemon status update byte count mismatch")
    sr = c.get("daemon_status_response")
    if not isinstance(sr, Mapping) or not sr.get("ok"):
        raise _CompletionError("worker daemon status report was not accepted")
    cr = c.get("daemon_cleanup_response")
    if not isinstance(cr, Mapping) or not cr.get("ok"):
        raise _CompletionError("worker lease release was not accepted")
    rel = c.get("staging_release")
    if not isinstance(rel, Mapping) or rel.get("transfer_id") != auth.transfer_id:
        raise _CompletionError("worker staging release does not match the transfer")
    return c


def require_daemon_complete(status: Mapping[str, object], expected_bytes: int) -> None:
    if not isinstance(status, Mapping):
        raise TypeError("final_status must be a mapping")
    s = status.get("state")
    s = str(getattr(s, "value", s))
    if s != "complete":
        raise RuntimeError(f"daemon transfer state is {s}, not complete")
    if int(status.get("bytes_completed", -1)) != int(expected_bytes):
        raise RuntimeError(f"daemon transfer completed {status.get('bytes_completed')} of {expected_bytes} bytes")


def make_worker_managed_transfer_client(*, daemon_socket_path: str, worker_socket_path: str, target_gpu: int,
                                        relay_gpus: Iterable[int], max_inflight_chunks: int = 8,
                                        worker_timeout_seconds: float | None = None,
                                        **kw) -> WorkerManagedTransferClient:
    from .daemon.client import TurboBusDaemonClient
    from .worker.socket_client import WorkerServiceSocketClient

    return WorkerManagedTransferClient(daemon_client=TurboBusDaemonClient(daemon_socket_path),
                                       worker_client=WorkerServiceSocketClient(worker_socket_path,
                                                                               worker_timeout_seconds),
                                       target_gpu=int(target_gpu), relay_gpus=[int(g) for g in relay_gpus],
                                       max_inflight_chunks=int(max_inflight_chunks), **kw)


__all__ = ["WorkerManagedTransferClient", "WorkerManagedTransferResult", "check_worker_completion",
           "is_direct_only_plan", "make_worker_managed_transfer_client", "require_daemon_complete",
           "submit_worker_execution"]
