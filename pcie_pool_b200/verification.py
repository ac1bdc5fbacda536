"""Live verification of the worker-managed path on real GPUs.

``python -m pcie_pool_b200.verification --direction h2d --mode relay
--target-gpu 0 --relay-gpu 1 --bytes N --chunk-bytes C`` starts a daemon
process (static verification topology, seeded profile) and, unless the
mode is ``direct``, a worker helper process; it then moves the byte pattern
``(i*131 + 17) & 0xFF`` from shared pinned host memory into a CUDA IPC
tensor (or back) through the daemon-approved plan and checks the bytes, the
direct/relay split the worker reports against the plan, and that every
reservation and relay quota was released (turbobus/verification.py:74-424,
:485-595).  Prints one JSON result line.
"""

from __future__ import annotations

from .planner_types import assignment_bytes, assignment_chunk_count

import argparse
import json
import multiprocessing
import os
import tempfile
import time
from dataclasses import asdict, dataclass
from collections.abc import Mapping
from typing import Sequence

PATTERN_MUL, PATTERN_ADD = 131, 17


@dataclass(frozen=True)
class WorkerManagedRelayVerificationResult:
    direction: str
    transfer_mode: str
    transfer_id: str
    job_id: str
    bytes_requested: int
    bytes_completed: int
    src_offset: int
    dst_offset: int
    source_buffer_bytes: int
    destination_buffer_bytes: int
    target_gpu: int
    relay_gpu: int
    state: str
    worker_final_state: str | None
    worker_path: str
    worker_direct_bytes: int
    worker_direct_chunks: int
    worker_relay_bytes: int
    worker_relay_chunks: int
    daemon_reservations_released: bool
    daemon_relay_active_chunks: int
    gb_per_s: float = 0.0          # end to end: daemon RPCs, worker start-up and binding included
    data_plane_gb_per_s: float = 0.0  # device-timed engine transfer as reported by the executor

    def as_dict(self) -> dict[str, object]:
        return asdict(self)


class WorkerManagedH2DRelayVerificationResult(WorkerManagedRelayVerificationResult):
    pass


class WorkerManagedD2HRelayVerificationResult(WorkerManagedRelayVerificationResult):
    pass


def make_pattern(n: int) -> bytes:
    import numpy as np

    i = np.arange(int(n), dtype=np.uint64)
    return ((i * PATTERN_MUL + PATTERN_ADD) & 0xFF).astype(np.uint8).tobytes()


def build_verification_daemon(target_gpu: int, relay_gpu: int, max_inflight_chunks: int, profile_bytes: int):
    from .daemon.server import TurboBusDaemon
    from .topology import (DaemonResourceInventory, FabricLinkRecord, GpuInventoryRecord, PciePathRecord,
                           StaticTopologyProvider)

    t, r = int(target_gpu), int(relay_gpu)
    inv = DaemonResourceInventory(
        gpus=(GpuInventoryRecord(t, backend="cuda", vendor="nvidia", role="target"),
              GpuInventoryRecord(r, backend="cuda", vendor="nvidia", role="relay")),
        pcie_paths=(PciePathRecord(t, bandwidth_gbps=55.0), PciePathRecord(r, bandwidth_gbps=55.0)),
        fabric_links=(FabricLinkRecord(r, t, fabric="nvswitch", bandwidth_gbps=770.0, enabled=True),),
        source="verification_static")
    daemon = TurboBusDaemon(relay_gpus=[r], max_sessions_per_relay=1,
                            max_inflight_chunks_per_relay=int(max_inflight_chunks),
                            topology_provider=StaticTopologyProvider(inventory=inv))
    resp = daemon.put_profile(target_gpu=t, relay_gpus=[r], profile={
        "target_device": t, "direct_h2d_bw_gbps": 1.0, "direct_d2h_bw_gbps": 1.0,
        "relays": [{"relay_device": r, "target_device": t, "h2d_bw_gbps": 16.0, "d2h_bw_gbps": 16.0,
                    "p2p_bw_gbps": 40.0, "effective_bw_gbps": 16.0, "effective_d2h_bw_gbps": 16.0,
                    "p2p_enabled": True}]}, profile_bytes=int(profile_bytes))
    if not resp.ok:
        raise RuntimeError(resp.error or "failed to seed daemon profile")
    return daemon


def _serve_daemon(socket_path: str, target: int, relay: int, inflight: int, profile_bytes: int) -> None:
    from .daemon.wire import serve_unix

    serve_unix(build_verification_daemon(target, relay, inflight, profile_bytes), socket_path)


def _serve_worker(daemon_socket: str, worker_socket: str) -> None:
    from .worker.process import run_worker_helper_process

    run_worker_helper_process(daemon_socket, worker_socket)


def _wait_for_socket(path: str, proc, timeout: float) -> None:
    end = time.monotonic() + timeout
    while time.monotonic() < end:
        if os.path.exists(path):
            return
        if proc is not None and not proc.is_alive():
            raise RuntimeError(f"process serving {path} exited with {proc.exitcode}")
        time.sleep(0.02)
    raise TimeoutError(f"socket {path} did not appear within {timeout} s")


def _stop(proc) -> None:
    if proc is None or not proc.is_alive():
        return
    proc.terminate()
    proc.join(5)
    if proc.is_alive():
        proc.kill()
        proc.join(5)


def _plan_split(plan: Mapping[str, object], kind: str) -> tuple[int, int]:
    b = c = 0
    for a in (plan.get("assignments") or ()):
        if str(a.get("path", {}).get("kind", "")).lower() == kind:
            b += assignment_bytes(a)
            c += assignment_chunk_count(a)
    return b, c


class _NoWorker:
    def submit(self, envelope):
        raise RuntimeError("direct mode must not reach the worker helper")


def verify(direction: str = "h2d", *, target_gpu: int = 0, relay_gpu: int = 1, bytes_to_copy: int = 1 << 20,
           chunk_bytes: int = 1 << 20, mode: str = "relay", src_offset: int = 0, dst_offset: int = 0,
           source_buffer_bytes: int | None = None, destination_buffer_bytes: int | None = None,
           max_inflight_chunks: int = 8, socket_dir: str | None = None,
           startup_timeout_seconds: float = 30.0) -> WorkerManagedRelayVerificationResult:
    direction, mode = str(direction).lower(), str(mode).lower()
    if direction not in ("h2d", "d2h"):
        raise ValueError("direction must be h2d or d2h")
    if mode not in ("direct", "relay", "pool"):
        raise ValueError("mode must be direct, relay, or pool")
    n, chunk = int(bytes_to_copy), int(chunk_bytes)
    if n <= 0 or chunk <= 0:
        raise ValueError("bytes_to_copy and chunk_bytes must be positive")
    if mode == "pool" and n <= chunk:
        raise ValueError("pool verification requires at least two chunks")
    src_size = int(source_buffer_bytes or src_offset + n)
    dst_size = int(destination_buffer_bytes or dst_offset + n)
    if src_offset + n > src_size or dst_offset + n > dst_size:
        raise ValueError("transfer range exceeds a verification buffer")
    import numpy as np
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available")
    need = max(int(target_gpu), int(relay_gpu) if mode != "direct" else 0) + 1
    if torch.cuda.device_count() < need:
        raise RuntimeError(f"CUDA verification needs at least {need} visible devices")
    from .backends.cuda import default_cuda_backend
    from .client import CudaIpcDeviceBuffer, SharedPinnedCpuBufferAllocator
    from .client_transfer import make_worker_managed_transfer_client

    pattern = np.frombuffer(make_pattern(n), dtype=np.uint8)
    job = f"verify-{direction}-{mode}-{os.getpid()}-{time.time_ns()}"
    alloc = SharedPinnedCpuBufferAllocator(name_prefix=f"ppb-verify-{direction}")
    ctx = multiprocessing.get_context("spawn")
    with tempfile.TemporaryDirectory(dir=socket_dir) as tmp:
        dsock, wsock = os.path.join(tmp, "daemon.sock"), os.path.join(tmp, "worker.sock")
        dproc = ctx.Process(target=_serve_daemon, args=(dsock, int(target_gpu), int(relay_gpu),
                                                         int(max_inflight_chunks), n), daemon=True)
        wproc = None if mode == "direct" else ctx.Process(target=_serve_worker, args=(dsock, wsock), daemon=True)
        cpu = None
        try:
            dproc.start()
            _wait_for_socket(dsock, dproc, startup_timeout_seconds)
            if wproc is not None:
                wproc.start()
                _wait_for_socket(wsock, wproc, startup_timeout_seconds)
            client = make_worker_managed_transfer_client(
                daemon_socket_path=dsock, worker_socket_path=wsock, target_gpu=int(target_gpu),
                relay_gpus=[int(relay_gpu)], max_inflight_chunks=int(max_inflight_chunks))
            if wproc is None:
                client.worker_client = _NoWorker()
            torch.cuda.set_device(int(target_gpu))
            rng = [{"src_offset": int(src_offset), "dst_offset": int(dst_offset), "bytes": n}]
            t0 = time.perf_counter()
            if direction == "h2d":
                cpu = alloc.allocate("verify-cpu-source", job, src_size)
                cpu.numpy()[:] = 0
                cpu.numpy()[src_offset:src_offset + n] = pattern
                dev_t = torch.zeros(dst_size, dtype=torch.uint8, device=f"cuda:{target_gpu}")
                torch.cuda.synchronize()
                gpu = CudaIpcDeviceBuffer.from_tensor("verify-gpu-target", job, dev_t, backend=default_cuda_backend)
                res = client.fetch_shared_cpu_to_cuda_ipc(cpu, gpu, ranges=rng, chunk_bytes=chunk, mode=mode, job_id=job)
                torch.cuda.synchronize()
                got = dev_t.cpu().numpy()
                want = np.zeros(dst_size, dtype=np.uint8)
                want[dst_offset:dst_offset + n] = pattern
            else:
                dev_t = torch.zeros(src_size, dtype=torch.uint8, device=f"cuda:{target_gpu}")
                dev_t[src_offset:src_offset + n] = torch.from_numpy(pattern.copy()).to(dev_t.device)
                torch.cuda.synchronize()
                gpu = CudaIpcDeviceBuffer.from_tensor("verify-gpu-source", job, dev_t, backend=default_cuda_backend)
                cpu = alloc.allocate("verify-cpu-destination", job, dst_size)
                cpu.numpy()[:] = 0
                res = client.offload_cuda_ipc_to_shared_cpu(gpu, cpu, ranges=rng, chunk_bytes=chunk, mode=mode,
                                                            job_id=job)
                got = cpu.numpy().copy()
                want = np.zeros(dst_size, dtype=np.uint8)
                want[dst_offset:dst_offset + n] = pattern
            secs = time.perf_counter() - t0
            if res.state != "complete" or res.bytes_completed != n:
                raise RuntimeError(f"daemon status {res.state} with {res.bytes_completed} of {n} bytes: "
                                   f"{getattr(res, 'final_status', '')}")
            if not np.array_equal(got, want):
                bad = int(np.flatnonzero(got != want)[0])
                raise RuntimeError(f"verification bytes differ first at offset {bad} "
                                   f"({int((got != want).sum())} bytes differ, {int((got == 0).sum())} zero; "
                                   f"got {got[bad:bad + 8].tolist()} want {want[bad:bad + 8].tolist()}; "
                                   f"status {res.state}, path {getattr(res, 'path', None)}, "
                                   f"measured {getattr(res, 'measured', None)})")
            d_b, d_c = _plan_split(res.plan["plan"], "direct")
            r_b, r_c = _plan_split(res.plan["plan"], "relay")
            wres = ((res.worker_completion or {}).get("worker_result") or {}).get("metadata") or {}
            if res.worker_completion is not None:
                reported = (int(wres.get("direct_bytes", -1)), int(wres.get("relay_bytes", -1)))
                if reported != (d_b, r_b):
                    raise RuntimeError(f"worker path split {reported} does not match the plan {(d_b, r_b)}")
            from .daemon.client import TurboBusDaemonClient

            desc = TurboBusDaemonClient(dsock).describe().payload
            quotas = desc.get("relay_quotas", {})
            q = quotas.get(str(relay_gpu), quotas.get(int(relay_gpu), {})) or {}
            released = not desc.get("reservations")
            active = int(q.get("active_chunks", 0))
            if not released or active:
                raise RuntimeError("daemon kept reservations or relay quota after the transfer")
            cls = WorkerManagedH2DRelayVerificationResult if direction == "h2d" else WorkerManagedD2HRelayVerificationResult
            return cls(direction=direction, transfer_mode=mode, transfer_id=res.transfer_id, job_id=job,
                       bytes_requested=n, bytes_completed=res.bytes_completed, src_offset=int(src_offset),
                       dst_offset=int(dst_offset), source_buffer_bytes=src_size, destination_buffer_bytes=dst_size,
                       target_gpu=int(target_gpu), relay_gpu=int(relay_gpu), state=res.state,
                       worker_final_state=None if res.worker_completion is None else
                       res.worker_completion.get("final_state"),
                       worker_path=res.path, worker_direct_bytes=d_b, worker_direct_chunks=d_c,
                       worker_relay_bytes=r_b, worker_relay_chunks=r_c, daemon_reservations_released=released,
                       daemon_relay_active_chunks=active, gb_per_s=round(n / secs / 1e9, 3),
                       data_plane_gb_per_s=round(float(wres.get("gb_per_s") or res.measured.get("gb_per_s") or 0.0),
                                                 3))
        finally:
            if cpu is not None:
                cpu.release()
            _stop(wproc)
            _stop(dproc)


def verify_worker_managed_h2d_relay(**kw) -> WorkerManagedRelayVerificationResult:
    return verify("h2d", **kw)


def verify_worker_managed_d2h_relay(**kw) -> WorkerManagedRelayVerificationResult:
    return verify("d2h", **kw)


def main(argv: Sequence[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Verify the worker-managed pooled path on real GPUs")
    ap.add_argument("--direction", choices=["h2d", "d2h"], default="h2d")
    ap.add_argument("--mode", choices=["direct", "relay", "pool"], default="relay")
    ap.add_argument("--target-gpu", type=int, default=0)
    ap.add_argument("--relay-gpu", type=int, default=1)
    ap.add_argument("--bytes", type=int, default=1 << 20)
    ap.add_argument("--chunk-bytes", type=int, default=1 << 20)
    ap.add_argument("--src-offset", type=int, default=0)
    ap.add_argument("--dst-offset", type=int, default=0)
    ap.add_argument("--source-buffer-bytes", type=int, default=None)
    ap.add_argument("--destination-buffer-bytes", type=int, default=None)
    ap.add_argument("--max-inflight-chunks", type=int, default=8)
    ap.add_argument("--socket-dir", default=None)
    ap.add_argument("--startup-timeout-seconds", type=float, default=30.0)
    a = ap.parse_args(argv)
    r = verify(a.direction, target_gpu=a.target_gpu, relay_gpu=a.relay_gpu, bytes_to_copy=a.bytes,
               chunk_bytes=a.chunk_bytes, mode=a.mode, src_offset=a.src_offset, dst_offset=a.dst_offset,
               source_buffer_bytes=a.source_buffer_bytes, destination_buffer_bytes=a.destination_buffer_bytes,
               max_inflight_chunks=a.max_inflight_chunks, socket_dir=a.socket_dir,
               startup_timeout_seconds=a.startup_timeout_seconds)
    print(json.dumps(r.as_dict(), sort_keys=True))
    return 0


__all__ = ["WorkerManagedD2HRelayVerificationResult", "WorkerManagedH2DRelayVerificationResult",
           "WorkerManagedRelayVerificationResult", "build_verification_daemon", "main", "make_pattern", "verify",
           "verify_worker_managed_d2h_relay", "verify_worker_managed_h2d_relay"]


if __name__ == "__main__":
    raise SystemExit(main())

