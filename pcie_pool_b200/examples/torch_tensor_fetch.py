"""Submit one generic transfer intent through the public client and print
its receipt line (``daemon_receipt ...``):

    python -m pcie_pool_b200.examples.torch_tensor_fetch --daemon-socket-path S \\
        --session-id SID --source-buffer-id HOST --destination-buffer-id GPU --bytes N

``--self-contained`` instead starts an in-process daemon over this GPU's
engine, registers a pinned torch CPU tensor and a CUDA tensor, fetches one
into the other and checks the bytes (the same call path a user makes)."""

from __future__ import annotations

import argparse

from .. import TransferIntent, TurboBusClient, WorkloadKind
from ..benchmarks.daemon_support import receipt_trace_line


def build_intent(args) -> TransferIntent:
    return TransferIntent(intent_id=args.intent_id, job_id=args.job_id, session_id=args.session_id,
                          source_buffer_id=args.source_buffer_id, destination_buffer_id=args.destination_buffer_id,
                          direction=args.direction, total_bytes=args.bytes,
                          ranges=({"src_offset": args.src_offset, "dst_offset": args.dst_offset, "bytes": args.bytes},),
                          workload_kind=WorkloadKind.GENERIC,
                          metadata={"example": "torch-tensor-fetch", "policy": args.policy})


def self_contained(nbytes: int) -> str:
    import torch

    from ..e2e import build_inprocess_node
    from ..parallel.engine import PoolEngine

    n = torch.cuda.device_count()
    eng = PoolEngine(list(range(n)))
    _d, dc = build_inprocess_node(eng, list(range(n)), 0)
    sid = dc.register_session(0, list(range(1, n)), max_inflight_chunks=4096).payload["session"]["session_id"]
    dc.register_job("fetch", session_id=sid)
    src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8).pin_memory()
    dst = torch.zeros(nbytes, dtype=torch.uint8, device="cuda:0")
    dc.register_buffer("cpu", "fetch", "cpu_pinned", nbytes, address=src.data_ptr(), pinned=True)
    dc.register_buffer("gpu", "fetch", "gpu", nbytes, device_index=0, address=dst.data_ptr())
    it = TransferIntent("fetch-0", "fetch", sid, "cpu", "gpu", "h2d", nbytes,
                        ({"src_offset": 0, "dst_offset": 0, "bytes": nbytes},))
    r = TurboBusClient(daemon=dc).transfer(it, timeout_seconds=120)
    ok = bool(torch.equal(dst.cpu(), src))
    return receipt_line(r) + f" bytes_match={ok}"


def receipt_line(receipt) -> str:
    """The receipt's trace line: intent, decision, topology snapshot and
    ticket ids, state, and the direct / relay byte and chunk split."""
    return receipt_trace_line(receipt)


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--self-contained", action="store_true")
    p.add_argument("--daemon-socket-path")
    p.add_argument("--session-id")
    p.add_argument("--job-id", default="example-torch-tensor-fetch")
    p.add_argument("--intent-id", default="example-torch-tensor-fetch-0")
    p.add_argument("--source-buffer-id")
    p.add_argument("--destination-buffer-id")
    p.add_argument("--direction", choices=["h2d", "d2h"], default="h2d")
    p.add_argument("--bytes", type=int, default=64 << 20)
    p.add_argument("--src-offset", type=int, default=0)
    p.add_argument("--dst-offset", type=int, default=0)
    p.add_argument("--policy", default="daemon-default")
    p.add_argument("--wait-timeout-seconds", type=float, default=120.0)
    return p


def main(argv=None) -> int:
    p = build_parser()
    a = p.parse_args(argv)
    if a.self_contained:
        print(self_contained(a.bytes))
        return 0
    for req in ("daemon_socket_path", "session_id", "source_buffer_id", "destination_buffer_id"):
        if not getattr(a, req):
            p.error(f"--{req.replace('_', '-')} is required without --self-contained")
    client = TurboBusClient(socket_path=a.daemon_socket_path)
    intent = build_intent(a)
    client.submit_transfer_intent(intent)
    print(receipt_line(client.wait_transfer_receipt(intent.intent_id, timeout_seconds=a.wait_timeout_seconds)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
