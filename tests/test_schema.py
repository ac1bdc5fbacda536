"""Contract schema rules, each as a small table of valid and invalid
objects: enums, ranges and totals, the no-physical-path rule for intents,
buffer handle metadata per handle type (shared pinned CPU, CUDA IPC),
decisions, tickets, receipts, statuses, leases, worker handles and the
data-plane request's direction and bounds rules, and ``contract_asdict``.
Behaviours follow unit/test_schema.py and unit/test_contract_schema.py of
the reference with independent cases."""

from __future__ import annotations

import pytest

from pcie_pool_b200.schema import (BufferHandle, BufferKind, BufferRegistration, CleanupRequest, ExecutionTicket,
                                   JobIdentity, LeaseToken, PeerIdentity, RelayQuota, RequestType,
                                   SchedulingDecision, SchedulingDecisionState, TransferIntent, TransferMode,
                                   TransferReceipt, TransferStatus, TransferStatusState, WorkerBufferHandle,
                                   WorkerDataPlaneCompletion, WorkloadKind, check_plan_chunk_bounds,
                                   contract_asdict)

R = ({"src_offset": 0, "dst_offset": 0, "bytes": 16},)
IPC = "ab" * 64


def test_enum_values_match_the_wire():
    assert {m.value for m in TransferMode} == {"auto", "pool", "direct", "relay"}
    assert len(list(RequestType)) == 23
    assert {s.value for s in TransferStatusState} >= {"submitted", "running", "complete", "failed", "canceled"}
    assert {k.value for k in WorkloadKind} == {"generic", "kv_cache", "model_weights", "training_state",
                                              "optimizer_state"}
    assert BufferKind("gpu") is BufferKind.GPU


def intent(**over):
    kw = dict(intent_id="i", job_id="j", session_id="s", source_buffer_id="a", destination_buffer_id="b",
              direction="h2d", total_bytes=16, ranges=R)
    kw.update(over)
    return TransferIntent(**kw)


@pytest.mark.parametrize("over,msg", [
    ({"direction": "sideways"}, "direction"),
    ({"total_bytes": 0}, "positive"),
    ({"total_bytes": 17}, "sum of range bytes"),
    ({"ranges": ()}, "at least one"),
    ({"ranges": ({"src_offset": -1, "dst_offset": 0, "bytes": 16},)}, "non-negative"),
    ({"ranges": ({"src_offset": 0, "dst_offset": 0, "bytes": 0},)}, "positive"),
    ({"destination_buffer_id": "a"}, "different"),
    ({"intent_id": " "}, "intent_id"),
    ({"workload_kind": "video"}, ""),
    ({"policy_hints": {"relay_gpus": [1]}}, "physical"),
    ({"policy_hints": {"Route": "x"}}, "physical"),
])
def test_intent_rejections(over, msg):
    with pytest.raises(ValueError, match=msg):
        intent(**over)


def test_intent_normalises_fields():
    it = intent(direction="H2D", workload_kind="kv_cache", policy_hints={"latency": "low"}, priority="3")
    assert it.direction == "h2d" and it.workload_kind is WorkloadKind.KV_CACHE and it.priority == 3


def test_buffer_handle_metadata_rules():
    shm = {"shared_memory_name": "x", "offset_bytes": 0, "shared_memory_size_bytes": 64}
    ok = BufferHandle("b", "j", "s", "cpu_pinned", 64, pinned=True, handle_type="shared_pinned_cpu", metadata=shm)
    assert ok.kind is BufferKind.CPU_PINNED
    with pytest.raises(ValueError, match="smaller"):
        BufferHandle("b", "j", "s", "cpu_pinned", 65, pinned=True, handle_type="shared_pinned_cpu", metadata=shm)
    with pytest.raises(ValueError, match="pinned"):
        BufferHandle("b", "j", "s", "cpu_pinned", 64, pinned=False, handle_type="shared_pinned_cpu", metadata=shm)
    with pytest.raises(ValueError, match="requires"):
        BufferHandle("b", "j", "s", "cpu_pinned", 64, pinned=True, handle_type="shared_pinned_cpu",
                     metadata={"shared_memory_name": "x"})
    with pytest.raises(ValueError, match="device_index"):
        BufferHandle("b", "j", "s", "gpu", 64)
    g = BufferHandle("b", "j", "s", "gpu", 64, device_index=1, handle_type="cuda_ipc_device",
                     metadata={"cuda_ipc_handle": IPC.upper()})
    assert g.metadata["cuda_ipc_handle"] == IPC, "hex is normalised"
    for bad in ("zz" * 64, "ab" * 63, 12):
        with pytest.raises(ValueError, match="cuda_ipc_handle"):
            BufferHandle("b", "j", "s", "gpu", 64, device_index=1, handle_type="cuda_ipc_device",
                         metadata={"cuda_ipc_handle": bad})
    with pytest.raises(ValueError, match="cuda_ipc_offset"):
        BufferRegistration("b", "j", "gpu", 64, device_index=0, handle_type="cuda_ipc_device",
                           metadata={"cuda_ipc_handle": IPC, "cuda_ipc_offset": -4})
    with pytest.raises(ValueError, match="gpu buffers"):
        BufferRegistration("b", "j", "cpu_pinned", 64, device_index=0, pinned=True, handle_type="cuda_ipc_device",
                           metadata={"cuda_ipc_handle": IPC})


def test_identities():
    with pytest.raises(ValueError, match="user_id"):
        PeerIdentity(authenticated=True, source="so_peercred")
    assert PeerIdentity(authenticated=False, source="none").user_id is None
    with pytest.raises(ValueError, match="weight"):
        JobIdentity("j", weight=0)
    with pytest.raises(ValueError):
        JobIdentity("")


def test_scheduling_decision_states():
    base = dict(decision_id="d", intent_id="i", topology_snapshot_id="t", job_id="j", session_id="s")
    assert SchedulingDecision(**base, state="planned", plan={"assignments": []}).state is \
        SchedulingDecisionState.PLANNED
    with pytest.raises(ValueError, match="require a plan"):
        SchedulingDecision(**base, state="planned")
    with pytest.raises(ValueError, match="fallback_reason"):
        SchedulingDecision(**base, state="fallback", plan={"a": 1})
    with pytest.raises(ValueError, match="must not include a plan"):
        SchedulingDecision(**base, state="rejected", plan={"a": 1}, rejection_reason="no")
    with pytest.raises(ValueError, match="rejection_reason"):
        SchedulingDecision(**base, state="rejected")


def ticket(**over):
    kw = dict(ticket_id="t", decision_id="d", intent_id="i", topology_snapshot_id="s", job_id="j", session_id="x",
              source_buffer_id="a", destination_buffer_id="b", direction="d2h", total_bytes=16, ranges=R,
              plan={"assignments": []}, issued_at=1.0, expires_at=2.0)
    kw.update(over)
    return ExecutionTicket(**kw)


@pytest.mark.parametrize("over,msg", [({"expires_at": 1.0}, "later"), ({"plan": {}}, "plan"),
                                      ({"total_bytes": 8}, "sum"), ({"destination_buffer_id": "a"}, "different"),
                                      ({"lease_ids": ("",)}, "")])
def test_ticket_rejections(over, msg):
    with pytest.raises(ValueError, match=msg):
        ticket(**over)


def receipt(**over):
    kw = dict(receipt_id="r", ticket_id="t", intent_id="i", decision_id="d", topology_snapshot_id="s", job_id="j",
              session_id="x", state="complete", bytes_total=16, bytes_completed=16)
    kw.update(over)
    return TransferReceipt(**kw)


def test_receipt_rules():
    assert receipt().state is TransferStatusState.COMPLETE
    with pytest.raises(ValueError, match="all bytes"):
        receipt(bytes_completed=8)
    with pytest.raises(ValueError, match="cannot include error"):
        receipt(error="x")
    with pytest.raises(ValueError, match="requires error"):
        receipt(state="failed", bytes_completed=0)
    with pytest.raises(ValueError, match="exceed"):
        receipt(state="running", bytes_completed=17)
    with pytest.raises(ValueError, match="earlier"):
        receipt(started_at=5.0, completed_at=4.0)


def test_status_and_lease_rules():
    with pytest.raises(ValueError, match="bytes_total completed"):
        TransferStatus("t", "j", "complete", 10, 9)
    with pytest.raises(ValueError, match="exceed"):
        TransferStatus("t", "j", "running", 10, 11)
    assert TransferStatus("t", "j", "running", 10, 3).state is TransferStatusState.RUNNING
    with pytest.raises(ValueError, match="earlier"):
        LeaseToken("l", "s", 1, "tok", issued_at=5.0, expires_at=4.0)
    assert LeaseToken("l", "s", 1, "tok", issued_at=5.0).expires_at == 0.0, "0 = no expiry"


def test_relay_quota_accounting():
    q = RelayQuota(relay_gpu=1, max_sessions=1, max_inflight_chunks=4)
    assert q.can_attach() and q.can_reserve(4) and not q.can_reserve(5)
    q.sessions.add("s")
    assert not q.can_attach()
    q.active_chunks = 3
    assert q.can_reserve(1) and not q.can_reserve(2)


def test_worker_handle_access_and_completion_rules():
    reg = BufferRegistration("b", "j", "gpu", 64, device_index=0, handle_type="cuda_ipc_device",
                             metadata={"cuda_ipc_handle": IPC})
    h = WorkerBufferHandle.from_buffer_registration(reg, "write")
    assert h.access == "write" and h.device_index == 0
    with pytest.raises(ValueError, match="access"):
        WorkerBufferHandle.from_buffer_registration(reg, "execute")
    with pytest.raises(ValueError, match="requires error"):
        WorkerDataPlaneCompletion(transfer_id="t", lease_id="l", state="failed", bytes_completed=0)
    with pytest.raises(ValueError, match="complete or failed"):
        WorkerDataPlaneCompletion(transfer_id="t", lease_id="l", state="running", bytes_completed=0)


def test_plan_chunk_bounds():
    plan = {"assignments": [{"chunks": [{"src_offset": 0, "dst_offset": 8, "bytes": 8}]}]}
    check_plan_chunk_bounds(plan, 16, 16)
    with pytest.raises(ValueError, match="dst buffer"):
        check_plan_chunk_bounds(plan, 16, 15)
    with pytest.raises(ValueError, match="src buffer"):
        check_plan_chunk_bounds({"assignments": [{"chunks": [{"src_offset": 10, "dst_offset": 0, "bytes": 8}]}]},
                                16, 16)
    with pytest.raises(ValueError, match="positive"):
        check_plan_chunk_bounds({"assignments": [{"chunks": [{"src_offset": 0, "dst_offset": 0, "bytes": 0}]}]},
                                16, 16)


def test_cleanup_request_and_asdict_roundtrip():
    c = CleanupRequest(target_kind="reservation", target_id="r", reason="x")
    assert contract_asdict(c)["target_kind"] == "reservation"
    it = intent(policy_hints={"latency": "low"})
    d = contract_asdict(it)
    assert d["ranges"][0]["bytes"] == 16 and TransferIntent(**d) == it
    t = ticket()
    assert ExecutionTicket(**contract_asdict(t)) == t
