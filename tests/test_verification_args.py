"""The verification harness without GPUs: argument checks that run before
any CUDA work, the no-CUDA error, the seeded verification daemon (its
relay, profile and a relay plan through it), the byte pattern and plan
splits.  Behaviours follow e2e/test_verification.py of the reference with
independent cases."""

from __future__ import annotations

import pytest

from pcie_pool_b200 import verification as V

MiB = 1 << 20


@pytest.mark.parametrize("kw,msg", [
    ({"direction": "sideways"}, "direction"),
    ({"mode": "teleport"}, "mode"),
    ({"bytes_to_copy": 0}, "positive"),
    ({"chunk_bytes": 0}, "positive"),
    ({"mode": "pool", "bytes_to_copy": MiB, "chunk_bytes": MiB}, "two chunks"),
    ({"src_offset": 4, "source_buffer_bytes": MiB}, "exceeds"),
    ({"dst_offset": 8, "destination_buffer_bytes": MiB}, "exceeds"),
])
def test_arguments_are_checked_before_any_cuda_work(kw, msg):
    direction = kw.pop("direction", "h2d")
    with pytest.raises(ValueError, match=msg):
        V.verify(direction, **kw)


def test_without_cuda_the_harness_says_so():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    with pytest.raises(RuntimeError, match="CUDA is not available"):
        V.verify("h2d", mode="relay")


def test_pattern_is_deterministic_and_wraps():
    p = V.make_pattern(1000)
    assert len(p) == 1000 and p == V.make_pattern(1000)
    assert all(p[i] == (i * 131 + 17) & 0xFF for i in range(1000))
    assert len(set(p[:256])) == 256, "every byte value appears once per 256-byte period"


def test_seeded_daemon_plans_through_its_relay():
    d = V.build_verification_daemon(0, 2, 8, 4 * MiB)
    assert d.relay_gpus == (2,)
    assert d.get_profile(0, [2]).payload["profile"] is not None
    s = d.register_session(0, [2], max_inflight_chunks=8)
    assert s.ok, s.error
    sid = s.payload["session"]["session_id"]
    assert d.register_job("j", session_id=sid).ok
    assert d.register_buffer("a", "j", "cpu_pinned", 4 * MiB, address=4096, pinned=True).ok
    assert d.register_buffer("b", "j", "gpu", 4 * MiB, device_index=0, address=8192).ok
    r = d.plan_transfer(sid, 4 * MiB, MiB, mode="relay", job_id="j", buffer_ids=["a", "b"])
    assert r.ok, r.error
    assert [t["relay_gpu"] for t in r.payload["lease_tokens"]] == [2]
    relay_b, relay_c = V._plan_split(r.payload["plan"], "relay")
    direct_b, _ = V._plan_split(r.payload["plan"], "direct")
    assert relay_b == 4 * MiB and relay_c == 4 and direct_b == 0


def test_cli_parses_and_forwards(monkeypatch, capsys):
    seen = {}

    class R:
        def as_dict(self):
            return {"ok": True}

    def fake_verify(direction, **kw):
        seen.update(kw, direction=direction)
        return R()

    monkeypatch.setattr(V, "verify", fake_verify)
    assert V.main(["--direction", "d2h", "--mode", "pool", "--bytes", "8", "--chunk-bytes", "2",
                   "--max-inflight-chunks", "4"]) == 0
    assert seen["direction"] == "d2h" and seen["mode"] == "pool" and seen["bytes_to_copy"] == 8
    assert seen["max_inflight_chunks"] == 4 and '"ok": true' in capsys.readouterr().out
