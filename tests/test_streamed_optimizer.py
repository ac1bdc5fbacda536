"""Streamed AdamW through the daemon on the CPU (mock data plane): the fp32
state lives in host memory in 24 KiB tiles, each step is one adamw landing
intent, and master weights, moments and the bf16 parameter copy follow
torch.optim.AdamW in fp32.  The GPU version (engine and daemon) is in
tests/test_gpu_streamed_optimizer.py."""

import pytest
import torch

from pcie_pool_b200 import TransferIntent, TurboBusClient
from pcie_pool_b200.adapters.streamed_optimizer import TILE_BYTES, TILE_PARAMS, StreamedAdamW
from pcie_pool_b200.daemon import InProcessDaemonClient, IntentExecutor, TurboBusDaemon
from pcie_pool_b200.mock import MockDataPlane, MockWorld
from pcie_pool_b200.topology import StaticTopologyProvider


def node():
    world = MockWorld(gpu_count=4)
    daemon = TurboBusDaemon(relay_gpus=range(1, 4), max_inflight_chunks_per_relay=4096,
                            topology_provider=StaticTopologyProvider(gpu_count=4),
                            executor=IntentExecutor(MockDataPlane(world, checksum=False)))
    daemon.put_profile(0, [1, 2, 3], world.profile(0))
    dc = InProcessDaemonClient(daemon)
    sid = dc.register_session(0, [1, 2, 3], max_inflight_chunks=1 << 16).payload["session"]["session_id"]
    assert dc.register_job("train", session_id=sid).ok
    return dc, sid


def torch_reference(p0, grads, **kw):
    p = torch.nn.Parameter(p0.float().clone())
    opt = torch.optim.AdamW([p], **kw)
    for g in grads:
        p.grad = g.float()
        opt.step()
    st = opt.state[p]
    return p.detach(), st["exp_avg"], st["exp_avg_sq"]


@pytest.mark.parametrize("nparams", [3 * TILE_PARAMS, 5 * TILE_PARAMS + 123])
def test_streamed_adamw_through_daemon_matches_torch(nparams):
    dc, sid = node()
    g = torch.Generator().manual_seed(1)
    params = (torch.randn(nparams, generator=g) * 0.1).to(torch.bfloat16)
    p0 = params.clone()
    grads_buf = torch.zeros(nparams, dtype=torch.bfloat16)
    kw = dict(lr=1e-2, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.05)
    opt = StreamedAdamW(params, client=TurboBusClient(daemon=dc), daemon_client=dc, session_id=sid, job_id="train",
                        chunk_bytes=TILE_BYTES, **kw)
    steps = [(torch.randn(nparams, generator=g) * 0.01).to(torch.bfloat16) for _ in range(3)]
    for gr in steps:
        grads_buf.copy_(gr)
        st = opt.step(grads_buf)
        assert st.bytes == opt.tiles * TILE_BYTES
    want_p, want_m, want_v = torch_reference(p0, steps, **kw)
    s = opt.state()
    torch.testing.assert_close(s["master"], want_p, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(s["exp_avg"], want_m, rtol=1e-5, atol=1e-9)
    torch.testing.assert_close(s["exp_avg_sq"], want_v, rtol=1e-5, atol=1e-12)
    assert torch.equal(params, s["master"].to(torch.bfloat16))
    d = dc.describe().payload
    assert not d.get("reservations")
    used = {int(p.get("relay_device", -1)) for m in d["measured_transfers"].values() for p in m.get("path_stats", ())}
    assert used - {-1}, "the optimizer steps should use relay lanes"


def test_adamw_spec_rejections():
    dc, sid = node()
    n = 2 * TILE_PARAMS
    host = torch.zeros(2 * TILE_BYTES, dtype=torch.uint8)
    params = torch.zeros(n, dtype=torch.bfloat16)
    grads = torch.zeros(n, dtype=torch.bfloat16)
    assert dc.register_buffer("st", "train", "cpu_pinned", host.numel(), address=host.data_ptr(), pinned=True).ok
    assert dc.register_buffer("p", "train", "gpu", 2 * n, device_index=0, address=params.data_ptr()).ok
    assert dc.register_buffer("g", "train", "gpu", n, device_index=0, address=grads.data_ptr()).ok  # too small

    def submit(adam, chunk=TILE_BYTES, direction="h2d"):
        src, dst = ("st", "p") if direction == "h2d" else ("p", "st")
        it = TransferIntent(f"x-{len(str(adam))}-{chunk}-{direction}", "train", sid, src, dst, direction, host.numel(),
                            ({"src_offset": 0, "dst_offset": 0, "bytes": host.numel()},),
                            metadata={"chunk_bytes": chunk, "landing": {"op": "adamw", "adam": adam}})
        return dc.submit_transfer_intent(it)

    r = submit({"grads_buffer": "g", "nparams": n})
    assert not r.ok and "nparams bf16" in r.error
    assert dc.register_buffer("g2", "train", "gpu", 2 * n, device_index=0, address=grads.data_ptr()).ok
    r = submit({"grads_buffer": "g2", "nparams": n}, chunk=TILE_BYTES + 16)
    assert not r.ok and "state tiles" in r.error
    r = submit({"grads_buffer": "g2", "nparams": n}, direction="d2h")
    assert not r.ok and "round trip" in r.error
    r = submit({"grads_buffer": "nope", "nparams": n})
    assert not r.ok and "not registered" in r.error
