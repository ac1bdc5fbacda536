"""Streamed AdamW on real GPUs: the landing kernel's fused optimizer op
(PoolEngine OP_ADAMW) over the direct lane and up to three relay lanes, and
the same step as a daemon intent.  Master weights, moments and the bf16
parameters follow torch.optim.AdamW in fp32 (CPU) after several steps; a
partial last tile keeps its padding untouched."""

import pytest
import torch

from pcie_pool_b200 import TurboBusClient
from pcie_pool_b200.adapters.streamed_optimizer import TILE_PARAMS, StreamedAdamW

pytestmark = pytest.mark.gpu


def torch_reference(p0, grads, **kw):
    p = torch.nn.Parameter(p0.float().cpu().clone())
    opt = torch.optim.AdamW([p], **kw)
    for g in grads:
        p.grad = g.float().cpu()
        opt.step()
    st = opt.state[p]
    return p.detach(), st["exp_avg"], st["exp_avg_sq"]


def _check(opt, params, p0, steps, kw):
    want_p, want_m, want_v = torch_reference(p0, steps, **kw)
    s = opt.state()
    torch.testing.assert_close(s["master"], want_p, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(s["exp_avg"], want_m, rtol=1e-5, atol=1e-9)
    torch.testing.assert_close(s["exp_avg_sq"], want_v, rtol=1e-5, atol=1e-12)
    assert torch.equal(params.cpu(), s["master"].to(torch.bfloat16))
    tiles = opt._tiled()
    last = tiles[-1, 0, :].numpy()
    tail = opt.nparams - (opt.tiles - 1) * TILE_PARAMS
    assert (last[tail:] == 0).all()


def test_streamed_adamw_engine_relays(need_gpu, gpu_count):
    from pcie_pool_b200.parallel.engine import PoolEngine

    devs = list(range(min(gpu_count, 4)))
    eng = PoolEngine(devs, slot_bytes=2 << 20, slots=3, timeout_s=10.0)
    n = 37 * TILE_PARAMS + 1001
    g = torch.Generator(device="cuda").manual_seed(3)
    params = (torch.randn(n, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    p0 = params.clone()
    kw = dict(lr=3e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    opt = StreamedAdamW(params, engine=eng, relays=devs[1:], chunk_bytes=5 * 24576, **kw)
    steps = [(torch.randn(n, device="cuda", generator=g) * 1e-2).to(torch.bfloat16) for _ in range(4)]
    grads = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    for gr in steps:
        grads.copy_(gr)
        st = opt.step(grads)
        torch.cuda.synchronize()
        assert st.cuda_ms > 0 and len(st.lanes) == len(devs)
    _check(opt, params, p0, steps, kw)


def test_streamed_adamw_through_daemon(need_gpu, gpu_count):
    from pcie_pool_b200.e2e import build_inprocess_node, nominal_profile
    from pcie_pool_b200.parallel.engine import PoolEngine

    devs = list(range(min(gpu_count, 4)))
    eng = PoolEngine(devs, slot_bytes=4 << 20, slots=3, timeout_s=10.0)
    daemon, dc = build_inprocess_node(eng, devs, 0, nominal_profile(0, devs[1:]) if len(devs) > 1 else None)
    sid = dc.register_session(0, devs[1:], max_inflight_chunks=1 << 16).payload["session"]["session_id"]
    assert dc.register_job("train", session_id=sid).ok
    n = 300 * TILE_PARAMS
    g = torch.Generator(device="cuda").manual_seed(4)
    params = (torch.randn(n, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    p0 = params.clone()
    kw = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    opt = StreamedAdamW(params, client=TurboBusClient(daemon=dc), daemon_client=dc, session_id=sid, job_id="train",
                        chunk_bytes=40 * 24576, **kw)
    grads = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    steps = []
    for _ in range(3):
        grads.copy_((torch.randn(n, device="cuda", generator=g) * 1e-2).to(torch.bfloat16))
        steps.append(grads.clone())
        opt.step(grads)
    torch.cuda.synchronize()
    _check(opt, params, p0, steps, kw)
    d = dc.describe().payload
    assert not d.get("reservations")
    assert all(int(q.get("active_chunks", 0)) == 0 for q in (d.get("relay_quotas") or {}).values())
