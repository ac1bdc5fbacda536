"""vLLM KV connector, scheduler side, with stand-in vLLM objects: the events
each hook records, restore caps, save requests that wait for their blocks,
metadata hand-off, finished-request reporting and the HMA variant; plus the
KV-cache layout the adapter infers.  Behaviours follow
e2e/test_vllm_kv_connector.py of the reference with independent fakes."""

from __future__ import annotations

from types import SimpleNamespace

import pytest

torch = pytest.importorskip("torch")

from pcie_pool_b200.adapters.vllm import kv_layout  # noqa: E402
from pcie_pool_b200.adapters.vllm_kv_connector import (TurboBusConnector, TurboBusSavedPrefix,  # noqa: E402
                                                       clear_connector_events, clear_saved_prefixes,
                                                       get_connector_events)


class Cfg:
    def __init__(self, extra=None, block_size=16):
        self.cache_config = SimpleNamespace(block_size=block_size)
        self.kv_transfer_config = SimpleNamespace(engine_id=None, kv_connector_extra_config=dict(extra or {}))


class Req:
    def __init__(self, rid="r0", params=None, num_tokens=512):
        self.request_id, self.kv_transfer_params, self.num_tokens = rid, dict(params or {}), num_tokens


def blocks(ids):
    return SimpleNamespace(get_block_ids=lambda allow_none=False: (list(ids),))


@pytest.fixture(autouse=True)
def _clean(monkeypatch):
    monkeypatch.setenv("TURBOBUS_CONNECTOR_EVENTS", "0")
    clear_saved_prefixes()
    clear_connector_events()
    yield
    clear_saved_prefixes()


def save_prefix(key="p", blocks_=8, tokens=128, session="s"):
    from pcie_pool_b200.adapters import vllm_kv_connector as K

    K._PREFIX_STORE.put(TurboBusSavedPrefix(key, [], blocks_, tokens, session_id=session))


def events(kind):
    return [e for e in get_connector_events() if e.get("event") == kind]


def sched(**extra):
    cfg = {"turbobus.session_id": "s", "turbobus.restore_enabled": True, **extra}
    return TurboBusConnector(Cfg(cfg), "scheduler")


def test_match_records_skipped_miss_and_hit_events():
    r = Req(params={"turbobus.do_restore": True, "turbobus.prefix_key": "p"})
    TurboBusConnector(Cfg({"turbobus.session_id": "s"}), "scheduler").get_num_new_matched_tokens(r, 0)
    assert events("match_skipped") and events("match_skipped")[0]["restore_enabled"] is False
    c = sched()
    assert c.get_num_new_matched_tokens(r, 0) == (0, False)
    assert events("match_miss")[0]["prefix_key"] == "p"
    save_prefix()
    assert c.get_num_new_matched_tokens(r, 0) == (128, False)
    hit = events("match")[-1]
    assert (hit["matched_tokens"], hit["available_tokens"], hit["session_id"]) == (128, 128, "s")


def test_requests_without_restore_params_are_ignored():
    c = sched()
    save_prefix()
    assert c.get_num_new_matched_tokens(Req(params={}), 0) == (0, False)
    assert not get_connector_events() or not events("match")


def test_matched_tokens_param_caps_and_computed_tokens_reduce():
    c = sched()
    save_prefix(tokens=128)
    r = Req(params={"turbobus.do_restore": True, "turbobus.prefix_key": "p", "turbobus.matched_tokens": 48})
    assert c.get_num_new_matched_tokens(r, 0) == (48, False)
    assert c.get_num_new_matched_tokens(r, 48) == (0, False), "nothing left beyond what vLLM computed"
    big = Req(params={"turbobus.do_restore": True, "turbobus.prefix_key": "p", "turbobus.matched_tokens": 4096})
    assert c.get_num_new_matched_tokens(big, 0) == (128, False), "never more than was saved"


def test_prefixes_are_isolated_by_session():
    save_prefix(session="other")
    r = Req(params={"turbobus.do_restore": True, "turbobus.prefix_key": "p"})
    assert sched().get_num_new_matched_tokens(r, 0) == (0, False)


def test_alloc_queues_a_load_capped_by_restore_blocks():
    c = sched(**{"turbobus.restore_block_limit": 3})
    save_prefix(blocks_=8, tokens=128)
    r = Req("L", {"turbobus.do_restore": True, "turbobus.prefix_key": "p"})
    n, _ = c.get_num_new_matched_tokens(r, 0)
    c.update_state_after_alloc(r, blocks(range(20, 30)), n)
    md = c.build_connector_meta(None)
    assert [(m.request_id, m.block_ids) for m in md.requests] == [("L", (20, 21, 22))]
    assert events("alloc")[-1]["block_count"] == 3
    assert len(c.build_connector_meta(None)) == 0, "metadata is handed over once"


def test_alloc_without_saved_prefix_or_tokens_queues_nothing():
    c = sched()
    r = Req("L", {"turbobus.do_restore": True, "turbobus.prefix_key": "missing"})
    c.update_state_after_alloc(r, blocks([1, 2]), 32)
    c.update_state_after_alloc(Req("M", {"turbobus.do_restore": True, "turbobus.prefix_key": "p"}), blocks([1]), 0)
    assert len(c.build_connector_meta(None)) == 0


def test_save_waits_for_enough_blocks_and_is_queued_once():
    c = sched()
    r = Req("S", {"turbobus.do_save": True, "turbobus.prefix_key": "k", "turbobus.save_blocks": 3})
    c.update_state_after_alloc(r, blocks([4, 5]), 0)
    assert events("save_waiting")[-1]["requested_blocks"] == 3
    out = SimpleNamespace(scheduled_new_reqs=[SimpleNamespace(req_id="S", block_ids=([4, 5, 6, 7],))],
                          scheduled_cached_reqs=SimpleNamespace(req_ids=[], new_block_ids=[]))
    md = c.build_connector_meta(out)
    assert [(m.request_id, m.block_ids) for m in md.save_requests] == [("S", (4, 5, 6))]
    c.update_state_after_alloc(r, blocks([4, 5, 6, 7]), 0)
    assert len(c.build_connector_meta(out)) == 0, "a request is saved once"


def test_save_blocks_default_to_matched_tokens_or_all_blocks():
    c = sched()
    c.update_state_after_alloc(Req("A", {"turbobus.do_save": True, "turbobus.prefix_key": "a",
                                         "turbobus.matched_tokens": 40}), blocks([1, 2, 3, 4]), 0)
    c.update_state_after_alloc(Req("B", {"turbobus.do_save": True, "turbobus.prefix_key": "b"}),
                               blocks([5, 6]), 0)
    saves = {m.request_id: m for m in c.build_connector_meta(None).save_requests}
    assert saves["A"].block_ids == (1, 2, 3) and saves["A"].matched_tokens == 40
    assert saves["B"].block_ids == (5, 6)


def test_finished_requests_never_hold_blocks():
    c = sched()
    r = Req("S", {"turbobus.do_save": True, "turbobus.prefix_key": "k", "turbobus.save_blocks": 1})
    c.update_state_after_alloc(r, blocks([9]), 0)
    held, params = c.request_finished(r, [9])
    assert held is False and params["turbobus.prefix_key"] == "k"
    assert c.request_finished_all_groups(r, ([9],))[0] is False
    w = TurboBusConnector(Cfg({"turbobus.session_id": "s"}), "worker")
    assert w.get_finished({"S"}) == (None, None)


@pytest.mark.parametrize("shape,planes", [((2, 10, 16, 8, 64), True), ((10, 2, 16, 8, 64), False)])
def test_kv_layout_detects_where_the_kv_axis_is(shape, planes):
    """``[2, blocks, ...]``: K and V are separate planes, two units per block;
    ``[blocks, 2, ...]``: K and V sit together in a block, one unit."""
    t = torch.zeros(shape, dtype=torch.bfloat16)
    lay = kv_layout(t)
    es = t.element_size()
    assert lay.num_blocks == 10
    if planes:
        assert (lay.lanes, lay.lane_stride, lay.block_stride) == (2, t.stride(0) * es, t.stride(1) * es)
        assert lay.unit_bytes == 16 * 8 * 64 * es
    else:
        assert (lay.lanes, lay.block_stride) == (1, t.stride(0) * es)
        assert lay.unit_bytes == 2 * 16 * 8 * 64 * es
