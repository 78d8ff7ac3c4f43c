"""Host-side logic of the gstar_evict mirror on CPU (no kernels are called):
configuration checks, entry lifecycle and the error paths of on_extend
(code/cache_eviction/sglang_evict_runtime.py:625-689, 719-747)."""
from types import SimpleNamespace

import pytest
import torch

from cache_eviction_b200 import policy
from cache_eviction_b200 import runtime as ge


def cpu_backend(rows=4, width=64, slots=100):
    keys = {l: torch.zeros((slots, 8, 64), dtype=torch.bfloat16) for l in range(2)}
    pool = SimpleNamespace(layers_mapping={0: (0, True), 1: (1, False)},
                           get_key_buffer=keys.__getitem__, get_value_buffer=keys.__getitem__)
    return SimpleNamespace(token_to_kv_pool=pool, req_to_token_pool=SimpleNamespace(
        req_to_token=torch.zeros((rows, width), dtype=torch.int32)),
        kv_indptr=torch.zeros(rows + 1, dtype=torch.int32))


@pytest.fixture(autouse=True)
def fresh(tmp_path, monkeypatch):
    monkeypatch.setenv("GSTAR_PAYLOAD_DIR", str(tmp_path))
    ge.STATE = None
    ge.RETRACTED.clear()
    yield
    ge.STATE = None


def req(rid="r", row=0, params=None, start=0, length=10, retraction=0, session=None):
    return SimpleNamespace(rid=rid, session=session, retraction_count=retraction,
                           origin_input_ids=[0] * 12, output_ids=[1, 2],
                           kv=SimpleNamespace(req_pool_idx=row, holds_kv=True),
                           sampling_params=SimpleNamespace(custom_params=params),
                           extend_range=SimpleNamespace(start=start, length=length))


def read_payload(key):
    import gzip
    import json
    import os
    from pathlib import Path
    return json.loads(gzip.decompress((Path(os.environ["GSTAR_PAYLOAD_DIR"]) / f"{key}.json.gz").read_bytes()))


CFG = {"name": "head_sum_2048", "budget": 1024, "prefix": 256, "recent": 256, "seed": 3}


@pytest.mark.parametrize("cfg,err", [
    ({"name": "nope", "budget": 8, "prefix": 1, "recent": 1}, "invalid gstar eviction settings"),
    ({"name": "head_sum_2048", "budget": 8, "prefix": 5, "recent": 5}, "invalid gstar eviction settings"),
    ({"name": "head_sum_2048", "budget": 8, "prefix": -1, "recent": 1}, "invalid gstar eviction settings"),
    ({"name": "prefix_sliding_2048", "budget": 8, "prefix": 2, "recent": 2}, "Prefix Sliding requires B = P + R"),
    ({"name": "head_sum_2048", "prefix": 2, "recent": 2}, "budget"),
])
def test_live_entry_rejects_bad_settings(cfg, err):
    e = ge._live_entry(SimpleNamespace(rid="r", session=None), cfg, "live")
    assert err in e["error"] and e["mode"] == 0


def test_policy_modes_and_aliases():
    assert policy.POLICIES["head_sum_2048"] == 1 and policy.POLICIES["head_max_sum_2048"] == 2
    assert policy.canonical("h2o_per_head") == "head_sum_2048"
    assert policy.canonical("recent") == "prefix_sliding_2048"
    assert policy.sweep_split(2048, "recent") == (512, 1536)
    assert policy.sweep_split(2048, "h2o_global") == (512, 512)
    with pytest.raises(ValueError, match="multiples of the page size"):
        policy.validate({"name": "head_sum_2048", "budget": 1000, "prefix": 8, "recent": 8}, 16)


def test_on_extend_creates_entry_and_mode():
    ge.state(cpu_backend())
    ge.on_extend(SimpleNamespace(reqs=[req(params={"gstar_eviction": CFG})]))
    st = ge.STATE
    assert st.entries[0]["kind"] == "live" and int(st.mode[0]) == 1
    ge.on_extend(SimpleNamespace(reqs=[req(row=1, params={"gstar_replay": dict(CFG, name="head_max_sum_2048")})]))
    assert st.entries[1]["kind"] == "replay" and int(st.mode[1]) == 2
    ge.on_extend(SimpleNamespace(reqs=[req(row=2, params={})]))
    assert 2 not in st.entries


def test_on_extend_rejects_chunk_crossing_a_boundary():
    ge.state(cpu_backend())
    r = req(params={"gstar_eviction": CFG}, start=2000, length=100)
    ge.on_extend(SimpleNamespace(reqs=[r]))
    e = ge.STATE.entries[0]
    assert "crosses a boundary" in e["error"] and int(ge.STATE.mode[0]) == 0


def test_retraction_disables_the_entry():
    ge.state(cpu_backend())
    ge.on_extend(SimpleNamespace(reqs=[req(params={"gstar_eviction": CFG})]))
    ge.on_extend(SimpleNamespace(reqs=[req(params={"gstar_eviction": CFG}, retraction=1)]))
    assert ge.STATE.entries[0]["error"] == "retracted" and "r" in ge.RETRACTED
    assert read_payload("r-retracted") == {"format": "gstar-payload-1", "key": "r-retracted", "kind": "retracted",
                                           "cfg": CFG}


def test_rewind_below_frontier_is_an_error():
    ge.state(cpu_backend())
    ge.on_extend(SimpleNamespace(reqs=[req(params={"gstar_eviction": CFG})]))
    ge.STATE.entries[0]["frontier"] = 2048
    ge.on_extend(SimpleNamespace(reqs=[req(params={"gstar_eviction": CFG}, start=100)]))
    assert "rewound" in ge.STATE.entries[0]["error"]


def test_row_reuse_by_another_request_resets_state():
    ge.state(cpu_backend())
    ge.on_extend(SimpleNamespace(reqs=[req(params={"gstar_eviction": CFG})]))
    ge.STATE.count[0] = 7
    ge.on_extend(SimpleNamespace(reqs=[req(rid="other", params={})]))
    assert 0 not in ge.STATE.entries and int(ge.STATE.count[0]) == 0


def test_release_keeps_session_rows_and_resets_others():
    ge.state(cpu_backend())
    sess = SimpleNamespace(streaming=True, session_id="s1")
    ge.on_extend(SimpleNamespace(reqs=[req(rid="a", params={"gstar_eviction": CFG}, session=sess)]))
    ge.release(req(rid="a", session=sess))
    assert 0 in ge.STATE.entries  # the session keeps its row
    ge.on_extend(SimpleNamespace(reqs=[req(rid="b", row=1, params={"gstar_eviction": CFG})]))
    ge.release(req(rid="b", row=1))
    assert 1 not in ge.STATE.entries and int(ge.STATE.mode[1]) == 0
    # the reference's event payloads (runtime:712-716, 738-741): the session's
    # under "<key>-events", a plain request's under its rid
    for key in ("session-s1-events", "b"):
        ev = read_payload(key)
        assert ev["kind"] == "events" and ev["cfg"] == CFG and ev["events"] == [] and ev["length"] == 14
        assert ev["retracted"] is False and ev["verify_steps"] is None and ev["peak_full_entries"] == 0


def test_filter_holes_and_freed():
    segs = [(torch.tensor([0, 5, 0, 7]), 3), (torch.tensor([0]), 9)]
    out = ge.filter_holes(segs)
    assert out[0][0].tolist() == [5, 7] and out[0][1] == 3 and out[1][0].numel() == 0
    ge.state(cpu_backend())
    ge.on_extend(SimpleNamespace(reqs=[req(params={"gstar_eviction": CFG})]))
    ge.STATE.entries[0]["freed"] = 12
    assert ge.freed(0) == 12 and ge.freed(3) == 0


def test_enabled_reads_environment(monkeypatch):
    monkeypatch.setenv("GSTAR_EVICT", "1")
    assert ge.enabled()
    monkeypatch.setenv("GSTAR_EVICT", "0")
    assert not ge.enabled()
