"""The gstar_evict mirror driven like the reference's own tests
(code/tests/test_sglang_evict.py), on the sm_100a kernels.

Where the reference test compares against core.Policy (which needs the
reference source), these compare against the CPU oracle, which
tests/test_oracle_golden.py pins to the reference's outputs.
"""
import random
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
FULL = (1, 3)


@pytest.fixture(autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import runtime as ge
    ge.STATE = None
    torch.manual_seed(0)
    yield ge
    ge.STATE = None


def backend(rows=4, width=8192, slots=20000, kv_heads=8, dim=64, page=1):
    """Two full layers (1, 3) and two sliding-window layers (test_sglang_evict.py:19-28).
    With page > 1 the pools are [slots / page, kv_heads, page, dim]."""
    shape = (slots, kv_heads, dim) if page == 1 else (slots // page, kv_heads, page, dim)
    keys = {l: torch.randn(shape, device="cuda").to(torch.bfloat16) for l in range(4)}
    values = {l: torch.randn(shape, device="cuda").to(torch.bfloat16) for l in range(4)}
    pool = SimpleNamespace(layers_mapping={l: (l, l not in FULL) for l in range(4)},
                           get_key_buffer=keys.__getitem__, get_value_buffer=values.__getitem__)
    return SimpleNamespace(token_to_kv_pool=pool, max_kv_splits=8, page_size=page,
                           req_to_token_pool=SimpleNamespace(req_to_token=torch.zeros(
                               (rows, width), dtype=torch.int32, device="cuda")),
                           kv_indptr=torch.zeros(rows + 1, dtype=torch.int32, device="cuda"))


def allocator(slots=20000):
    freed = []
    return freed, SimpleNamespace(free_full=lambda s: freed.append(s.clone()),
                                  full_to_swa_index_mapping=torch.zeros(slots, dtype=torch.int64, device="cuda"))


def entry(ge, name, budget, prefix, recent, seed, kind="live"):
    cfg = {"name": name, "budget": budget, "prefix": prefix, "recent": recent, "seed": seed}
    return ge._live_entry(SimpleNamespace(rid="r", session=None), cfg, kind)


def test_decode_scores_are_per_kv_head(_setup):
    """test_sglang_evict.py:48-78, with the fused kernel in place of SGLang's decode."""
    ge = _setup
    b = backend()
    st = ge.state(b)
    heads, kv_heads, dim, lengths = 64, 8, 64, [37, 1500, 3001]
    keys, values = b.token_to_kv_pool.get_key_buffer(1), b.token_to_kv_pool.get_value_buffer(1)
    q = torch.randn((3, heads, dim), device="cuda").to(torch.bfloat16)
    sinks = torch.randn(heads, device="cuda").to(torch.bfloat16)
    perm = (torch.randperm(19999, device="cuda")[:sum(lengths)] + 1).int()
    indptr = torch.tensor([0, 37, 1537, 4538], dtype=torch.int32, device="cuda")
    rows = torch.tensor([1, 2, 3], device="cuda")
    b.forward_metadata = SimpleNamespace(kv_indptr=indptr, kv_indices=perm)
    layer = SimpleNamespace(sliding_window_size=-1, tp_q_head_num=heads, tp_k_head_num=kv_heads,
                            qk_head_dim=dim, layer_id=1, scaling=0.125)
    for mode in (1, 2):
        st.mode[:] = mode
        st.scores.zero_()
        out = torch.empty((3, heads, dim), dtype=torch.bfloat16, device="cuda")
        ge.decode(b, q.reshape(3, -1), layer, SimpleNamespace(
            out_cache_loc=torch.zeros(3, dtype=torch.int64, device="cuda"), req_pool_indices=rows),
            sinks, out)
        expected = torch.zeros_like(st.scores)
        expected_out = torch.zeros((3, heads, dim), device="cuda")
        for i in range(3):
            slots = perm[indptr[i]:indptr[i + 1]].long()
            k = keys[slots].float().repeat_interleave(heads // kv_heads, 1)
            v = values[slots].float().repeat_interleave(heads // kv_heads, 1)
            logits = torch.einsum("hd,khd->hk", q[i].float(), k) * 0.125
            p = torch.softmax(torch.cat((logits, sinks.float()[:, None]), -1), -1)[:, :-1]
            expected_out[i] = torch.einsum("hk,khd->hd", p, v)
            p = p.view(kv_heads, 8, -1)
            expected[0][:, slots] += p.sum(1) if mode == 1 else p.amax(1)
        # the new slots (out_cache_loc = 0) were zeroed first, as in the reference
        torch.testing.assert_close(st.scores, expected, rtol=2e-3, atol=1e-6)
        rel = (out.float() - expected_out).norm() / expected_out.norm()
        assert float(rel) < 5e-3


def test_after_decode_matches_reference_hook_semantics(_setup):
    ge = _setup
    b = backend()
    st = ge.state(b)
    lengths = [100, 257]
    perm = (torch.randperm(19999, device="cuda")[:sum(lengths)] + 1).int()
    b.forward_metadata = SimpleNamespace(kv_indptr=torch.tensor([0, 100, 357], dtype=torch.int32, device="cuda"),
                                         kv_indices=perm)
    q = torch.randn((2, 64, 64), device="cuda").to(torch.bfloat16)
    sinks = torch.randn(64, device="cuda")
    layer = SimpleNamespace(sliding_window_size=-1, tp_q_head_num=64, tp_k_head_num=8, qk_head_dim=64,
                            layer_id=1, scaling=0.125)
    st.mode[:] = 1
    st.scores.fill_(5.0)
    loc = perm[[99, 356]].long()
    ge.after_decode(b, q.reshape(2, -1), layer, SimpleNamespace(out_cache_loc=loc,
                                                                req_pool_indices=torch.tensor([0, 1], device="cuda")), sinks)
    s = st.scores.cpu()
    # new slots zeroed on every full layer, then this layer's mass added
    assert float(s[1, :, loc.cpu()].abs().max()) == 0.0
    assert float(s[0, :, loc.cpu()].max()) < 1.0
    sliding = SimpleNamespace(sliding_window_size=128)
    ge.after_decode(b, q.reshape(2, -1), sliding, None, sinks)  # sliding layers are ignored


def test_fill_reads_compact_residents_then_tail(_setup):
    """test_sglang_evict.py:80-90 (golden vectors)."""
    ge = _setup
    b = backend()
    st = ge.state(b)
    st.req_to_token[1, :10] = torch.arange(101, 111, dtype=torch.int32)
    st.req_to_token[2, :6] = torch.arange(201, 207, dtype=torch.int32)
    st.table[1, :4] = torch.tensor([101, 102, 106, 107], dtype=torch.int32)
    st.count[1], st.frontier[1] = 4, 7
    out = torch.full((32,), -1, dtype=torch.int64, device="cuda")
    indptr = ge.fill(b, 2, torch.tensor([10, 6], device="cuda"), torch.tensor([1, 2], device="cuda"), out)
    assert indptr.tolist() == [0, 7, 13]
    assert out[:13].tolist() == [101, 102, 106, 107, 108, 109, 110, 201, 202, 203, 204, 205, 206]


def _oracle_state(st, b):
    state = {"table": st.table.cpu().numpy(), "r2u": st.req_to_token.cpu().numpy(),
             "frontier": st.frontier.cpu().numpy(), "count": st.count.cpu().numpy(),
             "pos": st.pos.cpu().numpy(), "scores": st.scores.cpu().numpy()}
    kl = [b.token_to_kv_pool.get_key_buffer(l).view(torch.int16).cpu().numpy().reshape(-1, 8, 1, 64) for l in FULL]
    vl = [b.token_to_kv_pool.get_value_buffer(l).view(torch.int16).cpu().numpy().reshape(-1, 8, 1, 64) for l in FULL]
    return state, [k.view(np.uint16) for k in kl], [v.view(np.uint16) for v in vl]


def check_boundaries(ge, name, kind):
    """test_sglang_evict.py:92-148: two boundaries with relocation, ownership and
    freeing checks; kept sets against the oracle run on the same state."""
    b = backend()
    st = ge.state(b)
    n, budget = 4096 + 300, 1024
    prefix = budget // 4
    recent = budget - prefix if name == "prefix_sliding_2048" else budget // 4
    slot_of = torch.randperm(19000, device="cuda")[:n] + 1
    st.req_to_token[1, :n] = slot_of.int()
    original = {l: b.token_to_kv_pool.get_key_buffer(l)[slot_of].clone() for l in FULL}
    original_v = {l: b.token_to_kv_pool.get_value_buffer(l)[slot_of].clone() for l in FULL}
    score = torch.rand((2, 8, n), device="cuda")
    st.scores[:, :, slot_of] = score
    e = entry(ge, name, budget, prefix, recent, seed=4, kind=kind)
    freed, alloc = allocator()
    ostate, okl, ovl = _oracle_state(st, b)
    for boundary in (2048, 4096):
        cursor = boundary - 200
        N = int(ostate["count"][1]) + boundary - int(ostate["frontier"][1])
        uni = None
        if name == "random_2048":
            g = torch.Generator(device="cuda").manual_seed((4 * 1000003 + boundary) & 0x7FFFFFFF)
            uni = torch.rand((2, 8, N), generator=g, device="cuda", dtype=torch.float64).cpu().numpy()[None]
        row = dict(n=boundary, budget=budget, prefix=prefix, recent=recent,
                   cursor=None if kind == "replay" else cursor, policy=name, seed=4)
        oracle.boundary(ostate, okl, ovl, [1], oracle.row_params([row]), N, live=kind == "live",
                        uniforms=uni)
        if kind == "replay":
            ge._boundary(st, 1, e, boundary)
        else:
            ge._boundary(st, 1, e, boundary, cursor, alloc)
        table = st.table[1, :e["count"]].long()
        assert e["count"] == (budget if name != "prefix_sliding_2048" else prefix + recent)
        np.testing.assert_array_equal(st.table.cpu().numpy(), ostate["table"])
        np.testing.assert_array_equal(st.pos.cpu().numpy(), ostate["pos"])
        for index, layer in enumerate(FULL):
            keys = b.token_to_kv_pool.get_key_buffer(layer)
            values = b.token_to_kv_pool.get_value_buffer(layer)
            for g in range(8):
                held = e["pos"][index, g]
                assert held.numel() == e["count"]
                # relocated keys, values and scores belong to the positions the head claims
                assert torch.equal(keys[table, g], original[layer][held, g])
                assert torch.equal(values[table, g], original_v[layer][held, g])
                torch.testing.assert_close(st.scores[index, g, table], score[index, g, held])
        assert int(st.frontier[1]) == boundary
    if kind == "replay":
        assert torch.equal(st.req_to_token[1, :n], slot_of.int())
        assert freed == []
        return
    row = st.req_to_token[1, :n].long()
    owned = row[row != 0]
    true = min(4096 - recent, 4096 - 200)
    assert torch.equal(row[true:], slot_of[true:])
    assert owned.numel() == torch.unique(owned).numel()
    assert set(owned.tolist()) == set(st.table[1, :e["count"]].tolist()) | set(slot_of[4096:].tolist())
    released = torch.cat(freed).tolist()
    assert len(released) == len(set(released))
    assert set(released) | set(owned.tolist()) == set(slot_of.tolist())
    assert e["freed"] == len(released)
    np.testing.assert_array_equal(st.req_to_token.cpu().numpy(), ostate["r2u"])


@pytest.mark.parametrize("name", ["head_sum_2048", "random_reservoir_2048", "prefix_sliding_2048",
                                  "random_2048", "h2o_global_2048"])
def test_live_boundaries_relocate_and_free(_setup, name):
    check_boundaries(_setup, name, "live")


@pytest.mark.parametrize("name", ["head_max_sum_2048", "random_reservoir_2048"])
def test_replay_boundaries_relocate_without_freeing(_setup, name):
    check_boundaries(_setup, name, "replay")


def test_random_redraws_but_reservoir_is_fixed(_setup):
    """test_sglang_evict.py:160-169."""
    ge = _setup
    pos = torch.arange(1000, device="cuda").expand(2, 8, -1)
    layers, heads = torch.arange(2, device="cuda"), torch.arange(8, device="cuda")
    fixed = ge.reservoir_scores(7, pos, layers, heads)
    assert float(fixed[1, 5, 321]) == oracle.reservoir53(7, 1, 5, 321) / float(1 << 53)
    assert float((fixed[0, 0] - fixed[1, 3]).abs().mean()) > 0.2
    st = SimpleNamespace(scores=None)
    a = ge._scores(st, {"cfg": {"seed": 7}}, "random_2048", pos, None, 2048)
    c = ge._scores(st, {"cfg": {"seed": 7}}, "random_2048", pos, None, 4096)
    assert float((a - c).abs().mean()) > 0.2


def test_reservoir_survival_does_not_decay_with_age(_setup):
    """test_sglang_evict.py:171-189, through the selection kernel."""
    ge = _setup
    budget, total = 2048, 2048 * 16
    layers, heads = torch.arange(1, device="cuda"), torch.arange(1, device="cuda")
    fractions = {}
    for name in ("random_reservoir_2048", "random_2048"):
        resident = torch.arange(0, device="cuda", dtype=torch.long).view(1, 1, 0)
        for n in range(2048, total + 1, 2048):
            pos = torch.cat((resident, torch.arange(n - 2048, n, device="cuda").view(1, 1, -1)), -1)
            if name == "random_2048":
                g = torch.Generator(device="cuda").manual_seed(n)
                score = torch.rand(pos.shape, generator=g, device="cuda", dtype=torch.float64)
            else:
                score = ge.reservoir_scores(3, pos, layers, heads)
            keep, _ = ge.choose(name, pos, n, budget, 0, 0, score)
            resident = torch.gather(pos, -1, keep)
        fractions[name] = float((resident < total // 2).float().mean())
    assert abs(fractions["random_reservoir_2048"] - 0.5) < 0.05
    assert fractions["random_2048"] < 0.1


def test_choose_deferred_and_mismatch(_setup):
    ge = _setup
    pos = torch.arange(600, device="cuda").expand(2, 8, -1).contiguous()
    score = torch.rand((2, 8, 600), device="cuda", dtype=torch.float64)
    keep, count = ge.choose("head_sum_2048", pos, 600, 100, 64, 64, score)
    assert keep is None and count == 128
    bad = pos.clone()
    bad[1, 3, 599] = 650  # at n = 700 only this head holds a recent-window position
    with pytest.raises(RuntimeError, match="protected positions differ"):
        ge.choose("head_sum_2048", bad, 700, 256, 64, 64, score)


def test_on_decode_runs_due_boundary_and_frees(_setup, tmp_path, monkeypatch):
    """The scheduler hook path: create the entry at extend, boundary at decode;
    release writes the request's event payload."""
    monkeypatch.setenv("GSTAR_PAYLOAD_DIR", str(tmp_path))
    ge = _setup
    b = backend(rows=2, slots=6000)
    st = ge.state(b)
    n = 2048
    slot_of = torch.randperm(5990, device="cuda")[:n] + 1
    st.req_to_token[0, :n] = slot_of.int()
    freed, alloc = allocator(6000)
    req = SimpleNamespace(rid="a", session=None, kv=SimpleNamespace(req_pool_idx=0, holds_kv=True),
                          sampling_params=SimpleNamespace(custom_params={"gstar_eviction": {
                              "name": "random_reservoir_2048", "budget": 512, "prefix": 128,
                              "recent": 128, "seed": 1}}),
                          extend_range=SimpleNamespace(start=0, length=2048),
                          origin_input_ids=[0] * 2000, output_ids=[0] * 48)
    batch = SimpleNamespace(reqs=[req], tree_cache=SimpleNamespace(token_to_kv_pool_allocator=alloc),
                            seq_lens_cpu=torch.tensor([n]))
    ge.on_extend(batch)
    e = st.entries[0]
    assert e["error"] is None and int(st.mode[0]) == 0
    ge.on_decode(batch)
    assert e["count"] == 512 and e["last_boundary"] == n
    assert sum(x.numel() for x in freed) == n - 512 == e["freed"]
    ge.on_decode(batch)  # same length again: no second boundary
    assert len(e["events"]) == 1
    ge.release(req)
    assert 0 not in st.entries
    import gzip
    import json
    obj = json.loads(gzip.decompress((tmp_path / "a.json.gz").read_bytes()))
    assert obj["kind"] == "events" and obj["length"] == n and obj["freed"] == n - 512
    assert [ev["boundary"] for ev in obj["events"]] == [n] and obj["peak_full_entries"] == n


def test_after_extend_scores_h2o_rows(_setup):
    """after_extend (runtime:277-311): new slots zeroed on every full layer,
    then each head_sum / head_max row adds its chunk's exact probabilities
    over prefix ++ chunk with the causal mask and sinks (_probabilities,
    runtime:314-324, in plain torch here)."""
    ge = _setup
    b = backend()
    st = ge.state(b)
    heads, kv_heads, dim = 64, 8, 64
    # row: (policy or None, prefix tokens, chunk tokens)
    spec = [("head_sum_2048", 300, 120), (None, 50, 17), ("head_max_sum_2048", 0, 64),
            ("random_2048", 10, 5)]
    for r, (name, _, _) in enumerate(spec):
        if name is not None:
            st.entries[r] = entry(ge, name, 1024, 256, 256, 7)
            st.mode[r] = st.entries[r]["mode"]
    perm = (torch.randperm(19999, device="cuda") + 1).long()
    prefixes, news, k = [], [], 0
    for _, p, n in spec:
        prefixes.append(perm[k:k + p])
        news.append(perm[k + p:k + p + n])
        k += p + n
    kv_indptr = torch.tensor([0] + list(np.cumsum([p for _, p, _ in spec])), dtype=torch.int32, device="cuda")
    qo_indptr = torch.tensor([0] + list(np.cumsum([n for _, _, n in spec])), dtype=torch.int32, device="cuda")
    b.forward_metadata = SimpleNamespace(kv_indptr=kv_indptr, kv_indices=torch.cat(prefixes),
                                         qo_indptr=qo_indptr)
    total = int(qo_indptr[-1])
    q = torch.randn((total, heads, dim), device="cuda").to(torch.bfloat16)
    sinks = torch.randn(heads, device="cuda").to(torch.bfloat16)
    batch = SimpleNamespace(out_cache_loc=torch.cat(news), req_pool_indices=torch.arange(4, device="cuda"),
                            extend_prefix_lens_cpu=[p for _, p, _ in spec])
    st.scores.fill_(5.0)
    expected = torch.full_like(st.scores, 5.0)
    expected[:, :, batch.out_cache_loc] = 0.0
    for layer_id in FULL:
        layer = SimpleNamespace(sliding_window_size=-1, tp_q_head_num=heads, tp_k_head_num=kv_heads,
                                qk_head_dim=dim, layer_id=layer_id, scaling=0.125)
        ge.after_extend(b, q.reshape(total, -1), layer, batch, sinks)
        keys = b.token_to_kv_pool.get_key_buffer(layer_id)
        for r, (name, p, n) in enumerate(spec):
            mode = st.entries[r]["mode"] if r in st.entries else 0
            if mode not in (1, 2):
                continue
            slots = torch.cat((prefixes[r], news[r]))
            kk = keys[slots].float().repeat_interleave(heads // kv_heads, 1)     # [T, H, D]
            qq = q[int(qo_indptr[r]):int(qo_indptr[r + 1])].float()             # [n, H, D]
            logits = torch.einsum("qhd,khd->hqk", qq, kk) * 0.125
            causal = torch.arange(p + n, device="cuda")[None, :] > (p + torch.arange(n, device="cuda"))[:, None]
            logits = logits.masked_fill(causal[None], -torch.inf)
            sink = sinks.float()[:, None, None].expand(heads, n, 1)
            prob = torch.softmax(torch.cat((logits, sink), -1), -1)[..., :-1].view(kv_heads, 8, n, -1)
            red = (prob.sum(1) if mode == 1 else prob.amax(1)).sum(1)             # [G, T]
            expected[FULL.index(layer_id)][:, slots] += red
    torch.testing.assert_close(st.scores, expected, rtol=1e-3, atol=1e-5)
    assert int(st.err.item()) == 0


def _read_payload(directory, key):
    import base64
    import gzip
    import json
    obj = json.loads(gzip.decompress((directory / f"{key}.json.gz").read_bytes()))
    dec = lambda a: np.frombuffer(base64.b64decode(a["data"]), a["dtype"])
    return obj, dec(obj["evicted_delta"]), dec(obj["evicted_counts"])


@pytest.mark.parametrize("name", ["head_sum_2048", "random_reservoir_2048", "random_2048"])
def test_retention_records_are_written_and_decode_to_the_kept_sets(_setup, name, tmp_path, monkeypatch):
    """cfg record=True (runtime:465-467, 500-507): one payload per evicting
    boundary; replaying the records like the reference's client
    (sglang_client.py:115-133) rebuilds every head's held positions."""
    monkeypatch.setenv("GSTAR_PAYLOAD_DIR", str(tmp_path))
    ge = _setup
    b = backend()
    st = ge.state(b)
    n, budget = 4096 + 300, 1024
    slot_of = torch.randperm(19000, device="cuda")[:n] + 1
    st.req_to_token[1, :n] = slot_of.int()
    st.scores[:, :, slot_of] = torch.rand((2, 8, n), device="cuda")
    cfg = {"name": name, "budget": budget, "prefix": budget // 4, "recent": budget // 4, "seed": 4,
           "record": True}
    e = ge._live_entry(SimpleNamespace(rid="req7", session=None), cfg, "live")
    freed, alloc = allocator()
    held, last = None, 0
    for boundary in (2048, 4096):
        before = (st.pos[1].cpu().numpy().copy(), e["count"], e["frontier"])
        ge._boundary(st, 1, e, boundary, boundary - 200, alloc)
        obj, delta, counts = _read_payload(tmp_path, f"req7-b{boundary}")
        assert obj["kind"] == "retention" and obj["boundary"] == boundary and obj["kv_heads"] == 8
        assert obj["format"] == "gstar-payload-1" and obj["cfg"]["record"] is True
        dw, cw = oracle.retention_record(before[0], before[1], before[2], boundary,
                                         st.pos[1].cpu().numpy(), e["count"])
        np.testing.assert_array_equal(counts, cw)
        np.testing.assert_array_equal(delta, dw)
        evicted = np.split(delta.astype(np.int64), np.cumsum(counts)[:-1])
        new = np.arange(last, boundary)
        held = [new.copy() for _ in counts] if held is None else [np.concatenate((h, new)) for h in held]
        held = [np.setdiff1d(h, np.cumsum(v), assume_unique=True) for h, v in zip(held, evicted)]
        last = boundary
        for s, h in enumerate(held):
            np.testing.assert_array_equal(np.sort(e["pos"][s // 8, s % 8].cpu().numpy()), h)


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _chunk(b, st, ge, row, start, count, slot_of, page):
    """Extend metadata of one chunk: the row's CSR for its prefix (built by
    fill, as SGLang's backend does) and the chunk's token slots."""
    kv_indptr = torch.zeros(2, dtype=torch.int32, device="cuda")
    b.kv_indptr = kv_indptr
    kv_indices = torch.zeros(8192, dtype=torch.int32, device="cuda")
    ge.fill(b, 1, torch.tensor([start], device="cuda"), torch.tensor([row], device="cuda"), kv_indices)
    b.forward_metadata = SimpleNamespace(kv_indptr=kv_indptr, kv_indices=kv_indices[:int(kv_indptr[1])],
                                         qo_indptr=torch.tensor([0, count], dtype=torch.int32, device="cuda"))
    return SimpleNamespace(out_cache_loc=slot_of[start:start + count], req_pool_indices=torch.tensor([row], device="cuda"),
                           extend_prefix_lens_cpu=[start], positions=torch.arange(start, start + count, device="cuda"))


def _layout(st, n, page, row=0):
    """Random units for the row's pages; returns the token slot of every logical position."""
    units = -(-n // page)
    unit_of = (torch.randperm(st.units - 1, device="cuda")[:units] + 1).int()
    st.req_to_token[row, :units] = unit_of
    t = torch.arange(n, device="cuda")
    return unit_of[t // page].long() * page + t % page


def _layer(layer_id):
    return SimpleNamespace(sliding_window_size=-1, tp_q_head_num=64, tp_k_head_num=8, qk_head_dim=64,
                           layer_id=layer_id, scaling=0.125)


def _visible_np(e, page, end):
    vis = np.zeros((8, end), bool)
    vis[:, e["frontier"] * page:] = True
    pos = e["pos"][0].cpu().numpy()
    for g in range(8):
        for u in pos[g]:
            vis[g, u * page:(u + 1) * page] = True
    return vis


@pytest.mark.parametrize("page", [1, 16])
def test_replay_entry_records_layer_error(_setup, page, tmp_path, monkeypatch):
    """Static replay (runtime:301-306, 520-546, 685-686, 732-736): the first
    full layer's chunks are copied into the shadow by position, the boundary
    at 2,048 relocates survivors without freeing, the chunk after it records
    each query's layer error against the unevicted keys, and release writes
    the replay payload.  Expected errors from the CPU oracle over the keys
    and values as they were written, with the entry's kept positions."""
    import base64
    import gzip
    import json
    monkeypatch.setenv("GSTAR_PAYLOAD_DIR", str(tmp_path))
    ge = _setup
    b = backend(page=page)
    st = ge.state(b)
    n0, n1 = 2048, 152
    slot_of = _layout(st, n0 + n1, page)
    cfg = {"name": "head_sum_2048", "budget": 1024, "prefix": 256, "recent": 256, "seed": 3}
    req = SimpleNamespace(rid="rep1", session=None, kv=SimpleNamespace(req_pool_idx=0, holds_kv=True),
                          sampling_params=SimpleNamespace(custom_params={"gstar_replay": cfg}),
                          extend_range=SimpleNamespace(start=0, length=n0), origin_input_ids=[0] * (n0 + n1),
                          output_ids=[])
    batch = SimpleNamespace(reqs=[req])
    q = torch.randn((n0 + n1, 64, 64), device="cuda").mul_(1.5).to(torch.bfloat16)
    sinks = torch.randn(64, device="cuda").to(torch.bfloat16)
    kpool, vpool = st.pools(1)
    orig_k = ge._token_rows(kpool, slot_of, page).clone()
    orig_v = ge._token_rows(vpool, slot_of, page).clone()
    ge.on_extend(batch)
    e = st.entries[0]
    assert e["kind"] == "replay" and e["error"] is None
    fb = _chunk(b, st, ge, 0, 0, n0, slot_of, page)
    for layer_id in FULL:
        ge.after_extend(b, q[:n0].reshape(n0, -1), _layer(layer_id), fb, sinks)
    req.extend_range = SimpleNamespace(start=n0, length=n1)
    ge.on_extend(batch)                        # static boundary at 2,048: nothing freed
    assert e["count"] == 1024 // page and e["events"][-1]["freed"] == 0
    fb = _chunk(b, st, ge, 0, n0, n1, slot_of, page)
    for layer_id in FULL:
        ge.after_extend(b, q[n0:].reshape(n1, -1), _layer(layer_id), fb, sinks)
    torch.cuda.synchronize()
    assert int(st.err.item()) == 0
    vis = _visible_np(e, page, n0 + n1)
    want = oracle.replay_error(_bits(q[n0:]), _bits(orig_k), _bits(orig_v), n0, 0.125, vis,
                               sinks.float().cpu().numpy())
    ge.release(req)
    obj = json.loads(gzip.decompress((tmp_path / "rep1.json.gz").read_bytes()))
    assert obj["kind"] == "replay" and obj["layer"] == 1 and obj["cfg"] == cfg and obj["error"] is None
    assert [ev["boundary"] for ev in obj["events"]] == [n0]
    err = np.frombuffer(base64.b64decode(obj["layer_error"]["data"]), np.float32)
    assert err.shape == (n0 + n1,)
    assert not err[:n0].any()                  # nothing evicted before the boundary
    assert (err[n0:] > 0).all()
    np.testing.assert_allclose(err[n0:], want, rtol=1e-3, atol=1e-6)


@pytest.mark.parametrize("page", [1, 16])
def test_verify_mode_checks_decode_and_relocation(_setup, page, tmp_path, monkeypatch):
    """GSTAR_EVICT_VERIFY=1 (runtime:110, 213-214, 250-274, 497-498, 510-515):
    live entries keep a shadow; the boundary event reports that every head's
    relocated keys equal the unevicted keys of its claimed positions, and a
    decode step's first-full-layer output matches attention over those
    positions."""
    monkeypatch.setenv("GSTAR_PAYLOAD_DIR", str(tmp_path))
    monkeypatch.setenv("GSTAR_EVICT_VERIFY", "1")
    ge = _setup
    b = backend(page=page)
    st = ge.state(b)
    assert st.verify
    n0, n1 = 2048, 160
    slot_of = _layout(st, n0 + n1 + 1, page)
    cfg = {"name": "head_sum_2048", "budget": 1024, "prefix": 256, "recent": 256, "seed": 3}
    req = SimpleNamespace(rid="v1", session=None, kv=SimpleNamespace(req_pool_idx=0, holds_kv=True),
                          sampling_params=SimpleNamespace(custom_params={"gstar_eviction": cfg}),
                          extend_range=SimpleNamespace(start=0, length=n0), origin_input_ids=[0] * (n0 + n1),
                          output_ids=[5])
    freed, alloc = allocator()
    batch = SimpleNamespace(reqs=[req], tree_cache=SimpleNamespace(token_to_kv_pool_allocator=alloc))
    q = torch.randn((n0 + n1 + 1, 64, 64), device="cuda").to(torch.bfloat16)
    sinks = torch.randn(64, device="cuda").to(torch.bfloat16)
    ge.on_extend(batch)
    e = st.entries[0]
    fb = _chunk(b, st, ge, 0, 0, n0, slot_of, page)
    for layer_id in FULL:
        ge.after_extend(b, q[:n0].reshape(n0, -1), _layer(layer_id), fb, sinks)
    req.extend_range = SimpleNamespace(start=n0, length=n1)
    ge.on_extend(batch)                        # live boundary at 2,048
    ev = e["events"][-1]
    assert ev["boundary"] == n0 and ev["freed"] > 0 and ev["relocation_ok"] is True
    fb = _chunk(b, st, ge, 0, n0, n1, slot_of, page)
    for layer_id in FULL:
        ge.after_extend(b, q[n0:n0 + n1].reshape(n1, -1), _layer(layer_id), fb, sinks)
    # one decode step for the token at position n0 + n1
    n = n0 + n1 + 1
    kv_indptr = torch.zeros(2, dtype=torch.int32, device="cuda")
    b.kv_indptr = kv_indptr
    kv_indices = torch.zeros(8192, dtype=torch.int32, device="cuda")
    ge.fill(b, 1, torch.tensor([n], device="cuda"), torch.tensor([0], device="cuda"), kv_indices)
    b.forward_metadata = SimpleNamespace(kv_indptr=kv_indptr, kv_indices=kv_indices[:int(kv_indptr[1])])
    dfb = SimpleNamespace(out_cache_loc=slot_of[n - 1:n], req_pool_indices=torch.tensor([0], device="cuda"),
                          positions=torch.tensor([n - 1], device="cuda"))
    out = torch.empty((1, 64, 64), dtype=torch.bfloat16, device="cuda")
    ge.decode(b, q[n - 1:n].reshape(1, -1), _layer(1), dfb, sinks, out)
    torch.cuda.synchronize()
    assert int(st.err.item()) == 0
    assert e["verify_steps"] == 1 and e["verify_max_error"] < 2e-2
    ge.release(req)
    import gzip
    import json
    obj = json.loads(gzip.decompress((tmp_path / "v1.json.gz").read_bytes()))
    assert obj["kind"] == "events" and obj["verify_steps"] == 1 and obj["length"] == n0 + n1 + 1
    assert obj["events"][0]["relocation_ok"] is True
