"""Pin the CPU oracle against the reference's own outputs (CPU only).

Fixtures in tests/golden/*.npz come from tonghuikang/cache-eviction's functions
(tests/golden/make_golden.py); inputs are rebuilt from tests/golden/scenarios.py.
"""
from pathlib import Path

import numpy as np
import pytest

from golden import scenarios as sc
from helpers import boundary_row, boundary_state, paged, prefill_inputs, prefill_want, sha16, sha_bytes
from oracle import oracle

GOLD = Path(__file__).resolve().parent / "golden"


def test_reservoir_matches_reference():
    z = np.load(GOLD / "reservoir.npz")
    assert oracle.reservoir53(7, 1, 5, 321) / float(1 << 53) == float(z["kat_7_1_5_321"])
    assert float(z["kat_7_1_5_321"]) == float(z["kat_runtime_7_1_5_321"])
    for key in z.files:
        if not key.startswith("seed_"):
            continue
        seed = int(key[5:])
        want = z[key]
        got = np.array([[[oracle.reservoir53(seed, l, g, p) for p in range(want.shape[2])]
                         for g in range(want.shape[1])] for l in range(want.shape[0])], np.uint64)
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("i", range(len(sc.choose_cases())))
def test_choose_matches_reference(i):
    c = sc.choose_cases()[i]
    z = np.load(GOLD / "choose.npz")
    L, G, N = c["pos"].shape
    row = dict(n=c["n"], budget=c["budget"], prefix=c["prefix"], recent=c["recent"],
               cursor=c["cursor"], policy=c["name"], seed=c.get("seed", 0))
    score = None if c["score"] is None else c["score"].reshape(1, L * G, N)
    kept, status, pcount = oracle.choose(c["pos"].reshape(1, L * G, N), score,
                                         oracle.row_params([row]), L, G,
                                         score_is_f32=c["name"] == "h2o_global_2048")
    assert int(status[0]) == int(z[f"case{i}_status"])
    if int(status[0]) == 0:
        assert int(pcount[0]) == int(z[f"case{i}_count"])
        want = z[f"case{i}_kept"]
        K = want.shape[-1]
        got = np.sort(kept[0, :, :K], -1).reshape(L, G, K)
        np.testing.assert_array_equal(got, want)
        assert (kept[0, :, K:] == -1).all() if kept.shape[-1] > K else True


@pytest.mark.parametrize("name,kind", sc.BOUNDARY_NAMES)
def test_boundary_matches_reference(name, kind):
    z = np.load(GOLD / "boundary.npz")
    setup = sc.boundary_setup()
    state, kl, vl = boundary_state(setup)
    key = f"{name}_{kind}"
    max_cols = 4096
    for k, b in enumerate((2048, 4096)):
        N = int(state["count"][1]) + b - int(state["frontier"][1])
        uni = None
        if name == "random_2048":
            uni = np.zeros((1, 2, sc.G, max_cols))
            uni[0, :, :, :N] = sc.random_uniforms(4, b, (2, sc.G, N))
        result, freed = oracle.boundary(state, kl, vl, [1], oracle.row_params([boundary_row(name, b)]),
                                        max_cols, live=kind == "live", uniforms=uni)
        assert result[0, 0] == 0, result
        cnt = int(state["count"][1])
        np.testing.assert_array_equal(state["table"][1, :cnt], z[f"{key}_b{k}_table"])
        np.testing.assert_array_equal(state["pos"][1, :, :, :cnt], z[f"{key}_b{k}_pos"])
        assert int(state["frontier"][1]) == int(z[f"{key}_b{k}_frontier"])
        np.testing.assert_array_equal(state["r2u"][1, :setup["n"]], z[f"{key}_b{k}_r2u"])
        if kind == "live":
            prev = 0 if k == 0 else len(z[f"{key}_b0_freed"])
            now = z[f"{key}_b{k}_freed"][prev:]
            np.testing.assert_array_equal(freed[0, :result[0, 3]], now)
    assert [sha16(a) for a in kl] == list(z[f"{key}_keys_sha"])
    assert [sha16(a) for a in vl] == list(z[f"{key}_values_sha"])
    assert sha_bytes(state["scores"]) == str(z[f"{key}_scores_sha"][0])


def _decode_inputs(page):
    d = sc.decode_setup()
    lists = [d["perm"][d["indptr"][i]:d["indptr"][i + 1]] for i in range(3)]
    if page == 1:
        kpool = d["keys"].reshape(-1, sc.G, 1, sc.D)
        vpool = d["values"].reshape(-1, sc.G, 1, sc.D)
        units = lists
    else:
        kpool, units = paged(d["keys"], lists, page)
        vpool, _ = paged(d["values"], lists, page)
    indptr = np.concatenate([[0], np.cumsum([len(u) for u in units])]).astype(np.int32)
    indices = np.concatenate(units).astype(np.int32)
    tokens = np.array(sc.DECODE_LENGTHS, np.int32)
    sinks = sc.bits_to_f32(d["sinks"])
    return d, kpool, vpool, indptr, indices, tokens, sinks, units


@pytest.mark.parametrize("page", [1, 16])
@pytest.mark.parametrize("mode", [1, 2])
def test_decode_matches_reference(page, mode):
    z = np.load(GOLD / "decode.npz")
    d, kpool, vpool, indptr, indices, tokens, sinks, units = _decode_inputs(page)
    scores = np.zeros((sc.G, kpool.shape[0]), np.float32)
    out, lse = oracle.decode(d["q"], kpool, vpool, indptr, indices, tokens, sinks,
                             np.full(3, mode, np.int32), d["scale"], page, scores, zero_new=False)
    for i, length in enumerate(sc.DECODE_LENGTHS):
        np.testing.assert_allclose(out[i], z[f"seq{i}_out"], rtol=1e-4, atol=1e-6)
        tok = z[f"seq{i}_{'sum' if mode == 1 else 'max'}"]  # [G, len]
        if page == 1:
            got = scores[:, units[i]]
            want = tok
        else:
            npg = len(units[i])
            pad = np.zeros((sc.G, npg * page), np.float32)
            pad[:, :length] = tok
            want = pad.reshape(sc.G, npg, page).sum(-1)
            got = scores[:, units[i]]
        np.testing.assert_allclose(got, want, rtol=2e-5, atol=1e-7)


@pytest.mark.parametrize("page", [1, 16])
@pytest.mark.parametrize("mode", [1, 2])
def test_prefill_matches_reference(page, mode):
    z = np.load(GOLD / "prefill.npz")
    d, kpool, units, indptr, indices, tokens = prefill_inputs(page)
    init = np.random.default_rng(3).random((sc.G, kpool.shape[0])).astype(np.float32)
    scores = init.copy()
    oracle.prefill(d["q"], kpool, d["qo_indptr"], indptr, indices, tokens, sc.bits_to_f32(d["sinks"]),
                   np.full(len(tokens), mode, np.int32), d["scale"], page, scores, zero_new=True)
    want = prefill_want(z, mode, page, units, init.astype(np.float64))
    np.testing.assert_allclose(scores, want, rtol=2e-5, atol=1e-6)


RECORD_NAMES = ("head_sum_2048", "random_reservoir_2048", "random_2048", "prefix_sliding_2048")


@pytest.mark.parametrize("name", RECORD_NAMES)
def test_retention_record_matches_reference(name):
    """The oracle's record, rebuilt from the reference's own positions before
    and after each boundary, equals the record the reference wrote."""
    rec = np.load(GOLD / "records.npz")
    bnd = np.load(GOLD / "boundary.npz")
    key = f"{name}_live"
    prev, prev_count, prev_frontier = np.zeros((2, sc.G, 0), np.int32), 0, 0
    for k, b in enumerate((2048, 4096)):
        after = bnd[f"{key}_b{k}_pos"]
        d, c = oracle.retention_record(prev, prev_count, prev_frontier, b, after, after.shape[-1])
        np.testing.assert_array_equal(c, rec[f"{name}_b{k}_evicted_counts"])
        np.testing.assert_array_equal(d, rec[f"{name}_b{k}_evicted_delta"])
        prev, prev_count, prev_frontier = after, after.shape[-1], b


def test_fill_reference_golden():
    # code/tests/test_sglang_evict.py:80-90
    table = np.zeros((4, 16), np.int32)
    r2u = np.zeros((4, 16), np.int32)
    r2u[1, :10] = np.arange(101, 111)
    r2u[2, :6] = np.arange(201, 207)
    table[1, :4] = [101, 102, 106, 107]
    frontier = np.array([0, 7, 0, 0], np.int32)
    count = np.array([0, 4, 0, 0], np.int32)
    indptr, indices, tokens = oracle.fill(table, r2u, frontier, count, [1, 2], [10, 6])
    assert indptr.tolist() == [0, 7, 13]
    assert indices.tolist() == [101, 102, 106, 107, 108, 109, 110, 201, 202, 203, 204, 205, 206]
    assert tokens.tolist() == [7, 6]


@pytest.mark.parametrize("chunk", range(len(sc.REPLAY_CHUNKS)))
def test_replay_error_matches_reference(chunk):
    """Per-token layer error of the reference's static replay
    (_replay_layer_difference, runtime:520-546) for a chunk before any
    eviction (all zeros) and two chunks after a boundary."""
    z = np.load(GOLD / "replay.npz")
    d = sc.replay_setup()
    lo, hi, evicted = sc.REPLAY_CHUNKS[chunk]
    vis = sc.replay_visible(d["pos"], sc.REPLAY_FRONTIER, hi) if evicted else None
    got = oracle.replay_error(d["q"][lo:hi], d["keys"], d["values"], lo, d["scale"], vis, d["sinks"])
    want = z[f"chunk{chunk}"]
    if not evicted:
        assert not got.any() and not want.any()
    np.testing.assert_allclose(got, want, rtol=5e-6, atol=1e-7)
