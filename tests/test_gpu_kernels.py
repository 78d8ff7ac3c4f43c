"""GPU parity of the sm_100a kernels, called through the C ABI, against the
CPU oracle and the reference's golden fixtures."""
from pathlib import Path

import numpy as np
import pytest
import torch

from golden import scenarios as sc
from helpers import boundary_row, boundary_state, paged, sha16, sha_bytes
from oracle import oracle

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi
    capi.load()


def K():
    from cache_eviction_b200 import kernels
    return kernels


def t16(bits):  # numpy bf16 bits -> device bf16 tensor
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(DEV).view(torch.bfloat16)


def err_ok(err):
    torch.cuda.synchronize()
    assert int(err.item()) == 0, hex(int(err.item()))


# ------------------------------------------------------------------------ fill
def test_fill_reference_golden():
    # code/tests/test_sglang_evict.py:80-90
    table = torch.zeros((4, 64), dtype=torch.int32, device=DEV)
    r2u = torch.zeros((4, 64), dtype=torch.int32, device=DEV)
    r2u[1, :10] = torch.arange(101, 111, dtype=torch.int32)
    r2u[2, :6] = torch.arange(201, 207, dtype=torch.int32)
    table[1, :4] = torch.tensor([101, 102, 106, 107], dtype=torch.int32)
    frontier = torch.tensor([0, 7, 0, 0], dtype=torch.int32, device=DEV)
    count = torch.tensor([0, 4, 0, 0], dtype=torch.int32, device=DEV)
    out = torch.full((32,), -1, dtype=torch.int64, device=DEV)
    indptr = torch.zeros(5, dtype=torch.int32, device=DEV)
    tokens = torch.zeros(2, dtype=torch.int32, device=DEV)
    K().fill(table, r2u, frontier, count, torch.tensor([1, 2], device=DEV),
             torch.tensor([10, 6], device=DEV), 1, indptr, out, tokens)
    assert indptr[:3].tolist() == [0, 7, 13]
    assert out[:13].tolist() == [101, 102, 106, 107, 108, 109, 110, 201, 202, 203, 204, 205, 206]
    assert tokens.tolist() == [7, 6]


@pytest.mark.parametrize("page", [1, 16])
def test_fill_random_vs_oracle(page):
    rng = np.random.default_rng(3)
    rows, width = 40, 512
    table = rng.integers(1, 10000, (rows, width)).astype(np.int32)
    r2u = rng.integers(1, 10000, (rows, width)).astype(np.int32)
    frontier = (rng.integers(0, 8, rows) * (128 // page if page > 1 else 128)).astype(np.int32)
    count = rng.integers(0, 100, rows).astype(np.int32)
    bsel = rng.permutation(rows)[:33].astype(np.int64)
    lens = np.array([frontier[r] * page + rng.integers(1, 300) for r in bsel], np.int64)
    ip, idx, tok = oracle.fill(table, r2u, frontier, count, bsel, lens, page)
    dt = lambda a: torch.from_numpy(a).to(DEV)
    indptr = torch.zeros(len(bsel) + 1, dtype=torch.int32, device=DEV)
    out = torch.full((len(idx) + 5,), -7, dtype=torch.int32, device=DEV)
    tokens = torch.zeros(len(bsel), dtype=torch.int32, device=DEV)
    err = K().error_word(DEV)
    K().fill(dt(table), dt(r2u), dt(frontier), dt(count), dt(bsel), dt(lens), page, indptr, out,
             tokens, err)
    err_ok(err)
    assert indptr.cpu().numpy().tolist() == ip.tolist()
    assert out[:len(idx)].cpu().numpy().tolist() == idx.tolist()
    assert tokens.cpu().numpy().tolist() == tok.tolist()


# ---------------------------------------------------------------------- decode
def _decode_case(lengths, G, page, modes, seed, scattered=True):
    """Random paged decode batch; returns numpy inputs for both implementations."""
    rng = np.random.default_rng(seed)
    H = 8 * G
    units_per = [(n + page - 1) // page for n in lengths]
    units = sum(units_per) + 3
    kp = sc.bf16_bits(rng.standard_normal((units, G, page, sc.D), dtype=np.float32))
    vp = sc.bf16_bits(rng.standard_normal((units, G, page, sc.D), dtype=np.float32))
    q = sc.bf16_bits(rng.standard_normal((len(lengths), H, sc.D), dtype=np.float32))
    sinks = sc.bits_to_f32(sc.bf16_bits(rng.standard_normal(H, dtype=np.float32)))
    order = (rng.permutation(units - 1) + 1) if scattered else np.arange(1, units)
    indices = order[:sum(units_per)].astype(np.int32)
    indptr = np.concatenate([[0], np.cumsum(units_per)]).astype(np.int32)
    tokens = np.array(lengths, np.int32)
    return dict(kp=kp, vp=vp, q=q, sinks=sinks, indices=indices, indptr=indptr, tokens=tokens,
                modes=np.array(modes, np.int32), H=H, G=G, page=page, units=units,
                scores0=rng.random((G, units), dtype=np.float32))


def _run_decode_gpu(c, scale, zero_new, out_f32=True, score_flags=3):
    kern = K()
    scores = torch.from_numpy(c["scores0"].copy()).to(DEV)
    err = kern.error_word(DEV)
    lse = torch.zeros((len(c["tokens"]), c["H"]), dtype=torch.float32, device=DEV)
    dt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    out = kern.decode_attn_score(
        t16(c["q"]), t16(c["kp"]), t16(c["vp"]), dt(c["indptr"]), dt(c["indices"]), dt(c["tokens"]),
        scale, c["page"], sinks=dt(c["sinks"]), mode_of_row=dt(c["modes"]), rows=None, scores=scores,
        zero_new=zero_new, out_f32=out_f32, lse=lse, score_flags=score_flags, err=err)
    err_ok(err)
    return out.float().cpu().numpy(), scores.cpu().numpy(), lse.cpu().numpy()


def _run_decode_oracle(c, scale, zero_new):
    scores = c["scores0"].copy()
    out, lse = oracle.decode(c["q"], c["kp"], c["vp"], c["indptr"], c["indices"], c["tokens"],
                             c["sinks"], c["modes"], scale, c["page"], scores, zero_new=zero_new)
    return out, scores, lse


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_decode_reference_golden_token_mode():
    """The reference's decode-score scenario (test_sglang_evict.py:48-78) at page 1."""
    z = np.load(GOLD / "decode.npz")
    d = sc.decode_setup()
    kern = K()
    dt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    kp = t16(d["keys"].reshape(-1, sc.G, 1, sc.D))
    vp = t16(d["values"].reshape(-1, sc.G, 1, sc.D))
    for mode in (1, 2):
        scores = torch.zeros((sc.G, d["slots"]), dtype=torch.float32, device=DEV)
        err = kern.error_word(DEV)
        out = kern.decode_attn_score(
            t16(d["q"]), kp, vp, dt(d["indptr"]), dt(d["perm"]), dt(np.array(sc.DECODE_LENGTHS, np.int32)),
            d["scale"], 1, sinks=dt(sc.bits_to_f32(d["sinks"])), mode_of_row=dt(np.full(3, mode, np.int32)),
            scores=scores, zero_new=False, out_f32=True, err=err)
        err_ok(err)
        o = out.cpu().numpy()
        s = scores.cpu().numpy()
        for i in range(3):
            sl = d["perm"][d["indptr"][i]:d["indptr"][i + 1]]
            # the reference test's tolerance for scores (test_sglang_evict.py:78)
            np.testing.assert_allclose(s[:, sl], z[f"seq{i}_{'sum' if mode == 1 else 'max'}"],
                                       rtol=2e-3, atol=1e-6)
            assert _rel(o[i], z[f"seq{i}_out"]) < 1e-3


@pytest.mark.parametrize("G", [8, 4, 2, 1])
def test_decode_paged_vs_oracle(G):
    lengths = [1, 15, 16, 17, 33, 255, 1000, 3001, 64, 4097]
    modes = [1, 2, 0, 1, 2, 1, 1, 2, 0, 1]
    c = _decode_case(lengths, G, 16, modes, seed=G)
    o_g, s_g, l_g = _run_decode_gpu(c, 0.125, zero_new=True)
    o_c, s_c, l_c = _run_decode_oracle(c, 0.125, zero_new=True)
    for i in range(len(lengths)):
        assert _rel(o_g[i], o_c[i]) < 1e-3, (i, _rel(o_g[i], o_c[i]))
    np.testing.assert_allclose(l_g, l_c, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(s_g, s_c, rtol=1e-3, atol=1e-6)


@pytest.mark.parametrize("G,page,mode", [(8, 16, 1), (8, 16, 2), (1, 16, 1), (2, 16, 2), (8, 1, 1)])
def test_decode_batch1_long_sequence_vs_oracle(G, page, mode):
    """One sequence spread over every attention CTA (config 4's decode shape):
    the combine splits each KV head's output merges and page scoring into
    chunks, and at one KV head per GPU merges more slots than it has threads."""
    c = _decode_case([28_700], G, page, [mode], seed=40 + G + page + mode)
    o_g, s_g, l_g = _run_decode_gpu(c, 0.125, zero_new=True)
    o_c, s_c, l_c = _run_decode_oracle(c, 0.125, zero_new=True)
    assert _rel(o_g[0], o_c[0]) < 1e-3
    np.testing.assert_allclose(l_g, l_c, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(s_g, s_c, rtol=1e-3, atol=1e-6)


@pytest.mark.parametrize("G,page,n", [(8, 16, 40), (2, 16, 90), (1, 16, 160), (8, 1, 40)])
def test_decode_large_batch_vs_oracle(G, page, n):
    """Batches with at least as many (sequence, KV head) pairs as attention
    CTAs (the combine's one-slot, 64-register variant) at 8, 2 and 1 KV heads
    and page size 1: ragged lengths, some spanning several CTAs, an empty and
    a one-token sequence."""
    rng = np.random.default_rng(70 + G + page)
    lengths = rng.integers(1, 2500 if page == 16 else 900, n).tolist()
    lengths[3], lengths[7], lengths[11] = 0, 1, 9000 if page == 16 else 3000
    modes = rng.integers(0, 3, n).tolist()
    c = _decode_case(lengths, G, page, modes, seed=70 + G + page)
    o_g, s_g, l_g = _run_decode_gpu(c, 0.125, zero_new=True)
    o_c, s_c, l_c = _run_decode_oracle(c, 0.125, zero_new=True)
    for i in range(n):
        assert _rel(o_g[i], o_c[i]) < 1e-3, (i, _rel(o_g[i], o_c[i]))
    np.testing.assert_allclose(l_g, l_c, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(s_g, s_c, rtol=1e-3, atol=1e-6)


def test_decode_token_mode_vs_oracle():
    lengths = [1, 2, 37, 1500, 3001, 513]
    c = _decode_case(lengths, 8, 1, [1, 2, 1, 2, 1, 0], seed=11)
    o_g, s_g, l_g = _run_decode_gpu(c, 0.125, zero_new=True)
    o_c, s_c, l_c = _run_decode_oracle(c, 0.125, zero_new=True)
    for i in range(len(lengths)):
        assert _rel(o_g[i], o_c[i]) < 1e-3
    np.testing.assert_allclose(s_g, s_c, rtol=1e-3, atol=1e-6)


def test_decode_bf16_output_and_many_sequences():
    rng = np.random.default_rng(21)
    lengths = rng.integers(1, 9000, 64).tolist()
    modes = rng.integers(0, 3, 64).tolist()
    c = _decode_case(lengths, 8, 16, modes, seed=21)
    o_g, s_g, _ = _run_decode_gpu(c, 0.125, zero_new=True, out_f32=False)
    o_c, s_c, _ = _run_decode_oracle(c, 0.125, zero_new=True)
    for i in range(len(lengths)):
        assert _rel(o_g[i], o_c[i]) < 5e-3  # bf16 rounding of the output
    np.testing.assert_allclose(s_g, s_c, rtol=1e-3, atol=1e-6)


def test_decode_without_score_workspace_flags_mode_error():
    c = _decode_case([40, 50], 8, 16, [1, 2], seed=5)
    kern = K()
    dt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    err = kern.error_word(DEV)
    scores = torch.from_numpy(c["scores0"].copy()).to(DEV)
    kern.decode_attn_score(t16(c["q"]), t16(c["kp"]), t16(c["vp"]), dt(c["indptr"]), dt(c["indices"]),
                           dt(c["tokens"]), 0.125, 16, sinks=dt(c["sinks"]),
                           mode_of_row=dt(c["modes"]), scores=scores, score_flags=0, err=err)
    torch.cuda.synchronize()
    from cache_eviction_b200 import capi
    assert int(err.item()) & capi.CE_EW_MODE
    np.testing.assert_array_equal(scores.cpu().numpy(), c["scores0"])


# ---------------------------------------------------------------------- choose
@pytest.mark.parametrize("i", range(len(sc.choose_cases())))
def test_choose_reference_golden(i):
    c = sc.choose_cases()[i]
    z = np.load(GOLD / "choose.npz")
    L, G, N = c["pos"].shape
    kern = K()
    row = dict(n=c["n"], budget=c["budget"], prefix=c["prefix"], recent=c["recent"],
               cursor=c["cursor"], policy=c["name"], seed=c.get("seed", 0))
    score = None
    if c["score"] is not None:
        a = c["score"].reshape(1, L * G, N)
        score = torch.from_numpy(a.astype(np.float32) if c["name"] == "h2o_global_2048" else a).to(DEV)
    pos = torch.from_numpy(c["pos"].reshape(1, L * G, N).astype(np.int32)).to(DEV)
    err = kern.error_word(DEV)
    kept, status, pcount = kern.choose(pos, score, kern.row_params([row], DEV), L, G, max_n=c["n"] + 1,
                                       err=err)
    torch.cuda.synchronize()
    assert int(status[0]) == int(z[f"case{i}_status"])
    if int(status[0]) == 0:
        err_ok(err)
        want = z[f"case{i}_kept"]
        k = want.shape[-1]
        got = np.sort(kept[0, :, :k].cpu().numpy(), -1).reshape(L, G, k)
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("policy", ["h2o_global_2048", "head_sum_2048", "random_2048",
                                    "random_reservoir_2048", "prefix_sliding_2048"])
def test_choose_config5_vs_oracle(policy):
    """Selection microbench shape: 32 sequences x 8 KV heads x 4096 pages, lognormal(0, 2)."""
    rng = np.random.default_rng(5)
    P, G, N = 32, 8, 4096
    pos = np.broadcast_to(np.arange(N, dtype=np.int32), (P, G, N)).copy()
    if policy == "random_2048":
        score = rng.random((P, G, N))
    else:
        score = rng.lognormal(0.0, 2.0, (P, G, N)).astype(np.float32)
    kern = K()
    for budget_tokens in (2048, 4096, 8192, 16384, 32768):
        b = budget_tokens // 16
        pre, rec = b // 4, (3 * b // 4 if policy == "prefix_sliding_2048" else b // 4)
        rows = [dict(n=N, budget=b, prefix=pre, recent=rec, cursor=None, policy=policy, seed=9 + i)
                for i in range(P)]
        kept_c, st_c, pc_c = oracle.choose(pos, score, oracle.row_params(rows), 1, G,
                                           score_is_f32=score.dtype == np.float32)
        sc_t = torch.from_numpy(score).to(DEV)
        kept_g, st_g, pc_g = kern.choose(torch.from_numpy(pos).to(DEV), sc_t,
                                         kern.row_params(rows, DEV), 1, G, max_n=N)
        torch.cuda.synchronize()
        assert st_g.cpu().numpy().tolist() == st_c.tolist()
        k = min(b, N) if policy != "prefix_sliding_2048" else int(pc_c[0])
        np.testing.assert_array_equal(kept_g[:, :, :k].cpu().numpy(), kept_c[:, :, :k])


def test_reservoir_reference_golden():
    z = np.load(GOLD / "reservoir.npz")
    pos = torch.arange(128, dtype=torch.int32, device=DEV).expand(2, 8, -1).contiguous()
    for key in z.files:
        if not key.startswith("seed_"):
            continue
        got = K().reservoir_scores53(pos, int(key[5:])).cpu().numpy().astype(np.uint64)
        np.testing.assert_array_equal(got, z[key])


# -------------------------------------------------------------------- boundary
def _gpu_state(state, kl, vl):
    dt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    g = {k: dt(v) for k, v in state.items()}
    g["k"] = [t16(a) for a in kl]
    g["v"] = [t16(a) for a in vl]
    kern = K()
    g["kp"] = kern.layer_pointers(g["k"], DEV)
    g["vp"] = kern.layer_pointers(g["v"], DEV)
    g["marks"] = torch.zeros(g["scores"].shape[2], dtype=torch.int32, device=DEV)
    return g


def _gpu_boundary(g, rows, params, max_cols, max_n, live, epoch, uniforms=None, swa=None,
                  hazard_bytes=256 << 20, page=1, max_width=0, record=None):
    kern = K()
    err = kern.error_word(DEV)
    res, freed = kern.boundary(g["table"], g["r2u"], g["frontier"], g["count"], g["pos"], g["scores"],
                               g["kp"], g["vp"], sc.G, page,
                               torch.tensor(rows, dtype=torch.int32, device=DEV),
                               kern.row_params(params, DEV), max_cols, max_n, live, marks=g["marks"],
                               epoch=epoch, uniforms=uniforms, swa=swa, hazard_bytes=hazard_bytes,
                               err=err, max_width=max_width, record=record)
    torch.cuda.synchronize()
    return res.cpu().numpy(), freed.cpu().numpy(), int(err.item())


def _record_buffers(rows, L, G, max_cols):
    return (torch.full((rows * L * G, max_cols), -1, dtype=torch.int32, device=DEV),
            torch.full((rows * L * G,), -1, dtype=torch.int32, device=DEV))


def _record_of_row(record, r, L, G):
    """(deltas uint32 concatenated over layer-major heads, counts) of row r."""
    delta, counts = record[0].cpu().numpy().view(np.uint32), record[1].cpu().numpy()
    segs = range(r * L * G, (r + 1) * L * G)
    return (np.concatenate([delta[s, :counts[s]] for s in segs]), counts[r * L * G:(r + 1) * L * G])


RECORD_NAMES = ("head_sum_2048", "random_reservoir_2048", "random_2048", "prefix_sliding_2048")


@pytest.mark.parametrize("name", RECORD_NAMES)
def test_boundary_record_reference_golden(name):
    """Retention records of the reference test's scenario (record=True),
    bit for bit against the records the reference itself wrote."""
    rec = np.load(GOLD / "records.npz")
    setup = sc.boundary_setup()
    state, kl, vl = boundary_state(setup)
    g = _gpu_state(state, kl, vl)
    max_cols = 4096
    for k, b in enumerate((2048, 4096)):
        N = int(g["count"][1]) + b - int(g["frontier"][1])
        uni = None
        if name == "random_2048":
            u = np.zeros((1, 2, sc.G, max_cols))
            u[0, :, :, :N] = sc.random_uniforms(4, b, (2, sc.G, N))
            uni = torch.from_numpy(u).to(DEV)
        record = _record_buffers(1, 2, sc.G, max_cols)
        res, _, err = _gpu_boundary(g, [1], [boundary_row(name, b)], max_cols, setup["n"] + 1, True,
                                    epoch=k + 1, uniforms=uni, record=record)
        assert err == 0 and res[0, 0] == 0, (res, hex(err))
        d, c = _record_of_row(record, 0, 2, sc.G)
        np.testing.assert_array_equal(c, rec[f"{name}_b{k}_evicted_counts"])
        np.testing.assert_array_equal(d, rec[f"{name}_b{k}_evicted_delta"])


@pytest.mark.parametrize("name,kind", sc.BOUNDARY_NAMES)
def test_boundary_reference_golden(name, kind):
    z = np.load(GOLD / "boundary.npz")
    setup = sc.boundary_setup()
    state, kl, vl = boundary_state(setup)
    g = _gpu_state(state, kl, vl)
    key = f"{name}_{kind}"
    max_cols = 4096
    for k, b in enumerate((2048, 4096)):
        N = int(g["count"][1]) + b - int(g["frontier"][1])
        uni = None
        if name == "random_2048":
            u = np.zeros((1, 2, sc.G, max_cols))
            u[0, :, :, :N] = sc.random_uniforms(4, b, (2, sc.G, N))
            uni = torch.from_numpy(u).to(DEV)
        # hazard budget of one layer forces the two-group path on the second boundary
        res, freed, err = _gpu_boundary(g, [1], [boundary_row(name, b)], max_cols, setup["n"] + 1,
                                        kind == "live", epoch=k + 1, uniforms=uni,
                                        hazard_bytes=1 if k else 256 << 20)
        assert err == 0 and res[0, 0] == 0, (res, hex(err))
        cnt = int(g["count"][1])
        assert cnt == res[0, 2]
        np.testing.assert_array_equal(g["table"][1, :cnt].cpu().numpy(), z[f"{key}_b{k}_table"])
        np.testing.assert_array_equal(g["pos"][1, :, :, :cnt].cpu().numpy(), z[f"{key}_b{k}_pos"])
        assert int(g["frontier"][1]) == int(z[f"{key}_b{k}_frontier"])
        np.testing.assert_array_equal(g["r2u"][1, :setup["n"]].cpu().numpy(), z[f"{key}_b{k}_r2u"])
        if kind == "live":
            prev = 0 if k == 0 else len(z[f"{key}_b0_freed"])
            np.testing.assert_array_equal(freed[0, :res[0, 3]], z[f"{key}_b{k}_freed"][prev:])
    k16 = lambda t: t.view(torch.int16).cpu().numpy()
    assert [sha16(k16(a)) for a in g["k"]] == list(z[f"{key}_keys_sha"])
    assert [sha16(k16(a)) for a in g["v"]] == list(z[f"{key}_values_sha"])
    assert sha_bytes(g["scores"].cpu().numpy()) == str(z[f"{key}_scores_sha"][0])


def _paged_state(rng, rows, L, G, page, units, width, pos_cap):
    kl = [sc.bf16_bits(rng.standard_normal((units, G, page, sc.D), dtype=np.float32)) for _ in range(L)]
    vl = [sc.bf16_bits(rng.standard_normal((units, G, page, sc.D), dtype=np.float32)) for _ in range(L)]
    state = {"table": np.zeros((rows, width), np.int32), "r2u": np.zeros((rows, width), np.int32),
             "frontier": np.zeros(rows, np.int32), "count": np.zeros(rows, np.int32),
             "pos": np.zeros((rows, L, G, pos_cap), np.int32),
             "scores": rng.lognormal(0, 2, (L, G, units)).astype(np.float32)}
    return state, kl, vl


@pytest.mark.parametrize("policy", ["head_sum_2048", "h2o_global_2048", "random_reservoir_2048",
                                    "random_2048", "prefix_sliding_2048", "head_max_sum_2048"])
def test_boundary_paged_multirow_vs_oracle(policy):
    """Three rows at page 16, three successive boundaries each, against the oracle."""
    rng = np.random.default_rng(17)
    rows, L, G, page = 3, 3, 8, 16
    units, width, pos_cap = 2000, 1024, 512
    state, kl, vl = _paged_state(rng, rows, L, G, page, units, width, pos_cap)
    perm = rng.permutation(units - 1) + 1
    for r in range(rows):
        state["r2u"][r, :500] = perm[r * 500:(r + 1) * 500]
    g = _gpu_state(state, kl, vl)
    budgets = [64, 128, 96]  # pages
    epoch = 0
    for k, n in enumerate((128, 256, 384)):
        params = []
        for r in range(rows):
            b = budgets[r]
            rec = b - b // 4 if policy == "prefix_sliding_2048" else b // 4
            params.append(dict(n=n, budget=b, prefix=b // 4, recent=rec, cursor=n - 13 + r,
                               policy=policy, seed=100 + r))
        max_cols = max(int(state["count"][r]) + n - int(state["frontier"][r]) for r in range(rows))
        uni = None
        if policy == "random_2048":
            u = rng.random((rows, L, G, max_cols))
            uni = u
        before = {k: state[k].copy() for k in ("pos", "count", "frontier")}
        res_c, fr_c = oracle.boundary(state, kl, vl, list(range(rows)), oracle.row_params(params),
                                      max_cols, live=True, uniforms=uni)
        epoch += 1
        record = _record_buffers(rows, L, G, max_cols)
        res_g, fr_g, err = _gpu_boundary(g, list(range(rows)), params, max_cols, n + 1, True, epoch,
                                         uniforms=None if uni is None else torch.from_numpy(uni).to(DEV),
                                         page=page, max_width=max(budgets), hazard_bytes=1, record=record)
        assert err == 0, hex(err)
        np.testing.assert_array_equal(res_g, res_c)
        for r in range(rows):
            d, c = _record_of_row(record, r, L, G)
            if res_c[r, 0] != 0:
                assert not c.any()
                continue
            dw, cw = oracle.retention_record(before["pos"][r], int(before["count"][r]),
                                             int(before["frontier"][r]), n, state["pos"][r],
                                             int(state["count"][r]))
            np.testing.assert_array_equal(c, cw)
            np.testing.assert_array_equal(d, dw)
        for r in range(rows):
            np.testing.assert_array_equal(fr_g[r, :res_c[r, 3]], fr_c[r, :res_c[r, 3]])
        for key in ("table", "r2u", "frontier", "count", "pos", "scores"):
            np.testing.assert_array_equal(g[key].cpu().numpy(), state[key], err_msg=key)
        for l in range(L):
            np.testing.assert_array_equal(g["k"][l].view(torch.int16).cpu().numpy(), kl[l].view(np.int16))
            np.testing.assert_array_equal(g["v"][l].view(torch.int16).cpu().numpy(), vl[l].view(np.int16))


def test_boundary_noop_deferred_and_mismatch():
    rng = np.random.default_rng(2)
    rows, L, G, page = 3, 2, 8, 16
    state, kl, vl = _paged_state(rng, rows, L, G, page, 600, 256, 256)
    for r in range(rows):
        state["r2u"][r, :150] = np.arange(1 + 150 * r, 151 + 150 * r)
    g = _gpu_state(state, kl, vl)
    params = [dict(n=128, budget=200, prefix=8, recent=8, cursor=None, policy="head_sum_2048"),  # noop
              dict(n=128, budget=20, prefix=16, recent=16, cursor=None, policy="head_sum_2048"),  # deferred
              dict(n=128, budget=64, prefix=16, recent=16, cursor=None, policy="head_sum_2048")]
    before = {k: v.clone() for k, v in g.items() if isinstance(v, torch.Tensor)}
    res, _, err = _gpu_boundary(g, [0, 1, 2], params, 128, 129, True, 1, page=page)
    res_c, _ = oracle.boundary(state, kl, vl, [0, 1, 2], oracle.row_params(params), 128, live=True)
    np.testing.assert_array_equal(res, res_c)
    assert res[0, 0] == 1 and res[1, 0] == 2 and res[2, 0] == 0
    for r in (0, 1):
        assert torch.equal(g["table"][r], before["table"][r])
        assert int(g["frontier"][r]) == 0


def test_boundary_random_row_without_uniforms_is_rejected():
    """A random row needs the caller's uniforms: without them the row gets
    status 6 and CE_EW_SHAPE, and nothing of it changes."""
    rng = np.random.default_rng(5)
    state, kl, vl = _paged_state(rng, 2, 1, 8, 16, 400, 256, 256)
    for r in range(2):
        state["r2u"][r, :150] = np.arange(1 + 150 * r, 151 + 150 * r)
    g = _gpu_state(state, kl, vl)
    params = [dict(n=128, budget=64, prefix=16, recent=16, cursor=None, policy="random_2048"),
              dict(n=128, budget=64, prefix=16, recent=16, cursor=None, policy="head_sum_2048")]
    before = {k: v.clone() for k, v in g.items() if isinstance(v, torch.Tensor)}
    res, _, err = _gpu_boundary(g, [0, 1], params, 128, 129, True, 1, page=16)
    assert res[0, 0] == 6 and res[1, 0] == 0, res
    from cache_eviction_b200 import capi
    assert err & capi.CE_EW_SHAPE
    for key in ("table", "r2u", "pos", "frontier", "count"):
        assert torch.equal(g[key][0], before[key][0]), key


def test_boundary_sliding_window_guard_error():
    rng = np.random.default_rng(8)
    state, kl, vl = _paged_state(rng, 1, 1, 8, 16, 400, 256, 256)
    state["r2u"][0, :128] = np.arange(1, 129)
    g = _gpu_state(state, kl, vl)
    swa = torch.zeros(400, dtype=torch.int64, device=DEV)
    swa[100] = 9  # unit 100 (column 99) is a leftover that still holds a sliding-window entry
    params = [dict(n=128, budget=32, prefix=8, recent=8, cursor=None, policy="head_sum_2048")]
    res, _, err = _gpu_boundary(g, [0], params, 128, 129, True, 1, swa=swa, page=16)
    res_c, _ = oracle.boundary(state, kl, vl, [0], oracle.row_params(params), 128, live=True,
                               swa=swa.cpu().numpy())
    assert res[0, 0] == 5 and res_c[0, 0] == 5
    from cache_eviction_b200 import capi
    assert err & capi.CE_EW_SWA
