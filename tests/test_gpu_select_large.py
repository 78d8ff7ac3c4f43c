"""Selection on large segments (4,097-65,536 columns per (row, layer, KV head):
the page-size-1 stress shapes) through the C ABI, bit for bit against the CPU
oracle: kept sets and statuses for ce_choose; results, tables, positions,
scores and pools for ce_boundary.  Covers fresh and compacted positions, exact
ties at the threshold (position decides), heavy ties (the candidate buffer
overflows and the general path takes over), f64 and f32 uniforms, reservoir
draws, H2O global and prefix-sliding rows."""
import numpy as np
import pytest
import torch

from golden import scenarios as sc
from oracle import oracle

pytestmark = pytest.mark.gpu
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


def _positions(rng, P, G, N, compacted):
    """Fresh columns (position = column) or a compacted layout: every head
    keeps the same first and last F positions (so protected counts agree
    across heads, as the reference requires) and its own random middle."""
    if not compacted:
        return np.broadcast_to(np.arange(N, dtype=np.int32), (P, G, N)).copy(), N
    n = 2 * N
    F = min(N // 2 - 1, 3 * N // 8 + 64)
    pos = np.empty((P, G, N), np.int32)
    for r in range(P):
        for g in range(G):
            mid = np.sort(rng.choice(np.arange(F, n - F), N - 2 * F, replace=False))
            pos[r, g] = np.concatenate([np.arange(F), mid, np.arange(n - F, n)])
    return pos, n


def _scores(rng, kind, shape):
    if kind == "lognormal":
        return rng.lognormal(0.0, 2.0, shape).astype(np.float32)
    if kind == "coarse":      # few distinct values: exact ties decide by position
        return np.round(rng.lognormal(0.0, 1.0, shape), 1).astype(np.float32)
    if kind == "equal":       # one value: every column is a candidate (overflow path)
        return np.full(shape, 0.5, np.float32)
    if kind == "u64":
        return rng.random(shape)
    if kind == "u32":
        return rng.random(shape).astype(np.float32)
    raise ValueError(kind)


CASES = [
    ("head_sum_2048", "lognormal", False),
    ("head_sum_2048", "coarse", True),
    ("head_sum_2048", "equal", False),
    ("h2o_global_2048", "lognormal", True),
    ("random_2048", "u64", False),
    ("random_2048", "u32", True),
    ("random_reservoir_2048", None, True),
    ("prefix_sliding_2048", None, False),
]


# 5000: one tile; 20000: three tiles, the last partial; 12347: no 16-byte
# quads (single-column loads); 65536: eight full tiles
@pytest.mark.parametrize("N", [5000, 12347, 20000, 65536])
@pytest.mark.parametrize("policy,skind,compacted", CASES)
def test_choose_large_vs_oracle(policy, skind, compacted, N):
    rng = np.random.default_rng(N + len(policy))
    P, G = 3, 8
    pos, n = _positions(rng, P, G, N, compacted)
    score = None if skind is None else _scores(rng, skind, (P, G, N))
    kern = K()
    for budget in (N // 16, N // 2 + 3):
        pre = budget // 4
        rec = budget - pre if policy == "prefix_sliding_2048" else budget // 4
        rows = [dict(n=n, budget=budget, prefix=pre, recent=rec, cursor=n - 7 * (r + 1) if r else None,
                     policy=policy, seed=31 + r) for r in range(P)]
        # prefix_sliding keeps only the protected set; with compacted positions
        # the protected count is what the policy allows
        kept_c, st_c, pc_c = oracle.choose(pos, score, oracle.row_params(rows), 1, G,
                                           score_is_f32=score is not None and score.dtype == np.float32)
        err = kern.error_word(DEV)
        sc_t = None if score is None else torch.from_numpy(score).to(DEV)
        kept_g, st_g, pc_g = kern.choose(torch.from_numpy(pos).to(DEV), sc_t, kern.row_params(rows, DEV),
                                         1, G, max_n=n + 1, err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0, hex(int(err.item()))
        assert st_g.cpu().numpy().tolist() == st_c.tolist()
        for r in range(P):
            if int(st_c[r]) != 0:
                continue
            k = budget if policy != "prefix_sliding_2048" else int(pc_c[r])
            np.testing.assert_array_equal(kept_g[r, :, :k].cpu().numpy(), kept_c[r, :, :k],
                                          err_msg=f"row {r} budget {budget}")


def _two_boundaries(policy, rows, L, n0, n1, budgets, seed, hazard_bytes=256 << 20, record=False):
    """Two successive page-size-1 boundaries of `rows` rows (n0 then n1
    positions), the GPU against the oracle after each: results, freed units,
    tables, positions, scores and the K/V pools bit for bit, and with record
    the retention record of every evicted row."""
    rng = np.random.default_rng(seed)
    G, page = 8, 1
    units, width, pos_cap = rows * n1 + 1, n1 + 64, max(budgets)
    # the boundary moves K/V bytes without reading them: any 16-bit patterns do
    kl = [rng.integers(0, 1 << 16, (units, G, page, sc.D), dtype=np.uint16) for _ in range(L)]
    vl = [rng.integers(0, 1 << 16, (units, G, page, sc.D), dtype=np.uint16) for _ in range(L)]
    state = {"table": np.zeros((rows, width), np.int32), "r2u": np.zeros((rows, width), np.int32),
             "frontier": np.zeros(rows, np.int32), "count": np.zeros(rows, np.int32),
             "pos": np.zeros((rows, L, G, pos_cap), np.int32),
             "scores": rng.lognormal(0, 2, (L, G, units)).astype(np.float32)}
    perm = rng.permutation(units - 1) + 1
    for r in range(rows):
        state["r2u"][r, :n1] = perm[r * n1:(r + 1) * n1]
    dt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    g = {k: dt(v) for k, v in state.items()}
    gk, gv = [dt(a.view(np.int16)).view(torch.bfloat16) for a in kl], [dt(a.view(np.int16)).view(torch.bfloat16) for a in vl]
    kern = K()
    kp, vp = kern.layer_pointers(gk, DEV), kern.layer_pointers(gv, DEV)
    marks = torch.zeros(units, dtype=torch.int32, device=DEV)
    for step, n in enumerate((n0, n1)):
        params = []
        for r in range(rows):
            b = budgets[r]
            rec = b - b // 4 if policy == "prefix_sliding_2048" else b // 4
            params.append(dict(n=n, budget=b, prefix=b // 4, recent=rec, cursor=n - 11, policy=policy,
                               seed=7 + r))
        max_cols = max(int(state["count"][r]) + n - int(state["frontier"][r]) for r in range(rows))
        assert max_cols > 4096
        uni = rng.random((rows, L, G, max_cols)) if policy == "random_2048" else None
        before = {k: state[k].copy() for k in ("pos", "count", "frontier")}
        rec = None
        if record:
            rec = (torch.full((rows * L * G, max_cols), -1, dtype=torch.int32, device=DEV),
                   torch.full((rows * L * G,), -1, dtype=torch.int32, device=DEV))
        res_c, fr_c = oracle.boundary(state, kl, vl, list(range(rows)), oracle.row_params(params),
                                      max_cols, live=True, uniforms=uni)
        err = kern.error_word(DEV)
        res_g, fr_g = kern.boundary(g["table"], g["r2u"], g["frontier"], g["count"], g["pos"], g["scores"],
                                    kp, vp, G, page, torch.arange(rows, dtype=torch.int32, device=DEV),
                                    kern.row_params(params, DEV), max_cols, n + 1, True, marks=marks,
                                    epoch=step + 1, uniforms=None if uni is None else dt(uni), err=err,
                                    max_width=max(budgets), hazard_bytes=hazard_bytes, record=rec)
        torch.cuda.synchronize()
        assert int(err.item()) == 0, hex(int(err.item()))
        np.testing.assert_array_equal(res_g.cpu().numpy(), res_c)
        for r in range(rows):
            np.testing.assert_array_equal(fr_g.cpu().numpy()[r, :res_c[r, 3]], fr_c[r, :res_c[r, 3]])
        for key in ("table", "r2u", "frontier", "count", "pos", "scores"):
            np.testing.assert_array_equal(g[key].cpu().numpy(), state[key], err_msg=key)
        for l in range(L):
            np.testing.assert_array_equal(gk[l].view(torch.int16).cpu().numpy(), kl[l].view(np.int16))
            np.testing.assert_array_equal(gv[l].view(torch.int16).cpu().numpy(), vl[l].view(np.int16))
        if record:
            delta, counts = rec[0].cpu().numpy().view(np.uint32), rec[1].cpu().numpy()
            for r in range(rows):
                segs = range(r * L * G, (r + 1) * L * G)
                if res_c[r, 0] != 0:
                    assert not counts[r * L * G:(r + 1) * L * G].any()
                    continue
                dw, cw = oracle.retention_record(before["pos"][r], int(before["count"][r]),
                                                 int(before["frontier"][r]), n, state["pos"][r],
                                                 int(state["count"][r]))
                np.testing.assert_array_equal(counts[r * L * G:(r + 1) * L * G], cw)
                np.testing.assert_array_equal(np.concatenate([delta[q, :counts[q]] for q in segs]), dw)


@pytest.mark.parametrize("policy", ["head_sum_2048", "h2o_global_2048", "random_reservoir_2048",
                                    "random_2048", "prefix_sliding_2048"])
def test_boundary_large_segments_vs_oracle(policy):
    """Two rows at page size 1, two successive boundaries with 5,000-8,000
    columns per (row, layer, head), against the oracle."""
    _two_boundaries(policy, rows=2, L=2, n0=8000, n1=10048, budgets=[3000, 2000], seed=41)


@pytest.mark.parametrize("policy", ["head_sum_2048", "h2o_global_2048", "random_2048"])
def test_boundary_page1_full_width_vs_oracle(policy):
    """Four rows at page size 1 with 65,536 columns per (row, head) -- the
    largest segment of the shared-memory path -- and budgets of 8K-40K
    tokens, so the candidate ranking, the packing and the compaction all run
    over many tiles and chunks; then a second boundary over the kept columns
    plus 9,000 new ones, with the hazard workspace forcing one row per copy
    launch.  The GPU against the oracle, bit for bit (and the retention
    record for head_sum)."""
    _two_boundaries(policy, rows=4, L=1, n0=65536, n1=74536, budgets=[40000, 8192, 20000, 32768], seed=43,
                    hazard_bytes=1, record=policy == "head_sum_2048")


@pytest.mark.parametrize("N", [5000, 65536])
@pytest.mark.parametrize("policy", ["head_sum_2048", "random_2048"])
def test_choose_large_unordered_positions_vs_oracle(policy, N):
    """Positions that do not ascend with the column index (each head's row a
    permutation of the same positions, so protected counts agree): the
    kept set must still come out ranked by position, through the bitmap
    ranking rather than the column-order one."""
    rng = np.random.default_rng(N + 7)
    P, G = 2, 8
    pos = np.stack([np.stack([rng.permutation(N).astype(np.int32) for _ in range(G)]) for _ in range(P)])
    pos[:, :, :4] = np.sort(pos[:, :, :4], -1)[..., ::-1]   # the first quad itself descends
    score = _scores(rng, "lognormal" if policy == "head_sum_2048" else "u64", (P, G, N))
    kern = K()
    budget = N // 3
    rows = [dict(n=N, budget=budget, prefix=budget // 4, recent=budget // 4, cursor=None, policy=policy,
                 seed=3 + r) for r in range(P)]
    kept_c, st_c, _ = oracle.choose(pos, score, oracle.row_params(rows), 1, G,
                                    score_is_f32=score.dtype == np.float32)
    err = kern.error_word(DEV)
    kept_g, st_g, _ = kern.choose(torch.from_numpy(pos).to(DEV), torch.from_numpy(score).to(DEV),
                                  kern.row_params(rows, DEV), 1, G, max_n=N + 1, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert st_g.cpu().numpy().tolist() == st_c.tolist() == [0] * P
    np.testing.assert_array_equal(kept_g[:, :, :budget].cpu().numpy(), kept_c[:, :, :budget])
