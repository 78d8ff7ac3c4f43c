"""Host bookkeeping of the ragged decode engine, on CPU (no kernels run):
due() with its skip-ahead counter against a plain scan of every row, over
advances, boundaries taken, rows added and retired; and bench.py's
per-step resident counter against a sum over the rows."""
import random
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from cache_eviction_b200.engine import RaggedDecodeEngine, Row  # noqa: E402
from cache_eviction_b200.policy import INTERVAL, EvictionConfig, sweep_split  # noqa: E402


def _engine():
    return RaggedDecodeEngine(layers=1, q_heads=64, kv_heads=8, page_size=16, pool_units=64, max_rows=16,
                              r2u_width=64, pos_cap=64, device="cpu", alloc_pools=False)


def _cfg(seed):
    p, r = sweep_split(2048, "head_sum_2048")
    return EvictionConfig("head_sum_2048", 2048, p, r, seed=seed)


def _scan(eng):
    return [r for r in eng.active if eng.rows[r].cfg is not None
            and eng.rows[r].n % INTERVAL == 0 and eng.rows[r].n > eng.rows[r].last_boundary]


def _add(eng, row, n, cfg):
    eng.rows[row] = Row(cfg=cfg, n=n, last_boundary=(n // INTERVAL) * INTERVAL)
    eng.active.append(row)
    eng._due_in = None


def test_due_skip_ahead_matches_full_scan():
    rnd = random.Random(3)
    eng = _engine()
    eng.free_top = 10 ** 9
    for row in range(10):
        _add(eng, row, rnd.randrange(2000, 9000), _cfg(row) if row % 3 else None)
    for step in range(6000):
        due = eng.due()
        assert due == _scan(eng), step
        for r in due:                      # what run_boundaries records
            eng.rows[r].last_boundary = eng.rows[r].n
        if due:
            eng._due_in = None
        if step % 997 == 5:                # a row leaves, another arrives
            gone = eng.active.pop(0)
            eng.rows.pop(gone)
            eng._due_in = None
            _add(eng, 100 + step, rnd.randrange(2000, 9000), _cfg(step))
        eng.advance_host()


def test_resident_counter_matches_row_sums():
    import bench

    class Eng:
        P = 16

    eng = Eng()
    eng.rows, eng.active, eng.boundary_ms = {}, [], []
    rnd = random.Random(5)
    for r in range(20):
        eng.rows[r] = Row(cfg=_cfg(r) if r % 2 else None, n=rnd.randrange(100, 5000),
                          count=rnd.randrange(0, 50), frontier=rnd.randrange(0, 5))
        eng.active.append(r)
    counter = bench.ResidentCounter(eng)
    for step in range(300):
        if step % 50 == 7:                 # a boundary batch changes some rows
            eng.rows[1].count, eng.rows[1].frontier = 40, eng.rows[1].n // 16
            eng.boundary_ms.append(0.1)
        tokens, pages = counter()
        want_t = sum(r.count * 16 + r.n - r.frontier * 16 for r in eng.rows.values())
        want_p = sum(r.count + max(0, -(-r.n // 16) - r.frontier) for r in eng.rows.values()
                     if r.cfg is not None and r.cfg.score_mode)
        assert (tokens, pages) == (want_t, want_p), step
        for r in eng.rows.values():
            r.n += 1


def test_csr_capacity_bound_never_undershoots():
    """_ensure_capacity skips its pass over the rows while a bound on the CSR
    need stays under capacity; the capacity must cover the exact need after
    every call."""
    rnd = random.Random(7)
    eng = _engine()
    eng.free_top = 10 ** 9
    for row in range(12):
        eng.add_row(row, None, rnd.randrange(1, 3000), frontier_units=0, count_units=0)
    for step in range(3000):
        eng.advance_host()
        eng._ensure_capacity(0)
        exact = sum(eng.resident_units(r, 0) for r in eng.active) + 16
        assert eng.kv_indices.numel() >= exact, step


def test_workload_spreads_boundaries_over_the_timed_window():
    """bench.workload(first_boundary_step=W): the evicting rows reach their
    boundaries one by one from step W on, evenly spaced, so a window of K
    timed steps holds ceil(K * E / 2048) of them; contexts stay >= 2,048 and
    move by less than 2,048 tokens."""
    import math
    import bench
    free = bench.workload(64)
    for W in (3, 5, 8):
        specs = bench.workload(64, first_boundary_step=W)
        evicting = [(a, b) for a, b in zip(free, specs) if b["cfg"] is not None]
        E = len(evicting)
        steps = sorted((-b["ctx"]) % INTERVAL for _, b in evicting)
        assert steps[0] == W
        for a, b in evicting:
            assert b["ctx"] >= 2048 and abs(a["ctx"] - b["ctx"]) < INTERVAL
        for K in (1, 20, 64, 512):
            assert sum(W <= s < W + K for s in steps) == math.ceil(K * E / INTERVAL), (W, K)
