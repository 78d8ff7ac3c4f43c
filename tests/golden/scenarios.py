"""Deterministic inputs shared by the fixture generator and the tests.

Everything here is numpy with fixed seeds, so tests/golden/make_golden.py (run
once in a container that has the reference source) and the tests (run anywhere)
rebuild bit-identical inputs; the fixtures then only hold the reference's
outputs.  Shapes follow the reference's own tests
(code/tests/test_sglang_evict.py:19-39, 48-158) at reduced pool sizes.
"""
from __future__ import annotations

import numpy as np

FULL = (1, 3)            # full-attention layers of the fake backend (test_sglang_evict.py:16)
H, G, D = 64, 8, 64      # query heads, KV heads, head dim
BOUNDARY_SLOTS = 6000    # pool slots for the boundary scenario (the reference test uses 20000)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- choose cases
def choose_cases():
    """List of dicts: name, pos [L,G,N] int64, score [L,G,N] float64 or None, n, budget,
    prefix, recent, cursor.  Scores are fp32-representable unless noted."""
    rng = np.random.default_rng(1234)
    cases = []
    L = 2

    def fresh(N):
        return np.broadcast_to(np.arange(N, dtype=np.int64), (L, G, N)).copy()

    def compacted(n, count_prot_prefix, recent_old, middle, tail_from):
        """Per-head positions after an earlier boundary: shared protected prefix and
        old-recent region, per-head middle subsets, then the tail."""
        out = []
        for _ in range(L * G):
            mid = np.sort(rng.choice(np.arange(count_prot_prefix, recent_old[0]), middle, replace=False))
            out.append(np.concatenate([np.arange(count_prot_prefix), recent_old, mid,
                                       np.arange(tail_from, n)]))
        return np.stack(out).reshape(L, G, -1).astype(np.int64)

    N = 600
    s = rng.random((L, G, N), dtype=np.float32).astype(np.float64)
    cases.append(dict(name="head_sum_2048", pos=fresh(N), score=s, n=N, budget=256, prefix=64,
                      recent=64, cursor=None))
    ties = rng.integers(0, 4, (L, G, N)).astype(np.float64)
    cases.append(dict(name="head_max_sum_2048", pos=fresh(N), score=ties, n=N, budget=300,
                      prefix=32, recent=32, cursor=None))
    cases.append(dict(name="head_sum_2048", pos=fresh(N), score=s, n=N, budget=256, prefix=64,
                      recent=64, cursor=N - 100))
    # after a previous boundary at 512: 64 prefix, old recent [448,512), 128 middle each
    pos = compacted(1024, 64, np.arange(448, 512), 128, 512)
    sc = rng.random(pos.shape, dtype=np.float32).astype(np.float64)
    cases.append(dict(name="head_sum_2048", pos=pos, score=sc, n=1024, budget=256, prefix=64,
                      recent=64, cursor=None))
    cases.append(dict(name="random_2048", pos=pos, score=rng.random(pos.shape), n=1024, budget=256,
                      prefix=64, recent=64, cursor=900))
    cases.append(dict(name="random_reservoir_2048", pos=pos, score=None, n=1024, budget=256,
                      prefix=64, recent=64, cursor=None, seed=7))
    cases.append(dict(name="prefix_sliding_2048", pos=fresh(N), score=None, n=N, budget=256,
                      prefix=64, recent=192, cursor=None))
    # signed zeros and exact ties must tie-break by position only
    z = np.where(rng.random((L, G, N)) < 0.5, -0.0, 0.0)
    z[..., ::7] = 1.0
    cases.append(dict(name="head_sum_2048", pos=fresh(N), score=z, n=N, budget=200, prefix=16,
                      recent=16, cursor=None))
    # H2O global: every head ranks the fp32 sum over the layer's KV heads (ascending head order)
    g32 = rng.random((L, G, N), dtype=np.float32)
    gsum = np.zeros((L, N), np.float32)
    for g in range(G):
        gsum = (gsum + g32[:, g]).astype(np.float32)
    cases.append(dict(name="h2o_global_2048", pos=fresh(N), score=g32.astype(np.float64),
                      global_key=np.broadcast_to(gsum[:, None, :], (L, G, N)).astype(np.float64),
                      n=N, budget=256, prefix=64, recent=64, cursor=None))
    # deferred: protection exceeds the budget
    cases.append(dict(name="head_sum_2048", pos=fresh(N), score=s, n=N, budget=100, prefix=64,
                      recent=64, cursor=None))
    # protected counts differ between heads -> error
    bad = compacted(1024, 64, np.arange(448, 512), 128, 512)
    # one head trades a protected recent position for an unprotected unused one
    col = int(np.nonzero(bad[1, 3] == 1000)[0][0])
    unused = np.setdiff1d(np.arange(64, 448), bad[1, 3])
    bad[1, 3, col] = unused[0]
    cases.append(dict(name="head_sum_2048", pos=bad, score=sc, n=1024, budget=256, prefix=64,
                      recent=64, cursor=None))
    return cases


# ------------------------------------------------------------ boundary scenario
def boundary_setup(seed: int = 0):
    """The reference's check_boundaries setup (test_sglang_evict.py:92-107) at
    BOUNDARY_SLOTS slots: pools for the 4 layers, scattered original slots,
    scores on the full layers."""
    rng = np.random.default_rng(seed)
    n = 4096 + 300
    slots = BOUNDARY_SLOTS
    keys = {l: bf16_bits(rng.standard_normal((slots, G, D), dtype=np.float32)) for l in range(4)}
    values = {l: bf16_bits(rng.standard_normal((slots, G, D), dtype=np.float32)) for l in range(4)}
    slot_of = (rng.permutation(slots - 1)[:n] + 1).astype(np.int64)
    score = rng.random((2, G, n), dtype=np.float32)
    return dict(n=n, keys=keys, values=values, slot_of=slot_of, score=score, rows=4,
                width=8192, slots=slots)


BOUNDARY_NAMES = [("head_sum_2048", "live"), ("random_reservoir_2048", "live"),
                  ("prefix_sliding_2048", "live"), ("random_2048", "live"),
                  ("head_max_sum_2048", "replay"), ("random_reservoir_2048", "replay"),
                  ("h2o_global_2048", "live")]


def boundary_cfg(name: str):
    budget = 1024
    prefix = budget // 4
    recent = budget - prefix if name == "prefix_sliding_2048" else budget // 4
    return dict(name=name, budget=budget, prefix=prefix, recent=recent, seed=4)


def random_uniforms(seed: int, n: int, shape):
    """The reference's random_2048 draw (runtime:403-406): a float64 torch.rand
    from a CPU generator seeded (seed*1000003 + n) & 0x7FFFFFFF."""
    import torch
    gen = torch.Generator(device="cpu").manual_seed((seed * 1000003 + n) & 0x7FFFFFFF)
    return torch.rand(shape, generator=gen, dtype=torch.float64).numpy()


# -------------------------------------------------------------- decode scenario
DECODE_LENGTHS = (37, 150, 301)


def decode_setup(seed: int = 5):
    """Three ragged sequences over scattered token slots (the reference's
    test_decode_scores_are_per_kv_head shape, test_sglang_evict.py:48-78, at
    shorter lengths)."""
    rng = np.random.default_rng(seed)
    slots = 1200
    keys = bf16_bits(rng.standard_normal((slots, G, D), dtype=np.float32))
    values = bf16_bits(rng.standard_normal((slots, G, D), dtype=np.float32))
    q = bf16_bits(rng.standard_normal((len(DECODE_LENGTHS), H, D), dtype=np.float32))
    sinks = bf16_bits(rng.standard_normal(H, dtype=np.float32))
    total = sum(DECODE_LENGTHS)
    perm = (rng.permutation(slots - 1)[:total] + 1).astype(np.int32)
    indptr = np.concatenate([[0], np.cumsum(DECODE_LENGTHS)]).astype(np.int32)
    return dict(keys=keys, values=values, q=q, sinks=sinks, perm=perm, indptr=indptr,
                scale=0.125, slots=slots)


# -------------------------------------------------------------- prefill scenario
# (prefix tokens, chunk queries) per entry: a chunk after a prefix, a fresh
# prompt, and a one-query chunk.
PREFILL_ENTRIES = ((150, 70), (0, 90), (333, 1))


def prefill_setup(seed: int = 11):
    """Extend chunks over scattered token slots, scored as _prefill_scores
    does (runtime:327-340): each entry's key list is its prefix slots followed
    by its chunk's new slots."""
    rng = np.random.default_rng(seed)
    slots = 1200
    keys = bf16_bits(rng.standard_normal((slots, G, D), dtype=np.float32))
    total_q = sum(nq for _, nq in PREFILL_ENTRIES)
    q = bf16_bits(rng.standard_normal((total_q, H, D), dtype=np.float32))
    sinks = bf16_bits(rng.standard_normal(H, dtype=np.float32))
    perm = rng.permutation(slots - 1) + 1
    lists, k = [], 0
    for prefix, nq in PREFILL_ENTRIES:
        lists.append(perm[k:k + prefix + nq].astype(np.int32))
        k += prefix + nq
    qo_indptr = np.concatenate([[0], np.cumsum([nq for _, nq in PREFILL_ENTRIES])]).astype(np.int32)
    return dict(keys=keys, q=q, sinks=sinks, lists=lists, qo_indptr=qo_indptr, scale=0.125,
                slots=slots)


# ------------------------------------------------------- diagnostic scenario
DIAG_SPECS = (("head_sum_2048", 900, 16, 64), ("head_max_sum_2048", 900, 16, 64),
              ("prefix_sliding_2048", 900, 16, 884), ("random_reservoir_2048", 900, 16, 64))
DIAG_H, DIAG_G, DIAG_LEN = 16, 2, 2200
DIAG_CHUNKS = ((0, 2048), (2048, 2200))


def diagnostic_setup(seed: int = 21):
    """The reference test's lost-mass scenario (test_sglang_evict.py:191-221)
    at head_dim 64: one full layer, GQA 8:1, a 2,200-token prompt in two
    chunks (the spec boundaries fall at 2,048), keys in slots 1..2200."""
    rng = np.random.default_rng(seed)
    keys = bf16_bits(rng.standard_normal((DIAG_LEN + 1, DIAG_G, D), dtype=np.float32) * 2)
    q = bf16_bits(rng.standard_normal((DIAG_LEN, DIAG_H, D), dtype=np.float32) * 2)
    sinks = rng.standard_normal(DIAG_H).astype(np.float32)
    policies = ",".join(f"{n}:{b}:{p}:{r}" for n, b, p, r in DIAG_SPECS)
    return dict(keys=keys, q=q, sinks=sinks, policies=policies, seed=5, scale=0.125)


# ---------------------------------------------------------- replay scenario
REPLAY_H, REPLAY_G, REPLAY_LEN = 16, 2, 2400
REPLAY_CHUNKS = ((0, 300, False), (2048, 2200, True), (2200, 2400, True))  # (start, end, evicted)
REPLAY_FRONTIER, REPLAY_KEEP = 2048, 900


def replay_setup(seed: int = 23):
    """Shadow keys/values of one request by position and, for the chunks after
    its boundary at 2,048, each KV head's kept positions (prefix 16, recent 64,
    a random middle; 900 per head), the state _replay_layer_difference reads
    (runtime:520-546).  Keys are scaled so attention is peaked and evicted
    mass is not negligible."""
    rng = np.random.default_rng(seed)
    keys = bf16_bits(rng.standard_normal((REPLAY_LEN, REPLAY_G, D), dtype=np.float32) * 2)
    values = bf16_bits(rng.standard_normal((REPLAY_LEN, REPLAY_G, D), dtype=np.float32))
    q = bf16_bits(rng.standard_normal((REPLAY_LEN, REPLAY_H, D), dtype=np.float32) * 2)
    sinks = rng.standard_normal(REPLAY_H).astype(np.float32)
    F, K = REPLAY_FRONTIER, REPLAY_KEEP
    pos = np.empty((REPLAY_G, K), np.int64)
    for g in range(REPLAY_G):
        mid = np.sort(rng.choice(np.arange(16, F - 64), K - 80, replace=False))
        pos[g] = np.concatenate([np.arange(16), mid, np.arange(F - 64, F)])
    return dict(keys=keys, values=values, q=q, sinks=sinks, pos=pos, scale=0.125)


def replay_visible(pos, frontier, end):
    """_visible (runtime:241-247) as [G, end] bool: each head's kept positions
    below the frontier, everything from the frontier on."""
    vis = np.zeros((pos.shape[0], end), bool)
    vis[:, frontier:] = True
    for g in range(pos.shape[0]):
        vis[g, pos[g]] = True
    return vis
