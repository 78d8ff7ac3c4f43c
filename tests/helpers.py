"""Shared builders for the parity tests (numpy state in the reference's layout)."""
from __future__ import annotations

import hashlib

import numpy as np

from golden import scenarios as sc

POS_CAP = 1024 + 64


def boundary_state(setup):
    """Host state of the reference's check_boundaries scenario
    (code/tests/test_sglang_evict.py:92-107) at page_size 1."""
    rows, width, n = setup["rows"], setup["width"], setup["n"]
    slots = setup["slots"]
    state = {
        "table": np.zeros((rows, width), np.int32),
        "r2u": np.zeros((rows, width), np.int32),
        "frontier": np.zeros(rows, np.int32),
        "count": np.zeros(rows, np.int32),
        "pos": np.zeros((rows, 2, sc.G, POS_CAP), np.int32),
        "scores": np.zeros((2, sc.G, slots), np.float32),
    }
    state["r2u"][1, :n] = setup["slot_of"]
    state["scores"][:, :, setup["slot_of"]] = setup["score"]
    k_layers = [setup["keys"][l].reshape(slots, sc.G, 1, sc.D).copy() for l in sc.FULL]
    v_layers = [setup["values"][l].reshape(slots, sc.G, 1, sc.D).copy() for l in sc.FULL]
    return state, k_layers, v_layers


def boundary_row(name, boundary, seed=4):
    cfg = sc.boundary_cfg(name)
    return dict(n=boundary, budget=cfg["budget"], prefix=cfg["prefix"], recent=cfg["recent"],
                cursor=boundary - 200, policy=name, seed=seed)


def sha16(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).view(np.int16).tobytes()).hexdigest()


def sha_bytes(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def paged(keys_tok: np.ndarray, slot_lists, page: int):
    """Copy token rows [slots, G, D] of each sequence into fresh pages
    [units, G, page, D] (head-major inside a page); returns (pool, per-seq units)."""
    G, D = keys_tok.shape[1], keys_tok.shape[2]
    units_per = [(len(s) + page - 1) // page for s in slot_lists]
    total = sum(units_per) + 1
    pool = np.zeros((total, G, page, D), keys_tok.dtype)
    order = np.random.default_rng(99).permutation(total - 1) + 1
    out, k = [], 0
    for s, u in zip(slot_lists, units_per):
        us = order[k:k + u]
        k += u
        for t, slot in enumerate(s):
            pool[us[t // page], :, t % page, :] = keys_tok[slot]
        out.append(us.astype(np.int32))
    return pool, out


def prefill_inputs(page):
    """The prefill scenario as pools/lists at `page` tokens per unit."""
    d = sc.prefill_setup()
    lists = d["lists"]
    if page == 1:
        kpool = d["keys"].reshape(-1, sc.G, 1, sc.D)
        units = lists
    else:
        kpool, units = paged(d["keys"], lists, page)
    indptr = np.concatenate([[0], np.cumsum([len(u) for u in units])]).astype(np.int32)
    tokens = np.array([p + n for p, n in sc.PREFILL_ENTRIES], np.int32)
    return d, kpool, units, indptr, np.concatenate(units).astype(np.int32), tokens


def prefill_want(z, mode, page, units, init):
    """Expected [G, units] scores: the reference's per-token scores summed per
    page, added to `init` except on units that start inside the chunk."""
    want = init.copy()
    for i, (prefix, nq) in enumerate(sc.PREFILL_ENTRIES):
        tok = z[f"mode{mode}_entry{i}"]  # [G, prefix + nq]
        ntok = prefix + nq
        pad = np.zeros((sc.G, len(units[i]) * page), np.float64)
        pad[:, :ntok] = tok
        per_unit = pad.reshape(sc.G, -1, page).sum(-1)
        for j, u in enumerate(units[i]):
            base = 0.0 if j * page >= prefix else want[:, u]
            want[:, u] = base + per_unit[:, j]
    return want
