"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the CPU checker.

Wraps oracle/ce_oracle.c, a plain-C restatement of the reference's eviction
path (tonghuikang/cache-eviction, code/cache_eviction/sglang_evict_runtime.py
and core.py).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline / reference arm may import this module; the product path never does.
Parity is pinned by tests/test_oracle_golden.py against fixtures generated
from the reference's own functions by tests/golden/make_golden.py.
"""
from __future__ import annotations

import ctypes as C
import shutil
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libce_oracle.so"

POLICY_IDS = {"prefix_sliding_2048": 0, "random_2048": 1, "random_reservoir_2048": 2,
              "head_sum_2048": 3, "head_max_sum_2048": 4, "h2o_global_2048": 5}

ROW_DTYPE = np.dtype([("n", "<i4"), ("budget", "<i4"), ("prefix", "<i4"), ("recent", "<i4"),
                      ("cursor", "<i4"), ("policy", "<i4"), ("seed", "<u8")])
assert ROW_DTYPE.itemsize == 32


def build(force: bool = False) -> Path:
    """Compile the checker with the system gcc (OpenMP when available)."""
    src = HERE / "ce_oracle.c"
    if LIB.exists() and not force and LIB.stat().st_mtime >= src.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    gcc = shutil.which("gcc", path="/usr/bin:/bin") or "gcc"
    base = [gcc, "-O2", "-fPIC", "-std=c11", "-shared", "-o", str(LIB), str(src), "-lm"]
    res = subprocess.run(base[:1] + ["-fopenmp"] + base[1:], capture_output=True, text=True)
    if res.returncode != 0:
        res = subprocess.run(base, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    return LIB


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()  # no-op when the library is newer than its source
        _lib = C.CDLL(str(LIB))
        _lib.or_reservoir53.restype = C.c_uint64
        _lib.or_reservoir53.argtypes = [C.c_uint64] * 4
        _lib.or_num_threads.restype = C.c_int
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def set_threads(n: int) -> int:
    lib().or_set_threads(int(n))
    return lib().or_num_threads()


def threads() -> int:
    return lib().or_num_threads()


def reservoir53(seed: int, layer: int, head: int, pos: int) -> int:
    """core.reservoir_score (core.py:23-30) as the 53-bit integer."""
    m = (1 << 64) - 1
    return int(lib().or_reservoir53(seed & m, layer & m, head & m, pos & m))


def row_params(rows: list[dict]) -> np.ndarray:
    out = np.zeros(len(rows), dtype=ROW_DTYPE)
    for i, r in enumerate(rows):
        for k in ("n", "budget", "prefix", "recent"):
            out[i][k] = int(r[k])
        out[i]["cursor"] = -1 if r.get("cursor") is None else int(r["cursor"])
        pol = r["policy"]
        out[i]["policy"] = POLICY_IDS[pol] if isinstance(pol, str) else int(pol)
        out[i]["seed"] = int(r.get("seed", 0)) & ((1 << 64) - 1)
    return out


def fill(table, r2u, frontier, count, rows, seq_lens, page=1):
    """fill (runtime:136-152): returns (indptr int32, indices int64, tokens int32)."""
    table = np.ascontiguousarray(table, np.int32)
    r2u = np.ascontiguousarray(r2u, np.int32)
    frontier = np.ascontiguousarray(frontier, np.int32)
    count = np.ascontiguousarray(count, np.int32)
    rows = np.ascontiguousarray(rows, np.int64)
    seq_lens = np.ascontiguousarray(seq_lens, np.int64)
    bs = len(rows)
    total = 0
    for b in range(bs):
        units = -(-int(seq_lens[b]) // page)
        total += int(count[rows[b]]) + max(0, units - int(frontier[rows[b]]))
    indptr = np.zeros(bs + 1, np.int32)
    indices = np.zeros(max(total, 1), np.int64)
    tokens = np.zeros(max(bs, 1), np.int32)
    lib().or_fill(_p(table), C.c_int64(table.shape[1]), _p(r2u), C.c_int64(r2u.shape[1]),
                  _p(frontier), _p(count), _p(rows), _p(seq_lens), C.c_int(bs), C.c_int(page),
                  _p(indptr), _p(indices), _p(tokens))
    return indptr, indices[:total], tokens[:bs]


def decode(q_bits, k_bits, v_bits, indptr, indices, tokens, sinks, modes, scale, page,
           scores=None, zero_new=True):
    """Decode attention + H2O scores in float64 (runtime:155-224, 266-271).

    q_bits [bs, H, D] uint16 (bf16 bits); k/v [units, G, P, D] uint16.
    scores [G, units] float32 is updated in place.  Returns (out fp32, lse fp32).
    """
    q_bits = np.ascontiguousarray(q_bits, np.uint16)
    k_bits = np.ascontiguousarray(k_bits, np.uint16)
    v_bits = np.ascontiguousarray(v_bits, np.uint16)
    bs, H, D = q_bits.shape
    units, G, P, D2 = k_bits.shape
    assert D == D2 and P == page
    indptr = np.ascontiguousarray(indptr, np.int32)
    indices = np.ascontiguousarray(indices, np.int32)
    tokens = np.ascontiguousarray(tokens, np.int32)
    sinks = None if sinks is None else np.ascontiguousarray(sinks, np.float32)
    modes = None if modes is None else np.ascontiguousarray(modes, np.int32)
    out = np.zeros((bs, H, D), np.float32)
    lse = np.zeros((bs, H), np.float32)
    if scores is not None:
        assert scores.dtype == np.float32 and scores.flags.c_contiguous
    lib().or_decode(_p(q_bits), _p(k_bits), _p(v_bits), C.c_int64(units), _p(indptr),
                    _p(indices), _p(tokens), _p(sinks), _p(modes), C.c_float(scale), C.c_int(bs),
                    C.c_int(H), C.c_int(G), C.c_int(D), C.c_int(P), _p(scores),
                    C.c_int64(scores.shape[1] if scores is not None else 0),
                    C.c_int(1 if zero_new else 0), _p(out), _p(lse))
    return out, lse


def prefill(q_bits, k_bits, qo_indptr, indptr, indices, tokens, sinks, modes, scale, page,
            scores, zero_new=True):
    """Prefill / extend H2O scores in float64 (runtime:314-340).

    q_bits [total_q, H, D] uint16; k_bits [units, G, P, D] uint16; scores
    [G, units] float32 updated in place (see or_prefill)."""
    q_bits = np.ascontiguousarray(q_bits, np.uint16)
    k_bits = np.ascontiguousarray(k_bits, np.uint16)
    total_q, H, D = q_bits.shape
    units, G, P, D2 = k_bits.shape
    assert D == D2 and P == page and scores.dtype == np.float32 and scores.flags.c_contiguous
    qo_indptr = np.ascontiguousarray(qo_indptr, np.int32)
    indptr = np.ascontiguousarray(indptr, np.int32)
    indices = np.ascontiguousarray(indices, np.int32)
    tokens = np.ascontiguousarray(tokens, np.int32)
    modes = np.ascontiguousarray(modes, np.int32)
    sinks = None if sinks is None else np.ascontiguousarray(sinks, np.float32)
    lib().or_prefill(_p(q_bits), C.c_int64(H * D), C.c_int64(D), _p(k_bits), _p(qo_indptr),
                     _p(indptr), _p(indices), _p(tokens), _p(sinks), _p(modes), C.c_float(scale),
                     C.c_int(len(tokens)), C.c_int(H), C.c_int(G), C.c_int(D), C.c_int(P),
                     _p(scores), C.c_int64(scores.shape[1]), C.c_int(1 if zero_new else 0))
    return scores


def replay_error(q_bits, k_bits, v_bits, start, scale, visible=None, sinks=None, want_out=False):
    """Replay layer error of one chunk in float64 (runtime:520-546).

    q_bits [count, H, D] uint16 at positions start..; k_bits / v_bits
    [>= start + count, G, D] uint16 by position; visible [G, start + count]
    bool or None.  Returns error [count] (and the masked output [count, H, D]
    with want_out); see or_replay_error."""
    q_bits = np.ascontiguousarray(q_bits, np.uint16)
    k_bits = np.ascontiguousarray(k_bits, np.uint16)
    v_bits = np.ascontiguousarray(v_bits, np.uint16)
    count, H, D = q_bits.shape
    G = k_bits.shape[1]
    end = start + count
    assert k_bits.shape[0] >= end and v_bits.shape == k_bits.shape
    vis = None if visible is None else np.ascontiguousarray(np.asarray(visible)[:, :end], np.uint8)
    sinks = None if sinks is None else np.ascontiguousarray(sinks, np.float32)
    error = np.zeros(count, np.float64)
    out = np.zeros((count, H, D), np.float64) if want_out else None
    lib().or_replay_error(_p(q_bits), C.c_int64(H * D), C.c_int64(D), _p(k_bits), _p(v_bits), _p(vis),
                          _p(sinks), C.c_float(scale), C.c_int(H), C.c_int(G), C.c_int(D), C.c_int(start),
                          C.c_int(count), _p(error), _p(out))
    return (error, out) if want_out else error


def retention_record(pos_before, count_before, frontier_before, n, pos_after, count_after):
    """Retention record of one row's boundary (runtime:465-467, 500-507).

    pos_* [L, G, cap] int (the row's compacted positions before and after);
    the columns before the boundary are the count_before compacted ones then
    positions frontier_before .. n-1.  Victims of (layer, head) = positions
    it held before and does not hold after, ascending; returns (deltas
    uint32 concatenated over layer-major heads, first value of each head the
    position itself; counts int32 [L * G])."""
    L, G = pos_before.shape[:2]
    tail = np.arange(frontier_before, n, dtype=np.int64)
    deltas, counts = [], []
    for l in range(L):
        for g in range(G):
            before = np.concatenate([np.asarray(pos_before[l, g, :count_before], np.int64), tail])
            v = np.setdiff1d(before, np.asarray(pos_after[l, g, :count_after], np.int64))
            counts.append(len(v))
            deltas.append(np.diff(v, prepend=0))
    d = np.concatenate(deltas) if deltas else np.zeros(0, np.int64)
    return d.astype(np.uint32), np.array(counts, np.int32)


def choose(pos, score, params, layers, heads, ncols=None, head_offset=0, kept_stride=None,
           score_is_f32=False):
    """ce_choose restated (runtime:376-412): returns (kept cols, status, protected_count)."""
    pos = np.ascontiguousarray(pos, np.int32)
    problems, segs, n_cols = pos.shape
    assert segs == layers * heads
    sc = None if score is None else np.ascontiguousarray(score, np.float64)
    kept_stride = kept_stride or n_cols
    kept = np.full((problems, segs, kept_stride), -1, np.int32)
    status = np.zeros(problems, np.int32)
    pcount = np.zeros(problems, np.int32)
    params = np.ascontiguousarray(params, ROW_DTYPE)
    nc = None if ncols is None else np.ascontiguousarray(ncols, np.int32)
    lib().or_choose(_p(pos), _p(nc), C.c_int(n_cols), _p(sc), C.c_int(1 if score_is_f32 else 0),
                    _p(params), C.c_int(problems), C.c_int(layers), C.c_int(heads),
                    C.c_int(head_offset), _p(kept), C.c_int(kept_stride), _p(status), _p(pcount))
    return kept, status, pcount


def boundary(state: dict, k_layers: list, v_layers: list, rows, params, max_cols, live,
             uniforms=None, swa=None, head_offset=0):
    """_boundary (runtime:415-507) on host arrays; mutates `state` and the pools.

    state: table, r2u, frontier, count, pos [rows, L, G, cap], scores [L, G, units].
    Returns (result [R, 4], freed [R, max_cols]).
    """
    table, r2u = state["table"], state["r2u"]
    pos, scores = state["pos"], state["scores"]
    for a in (table, r2u, state["frontier"], state["count"], pos):
        assert a.dtype == np.int32 and a.flags.c_contiguous
    assert scores.dtype == np.float32 and scores.flags.c_contiguous
    L, G, units = scores.shape
    P = k_layers[0].shape[2]
    D = k_layers[0].shape[3]
    rows = np.ascontiguousarray(rows, np.int32)
    params = np.ascontiguousarray(params, ROW_DTYPE)
    R = len(rows)
    result = np.zeros((R, 4), np.int32)
    freed = np.full((R, max(max_cols, 1)), -1, np.int32)
    kp = (C.c_void_p * L)(*[k.ctypes.data for k in k_layers])
    vp = (C.c_void_p * L)(*[v.ctypes.data for v in v_layers])
    uni = None if uniforms is None else np.ascontiguousarray(uniforms, np.float64)
    sw = None if swa is None else np.ascontiguousarray(swa, np.int64)
    lib().or_boundary(_p(table), C.c_int64(table.shape[1]), _p(r2u), C.c_int64(r2u.shape[1]),
                      _p(state["frontier"]), _p(state["count"]), _p(pos),
                      C.c_int64(pos.shape[1] * pos.shape[2] * pos.shape[3]), C.c_int(pos.shape[3]),
                      _p(scores), C.c_int64(G * units), C.c_int64(units), C.c_int64(units), kp, vp,
                      C.c_int(L), C.c_int(G), C.c_int(P), C.c_int(D), C.c_int(head_offset),
                      _p(sw), _p(rows), _p(params), C.c_int(R), _p(uni), C.c_int(max_cols),
                      C.c_int(1 if live else 0), _p(result), _p(freed),
                      C.c_int64(freed.shape[1]))
    return result, freed
