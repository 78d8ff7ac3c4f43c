"""torch-tensor front end of the C ABI (libce_b200.so).

torch supplies device memory and the current CUDA stream; every call goes
through capi (ctypes) into the sm_100a kernels.  Workspaces are cached per
device and grown on demand from torch's caching allocator, so steady-state
calls allocate nothing.
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Optional, Sequence

import numpy as np
import torch

from . import capi

ROW_DTYPE = np.dtype([("n", "<i4"), ("budget", "<i4"), ("prefix", "<i4"), ("recent", "<i4"),
                      ("cursor", "<i4"), ("policy", "<i4"), ("seed", "<u8")])
POLICY_IDS = {"prefix_sliding_2048": capi.CE_POLICY_PREFIX_SLIDING,
              "random_2048": capi.CE_POLICY_RANDOM,
              "random_reservoir_2048": capi.CE_POLICY_RESERVOIR,
              "head_sum_2048": capi.CE_POLICY_HEAD_SUM,
              "head_max_sum_2048": capi.CE_POLICY_HEAD_MAX,
              "h2o_global_2048": capi.CE_POLICY_H2O_GLOBAL}
U64_MASK = (1 << 64) - 1


def _p(t: Optional[torch.Tensor]):
    if t is None:
        return None
    return C.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class _Workspaces:
    def __init__(self):
        self._bufs: dict = {}

    def get(self, device: torch.device, key: str, nbytes: int) -> torch.Tensor:
        k = (device.index if device.index is not None else torch.cuda.current_device(), key)
        buf = self._bufs.get(k)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(int(nbytes * 1.25), 256), dtype=torch.uint8, device=device)
            self._bufs[k] = buf
        return buf


WORKSPACES = _Workspaces()

# Kernel launches issued through this module (the C entry points' own
# kernels, not torch's); bench.py reports the count over its timed region.
LAUNCHES = [0]


def _count(n: int) -> None:
    LAUNCHES[0] += n


def row_params(rows: Sequence[dict], device) -> torch.Tensor:
    """Pack boundary parameters (units) into a device array of ce_row_params."""
    arr = np.zeros(len(rows), dtype=ROW_DTYPE)
    for i, r in enumerate(rows):
        for k in ("n", "budget", "prefix", "recent"):
            arr[i][k] = int(r[k])
        arr[i]["cursor"] = -1 if r.get("cursor") is None else int(r["cursor"])
        pol = r["policy"]
        arr[i]["policy"] = POLICY_IDS[pol] if isinstance(pol, str) else int(pol)
        arr[i]["seed"] = int(r.get("seed", 0)) & U64_MASK
    return torch.from_numpy(arr.view(np.uint8).copy()).to(device)


def error_word(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def fill(table, req_to_unit, frontier, count, rows, seq_lens, page_size, kv_indptr, kv_indices,
         kv_tokens=None, err=None):
    """CSR of compacted residents then the tail (runtime:136-152)."""
    lib = capi.load()
    bs = int(rows.numel())
    assert rows.dtype == torch.int64 and seq_lens.dtype == torch.int64
    assert kv_indices.dtype in (torch.int32, torch.int64)
    st = lib.ce_fill(_p(table), table.stride(0), _p(req_to_unit), req_to_unit.stride(0),
                     _p(frontier), _p(count), _p(rows), _p(seq_lens), bs, page_size,
                     _p(kv_indptr), _p(kv_indices), 1 if kv_indices.dtype == torch.int64 else 0,
                     kv_indices.numel(), _p(kv_tokens), _p(err), _stream(kv_indptr.device))
    capi.check(st, "ce_fill")
    _count(1 if bs else 0)
    return kv_indptr


def pool_alloc(units, top, req_to_unit, rows, seq_lens, page_size, err=None):
    """Pop a unit for every entry whose newest token starts one and write it
    to req_to_unit (ce_pool_alloc); units/top: the free-unit stack."""
    lib = capi.load()
    bs = int(rows.numel())
    assert units.dtype == torch.int32 and top.dtype == torch.int32 and req_to_unit.dtype == torch.int32
    assert rows.dtype == torch.int64 and seq_lens.dtype == torch.int64
    st = lib.ce_pool_alloc(_p(units), _p(top), _p(req_to_unit), req_to_unit.stride(0), req_to_unit.shape[1],
                           _p(rows), _p(seq_lens), bs, page_size, _p(err), _stream(units.device))
    capi.check(st, "ce_pool_alloc")
    _count(1 if bs else 0)


def pool_push(units, top, lists, counts, err=None):
    """Push lists[r, :counts[r]] for every row r onto the free-unit stack
    (ce_pool_push); counts may be a strided column (e.g. result[:, 3])."""
    lib = capi.load()
    nrows = int(lists.shape[0])
    assert lists.dtype == torch.int32 and counts.dtype == torch.int32 and lists.stride(1) == 1
    st = lib.ce_pool_push(_p(units), _p(top), units.numel(), _p(lists), lists.stride(0), _p(counts),
                          counts.stride(0), nrows, _p(err), _stream(units.device))
    capi.check(st, "ce_pool_push")
    _count(1 if nrows else 0)


def decode_attn_score(q, k_pool, v_pool, kv_indptr, kv_indices, kv_tokens, sm_scale, page_size,
                      sinks=None, mode_of_row=None, rows=None, scores=None, zero_new=True,
                      out=None, out_f32=False, lse=None, score_flags=3, err=None, workspace=None):
    """Fused decode attention + H2O score over one layer.

    q [bs, H, 64] bf16; pools [units, G, page, 64] bf16; scores [G, units] fp32.
    Returns out [bs, H, 64] (bf16, or fp32 with out_f32).  With
    capi.CE_SCORE_DEFER in score_flags the page scores are left to
    decode_scores, which must get the same workspace (then pass one here:
    a uint8 device tensor of at least decode_workspace_bytes()).
    """
    lib = capi.load()
    bs, H, D = q.shape
    G = k_pool.shape[1]
    assert q.dtype == torch.bfloat16 and q.stride(2) == 1
    assert k_pool.is_contiguous() and v_pool.is_contiguous()
    assert kv_indices.dtype == torch.int32 and kv_indptr.dtype == torch.int32
    dev = q.device
    if out is None:
        out = torch.empty((bs, H, D), dtype=torch.float32 if out_f32 else torch.bfloat16, device=dev)
    if sinks is not None and sinks.dtype != torch.float32:
        sinks = sinks.float()
    if scores is not None:
        assert scores.dtype == torch.float32 and scores.stride(1) == 1
    cap = kv_indices.numel()
    need = lib.ce_decode_workspace_bytes(bs, cap, H, G, page_size, score_flags)
    if need < 0:
        raise capi.CeError("ce_decode_workspace_bytes failed")
    if workspace is not None:
        assert workspace.dtype == torch.uint8 and workspace.numel() >= need
        ws = workspace
    else:
        ws = WORKSPACES.get(dev, "decode", need)
    st = lib.ce_decode_attn_score(
        _p(q), q.stride(0), q.stride(1), _p(k_pool), _p(v_pool), k_pool.shape[0], _p(kv_indptr),
        _p(kv_indices), _p(kv_tokens), cap, _p(sinks), _p(mode_of_row), _p(rows), float(sm_scale),
        bs, H, G, D, page_size, _p(scores), scores.stride(0) if scores is not None else 0,
        1 if zero_new else 0, _p(out), 1 if out.dtype == torch.float32 else 0, out.stride(0),
        out.stride(1), _p(lse), score_flags, _p(ws), ws.numel(), _p(err), _stream(dev))
    capi.check(st, "ce_decode_attn_score")
    _count(2 if bs else 0)
    return out


def decode_workspace_bytes(bs, kv_capacity, H, G, page_size, score_flags=3):
    need = capi.load().ce_decode_workspace_bytes(bs, kv_capacity, H, G, page_size, score_flags)
    if need < 0:
        raise capi.CeError("ce_decode_workspace_bytes failed")
    return need


def decode_scores(kv_indptr, kv_indices, kv_tokens, pool_units, page_size, H, G, bs, mode_of_row, rows,
                  scores, workspace, zero_new=True, score_flags=3, err=None, stream=None):
    """The page scores a decode_attn_score(..., CE_SCORE_DEFER) call left out,
    from that call's workspace and CSR, on `stream` (a torch.cuda.Stream;
    default the current stream)."""
    lib = capi.load()
    if bs == 0 or scores is None or mode_of_row is None:
        return
    assert scores.dtype == torch.float32 and scores.stride(1) == 1
    st = lib.ce_decode_scores(_p(kv_indptr), _p(kv_indices), _p(kv_tokens), kv_indices.numel(), pool_units,
                              _p(mode_of_row), _p(rows), bs, H, G, page_size, _p(scores), scores.stride(0),
                              1 if zero_new else 0, score_flags & 3, _p(workspace), workspace.numel(), _p(err),
                              _stream(workspace.device) if stream is None else C.c_void_p(stream.cuda_stream))
    capi.check(st, "ce_decode_scores")
    _count(1 if score_flags & 3 else 0)


def prefill_scores(q, k_pool, qo_indptr, kv_indptr, kv_indices, kv_tokens, sm_scale, page_size,
                   max_q, max_tokens, sinks=None, mode_of_row=None, rows=None, scores=None,
                   zero_new=True, err=None):
    """Prefill / extend H2O scores of one layer (runtime:314-340) into `scores`.

    q [total_q, H, 64] bf16; k_pool [units, G, page, 64] bf16; scores [G, units]
    fp32; qo_indptr/kv_indptr/kv_indices/kv_tokens int32 as ce_prefill_scores
    documents; max_q / max_tokens bound the chunk and list lengths (host ints).
    """
    lib = capi.load()
    total_q, H, D = q.shape
    G = k_pool.shape[1]
    assert q.dtype == torch.bfloat16 and q.stride(2) == 1
    assert k_pool.is_contiguous() and scores is not None and scores.dtype == torch.float32
    assert scores.stride(1) == 1
    for t in (qo_indptr, kv_indptr, kv_indices, kv_tokens):
        assert t.dtype == torch.int32
    dev = q.device
    if sinks is not None and sinks.dtype != torch.float32:
        sinks = sinks.float()
    bs = int(kv_tokens.numel())
    need = lib.ce_prefill_workspace_bytes(total_q, H)
    if need < 0:
        raise capi.CeError("ce_prefill_workspace_bytes failed")
    ws = WORKSPACES.get(dev, "prefill", need)
    st = lib.ce_prefill_scores(
        _p(q), q.stride(0), q.stride(1), _p(k_pool), k_pool.shape[0], _p(qo_indptr), _p(kv_indptr),
        _p(kv_indices), _p(kv_tokens), kv_indices.numel(), _p(sinks), _p(mode_of_row), _p(rows),
        float(sm_scale), bs, H, G, D, page_size, total_q, int(max_q), int(max_tokens), _p(scores),
        scores.stride(0), 1 if zero_new else 0, _p(ws), ws.numel(), _p(err), _stream(dev))
    capi.check(st, "ce_prefill_scores")
    if bs and max_q and mode_of_row is not None and total_q:
        _count(2 if max_tokens else 1)
    return scores


def prefill_lost(q, k_pool, qo_indptr, kv_indptr, kv_indices, kv_tokens, sm_scale, page_size, max_q,
                 max_tokens, evicted_bits, lost, lost_scale, sinks=None, err=None):
    """Lost-mass diagnostic of one entry's chunk (runtime:587-613), accumulated
    into lost [S, >= max_q]; evicted_bits [S, G, words] int32 bit masks."""
    lib = capi.load()
    total_q, H, D = q.shape
    G = k_pool.shape[1]
    assert q.dtype == torch.bfloat16 and q.stride(2) == 1 and k_pool.is_contiguous()
    assert evicted_bits.dtype == torch.int32 and evicted_bits.is_contiguous()
    assert lost.dtype == torch.float32 and lost.stride(1) == 1
    S = int(evicted_bits.shape[0])
    dev = q.device
    if sinks is not None and sinks.dtype != torch.float32:
        sinks = sinks.float()
    need = lib.ce_prefill_workspace_bytes(total_q, H)
    ws = WORKSPACES.get(dev, "prefill", need)
    st = lib.ce_prefill_lost(
        _p(q), q.stride(0), q.stride(1), _p(k_pool), k_pool.shape[0], _p(qo_indptr), _p(kv_indptr),
        _p(kv_indices), _p(kv_tokens), kv_indices.numel(), _p(sinks), float(sm_scale), H, G, D, page_size,
        total_q, int(max_q), int(max_tokens), _p(evicted_bits), S, evicted_bits.shape[2], _p(lost),
        lost.stride(0), float(lost_scale), _p(ws), ws.numel(), _p(err), _stream(dev))
    capi.check(st, "ce_prefill_lost")
    _count(2 if S and total_q else 0)
    return lost


def replay_error(q, k_shadow, v_shadow, start, sm_scale, visible_bits=None, sinks=None, out_masked=None,
                 err=None):
    """Per-query relative output error of eviction (runtime:520-546) for one
    chunk: q [count, H, 64] bf16 at positions start.., k/v shadows
    [>= start + count, G, 64] bf16 by position, visible_bits [G, words] int32
    (None = all visible).  Returns error [count] fp32; fills out_masked
    [count, H, 64] fp32 with the masked output when given."""
    lib = capi.load()
    count, H, D = q.shape
    G = k_shadow.shape[1]
    assert q.dtype == torch.bfloat16 and q.stride(2) == 1
    assert k_shadow.is_contiguous() and v_shadow.is_contiguous() and k_shadow.shape == v_shadow.shape
    if visible_bits is not None:
        assert visible_bits.dtype == torch.int32 and visible_bits.is_contiguous() and visible_bits.shape[0] == G
    if out_masked is not None:
        assert out_masked.dtype == torch.float32 and out_masked.is_contiguous()
        assert tuple(out_masked.shape) == (count, H, D)
    dev = q.device
    if sinks is not None and sinks.dtype != torch.float32:
        sinks = sinks.float()
    error = torch.empty(count, dtype=torch.float32, device=dev)
    need = lib.ce_replay_workspace_bytes(count, H)
    ws = WORKSPACES.get(dev, "replay", need)
    words = 0 if visible_bits is None else visible_bits.shape[1]
    st = lib.ce_replay_error(_p(q), q.stride(0), q.stride(1), _p(k_shadow), _p(v_shadow), k_shadow.shape[0],
                             _p(visible_bits), words, _p(sinks), float(sm_scale), H, G, D, int(start), count,
                             _p(error), _p(out_masked), _p(ws), ws.numel(), _p(err), _stream(dev))
    capi.check(st, "ce_replay_error")
    _count(3 if count else 0)
    return error


def choose(pos, score, params: torch.Tensor, layers, heads, max_n, ncols=None, head_offset=0,
           kept_stride=None, err=None):
    """Kept columns [problems, segs, kept_stride] in ascending position (runtime:376-412)."""
    lib = capi.load()
    problems, segs, n_cols = pos.shape
    dev = pos.device
    kept_stride = kept_stride or n_cols
    # ce_choose writes every status and protected count and the first
    # min(budget, ncols) kept columns of each chosen segment; the rest of
    # `kept` is left as allocated.
    kept = torch.empty((problems, segs, kept_stride), dtype=torch.int32, device=dev)
    status = torch.empty(problems, dtype=torch.int32, device=dev)
    pcount = torch.empty(problems, dtype=torch.int32, device=dev)
    sdt = capi.CE_DTYPE_NONE
    if score is not None:
        sdt = capi.CE_DTYPE_F64 if score.dtype == torch.float64 else capi.CE_DTYPE_F32
        assert score.is_contiguous() and score.shape == pos.shape
    need = lib.ce_choose_workspace_bytes(problems, segs, n_cols)
    ws = WORKSPACES.get(dev, "choose", need)
    st = lib.ce_choose(_p(pos.contiguous()), _p(ncols), n_cols, _p(score), sdt, _p(params), problems,
                       int(max_n), layers, heads, head_offset, _p(kept), kept_stride, _p(status),
                       _p(pcount), _p(ws), ws.numel(), _p(err), _stream(dev))
    capi.check(st, "ce_choose")
    _count(2 if problems else 0)
    return kept, status, pcount


def layer_pointers(tensors: Sequence[torch.Tensor], device) -> torch.Tensor:
    return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64, device=device)


def boundary(table, req_to_unit, frontier, count, pos, scores, k_ptrs, v_ptrs, kv_heads, page_size,
             rows, params, max_cols, max_n, live, marks=None, epoch=0, swa=None, uniforms=None,
             global_scores=None, head_offset=0, freed=None, hazard_bytes=256 << 20, err=None,
             max_width=0, record=None):
    """One eviction boundary for a batch of rows (runtime:415-507).

    record: None, or (delta [R * L * G, >= max_cols] int32 device tensor,
    counts [R * L * G] int32) to receive the retention record
    (runtime:465-467, 500-507; deltas are uint32 bit patterns).
    Returns (result [R, 4] int32 device tensor, freed [R, max_cols] int32).
    """
    lib = capi.load()
    dev = table.device
    R = int(rows.numel())
    L = int(k_ptrs.numel())
    result = torch.zeros((max(R, 1), 4), dtype=torch.int32, device=dev)
    if freed is None:
        freed = torch.full((max(R, 1), max(max_cols, 1)), -1, dtype=torch.int32, device=dev)
    need = lib.ce_boundary_workspace_bytes(R, L, kv_heads, 64, page_size, max_cols, int(max_width),
                                           global_scores.shape[2] if global_scores is not None else 0,
                                           hazard_bytes)
    if need < 0:
        raise capi.CeError("ce_boundary_workspace_bytes failed")
    ws = WORKSPACES.get(dev, "boundary", need)
    udt = capi.CE_DTYPE_NONE
    if uniforms is not None:
        udt = capi.CE_DTYPE_F64 if uniforms.dtype == torch.float64 else capi.CE_DTYPE_F32
    st = lib.ce_boundary(
        _p(table), table.stride(0), table.shape[1], _p(req_to_unit), req_to_unit.stride(0),
        req_to_unit.shape[1], _p(frontier), _p(count), _p(pos), pos.stride(0), pos.shape[3],
        _p(scores), scores.stride(0), scores.stride(1), scores.shape[2], _p(k_ptrs), _p(v_ptrs), L,
        kv_heads, 64, page_size, head_offset, _p(marks), int(epoch), _p(swa), _p(rows), _p(params),
        R, _p(uniforms), udt, _p(global_scores),
        global_scores.shape[2] if global_scores is not None else 0, 1 if live else 0, max_cols,
        int(max_width), int(max_n), _p(result), _p(freed), freed.stride(0), _p(ws), ws.numel(), int(hazard_bytes),
        _p(record[0]) if record else None, record[0].stride(0) if record else 0,
        _p(record[1]) if record else None, _p(err), _stream(dev))
    capi.check(st, "ce_boundary")
    if R:
        # bsel, bvalidate, bfinish; hsum (and unit_sum for long rows that own
        # most of the pool) without global scores; bzero when
        # live; a gather and a scatter per launch group (rows x layers fitting
        # the hazard scratch)
        width = max_width if 0 < max_width < max_cols else max_cols
        row_layer = max(1, kv_heads * width * 2 * page_size * 128)
        hz = max(int(hazard_bytes), row_layer)
        rows_per = min(R, max(1, hz // row_layer))
        group = min(L, max(1, hz // (rows_per * row_layer)))
        units = scores.shape[2]
        hsum = 0 if global_scores is not None else (2 if max_cols > 4096 and 0 < units <= 2 * R * max_cols else 1)
        _count(3 + hsum + (1 if live and units > 0 else 0)
               + 2 * ceil_div(R, rows_per) * ceil_div(L, group) + (1 if record else 0))
    return result, freed


def prepare_device(device):
    """Load the library's decode, boundary, CSR and pool kernels on `device`
    (ce_prepare_device), so that no later call pays the module load."""
    with torch.cuda.device(torch.device(device)):
        capi.check(capi.load().ce_prepare_device(), "ce_prepare_device")


def reserve_boundary(device, rows, layers, kv_heads, page_size, max_cols, max_width, global_heads,
                     hazard_bytes):
    """Allocate the ce_boundary workspace for the given batch bounds ahead of use."""
    need = capi.load().ce_boundary_workspace_bytes(rows, layers, kv_heads, 64, page_size, max_cols,
                                                   max_width, global_heads, hazard_bytes)
    if need < 0:
        raise capi.CeError("ce_boundary_workspace_bytes failed")
    return WORKSPACES.get(torch.device(device), "boundary", need)


def gather_row_scores(table, req_to_unit, frontier, count, scores, rows, params, max_cols, err=None):
    lib = capi.load()
    dev = table.device
    R = int(rows.numel())
    L, G, units = scores.shape
    out = torch.zeros((R, L, G, max_cols), dtype=torch.float32, device=dev)
    st = lib.ce_gather_row_scores(_p(table), table.stride(0), _p(req_to_unit), req_to_unit.stride(0),
                                  _p(frontier), _p(count), _p(scores), scores.stride(0),
                                  scores.stride(1), units, L, G, _p(rows), _p(params), R, max_cols,
                                  _p(out), _p(err), _stream(dev))
    capi.check(st, "ce_gather_row_scores")
    return out


def reservoir_scores53(pos: torch.Tensor, seed: int, head_offset: int = 0) -> torch.Tensor:
    """splitmix64 draws as 53-bit integers [L, G, N] (int64 storage of the uint64)."""
    lib = capi.load()
    L, G, N = pos.shape
    pos32 = pos.to(torch.int32).contiguous()
    out = torch.empty((L, G, N), dtype=torch.int64, device=pos.device)
    st = lib.ce_reservoir_scores(_p(pos32), L, G, N, head_offset, int(seed) & U64_MASK, _p(out),
                                 _stream(pos.device))
    capi.check(st, "ce_reservoir_scores")
    return out


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def next_pow2(x: int) -> int:
    return 1 << max(0, math.ceil(math.log2(max(1, x))))
