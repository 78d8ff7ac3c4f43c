"""Drop-in mirror of the overlay module ``sglang.srt.gstar_evict``.

Same hook names, arguments and error behaviour as the reference's
code/cache_eviction/sglang_evict_runtime.py ("runtime:" below), with the work
done by the sm_100a kernels behind include/ce_api.h:

  enabled()                                  runtime:53-54
  fill(backend, bs, seq_lens, rows, kv_indices) -> kv_indptr       runtime:136-152
  decode(backend, q, layer, forward_batch, sinks, out)   fused attention + score
  after_decode(backend, q, layer, forward_batch, sinks, out=None)  runtime:203-224
  after_extend(backend, q, layer, forward_batch, sinks)            runtime:277-311
  on_extend(batch), on_decode(batch), release(req)                runtime:640-742
  filter_holes(segments), freed(row)                               runtime:128-131, 745-747
  choose(...), reservoir_scores(...), _scores(...), _boundary(...) runtime:358-507

Backends, layers, batches, requests and allocators are the duck-typed SGLang
objects the reference reads (fields as in code/tests/test_sglang_evict.py:19-39).
A backend may carry ``page_size`` (units of that many tokens; default 1, the
reference's token slots) and ``gstar_pos_cap`` (retained units per row).

Differences by design: choose() returns each head's kept columns in ascending
position order (the reference returns them in key order; the kept sets are
identical and every caller only uses the sets), and decode() computes the
attention output together with the scores in one pass over K and V.
"""
from __future__ import annotations

import base64
import gzip
import json
import logging
import os
import time
from pathlib import Path

import numpy as np
import torch

from . import capi, kernels
from .policy import INTERVAL, POLICIES, SCORE_MODE, canonical, validate

logger = logging.getLogger(__name__)

STATE = None
RETRACTED: set = set()
POS_CAP_DEFAULT = 32768


def enabled() -> bool:
    return os.environ.get("GSTAR_EVICT") == "1"


# ------------------------------------------------------------- payloads
# The retention record's file format (runtime:59-73): gzip'd JSON with base64
# arrays, one file per key, written atomically.  Serving the files over HTTP
# is outside this path.
def payload_dir() -> Path:
    return Path(os.environ.get("GSTAR_PAYLOAD_DIR", "/tmp/gstar-payload"))


def array(values, dtype):
    data = np.ascontiguousarray(np.asarray(values, dtype=dtype))
    return {"dtype": dtype, "shape": list(data.shape), "data": base64.b64encode(data.tobytes()).decode()}


def write_payload(key, obj):
    directory = payload_dir()
    directory.mkdir(parents=True, exist_ok=True)
    temporary = directory / f".{key}.tmp"
    temporary.write_bytes(gzip.compress(json.dumps({"format": "gstar-payload-1", "key": key, **obj}).encode()))
    temporary.rename(directory / f"{key}.json.gz")


# ---------------------------------------------------------------- state
class State:
    """Per-process eviction state on the device (runtime:89-110)."""

    def __init__(self, backend):
        self.pool = backend.token_to_kv_pool
        self.req_to_token = backend.req_to_token_pool.req_to_token
        rows, width = self.req_to_token.shape
        device = self.req_to_token.device
        self.device = device
        if device.type == "cuda":
            # the library's kernels are loaded now, not inside the first boundary
            kernels.prepare_device(device)
        self.page_size = int(getattr(backend, "page_size", 1) or 1)
        self.full_layers = sorted(i for i, (_, swa) in self.pool.layers_mapping.items() if not swa)
        self.index = {layer: i for i, layer in enumerate(self.full_layers)}
        self.first_full = self.full_layers[0]
        keys = self.pool.get_key_buffer(self.first_full)
        self.kv_heads, self.dim = keys.shape[1], keys.shape[-1]
        self.units = keys.shape[0]
        self.head_offset = int(getattr(backend, "gstar_head_offset", 0))
        self.frontier = torch.zeros(rows, dtype=torch.int32, device=device)
        self.count = torch.zeros(rows, dtype=torch.int32, device=device)
        self.mode = torch.zeros(rows, dtype=torch.int32, device=device)
        self.table = torch.zeros((rows, width), dtype=torch.int32, device=device)
        self.scores = torch.zeros((len(self.full_layers), self.kv_heads, self.units),
                                  dtype=torch.float32, device=device)
        self.pos_cap = int(getattr(backend, "gstar_pos_cap", min(width, POS_CAP_DEFAULT)))
        self.pos = torch.zeros((rows, len(self.full_layers), self.kv_heads, self.pos_cap),
                               dtype=torch.int32, device=device)
        self.marks = torch.zeros(self.units, dtype=torch.int32, device=device)
        self.epoch = 0
        self.kv_tokens = torch.zeros(rows + 1, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.entries: dict = {}
        self.verify = os.environ.get("GSTAR_EVICT_VERIFY") == "1"
        self._ptrs = None

    def pools(self, layer_id):
        """One layer's K and V as [units, G, page, D] views."""
        k = self.pool.get_key_buffer(layer_id)
        v = self.pool.get_value_buffer(layer_id)
        shape = (k.shape[0], self.kv_heads, self.page_size, self.dim)
        return k.view(shape), v.view(shape)

    def layer_pointers(self):
        ptrs = ([self.pool.get_key_buffer(l).data_ptr() for l in self.full_layers],
                [self.pool.get_value_buffer(l).data_ptr() for l in self.full_layers])
        if self._ptrs is None or self._ptrs[0] != ptrs:
            self._ptrs = (ptrs, torch.tensor(ptrs[0], dtype=torch.int64, device=self.device),
                          torch.tensor(ptrs[1], dtype=torch.int64, device=self.device))
        return self._ptrs[1], self._ptrs[2]


def state(backend=None):
    global STATE
    if STATE is None and backend is not None:
        STATE = State(backend)
        logger.info("gstar_evict (B200) active: full layers %s, %d KV heads, page %d",
                    STATE.full_layers, STATE.kv_heads, STATE.page_size)
    return STATE


def _reset(st, row):
    st.entries.pop(row, None)
    st.mode[row] = 0
    st.frontier[row] = 0
    st.count[row] = 0


def freed(row):
    """Slots this row's evictions returned to the allocator (runtime:128-131)."""
    entry = STATE.entries.get(row) if STATE is not None else None
    return entry.get("freed", 0) if entry is not None else 0


# ------------------------------------------------------- attention metadata
def fill(backend, bs, seq_lens, req_pool_indices, kv_indices):
    """Full-layer CSR: shared resident units below the frontier, then the tail."""
    st = state(backend)
    kv_indptr = backend.kv_indptr[: bs + 1]
    rows = req_pool_indices[:bs].to(torch.int64).contiguous()
    lens = seq_lens[:bs].to(torch.int64).contiguous()
    kernels.fill(st.table, st.req_to_token, st.frontier, st.count, rows, lens, st.page_size,
                 kv_indptr, kv_indices, st.kv_tokens[:bs], st.err)
    return kv_indptr


def _layer_is_sliding(layer):
    return layer.sliding_window_size is not None and layer.sliding_window_size > -1


def _decode(backend, q, layer, forward_batch, sinks, out, zero_new):
    st = state(backend)
    meta = backend.forward_metadata
    heads, dim = layer.tp_q_head_num, layer.qk_head_dim
    queries = q.view(-1, heads, dim)
    bs = queries.shape[0]
    kpool, vpool = st.pools(layer.layer_id)
    indices = meta.kv_indices
    if indices.dtype != torch.int32:
        indices = indices.to(torch.int32)
    tokens = None if st.page_size == 1 else st.kv_tokens[:bs]
    rows = forward_batch.req_pool_indices.to(torch.int64)
    scores = st.scores[st.index[layer.layer_id]]
    o = None if out is None else out.view(bs, heads, dim)
    if o is None and st.verify and layer.layer_id == st.first_full:
        o = torch.empty((bs, heads, dim), dtype=torch.bfloat16, device=queries.device)
    result = kernels.decode_attn_score(
        queries, kpool, vpool, meta.kv_indptr[: bs + 1].to(torch.int32), indices, tokens,
        layer.scaling, st.page_size, sinks=sinks, mode_of_row=st.mode, rows=rows, scores=scores,
        zero_new=zero_new, out=o, err=st.err)
    if st.verify and layer.layer_id == st.first_full:
        _verify_decode(st, queries, result, layer, forward_batch, sinks)
    return result


def decode(backend, q, layer, forward_batch, sinks, out=None):
    """Fused replacement for decode_attention_fwd + after_decode on a full layer.

    Writes the attention output into ``out`` (allocated when None) and adds
    this step's H2O mass to the layer's scores in the same pass; the unit that
    the new token starts is zeroed first (runtime:211-212).
    """
    return _decode(backend, q, layer, forward_batch, sinks, out, zero_new=True)


def after_decode(backend, q, layer, forward_batch, sinks, out=None):
    """Scores of one decode step for a layer whose output SGLang already wrote.

    Same effect on the scores as the reference hook: on the first full layer
    every new slot's score is zeroed for all layers, then each H2O row adds
    p summed (head_sum) or maxed (head_max) over the KV head's query heads.
    """
    if _layer_is_sliding(layer):
        return
    st = state(backend)
    if layer.layer_id == st.first_full:
        st.scores.index_fill_(2, _new_units(st, forward_batch.out_cache_loc.long()), 0.0)
    _decode(backend, q, layer, forward_batch, sinks, None, zero_new=False)


def _new_units(st, loc):
    """Units that tokens at pool locations `loc` start (loc % page == 0); other
    tokens map to unit 0, SGLang's padding slot, so the result keeps its shape
    and needs no host sync."""
    P = st.page_size
    if P == 1:
        return loc
    return torch.where(loc % P == 0, loc // P, torch.zeros_like(loc))


def after_extend(backend, q, layer, forward_batch, sinks):
    """Prefill scores (runtime:277-311) for H2O rows of an extend batch.

    On the first full layer every unit that a new token starts is zeroed for
    all layers (runtime:293-294); replay entries (and live ones under
    GSTAR_EVICT_VERIFY=1) copy the chunk's keys and values into their shadow
    by logical position, and replay entries record the layer error of the
    chunk (runtime:301-306).  Diagnostic entries run _diagnose.  Then
    ce_prefill_scores adds each head_sum / head_max row's chunk probabilities
    over its resident prefix and the chunk itself (_prefill_scores,
    runtime:327-340).
    """
    if _layer_is_sliding(layer):
        return
    st = state(backend)
    rows = forward_batch.req_pool_indices.tolist()
    entries = [st.entries.get(r) for r in rows]
    if not any(entries):
        return
    loc = forward_batch.out_cache_loc.long()
    if layer.layer_id == st.first_full:
        st.scores.index_fill_(2, _new_units(st, loc), 0.0)
    meta = backend.forward_metadata
    qo_host = None
    for i, e in enumerate(entries):
        if e is None or e["error"]:
            continue
        if qo_host is None:
            qo_host = meta.qo_indptr.tolist()
        lo, hi = qo_host[i], qo_host[i + 1]
        start = int(forward_batch.extend_prefix_lens_cpu[i])
        chunk = q.view(-1, layer.tp_q_head_num, layer.qk_head_dim)[lo:hi]
        if layer.layer_id == st.first_full and (e["kind"] == "replay" or st.verify and e["kind"] == "live"):
            kpool, vpool = st.pools(layer.layer_id)
            shadow = e.setdefault("shadow", ShadowKV(st.kv_heads, st.dim, st.device))
            shadow.put(start, _token_rows(kpool, loc[lo:hi], st.page_size),
                       _token_rows(vpool, loc[lo:hi], st.page_size))
            if e["kind"] == "replay":
                _replay_layer_difference(st, e, chunk, layer, sinks, start)
        if e["kind"] == "diagnostic":
            kv = meta.kv_indptr.tolist()
            prefix = meta.kv_indices[kv[i]:kv[i + 1]].long()
            _diagnose(st, e, st.index[layer.layer_id], layer, chunk,
                      backend.token_to_kv_pool.get_key_buffer(layer.layer_id), sinks,
                      torch.cat((prefix, loc[lo:hi])), start)
    scored = [i for i, e in enumerate(entries) if e is not None and not e["error"] and e["mode"] in (1, 2)
              and e["kind"] != "diagnostic"]
    if not scored:
        return
    heads, dim = layer.tp_q_head_num, layer.qk_head_dim
    queries = q.view(-1, heads, dim)
    qo, kv = meta.qo_indptr.tolist(), meta.kv_indptr.tolist()
    P = st.page_size
    starts = forward_batch.extend_prefix_lens_cpu
    parts, indptr, tokens, modes = [], [0], [], []
    for i, e in enumerate(entries):
        nnew = qo[i + 1] - qo[i]
        if i not in scored:
            tokens.append(nnew)         # an empty list: skipped by mode 0
            modes.append(0)
            indptr.append(indptr[-1])
            continue
        start = int(starts[i])
        resident = e["count"] * P + start - e["frontier"] * P   # prefix tokens in the CSR
        prefix = meta.kv_indices[kv[i]:kv[i + 1]].to(torch.int32)
        new = loc[qo[i]:qo[i + 1]]
        if P > 1:
            first = (torch.arange(start, start + nnew, device=new.device) % P) == 0
            new = new[first] // P
        parts += [prefix, new.to(torch.int32)]
        indptr.append(indptr[-1] + prefix.numel() + new.numel())
        tokens.append(resident + nnew)
        modes.append(e["mode"])
    dev = queries.device
    kpool, _ = st.pools(layer.layer_id)
    kernels.prefill_scores(
        queries, kpool, meta.qo_indptr[: len(rows) + 1].to(torch.int32),
        torch.tensor(indptr, dtype=torch.int32, device=dev), torch.cat(parts),
        torch.tensor(tokens, dtype=torch.int32, device=dev), layer.scaling, P,
        max_q=max(qo[i + 1] - qo[i] for i in range(len(rows))), max_tokens=max(tokens),
        sinks=sinks, mode_of_row=torch.tensor(modes, dtype=torch.int32, device=dev),
        scores=st.scores[st.index[layer.layer_id]], zero_new=False, err=st.err)


# ------------------------------------------- static replay and verification
def _token_rows(pool, loc, page):
    """[n, G, D] rows of the tokens at pool slots `loc` from a [units, G, page, D] pool."""
    if page == 1:
        return pool[loc, :, 0]
    return pool[loc // page, :, loc % page]


class ShadowKV:
    """The first full layer's keys and values indexed by logical position:
    the unevicted cache that the replay metric and the verify checks compare
    against (runtime:227-238).  Storage is [capacity, G, D] bf16 per side,
    the capacity a whole number of INTERVAL blocks, so a request's shadow is
    reallocated at most once per 2,048 tokens."""

    def __init__(self, kv_heads, dim, device):
        self.k = torch.zeros((0, kv_heads, dim), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)

    def put(self, start, k_rows, v_rows):
        """Write the rows of positions start .. start + len(k_rows) - 1."""
        end = start + k_rows.shape[0]
        if end > self.k.shape[0]:
            cap = -(-end // INTERVAL) * INTERVAL
            for side in ("k", "v"):
                old = getattr(self, side)
                grown = torch.zeros((cap,) + tuple(old.shape[1:]), dtype=old.dtype, device=old.device)
                grown[:old.shape[0]].copy_(old)
                setattr(self, side, grown)
        self.k[start:end].copy_(k_rows)
        self.v[start:end].copy_(v_rows)


def _visible(st, entry, end):
    """Per-KV-head visibility of logical tokens [0, end) as [G, words] int32
    bit words (runtime:241-247): each head's survivors below the frontier
    (their pages' tokens at page sizes > 1), then the tail; None when nothing
    was evicted yet."""
    if not entry["count"]:
        return None
    P = st.page_size
    visible = torch.zeros((st.kv_heads, end), dtype=torch.bool, device=st.device)
    visible[:, entry["frontier"] * P:] = True
    # kept units lie below the frontier, so their tokens lie below end
    tokens = (entry["pos"][0][..., None] * P + torch.arange(P, device=st.device)).reshape(st.kv_heads, -1)
    visible.scatter_(1, tokens, True)
    return _pack_bits(visible)


def _replay_layer_difference(st, entry, queries, layer, sinks, start):
    """Per-token relative L2 error of the first full layer's attention output,
    evicted against full (runtime:520-546), by ce_replay_error over the
    shadow: both outputs use the unevicted keys, the evicted one restricted to
    each head's visible positions."""
    end = start + queries.shape[0]
    shadow = entry["shadow"]
    error = kernels.replay_error(queries, shadow.k, shadow.v, start, layer.scaling,
                                 visible_bits=_visible(st, entry, end), sinks=sinks, err=st.err)
    entry["layer_error"].append(error)


def _verify_decode(st, queries, out, layer, forward_batch, sinks):
    """GSTAR_EVICT_VERIFY=1, eager only (runtime:250-274): the first full
    layer's output of every live row with a shadow equals attention over each
    head's claimed positions; the largest absolute difference is kept.  The
    new token's key and value join the shadow first; ce_replay_error's masked
    output over the shadow is the expected output."""
    rows = forward_batch.req_pool_indices.tolist()
    checked = [(i, st.entries[r]) for i, r in enumerate(rows)
               if r in st.entries and st.entries[r]["kind"] == "live" and "shadow" in st.entries[r]]
    if not checked:
        return
    heads, dim = layer.tp_q_head_num, layer.qk_head_dim
    kpool, vpool = st.pools(st.first_full)
    new_loc = forward_batch.out_cache_loc.long()
    new_pos = forward_batch.positions.tolist()
    got = out.view(-1, heads, dim).float()
    expected = torch.empty((1, heads, dim), dtype=torch.float32, device=st.device)
    for i, entry in checked:
        p = int(new_pos[i])
        shadow = entry["shadow"]
        shadow.put(p, _token_rows(kpool, new_loc[i:i + 1], st.page_size),
                   _token_rows(vpool, new_loc[i:i + 1], st.page_size))
        kernels.replay_error(queries[i:i + 1], shadow.k, shadow.v, p, layer.scaling,
                             visible_bits=_visible(st, entry, p + 1), sinks=sinks, out_masked=expected,
                             err=st.err)
        gap = float((got[i] - expected[0]).abs().max())
        entry["verify_max_error"] = max(entry.get("verify_max_error", 0.0), gap)
        entry["verify_steps"] = entry.get("verify_steps", 0) + 1


def _relocation_ok(st, entry, table):
    """Each head's keys at the table's units equal the unevicted keys of the
    positions it claims (runtime:510-515), token by token."""
    P = st.page_size
    kpool, _ = st.pools(st.first_full)
    pos = entry["pos"][0]                                             # [G, count] units
    heads = torch.arange(st.kv_heads, device=st.device)[:, None]
    stored = kpool[table.long()[None, :].expand(st.kv_heads, -1), heads]   # [G, count, P, D]
    tokens = pos[..., None] * P + torch.arange(P, device=st.device)       # [G, count, P]
    want = entry["shadow"].k[tokens, heads[..., None]]                       # [G, count, P, D]
    return bool(torch.equal(stored, want))


def _events(entry, req):
    """A live request's event payload (runtime:712-716)."""
    keys = ("cfg", "error", "events", "peak_full_entries", "freed", "verify_max_error", "verify_steps")
    return {"kind": "events", **{k: entry.get(k) for k in keys},
            "length": len(req.origin_input_ids) + len(req.output_ids), "retracted": entry["key"] in RETRACTED}


# ------------------------------------------------------ regret diagnostic
# A diagnostic request (runtime:549-613) evicts nothing.  At each boundary it
# asks every "name:budget:prefix:recent" spec which positions it would keep,
# ranked by the unevicted cache's exact per-token tables, and then measures the
# softmax mass that each prefill query puts on the positions the spec dropped.
# A spec's state is the same positions-first form the live path keeps in
# State.pos: its kept positions [L, G, K] below the diagnostic frontier (None
# while nothing was dropped), everything from the frontier on resident.
def _diagnostic_entry(req, cfg, device, layers, heads):
    """A prefill-only entry scoring several eviction specs against the
    unevicted cache (runtime:549-560)."""
    specs = [(name, int(budget), int(prefix), int(recent))
             for name, budget, prefix, recent in (item.split(":") for item in str(cfg["policies"]).split(","))]
    length = len(req.origin_input_ids)
    tables = torch.zeros((2, layers, heads, length), device=device)   # head_sum, head_max per token
    return {"kind": "diagnostic", "key": _identity(req), "mode": 0, "specs": specs, "error": None,
            "frontier": 0, "seed": int(cfg.get("seed", 0)), "kept": [None] * len(specs),
            "score_sum": tables[0], "score_max": tables[1], "layers_seen": set(),
            "lost": torch.zeros((len(specs), length), device=device)}


def _diagnostic_draws(entry, j, n, name, pos):
    """The ranking key of spec j's candidates at a boundary at n (the
    reference draws its random keys with seed * 1000003 + 31 n + j)."""
    dev = pos.device
    L, G = pos.shape[:2]
    if name == "random_2048":
        gen = torch.Generator(device=dev).manual_seed((entry["seed"] * 1000003 + n * 31 + j) & 0x7FFFFFFF)
        return torch.rand(tuple(pos.shape), generator=gen, device=dev, dtype=torch.float64)
    if name == "random_reservoir_2048":
        return reservoir_scores(entry["seed"], pos, torch.arange(L, device=dev), torch.arange(G, device=dev))
    table = entry["score_max" if name == "head_max_sum_2048" else "score_sum"]
    return torch.gather(table, 2, pos).double()


def _diagnostic_boundary(entry, n):
    """Every spec's per-head boundary at n, ranked by the unevicted tables
    (runtime:563-584): candidates are the spec's kept positions and the new
    positions [frontier, n); the survivors become its kept positions."""
    L, G = entry["score_sum"].shape[:2]
    dev = entry["score_sum"].device
    fresh = torch.arange(entry["frontier"], n, device=dev).expand(L, G, -1)
    for j, (name, budget, prefix, recent) in enumerate(entry["specs"]):
        kept = entry["kept"][j]
        if kept is None:
            kept = torch.zeros((L, G, 0), dtype=torch.long, device=dev)
            pos = torch.arange(0, n, device=dev).expand(L, G, -1)
        else:
            pos = torch.cat((kept, fresh), -1)
        if pos.shape[-1] <= budget:
            if entry["kept"][j] is not None:
                entry["kept"][j] = pos.contiguous()
            continue
        cols, _ = choose(name, pos, n, budget, prefix, recent, _diagnostic_draws(entry, j, n, name, pos))
        entry["kept"][j] = torch.gather(pos, 2, cols)
    entry["frontier"] = n


def _diagnostic_resident(entry, j, layer_index, end):
    """Spec j's resident positions [G, end) of one layer as booleans."""
    G = entry["score_sum"].shape[1]
    dev = entry["score_sum"].device
    kept = entry["kept"][j]
    if kept is None:
        return torch.ones((G, end), dtype=torch.bool, device=dev)
    resident = torch.zeros((G, end), dtype=torch.bool, device=dev)
    resident[:, entry["frontier"]:] = True
    resident.scatter_(1, kept[layer_index], True)
    return resident


def _pack_bits(mask):
    """[..., T] bool -> [..., ceil(T/32)] int32 bit words (bit t of word t/32)."""
    T = mask.shape[-1]
    W = max(1, -(-T // 32))
    padded = torch.zeros(mask.shape[:-1] + (W * 32,), dtype=torch.int64, device=mask.device)
    padded[..., :T] = mask.to(torch.int64)
    words = (padded.view(mask.shape[:-1] + (W, 32)) << torch.arange(32, device=mask.device)).sum(-1)
    return torch.where(words >= 1 << 31, words - (1 << 32), words).to(torch.int32).contiguous()


def _diagnose(st, entry, index, layer, queries, keys, sinks, slots, start):
    """One full layer of one prefill chunk (runtime:587-613): the exact
    per-token head_sum / head_max tables (ce_prefill_scores over the whole
    unevicted prefix) and each spec's lost mass (ce_prefill_lost)."""
    count = queries.shape[0]
    end = start + count
    if start // INTERVAL != (end - 1) // INTERVAL:
        entry["error"] = "prefill chunk crosses a boundary; use --chunked-prefill-size 2048 and run alone"
        return
    if st.page_size != 1:
        raise NotImplementedError("the regret diagnostic works on token slots (page size 1)")
    if layer.layer_id == st.first_full and start % INTERVAL == 0 and start > entry["frontier"]:
        _diagnostic_boundary(entry, start)
    heads, kv_heads = layer.tp_q_head_num, layer.tp_k_head_num
    dev = queries.device
    kpool = keys.view(keys.shape[0], kv_heads, 1, keys.shape[-1])
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)
    qo, kvp, tok = i32([0, count]), i32([0, end]), i32([end])
    idx = slots.to(torch.int32).contiguous()
    q = queries.contiguous()
    for table, mode in (("score_sum", capi.CE_MODE_SUM), ("score_max", capi.CE_MODE_MAX)):
        scratch = torch.zeros((kv_heads, kpool.shape[0]), dtype=torch.float32, device=dev)
        kernels.prefill_scores(q, kpool, qo, kvp, idx, tok, layer.scaling, 1, count, end, sinks=sinks,
                               mode_of_row=i32([mode]), scores=scratch, zero_new=False, err=st.err)
        entry[table][index, :, :end] += scratch[:, slots.long()]
    evicted = _pack_bits(torch.stack([~_diagnostic_resident(entry, j, index, end)
                                      for j in range(len(entry["specs"]))]))
    kernels.prefill_lost(q, kpool, qo, kvp, idx, tok, layer.scaling, 1, count, end, evicted,
                         entry["lost"][:, start:end], 1.0 / (heads * len(st.full_layers)),
                         sinks=sinks, err=st.err)
    entry["layers_seen"].add(layer.layer_id)


# ------------------------------------------------------------- selection
_MASK = (1 << 64) - 1


def reservoir_scores(seed, pos, layers, heads):
    """splitmix64 score per (seed, layer, KV head, position) (runtime:358-373)."""
    L, G = int(layers.numel()), int(heads.numel())
    if not (torch.equal(layers.cpu(), torch.arange(L)) and
            torch.equal(heads.cpu(), torch.arange(int(heads[0]), int(heads[0]) + G))):
        raise ValueError("reservoir_scores expects arange layers and contiguous heads")
    p = pos.expand(L, G, pos.shape[-1]) if pos.dim() == 3 else pos
    ints = kernels.reservoir_scores53(p.contiguous(), int(seed) & _MASK, int(heads[0]))
    return ints.double() / float(1 << 53)


def choose(name, pos, n, budget, prefix, recent, score, cursor=None):
    """Survivors of one boundary for every (layer, KV head) row of pos [L, G, N].

    Returns (kept columns [L, G, K] in ascending position, protected count),
    or (None, count) when protection exceeds the budget; raises RuntimeError
    when heads protect different counts (runtime:384-397).
    """
    name = canonical(name)
    L, G, N = pos.shape
    dev = pos.device
    pos32 = pos.to(torch.int32).reshape(1, L * G, N).contiguous()
    sc = None
    if name not in ("prefix_sliding_2048", "random_reservoir_2048") and score is not None:
        sc = score.reshape(1, L * G, N).contiguous()
        if sc.dtype not in (torch.float32, torch.float64):
            sc = sc.double()
    row = dict(n=int(n), budget=int(budget), prefix=int(prefix), recent=int(recent),
               cursor=cursor, policy=name, seed=0)
    if name == "random_reservoir_2048" and score is not None:
        # the caller supplied reservoir draws: rank them as explicit doubles
        sc = score.reshape(1, L * G, N).double().contiguous()
        row["policy"] = "random_2048"
    max_n = max(int(n), int(pos.max().item()) + 1 if N else 1)
    kept, status, pcount = kernels.choose(pos32, sc, kernels.row_params([row], dev), L, G, max_n)
    st, count = int(status[0]), int(pcount[0])
    if st == 3:
        raise RuntimeError("protected positions differ between heads")
    if st == 2:
        return None, count
    k = count if name == "prefix_sliding_2048" else min(int(budget), N)
    return kept[0, :, :k].reshape(L, G, k).long(), count


def _scores(st, entry, name, pos, slots, n):
    """Per-column keys of a boundary, as the reference builds them (runtime:400-412)."""
    device = pos.device
    seed = int(entry["cfg"].get("seed", 0))
    name = canonical(name)
    if name == "random_2048":
        generator = torch.Generator(device=device).manual_seed((seed * 1000003 + n) & 0x7FFFFFFF)
        return torch.rand(pos.shape, generator=generator, device=device, dtype=torch.float64)
    if name == "random_reservoir_2048":
        return reservoir_scores(seed, pos, torch.arange(pos.shape[0], device=device),
                                torch.arange(pos.shape[1], device=device))
    if name in ("head_sum_2048", "head_max_sum_2048"):
        return st.scores[:, :, slots].double()
    if name == "h2o_global_2048":
        s = st.scores[:, :, slots]
        acc = torch.zeros((s.shape[0], s.shape[2]), dtype=torch.float32, device=device)
        for g in range(s.shape[1]):
            acc = acc + s[:, g]
        return acc[:, None, :].expand(-1, s.shape[1], -1).double()
    return torch.zeros(pos.shape, device=device, dtype=torch.float64)


def _units(st, tokens, what):
    if tokens % st.page_size:
        raise ValueError(f"{what}={tokens} is not a multiple of the page size {st.page_size}")
    return tokens // st.page_size


def _boundary(st, row, entry, n, cursor=None, allocator=None):
    """Evict at logical length n: choose per head, relocate survivors, free the rest.

    With allocator=None (static replay) survivors are relocated but nothing is
    freed and req_to_token is untouched (runtime:415-421).
    """
    cfg = entry["cfg"]
    name = canonical(cfg["name"])
    page = st.page_size
    budget, prefix, recent = (_units(st, int(cfg[k]), k) for k in ("budget", "prefix", "recent"))
    n_u = _units(st, int(n), "n")
    cur_u = None if cursor is None else int(cursor) // page
    frontier, count = entry["frontier"], entry["count"]
    started = time.perf_counter()
    N = count + n_u - frontier
    entry["last_boundary"] = n
    if N <= budget:
        entry["events"].append({"boundary": n, "before": int(N), "after": int(N)})
        return
    L, G = len(st.full_layers), st.kv_heads
    uniforms = None
    if name == "random_2048":
        generator = torch.Generator(device=st.device).manual_seed(
            (int(cfg.get("seed", 0)) * 1000003 + n) & 0x7FFFFFFF)
        draw = torch.rand((L, G, N), generator=generator, device=st.device, dtype=torch.float64)
        uniforms = draw.reshape(1, L, G, N)
    st.epoch += 1
    kptr, vptr = st.layer_pointers()
    live = allocator is not None
    swa = getattr(allocator, "full_to_swa_index_mapping", None) if live else None
    rows = torch.tensor([row], dtype=torch.int32, device=st.device)
    params = kernels.row_params([dict(n=n_u, budget=budget, prefix=prefix, recent=recent,
                                      cursor=cur_u, policy=name, seed=int(cfg.get("seed", 0)))],
                                st.device)
    record = None
    if cfg.get("record"):
        record = (torch.empty((L * G, N), dtype=torch.int32, device=st.device),
                  torch.empty(L * G, dtype=torch.int32, device=st.device))
    result, leftover = kernels.boundary(
        st.table, st.req_to_token, st.frontier, st.count, st.pos, st.scores, kptr, vptr, G, page,
        rows, params, N, n_u + 1, live, marks=st.marks, epoch=st.epoch, swa=swa,
        uniforms=uniforms, head_offset=st.head_offset, err=st.err, max_width=budget, record=record)
    res = result[0].tolist()  # synchronises, as the reference does (runtime:474, 492)
    finished = time.perf_counter()
    status, before, after, nfreed = res
    if status == 2:
        entry["events"].append({"boundary": n, "deferred": True, "protected": after})
        return
    if status == 3:
        raise RuntimeError("protected positions differ between heads")
    if status == 6:
        raise RuntimeError(f"boundary sizes exceed the state capacity (pos_cap {st.pos_cap})")
    entry["pos"] = st.pos[row, :, :, :after].long()
    entry.update(frontier=n_u, count=after)
    if status == 5:
        raise RuntimeError("gstar_evict would free a slot that still holds a sliding-window entry")
    if live:
        allocator.free_full(leftover[0, :nfreed].long())
        entry["freed"] = entry.get("freed", 0) + nfreed
    if status == 4:
        raise RuntimeError("packed ownership overlaps the sliding-window region")
    elapsed = 1000 * (finished - started)
    event = {"boundary": n, "before": before, "after": after, "freed": nfreed,
             "swa_cursor": cursor, "ranking_ms": elapsed, "compaction_ms": 0.0}
    if st.verify and "shadow" in entry:
        event["relocation_ok"] = _relocation_ok(st, entry, st.table[row, :after])
    entry["events"].append(event)
    if record is not None:
        _write_record(st, entry, cfg, n, record)


def _write_record(st, entry, cfg, n, record):
    """Retention payload of one boundary (runtime:465-467, 500-507): victims
    per (full layer, KV head), ascending, delta-coded.  With pages of P tokens
    an evicted page stands for its P token positions (boundaries fall on
    page multiples), so the record keeps the reference's token positions."""
    counts = record[1].cpu().numpy()
    delta = record[0].cpu().numpy().view(np.uint32)
    P = st.page_size
    lengths, deltas = [], []
    for s, c in enumerate(counts):
        victims = np.cumsum(delta[s, :c].astype(np.int64))
        if P > 1:
            victims = (victims[:, None] * P + np.arange(P)).ravel()
        lengths.append(len(victims))
        deltas.append(np.diff(victims, prepend=0))
    write_payload(f"{entry['key']}-b{n}", {
        "kind": "retention", "boundary": n, "cfg": cfg, "layers": st.full_layers,
        "kv_heads": st.kv_heads,
        "evicted_delta": array(np.concatenate(deltas) if deltas else np.zeros(0), "uint32"),
        "evicted_counts": array(lengths, "int32")})


# ------------------------------------------------------------ scheduler hooks
def _identity(req):
    session = getattr(req, "session", None)
    if session is not None and getattr(session, "streaming", False):
        return f"session-{session.session_id}"
    return req.rid


def _live_entry(req, cfg, kind):
    entry = {"kind": kind, "key": _identity(req), "cfg": dict(cfg),
             "mode": POLICIES.get(canonical(str(cfg.get("name"))), 0), "events": [], "error": None,
             "frontier": 0, "count": 0, "last_boundary": 0, "peak_full_entries": 0,
             "layer_error": []}
    try:
        validate(cfg, getattr(STATE, "page_size", 1) if STATE is not None else 1)
    except ValueError as error:
        entry["error"], entry["mode"] = str(error), 0
    return entry


def on_extend(batch):
    """Create entries from custom_params and run boundaries at chunk starts (runtime:640-689)."""
    st = STATE
    if st is None:
        return
    for req in batch.reqs:
        row = req.kv.req_pool_idx
        params = getattr(req.sampling_params, "custom_params", None) or {}
        entry = st.entries.get(row)
        if entry is not None and entry["key"] != _identity(req):
            _reset(st, row)  # the row now belongs to another request or session
            entry = None
        if entry is None:
            if "gstar_diagnostic" in params:
                entry = _diagnostic_entry(req, params["gstar_diagnostic"], st.req_to_token.device,
                                          len(st.full_layers), st.kv_heads)
            elif "gstar_replay" in params:
                entry = _live_entry(req, params["gstar_replay"], "replay")
            elif "gstar_eviction" in params:
                entry = _live_entry(req, params["gstar_eviction"], "live")
            else:
                continue
            st.entries[row] = entry
            st.mode[row] = 0 if entry["kind"] == "diagnostic" or entry["error"] else \
                SCORE_MODE.get(canonical(str(entry["cfg"].get("name"))), 0)
            st.frontier[row], st.count[row] = 0, 0
        if entry["kind"] == "diagnostic" or entry["error"]:
            continue
        if getattr(req, "retraction_count", 0) or entry["key"] in RETRACTED:
            # a retracted request recomputes its KV from scratch, which evicted state cannot survive
            RETRACTED.add(entry["key"])
            entry["error"] = "retracted"
            write_payload(f"{entry['key']}-retracted", {"kind": "retracted", "cfg": entry["cfg"]})
            st.mode[row] = 0
            continue
        start, length = req.extend_range.start, req.extend_range.length
        if start < entry["frontier"] * st.page_size:
            entry["error"] = "the session rewound below the eviction frontier"
        elif length and start // INTERVAL != (start + length - 1) // INTERVAL:
            entry["error"] = "prefill chunk crosses a boundary; use --chunked-prefill-size 2048"
        if entry["error"]:
            st.mode[row] = 0
            continue
        if start and start % INTERVAL == 0 and start > entry["last_boundary"]:
            torch.cuda.synchronize()  # the previous chunk's keys and scores are complete
            if entry["kind"] == "replay":
                _boundary(st, row, entry, start)
            else:
                _boundary(st, row, entry, start, _swa_cursor(req),
                          batch.tree_cache.token_to_kv_pool_allocator)


def _swa_cursor(req):
    getter = getattr(req.kv, "get_evicted_seqlen", None)
    if getter is None:
        return None
    try:
        from sglang.srt.mem_cache.unified_cache.component_type import ComponentType
        return getter(ComponentType.SWA)
    except ImportError:
        return getter("swa")


def on_decode(batch):
    """Run due boundaries before the decode step (runtime:692-710)."""
    st = STATE
    if st is None or not st.entries:
        return
    lengths = batch.seq_lens_cpu.tolist()
    for i, req in enumerate(batch.reqs):
        row = req.kv.req_pool_idx
        entry = st.entries.get(row)
        if entry is None or entry["kind"] != "live" or entry["error"] or entry["key"] != _identity(req):
            continue
        n = lengths[i]
        entry["peak_full_entries"] = max(entry["peak_full_entries"],
                                         entry["count"] * st.page_size + n - entry["frontier"] * st.page_size)
        if n % INTERVAL or n <= entry["last_boundary"]:
            continue
        torch.cuda.synchronize()  # the previous decode step wrote query n-1's key and scores
        _boundary(st, row, entry, n, _swa_cursor(req), batch.tree_cache.token_to_kv_pool_allocator)


def release(req):
    """At a request's KV release drop its state unless its session keeps the row (runtime:719-742)."""
    st = STATE
    if st is None or not req.kv.holds_kv:
        return
    row = req.kv.req_pool_idx
    entry = st.entries.get(row)
    if entry is None or entry["key"] != _identity(req):
        return
    if entry["kind"] == "diagnostic":
        lost = entry["lost"][:, :len(req.origin_input_ids)].cpu().numpy()
        write_payload(req.rid, {"kind": "diagnostic", "error": entry["error"], "specs": entry["specs"],
                                "layers": sorted(entry["layers_seen"]), "lost": array(lost, "float32")})
    elif entry["kind"] == "replay":
        error = torch.cat(entry["layer_error"]).cpu().numpy() if entry["layer_error"] else np.zeros(0)
        write_payload(req.rid, {"kind": "replay", "cfg": entry["cfg"], "error": entry["error"],
                                "events": entry["events"], "layer": st.first_full,
                                "layer_error": array(error, "float32")})
    else:
        session = entry["key"] != req.rid
        write_payload(f"{entry['key']}-events" if session else req.rid, _events(entry, req))
        if session:
            return  # the session keeps its row and eviction state for the next call
    _reset(st, row)


def filter_holes(segments):
    """Holes are zero and below the sliding-window cursor, so only full-side frees see them."""
    return [(kv[kv != 0], start) for kv, start in segments]
