"""Ragged continuous-batch decode with per-row KV eviction, on the device.

The engine keeps every row of a continuous batch packed in one paged pool per
full-attention layer and drives the four kernels through the C ABI:

  * per step: ce_fill builds one CSR over all rows (compacted residents then
    the tail, runtime:136-152), and ce_decode_attn_score runs the fused decode
    attention + H2O score for each full layer;
  * at boundaries (a row's length hits a multiple of 2048, runtime:692-710):
    ce_boundary selects and compacts every due row in one batched call;
  * units come from a free-unit stack on the device (ce_pool_alloc pops one
    for every row whose new token starts a unit, ce_pool_push returns a
    boundary's leftovers and a retired row's units), so rows can be admitted
    and retired between steps and the pool is sized to what is resident, as
    SGLang's allocator serves the reference (runtime:476-482, 719-742).

Rows, their policies and lengths live on the host (like SGLang's scheduler);
eviction state (tables, positions, scores, pools) lives on the device.  With
tensor parallelism each rank holds kv_heads/tp heads of every row; the only
cross-rank exchange on the eviction path is the all-gather of per-head scores
that H2O global needs at a boundary (tp.py adds the attention-output reduction).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from . import capi, kernels
from .policy import INTERVAL, EvictionConfig

D = 64


@dataclass
class Row:
    cfg: Optional[EvictionConfig]    # None = full cache, no eviction
    n: int                           # tokens in the cache
    last_boundary: int = 0
    frontier: int = 0                # units
    count: int = 0                   # units
    events: list = field(default_factory=list)
    freed: int = 0


class RaggedDecodeEngine:
    def __init__(self, *, layers: int, q_heads: int, kv_heads: int, page_size: int,
                 pool_units: int, max_rows: int, r2u_width: int, pos_cap: int,
                 device="cuda", head_offset: int = 0, global_kv_heads: Optional[int] = None,
                 process_group=None, alloc_pools: bool = True, boundary_rows: int = 8,
                 hazard_bytes: int = 512 << 20, overlap_scores: bool = False):
        self.L, self.H, self.G, self.P = layers, q_heads, kv_heads, page_size
        self.units = pool_units
        self.device = torch.device(device)
        self.head_offset = head_offset
        self.global_G = global_kv_heads or kv_heads
        self.group = process_group
        dev = self.device
        if alloc_pools:
            shape = (pool_units, kv_heads, page_size, D)
            self.k = [torch.empty(shape, dtype=torch.bfloat16, device=dev) for _ in range(layers)]
            self.v = [torch.empty(shape, dtype=torch.bfloat16, device=dev) for _ in range(layers)]
            self.kptr = kernels.layer_pointers(self.k, dev)
            self.vptr = kernels.layer_pointers(self.v, dev)
        self.scores = torch.zeros((layers, kv_heads, pool_units), dtype=torch.float32, device=dev)
        self.table = torch.zeros((max_rows, pos_cap), dtype=torch.int32, device=dev)
        self.r2u = torch.zeros((max_rows, r2u_width), dtype=torch.int32, device=dev)
        self.frontier = torch.zeros(max_rows, dtype=torch.int32, device=dev)
        self.count = torch.zeros(max_rows, dtype=torch.int32, device=dev)
        self.mode = torch.zeros(max_rows, dtype=torch.int32, device=dev)
        self.pos = torch.zeros((max_rows, layers, kv_heads, pos_cap), dtype=torch.int32, device=dev)
        self.marks = torch.zeros(pool_units, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = 0
        self.pos_cap = pos_cap
        self.rows: dict[int, Row] = {}
        self.active: list[int] = []
        self.kv_indptr = torch.zeros(max_rows + 1, dtype=torch.int32, device=dev)
        self.kv_tokens = torch.zeros(max_rows, dtype=torch.int32, device=dev)
        self.kv_indices = torch.zeros(1, dtype=torch.int32, device=dev)
        self.rows_dev = torch.zeros(0, dtype=torch.int64, device=dev)
        self.seq_lens_dev = torch.zeros(0, dtype=torch.int64, device=dev)
        # free-unit stack: units[0 .. top) on the device; free_top mirrors top
        # on the host exactly (every push and pop count is known there)
        self.free_stack = torch.zeros(pool_units, dtype=torch.int32, device=dev)
        self.free_top_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        self.free_top = 0
        self.boundary_ms: list = []
        # advance() calls until some evicting row reaches a boundary (None:
        # unknown), so due() scans the rows only when one can be due
        self._due_in = None
        # exact CSR need at some advance count (_ensure_capacity); None: unknown
        self._cap_base = None
        self._advances = 0
        self.last_batch: Optional[dict] = None
        # The boundary workspace is sized up front for batches of up to
        # `boundary_rows` rows, so no device allocation falls inside the decode
        # loop (a larger batch grows it once).
        self.hazard_bytes = hazard_bytes
        self.r2u_width = r2u_width
        # With overlap_scores a layer's H2O page scores (ce_decode_scores) run
        # on their own stream beside the next layer's attention, from one of
        # two decode workspaces alternating by layer (decode_layer).  Off by
        # default: measured against scoring inside the decode call it gained
        # 0-1 % at a batch of 64 and at batch 1 (CUDA-graph steps) and lost
        # ~3 % end to end in a host-driven loop with per-layer copies.
        self.overlap_scores = overlap_scores
        # score_flags of every decode call: 0 makes the engine a plain
        # full-cache decode (no score workspace, no score launches)
        self.score_flags = 3
        self._score_stream = torch.cuda.Stream(dev) if overlap_scores else None
        self._dec_ws = [None, None]
        self._ws_need = (None, 0)
        self.new_score_events()
        self._scores_pending = False
        if alloc_pools:
            # kernels loaded now rather than inside the first step that needs them
            kernels.prepare_device(dev)
            kernels.reserve_boundary(dev, min(max_rows, boundary_rows), layers, kv_heads, page_size,
                                     r2u_width, pos_cap,
                                     self.global_G if process_group is not None else 0, hazard_bytes)

    def new_score_events(self):
        """Fresh ordering events for the score stream.  Also for a CUDA-graph
        capture: a capture may not wait on an event recorded outside it, and
        no stream may wait on an event last recorded inside one, so call this
        (after join_scores) right before a capture and again right after."""
        self._ws_free = [torch.cuda.Event(), torch.cuda.Event()]
        self._attn_done = [torch.cuda.Event(), torch.cuda.Event()]

    def join_scores(self):
        """Order the current stream after every deferred page-score launch.
        Called before anything rewrites the CSR, the row lists or the decode
        workspaces, and before the scores are read."""
        if self._scores_pending:
            torch.cuda.current_stream(self.device).wait_stream(self._score_stream)
            self._scores_pending = False

    # ------------------------------------------------------------- rows
    def add_row(self, row: int, cfg: Optional[EvictionConfig], n: int, last_boundary: int = 0,
                frontier_units: int = 0, count_units: int = 0):
        self.join_scores()
        self.rows[row] = Row(cfg=cfg, n=n, last_boundary=last_boundary, frontier=frontier_units,
                             count=count_units)
        self._due_in = self._cap_base = None
        self.mode[row] = cfg.score_mode if cfg is not None else capi.CE_MODE_NONE
        self.frontier[row] = frontier_units
        self.count[row] = count_units
        if row not in self.active:
            self.active.append(row)

    def seed_free_units(self, units):
        """Make `units` (host ints) the free stack's contents (bottom first)."""
        units = np.asarray(units, dtype=np.int32)
        if len(units) > self.units:
            raise ValueError("more free units than the pool holds")
        self.free_stack[:len(units)] = torch.from_numpy(units).to(self.device)
        self.free_top_dev.fill_(len(units))
        self.free_top = len(units)

    def admit(self, row: int, cfg: Optional[EvictionConfig], n: int, prompt=None,
              settle: bool = True) -> torch.Tensor:
        """A new request whose n-token prompt is in the cache: ceil(n / P) units
        from the free stack become its req_to_unit row; prompt(units), if
        given, then fills them (K/V, prefill scores); then, as the chunked
        prefill would have done, the boundary at the last multiple of 2048
        at or below n runs (live: its leftovers go back to the stack) -- or,
        with settle=False, later in settle() together with other admissions.
        Returns the prompt's units (device int32).  Call commit_rows() after
        the admissions and retirements of a step."""
        k = -(-n // self.P)
        if k > self.free_top:
            raise RuntimeError(f"unit pool exhausted: {k} units wanted, {self.free_top} free")
        if k > self.r2u.shape[1]:
            raise ValueError("prompt longer than the req_to_unit width")
        dev = self.device
        seq = torch.arange(k, dtype=torch.int64, device=dev) * self.P + 1   # token j*P starts unit j
        kernels.pool_alloc(self.free_stack, self.free_top_dev, self.r2u,
                           torch.full((k,), row, dtype=torch.int64, device=dev), seq, self.P, self.err)
        self.free_top -= k
        units = self.r2u[row, :k].clone()
        if prompt is not None:
            prompt(units)
        self.add_row(row, cfg, n, last_boundary=0)
        if settle:
            self.settle([row])
        return units

    def settle(self, rows: list):
        """The prefill's last boundary (at the last multiple of 2048 at or
        below each row's length) for newly admitted rows, in one batch."""
        due = [r for r in rows if self.rows[r].cfg is not None and self.rows[r].n >= INTERVAL]
        if not due:
            return []
        lengths = {r: self.rows[r].n for r in due}
        for r in due:
            self.rows[r].n = (lengths[r] // INTERVAL) * INTERVAL
        try:
            return self.run_boundaries(due)
        finally:
            for r in due:
                self.rows[r].n = lengths[r]
            self._due_in = self._cap_base = None

    def retire(self, row: int):
        """A finished request: its resident units (compacted table and tail)
        return to the free stack; the row leaves the batch."""
        self.join_scores()
        r = self.rows.pop(row)
        self._due_in = self._cap_base = None
        tail_end = -(-r.n // self.P)
        owned = torch.cat([self.table[row, :r.count], self.r2u[row, r.frontier:tail_end]]).view(1, -1)
        k = int(owned.shape[1])
        if k:
            counts = torch.tensor([k], dtype=torch.int32, device=self.device)
            kernels.pool_push(self.free_stack, self.free_top_dev, owned.contiguous(), counts, self.err)
            self.free_top += k
        self.mode[row] = capi.CE_MODE_NONE
        self.frontier[row] = 0
        self.count[row] = 0
        self.active.remove(row)

    def owned_units(self, row: int) -> torch.Tensor:
        """The units row holds now (device int32): compacted table, then tail."""
        r = self.rows[row]
        return torch.cat([self.table[row, :r.count], self.r2u[row, r.frontier:-(-r.n // self.P)]])

    def commit_rows(self):
        """Upload the active row list and lengths (after rows were added)."""
        self.join_scores()
        self.rows_dev = torch.tensor(self.active, dtype=torch.int64, device=self.device)
        self.seq_lens_dev = torch.tensor([self.rows[r].n for r in self.active], dtype=torch.int64,
                                         device=self.device)
        self._ensure_capacity()

    def resident_units(self, r: int, extra_tokens: int = 0) -> int:
        row = self.rows[r]
        units = -(-(row.n + extra_tokens) // self.P)
        return row.count + max(0, units - row.frontier)

    def resident_tokens(self, r: int) -> int:
        row = self.rows[r]
        return row.count * self.P + row.n - row.frontier * self.P

    def _ensure_capacity(self, extra_tokens: int = 1):
        # A row gains at most one unit per P tokens, so from the last exact
        # count the need is bounded without a pass over the rows; the pass
        # (512 rows at eight ranks) runs only when the bound nears capacity.
        if self._cap_base is not None:
            need0, adv0, e0, nrows = self._cap_base
            grown = max(0, self._advances - adv0 + extra_tokens - e0)
            if need0 + nrows * (grown // self.P + 1) <= self.kv_indices.numel():
                return
        need = sum(self.resident_units(r, extra_tokens) for r in self.active) + 16
        self._cap_base = (need, self._advances, extra_tokens, len(self.active))
        if self.kv_indices.numel() < need:
            self.join_scores()
            self.kv_indices = torch.zeros(int(need * 1.25), dtype=torch.int32, device=self.device)

    # -------------------------------------------------------- boundaries
    def due(self) -> list:
        """Rows whose length sits on a boundary not yet taken (runtime:706).
        Every row grows by one token per advance(), so the scan also notes how
        many advances it is until the next row can be due; until then due()
        returns at once (a 512-row scan per step was host time the GPU waited
        for at eight ranks)."""
        if self._due_in is not None and self._due_in > 0:
            return []
        out, nxt = [], INTERVAL
        for r in self.active:
            row = self.rows[r]
            if row.cfg is None:
                continue
            k = row.n % INTERVAL
            if k == 0 and row.n > row.last_boundary:
                out.append(r)
            else:
                nxt = min(nxt, INTERVAL - k if k else INTERVAL)
        self._due_in = None if out else nxt
        return out

    def run_boundaries(self, rows: list, cursors: Optional[dict] = None, live: bool = True,
                       swa: Optional[torch.Tensor] = None, hazard_bytes: Optional[int] = None):
        """One batched ce_boundary over `rows`; returns the per-row results (host)."""
        if not rows:
            return []
        self.join_scores()
        P = self.P
        hazard_bytes = self.hazard_bytes if hazard_bytes is None else hazard_bytes
        params, ncols = [], []
        for r in rows:
            row = self.rows[r]
            b, p, q = row.cfg.units(P)
            n_u = row.n // P
            cur = None if not cursors or cursors.get(r) is None else cursors[r] // P
            params.append(dict(n=n_u, budget=b, prefix=p, recent=q, cursor=cur,
                               policy=row.cfg.policy_id, seed=row.cfg.seed))
            ncols.append(row.count + n_u - row.frontier)
            row.last_boundary = row.n
        max_cols = max(ncols)
        max_n = max(prm["n"] for prm in params) + 1
        dev = self.device
        uniforms = None
        if any(self.rows[r].cfg.name == "random_2048" for r in rows):
            uniforms = torch.zeros((len(rows), self.L, self.G, max_cols), dtype=torch.float64, device=dev)
            for i, r in enumerate(rows):
                row = self.rows[r]
                if row.cfg.name != "random_2048":
                    continue
                gen = torch.Generator(device=dev).manual_seed((row.cfg.seed * 1000003 + row.n) & 0x7FFFFFFF)
                draw = torch.rand((self.L, self.global_G, ncols[i]), generator=gen, device=dev,
                                  dtype=torch.float64)
                h0 = self.head_offset
                uniforms[i, :, :, :ncols[i]] = draw[:, h0:h0 + self.G]
        rows_t = torch.tensor(rows, dtype=torch.int32, device=dev)
        params_t = kernels.row_params(params, dev)
        gscores = None
        if self.group is not None and any(self.rows[r].cfg.name == "h2o_global_2048" for r in rows):
            from . import tp
            local = kernels.gather_row_scores(self.table, self.r2u, self.frontier, self.count,
                                              self.scores, rows_t, params_t, max_cols, self.err)
            gscores = tp.all_gather_heads(local, self.group)
        self.epoch += 1
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        result, freed = kernels.boundary(
            self.table, self.r2u, self.frontier, self.count, self.pos, self.scores, self.kptr,
            self.vptr, self.G, P, rows_t, params_t, max_cols, max_n, live, marks=self.marks,
            epoch=self.epoch, swa=swa, uniforms=uniforms, global_scores=gscores,
            head_offset=self.head_offset, hazard_bytes=hazard_bytes, err=self.err,
            max_width=max(prm["budget"] for prm in params))
        end.record()
        res = result.cpu().numpy()   # one readback per boundary batch, as the reference syncs
        self.boundary_ms.append(start.elapsed_time(end))
        # what this batch was given and returned (the uniforms are the exact
        # draws of the random rows), for callers that audit or replay it
        self.last_batch = dict(rows=list(rows), params=params, max_cols=max_cols, uniforms=uniforms,
                               result=res, freed=freed)
        pushed = 0
        for i, r in enumerate(rows):
            row = self.rows[r]
            status, before, after, nfreed = (int(x) for x in res[i])
            row.events.append(dict(boundary=row.n, status=status, before=before, after=after,
                                   freed=nfreed))
            if status == 0:
                row.frontier, row.count = row.n // P, after
                if live:
                    pushed += nfreed
                    row.freed += nfreed
            elif status not in (1, 2):
                raise RuntimeError(f"boundary for row {r} failed with status {status}")
        if live and pushed:
            # the leftovers go back to the free stack straight from the device result
            kernels.pool_push(self.free_stack, self.free_top_dev, freed, result[:, 3], self.err)
            self.free_top += pushed
        self._due_in = self._cap_base = None
        return res

    # ------------------------------------------------------------ decode
    def fill(self):
        self.join_scores()
        bs = len(self.active)
        kernels.fill(self.table, self.r2u, self.frontier, self.count, self.rows_dev,
                     self.seq_lens_dev, self.P, self.kv_indptr[:bs + 1], self.kv_indices,
                     self.kv_tokens[:bs], self.err)

    def _decode_workspace(self, k: int, bs: int, score_flags: int) -> torch.Tensor:
        """Decode workspace k of this engine (k = layer % 2 with overlap_scores,
        else 0), grown when the batch or the CSR capacity grew.  Each engine
        owns its workspaces, so a CUDA graph captured from one engine never
        depends on a buffer that another engine may regrow."""
        key = (bs, self.kv_indices.numel(), score_flags)
        if self._ws_need[0] != key:      # the same for every layer of a step
            self._ws_need = (key, kernels.decode_workspace_bytes(bs, key[1], self.H, self.G, self.P,
                                                                 score_flags))
        need = self._ws_need[1]
        if self._dec_ws[k] is None or self._dec_ws[k].numel() < need:
            self.join_scores()
            self._dec_ws[k] = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._dec_ws[k]

    def decode_layer(self, layer: int, q: torch.Tensor, out: torch.Tensor, sinks, scale: float,
                     score_flags: Optional[int] = None):
        bs = len(self.active)
        score_flags = self.score_flags if score_flags is None else score_flags
        if not (self.overlap_scores and score_flags & 3 and bs):
            ws = self._decode_workspace(0, bs, score_flags) if bs else None
            return kernels.decode_attn_score(
                q, self.k[layer], self.v[layer], self.kv_indptr[:bs + 1], self.kv_indices,
                self.kv_tokens[:bs], scale, self.P, sinks=sinks, mode_of_row=self.mode,
                rows=self.rows_dev, scores=self.scores[layer], zero_new=True, out=out,
                score_flags=score_flags, err=self.err, workspace=ws)
        # Attention and outputs on the current stream; this layer's page scores
        # on the score stream once they are done, overlapping the next layer.
        # Workspace k is reused two layers later, after its scores have run.
        k = layer % 2
        ws = self._decode_workspace(k, bs, score_flags)
        main = torch.cuda.current_stream(self.device)
        main.wait_event(self._ws_free[k])
        res = kernels.decode_attn_score(
            q, self.k[layer], self.v[layer], self.kv_indptr[:bs + 1], self.kv_indices,
            self.kv_tokens[:bs], scale, self.P, sinks=sinks, mode_of_row=self.mode,
            rows=self.rows_dev, scores=self.scores[layer], zero_new=True, out=out,
            score_flags=score_flags | capi.CE_SCORE_DEFER, err=self.err, workspace=ws)
        self._attn_done[k].record(main)
        side = self._score_stream
        side.wait_event(self._attn_done[k])
        kernels.decode_scores(self.kv_indptr[:bs + 1], self.kv_indices, self.kv_tokens[:bs], self.units,
                              self.P, self.H, self.G, bs, self.mode, self.rows_dev, self.scores[layer], ws,
                              zero_new=True, score_flags=score_flags, err=self.err, stream=side)
        self._ws_free[k].record(side)
        self._scores_pending = True
        return res

    def advance(self):
        """Append one token to every active row: host lengths, then the device
        lengths and a unit for every row whose new token starts one."""
        self.advance_host()
        self.advance_device()

    def advance_host(self):
        """The host side of advance (also what a replayed CUDA graph that
        captured advance_device needs)."""
        need = 0
        for r in self.active:
            row = self.rows[r]
            row.n += 1
            need += (row.n - 1) % self.P == 0
        self._advances += 1
        if self._due_in is not None:
            self._due_in -= 1
        if need > self.free_top:
            raise RuntimeError(f"unit pool exhausted: {need} units wanted, {self.free_top} free")
        self.free_top -= need

    def advance_device(self):
        """Device lengths + 1 and the new units (ce_pool_alloc); capturable."""
        self.seq_lens_dev.add_(1)
        if self.active:
            kernels.pool_alloc(self.free_stack, self.free_top_dev, self.r2u, self.rows_dev, self.seq_lens_dev,
                               self.P, self.err)

    def step(self, q_layers, out_layers, sinks, scale, after_layer=None, before_layer=None):
        """One decode step: due boundaries, one token appended, CSR, every layer.

        before_layer(l) / after_layer(l, out) run on the host around layer l's
        launches (e.g. to make the compute stream wait for layer l's query
        upload, or to queue layer l's output download on another stream)."""
        self.run_boundaries(self.due())
        self.advance()
        self._ensure_capacity(0)
        self.fill()
        for l in range(self.L):
            if before_layer is not None:
                before_layer(l)
            self.decode_layer(l, q_layers[l], out_layers[l], sinks[l], scale)
            if after_layer is not None:
                after_layer(l, out_layers[l])

    def check_errors(self):
        torch.cuda.synchronize(self.device)
        word = int(self.err.item())
        if word:
            raise RuntimeError(f"device error word 0x{word:x}")


# -------------------------------------------------------------- synthesis
def synth_rows(specs: list, seed: int, *, layers: int, kv_heads: int, page_size: int,
               pool_units: int, max_rows: int, pos_cap: int, r2u_width: int, shuffle: bool = True):
    """Host arrays of rows initialised as if every boundary up to each context
    had been taken (the state synth_state uploads).

    specs: dicts with ctx (tokens), cfg (EvictionConfig or None).  Each evicting
    row holds prefix + recent + budget-remainder residents after its last
    evicting boundary (ascending positions, per-head middle picks for per-head
    policies, shared picks for H2O global) and its tail since that boundary.
    Units are drawn from a shuffled pool (in order with shuffle=False, so a
    row's pages are consecutive in memory).  Returns (arrays dict with table,
    r2u, pos, frontier, count; rows list of (row, cfg, n, last_boundary,
    frontier, count); owned units of each H2O row; the units left free).
    """
    rng = np.random.default_rng(seed)
    P, L, G = page_size, layers, kv_heads
    order = rng.permutation(np.arange(1, pool_units)).astype(np.int32) if shuffle else \
        np.arange(1, pool_units, dtype=np.int32)
    cursor = 0

    def take(k):
        nonlocal cursor
        out = order[cursor:cursor + k]
        cursor += k
        if len(out) < k:
            raise RuntimeError("pool too small for the synthetic state")
        return out

    table = np.zeros((max_rows, pos_cap), np.int32)
    r2u = np.zeros((max_rows, r2u_width), np.int32)
    pos = np.zeros((max_rows, L, G, pos_cap), np.int32)
    frontier_a = np.zeros(max_rows, np.int32)
    count_a = np.zeros(max_rows, np.int32)
    rows, scored = [], []
    for r, sp in enumerate(specs):
        cfg, ctx = sp["cfg"], int(sp["ctx"])
        end_units = -(-ctx // P)
        frontier = count = 0
        last = (ctx // INTERVAL) * INTERVAL
        if cfg is not None and last > cfg.budget:
            b_u, p_u, r_u = cfg.units(P)
            f_u = last // P
            w_u = b_u - p_u - r_u
            units = take(b_u)
            table[r, :b_u] = units
            recent = np.arange(f_u - r_u, f_u)
            prefix = np.arange(p_u)
            middle_pool = np.arange(p_u, f_u - r_u)
            shared = cfg.name in ("h2o_global_2048", "prefix_sliding_2048")
            if shared:
                mid = np.sort(rng.choice(middle_pool, w_u, replace=False)) if w_u else np.zeros(0, int)
            for l in range(L):
                for g in range(G):
                    if not shared:
                        mid = np.sort(rng.choice(middle_pool, w_u, replace=False)) if w_u else np.zeros(0, int)
                    pos[r, l, g, :b_u] = np.concatenate([prefix, recent, mid])
            # req_to_unit: real units at the protected recent positions, the rest packed
            true_u = f_u - r_u
            r2u[r, true_u:f_u] = units[p_u:p_u + r_u]
            packed = np.concatenate([units[:p_u], units[p_u + r_u:]])
            r2u[r, :len(packed)] = packed
            tail = take(end_units - f_u)
            r2u[r, f_u:end_units] = tail
            frontier, count = f_u, b_u
            owned = np.concatenate([units, tail])
        else:
            owned = take(end_units)
            r2u[r, :end_units] = owned
            last = last if cfg is not None else 0
        frontier_a[r], count_a[r] = frontier, count
        rows.append((r, cfg, ctx, last if cfg is not None else 0, frontier, count))
        if cfg is not None and cfg.score_mode != capi.CE_MODE_NONE:
            scored.append(owned)
    arrays = dict(table=table, r2u=r2u, pos=pos, frontier=frontier_a, count=count_a)
    return arrays, rows, scored, order[cursor:]


def synth_state(engine: RaggedDecodeEngine, specs: list, seed: int, score_sigma: float = 2.0,
                fill_pools: bool = True, shuffle: bool = True):
    """Initialise the engine's rows with synth_rows' state; the units it does
    not use become the free stack.  Scores of H2O rows are lognormal(0,
    sigma), the pools N(0, 1)."""
    arrays, rows, scored, free = synth_rows(
        specs, seed, layers=engine.L, kv_heads=engine.G, page_size=engine.P, pool_units=engine.units,
        max_rows=engine.table.shape[0], pos_cap=engine.pos_cap, r2u_width=engine.r2u.shape[1],
        shuffle=shuffle)
    for r, cfg, n, last, frontier, count in rows:
        engine.add_row(r, cfg, n, last_boundary=last, frontier_units=frontier, count_units=count)
    engine.table.copy_(torch.from_numpy(arrays["table"]))
    engine.r2u.copy_(torch.from_numpy(arrays["r2u"]))
    engine.pos.copy_(torch.from_numpy(arrays["pos"]))
    engine.seed_free_units(free)
    L, G = engine.L, engine.G
    if scored:
        idx = torch.from_numpy(np.concatenate(scored).astype(np.int64)).to(engine.device)
        gen = torch.Generator(device=engine.device).manual_seed(seed + 7)
        vals = torch.randn((L, G, idx.numel()), generator=gen, device=engine.device) * score_sigma
        engine.scores[:, :, idx] = vals.exp_()
    if fill_pools:
        gen = torch.Generator(device=engine.device).manual_seed(seed + 11)
        for t in engine.k + engine.v:
            t.normal_(generator=gen)
    engine.commit_rows()
