"""Decode throughput of the eviction hot path on B200 (one JSON line on rank 0).

Workload (benchmark config 3, "ragged continuous batch"): 64 sequences per GPU
with contexts log-uniform over 2K-64K tokens in 16-token pages, per-sequence
budgets from {2K, 4K, 8K, 16K, 32K} (P = R = B/4, recent: R = 3B/4) and
policies mixed over full / recent / random / H2O global / H2O per-head, on the
12 full-attention layers of a gpt-oss-20b-shaped attention (64 query heads,
8 KV heads, head_dim 64, bf16).  Every step appends one token to every
sequence, runs due eviction boundaries (select + compact), builds the CSR page
table and runs the fused decode attention + H2O score kernel on each layer,
followed by the row-parallel output projection and its NCCL all-reduce across
ranks.  Synthetic seeded data; the KV state is larger than L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Tensor parallel over KV heads: rank r holds 8/N KV heads of every sequence and
the global batch is 64*N sequences (per-GPU work fixed: weak scaling).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("decode tok/s with eviction, config-3 ragged batch (64 seqs/GPU, budgets 2K-32K, "
          "policies full/recent/random/H2O global/H2O per-head)")
UNIT = "tok/s"
H_TOTAL, G_TOTAL, D, PAGE, LAYERS, HIDDEN = 64, 8, 64, 16, 12, 2880
SEQS_PER_GPU = 64
# DRAM bytes (read + write, attn_kernel + combine_kernel) per resident token
# from one ncu capture of the 8-sequence config-3 case (dram__bytes_read.sum +
# dram__bytes_write.sum over the launch's resident tokens); the traffic of this
# streaming kernel grows with resident tokens, so a full launch scales by its
# tokens.
TRAFFIC_BYTES_PER_RESIDENT_TOKEN = 2174.0
BUDGETS = [2048, 4096, 8192, 16384, 32768]
POLICY_MIX = ["full", "recent", "random", "h2o_global", "h2o_per_head"]
SLEEP_CYCLES = 2_000_000   # ~1 ms spin ahead of a timed call


def workload(n_seqs: int, seed: int = 2026, first_boundary_step=None):
    """Seeded per-sequence (ctx, policy, budget) of benchmark config 3.

    With first_boundary_step = t0, the evicting rows' boundaries are spread
    evenly over the 2,048 steps from step t0 on (row i of E reaches one at
    step t0 + i * 2048 // E): each context is lowered by less than 2,048
    tokens (raised by 2,048 if that would leave it under 2,048) so that its
    length then sits on a multiple of 2,048.  A run timed from step t0 then
    meets its share of the eviction work -- E boundaries per 2,048 steps,
    rounded up -- however few steps it times; with free phases a short
    window often saw none."""
    from cache_eviction_b200.policy import EvictionConfig, canonical, sweep_split
    rng = np.random.default_rng(seed)
    specs = []
    for _ in range(n_seqs):
        ctx = int(np.exp(rng.uniform(np.log(2048), np.log(65536)))) // PAGE * PAGE
        budget = int(rng.choice(BUDGETS))
        pol = str(rng.choice(POLICY_MIX))
        if pol == "full":
            cfg = None
        else:
            name = canonical(pol)
            p, r = sweep_split(budget, name)
            cfg = EvictionConfig(name, budget, p, r, seed=int(rng.integers(0, 1 << 31)))
        specs.append(dict(ctx=ctx, cfg=cfg, policy=pol, budget=budget))
    if first_boundary_step is not None:
        from cache_eviction_b200.policy import INTERVAL
        evicting = [sp for sp in specs if sp["cfg"] is not None]
        for i, sp in enumerate(evicting):
            t = int(first_boundary_step) + (i * INTERVAL) // len(evicting)
            ctx = sp["ctx"] - (sp["ctx"] + t) % INTERVAL
            sp["ctx"] = ctx if ctx >= 2048 else ctx + INTERVAL
    return specs


def pool_units_needed(specs, steps):
    """Units the engine's pool needs: what each row can hold at once over
    `steps` decode steps (units come and go through the free stack, so an
    evicting row needs its budget plus one boundary interval of new pages,
    not every token it ever saw), plus slack."""
    total = 1
    for sp in specs:
        cfg, ctx = sp["cfg"], sp["ctx"]
        grown = -(-(ctx + steps) // PAGE) + 1
        if cfg is None:
            total += grown
        elif (ctx // 2048) * 2048 > cfg.budget:       # evicted: budget + one interval of new pages
            total += min(grown, cfg.budget // PAGE + 2048 // PAGE + 1)
        else:                                         # not yet: its context until the first eviction
            total += min(grown, -(-(max(ctx, cfg.budget) + 2048) // PAGE) + 1)
    return total + 64


# --shard-of N (profiling): one process runs rank 0's shard of an N-GPU run
# (its KV heads of 64 N sequences) with no collectives, so a single GPU, and
# ncu, can see the per-rank workload of the scaling run.
SHARD_OF = [1]
# --ordered-units (profiling): each row's pages on consecutive units, for
# telling DRAM locality effects from kernel effects
ORDERED_UNITS = [False]


def _shard(rank, world):
    from cache_eviction_b200 import tp
    return tp.shard(G_TOTAL, H_TOTAL, rank, max(world, SHARD_OF[0]))


# ---------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"ce_bench_clocks_gpu{gpu_index}_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu),
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


# ------------------------------------------------------------ CPU baseline
def cpu_steps(specs, warmup, steps, budget_s, seed=2026 + 17):
    """Time the oracle (the reference's eviction path restated in C, on all
    host cores) on the whole config-3 workload, step by step, as the GPU arm's
    step runs it: the due boundaries (oracle.boundary, the engine's due rule
    and parameters), one token appended to every row, the CSR (oracle.fill)
    and decode attention + H2O scores of every row on every layer
    (oracle.decode).  The rows start from the same synthetic state as the GPU
    arm's (engine.synth_rows).  The twelve layers share one host K and one V
    pool: values do not change the CPU time, and the 12 x 1.3 GB a layer each
    would take is saved.  Stops once budget_s of host time is spent (at least
    one timed step).  Returns (seconds per timed step, info)."""
    from oracle import oracle
    from cache_eviction_b200.engine import synth_rows
    from cache_eviction_b200.policy import INTERVAL
    P, L, G, H = PAGE, LAYERS, G_TOTAL, H_TOTAL
    total = warmup + steps
    units = pool_units_needed(specs, total)
    pos_cap = 32768 // P
    width = -(-(max([65536] + [sp["ctx"] for sp in specs]) + total + 4096) // P)
    t_setup = time.perf_counter()
    arrays, rows, scored, free = synth_rows(specs, seed, layers=L, kv_heads=G, page_size=P,
                                            pool_units=units, max_rows=len(specs), pos_cap=pos_cap,
                                            r2u_width=width)
    free = list(free)      # the host allocator: a stack of free units
    rng = np.random.default_rng(seed)
    state = dict(arrays)
    state["scores"] = np.zeros((L, G, units), np.float32)
    for owned in scored:
        state["scores"][:, :, owned] = rng.lognormal(0.0, 2.0, (L, G, len(owned))).astype(np.float32)
    kp = rng.integers(0, 1 << 16, (units, G, P, D), dtype=np.uint16) & 0xBFFF
    vp = rng.integers(0, 1 << 16, (units, G, P, D), dtype=np.uint16) & 0xBFFF
    B = len(specs)
    q = (rng.integers(0, 1 << 16, (L, B, H, D), dtype=np.uint16) & 0x3FFF) | 0x3800
    sinks = rng.standard_normal((L, H)).astype(np.float32)
    cfgs = [r[1] for r in rows]
    n = [r[2] for r in rows]
    last = [r[3] for r in rows]
    modes = np.array([c.score_mode if c is not None else 0 for c in cfgs], np.int32)
    order = np.arange(B, dtype=np.int64)
    setup_s = time.perf_counter() - t_setup
    times, bound_rows = [], 0
    t0_all = time.perf_counter()
    for s in range(total):
        if s < warmup and times == [] and s > 0 and time.perf_counter() - t0_all > budget_s / 2:
            continue                       # warm-up cut short: keep the budget for timed steps
        t0 = time.perf_counter()
        due = [r for r in range(B) if cfgs[r] is not None and n[r] % INTERVAL == 0 and n[r] > last[r]]
        if due:
            params, ncols = [], []
            for r in due:
                b, pre, rec = cfgs[r].units(P)
                n_u = n[r] // P
                params.append(dict(n=n_u, budget=b, prefix=pre, recent=rec, cursor=None,
                                   policy=cfgs[r].policy_id, seed=cfgs[r].seed))
                ncols.append(int(state["count"][r]) + n_u - int(state["frontier"][r]))
                last[r] = n[r]
            max_cols = max(ncols)
            uni = None
            if any(cfgs[r].name == "random_2048" for r in due):
                uni = rng.random((len(due), L, G, max_cols))
            res, freed = oracle.boundary(state, [kp] * L, [vp] * L, due, oracle.row_params(params), max_cols,
                                         live=True, uniforms=uni)
            for i in range(len(due)):
                free.extend(freed[i, :res[i, 3]].tolist())
            bound_rows += len(due)
        for r in range(B):
            n[r] += 1
            if (n[r] - 1) % P == 0:
                state["r2u"][r, (n[r] - 1) // P] = free.pop()
        indptr, indices, tokens = oracle.fill(state["table"], state["r2u"], state["frontier"], state["count"],
                                              order, np.array(n, np.int64), page=P)
        indices = indices.astype(np.int32)
        for l in range(L):
            oracle.decode(q[l], kp, vp, indptr, indices, tokens, sinks[l], modes, D ** -0.5, P,
                          scores=state["scores"][l], zero_new=True)
        dt = time.perf_counter() - t0
        if s >= warmup:
            times.append(dt)
        if times and time.perf_counter() - t0_all > budget_s:
            break
    info = {"timed_steps": len(times), "resident_tokens": int(tokens.sum()), "boundary_rows": bound_rows,
            "setup_s": setup_s}
    return statistics.mean(times), info


def cpu_sample_text(info, B, steps_requested):
    return (f"oracle (C restatement of the reference path) on the whole config-3 step: due boundaries "
            f"(oracle.boundary), CSR fill and decode attention + H2O scores of all {B} sequences "
            f"({info['resident_tokens']} resident tokens) on all {LAYERS} layers; "
            f"{info['timed_steps']} of {steps_requested} steps timed in full, {info['boundary_rows']} boundary "
            f"rows in the run; the layers share one host K/V pool")


def reference_arm(args, world, rank):
    """--impl reference: the reference's path (its CPU restatement, the
    oracle) on the host cores, timed on this arm's workload step by step."""
    if rank != 0:
        return 0
    from oracle import oracle
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    specs = workload(SEQS_PER_GPU * world, first_boundary_step=args.warmup)
    per_step, info = cpu_steps(specs, args.warmup, args.steps, budget_s=REFERENCE_BUDGET_S)
    value = len(specs) / per_step
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic", "config": config_block(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": cpu_sample_text(info, len(specs), args.steps)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# Host seconds the reference arm spends on its warm-up and timed steps (each a
# full step of the workload); setting up the host state comes on top.
REFERENCE_BUDGET_S = 150.0


def config_block(world):
    return {"workload": "config3 ragged continuous batch: 64 seqs/GPU, ctx log-uniform 2K-64K, "
                        "budgets {2K..32K}, policies {full, recent, random, h2o_global, h2o_per_head}, "
                        "12 full-attention layers, 64q/8kv heads, head_dim 64, 16-token pages",
            "global_batch": SEQS_PER_GPU * world, "page_size": PAGE, "layers": LAYERS,
            "kv_heads_per_gpu": G_TOTAL // world, "parallelism": f"tp{world} over KV heads",
            "l2": "KV state far larger than L2 (no flush needed)"}


# ---------------------------------------------------------------- our arm
# Page scores of a layer on a second stream beside the next layer's attention
# (engine overlap_scores), with --score-overlap; off by default.
SCORE_OVERLAP = [False]


class ResidentCounter:
    """Resident tokens and scored (H2O) pages of an engine's active rows, once
    per step after advance(): numpy copies of the rows' state are taken again
    only after a boundary batch, since between boundaries every row just grows
    by one token per step (a Python pass over 512 rows per step was host time
    that the GPUs waited for at eight ranks)."""

    def __init__(self, eng):
        self.eng, self.batches, self.t = eng, -1, 0

    def __call__(self):
        eng = self.eng
        if len(eng.boundary_ms) != self.batches:
            rows = [eng.rows[r] for r in eng.active]
            self.cnt = np.array([r.count for r in rows], np.int64)
            self.fr = np.array([r.frontier for r in rows], np.int64)
            self.n = np.array([r.n for r in rows], np.int64)
            self.scored = np.array([r.cfg is not None and bool(r.cfg.score_mode) for r in rows], bool)
            self.batches, self.t = len(eng.boundary_ms), 0
        else:
            self.t += 1
        P = eng.P
        n = self.n + self.t
        tokens = int(P * self.cnt.sum() + n.sum() - P * self.fr.sum())
        units = self.cnt + np.maximum(0, (n + P - 1) // P - self.fr)
        return tokens, int(units[self.scored].sum())


def build_engine(specs, steps_total, world, rank, group, device):
    import torch
    from cache_eviction_b200.engine import RaggedDecodeEngine, synth_state
    from cache_eviction_b200 import tp
    G, H, off = _shard(rank, world)
    units = pool_units_needed(specs, steps_total)
    eng = RaggedDecodeEngine(layers=LAYERS, q_heads=H, kv_heads=G, page_size=PAGE, pool_units=units,
                             max_rows=len(specs),
                             r2u_width=-(-(max([65536] + [sp["ctx"] for sp in specs]) + steps_total + 4096) // PAGE),
                             pos_cap=32768 // PAGE, device=device, head_offset=off,
                             global_kv_heads=G_TOTAL, process_group=group,
                             overlap_scores=SCORE_OVERLAP[0])
    synth_state(eng, specs, seed=2026 + 17, shuffle=not ORDERED_UNITS[0])
    torch.cuda.synchronize()
    return eng


def run_e2e(args, specs, steps_total, world, rank, group, device, q, out, sinks, scale,
            after_layer, barrier, max_over_ranks, e2e_steps):
    """End-to-end pass through the public engine API from a fresh state: every
    step uploads all layers' queries from pinned host memory and downloads all
    attention outputs into pinned host memory.  The copies run on their own
    streams, per layer, overlapped with the decode: layer l waits only for its
    own query upload, and its output download starts as soon as layer l is
    done (and after the previous step's download of that buffer)."""
    import torch
    B = len(specs)
    L = q.shape[0]
    eng = build_engine(specs, steps_total, world, rank, group, device)
    q_host = torch.empty(tuple(q.shape), dtype=torch.bfloat16).pin_memory()
    q_host.copy_(q.cpu())
    out_host = torch.empty(tuple(out.shape), dtype=torch.bfloat16).pin_memory()
    q_dev = torch.empty_like(q)
    compute = torch.cuda.current_stream(device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    q_ready = [torch.cuda.Event() for _ in range(L)]
    out_ready = [torch.cuda.Event() for _ in range(L)]
    q_free = [torch.cuda.Event() for _ in range(L)]
    out_free = [torch.cuda.Event() for _ in range(L)]

    def one_step():
        for l in range(L):
            up.wait_event(q_free[l])                # the previous step's layer l read q_dev[l]
            with torch.cuda.stream(up):
                q_dev[l].copy_(q_host[l], non_blocking=True)
            q_ready[l].record(up)

        def before(l):
            compute.wait_event(q_ready[l])
            compute.wait_event(out_free[l])         # out[l] was downloaded last step

        def after(l, o):
            after_layer(l, o)
            q_free[l].record(compute)
            out_ready[l].record(compute)
            down.wait_event(out_ready[l])
            with torch.cuda.stream(down):
                out_host[l].copy_(out[l], non_blocking=True)
            out_free[l].record(down)

        eng.step(q_dev, out, sinks, scale, after, before_layer=before)

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(e2e_steps):
        one_step()
    compute.wait_stream(up)
    compute.wait_stream(down)                       # every download is inside the timed region
    eng.join_scores()
    e2.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2))
    del eng
    torch.cuda.empty_cache()
    return B * e2e_steps / (e2e_ms * 1e-3)


def paired_segments(run_a, run_b, steps, seg):
    """Alternate `seg`-step segments of two passes (a then b, then b then a,
    ...) until each has run `steps` steps, as the reference's paired off/on
    timing does (code/cache_eviction/sglang_timing.py:69-87): box drift then
    falls on both sides alike.  Each segment is bracketed by CUDA events on
    the current stream.  Returns (ms of a, ms of b, pairs)."""
    import torch
    done, i, marks = 0, 0, []
    while done < steps:
        n = min(seg, steps - done)
        order = (("a", run_a), ("b", run_b)) if i % 2 == 0 else (("b", run_b), ("a", run_a))
        for name, fn in order:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn(n)
            e1.record()
            marks.append((i, name, e0, e1))
        done += n
        i += 1
    torch.cuda.synchronize()
    pairs = {}
    for i, name, e0, e1 in marks:
        pairs.setdefault(i, {})[name] = e0.elapsed_time(e1)
    ms_a = sum(p["a"] for p in pairs.values())
    ms_b = sum(p["b"] for p in pairs.values())
    return ms_a, ms_b, list(pairs.values())


def run_no_score(args, specs, steps_total, world, rank, group, device, q, out, sinks, scale,
                 after_layer, barrier, max_over_ranks):
    """Scored against unscored decode at the same resident KV, in alternating
    segments: two engines from the same fresh state, one with H2O scoring off
    for every row (mode NONE, no score work at all) and the same boundaries, so
    the resident KV matches step for step.  The unscored rate is the
    full-cache decode rate at the same resident size that the north star
    compares the scored rate with."""
    import torch
    from cache_eviction_b200 import capi
    B = len(specs)
    eng_s = build_engine(specs, steps_total, world, rank, group, device)
    eng_u = build_engine(specs, steps_total, world, rank, group, device)
    eng_u.mode.fill_(capi.CE_MODE_NONE)
    eng_u.score_flags = 0        # a plain full-cache decode: no score work or launches
    for eng in (eng_s, eng_u):
        for _ in range(args.warmup):
            eng.step(q, out, sinks, scale, after_layer)

    def runner(eng):
        def fn(n):
            for _ in range(n):
                eng.step(q, out, sinks, scale, after_layer)
            eng.join_scores()
        return fn

    barrier()
    torch.cuda.synchronize()
    ms_s, ms_u, pairs = paired_segments(runner(eng_s), runner(eng_u), args.steps, seg=16)
    barrier()
    ms_s, ms_u = max_over_ranks(ms_s), max_over_ranks(ms_u)
    del eng_s, eng_u
    torch.cuda.empty_cache()
    return {"value": B * args.steps / (ms_u * 1e-3), "scored_value": B * args.steps / (ms_s * 1e-3),
            "scored_over_no_score": ms_u / ms_s, "pairs": len(pairs), "segment_steps": 16}


def decode4_microbench(world, rank, group, device, barrier, max_over_ranks, steps=2048, warmup=8, seg=64):
    """benchmark config 4's decode phase: one sequence after an 80,000-token
    prompt, per-head H2O (head_sum) with 512 prefix + 4,096 recent + 24,064
    scored tokens (28,672 resident after each boundary), 12 full layers of
    this rank's heads (attention + H2O score, no output projection), `steps`
    decode steps including the boundary at 81,920 tokens.  Each step without a
    boundary replays one CUDA graph (position advance, CSR fill, the 12 fused
    decode layers); the boundary step runs eagerly through engine.step.  The
    same steps with scoring off at the same resident KV (a second engine, the
    full-cache rate) are timed in alternating `seg`-step segments with the
    scored ones.  Algorithmic bytes per step: K + V of every resident token
    (2,048 B at 8 KV heads) + Q/O + the page-score read-modify-write, per
    layer."""
    import torch
    from cache_eviction_b200 import capi, tp
    from cache_eviction_b200.policy import EvictionConfig
    G, H, _ = _shard(rank, world)
    ctx, budget, prefix, recent = 80000, 28672, 512, 4096
    cfg = EvictionConfig("head_sum_2048", budget, prefix, recent, seed=4)
    specs = [dict(ctx=ctx, cfg=cfg, policy="h2o_per_head", budget=budget)]
    scale = D ** -0.5
    gen = torch.Generator(device=device).manual_seed(4321 + rank)
    q = torch.randn((LAYERS, 1, H, D), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty((LAYERS, 1, H, D), dtype=torch.bfloat16, device=device)
    sinks = [torch.randn(H, generator=gen, device=device) for _ in range(LAYERS)]
    passes = {}
    for scored in (True, False):
        eng = build_engine(specs, warmup + steps, world, rank, group, device)
        if not scored:
            eng.mode.fill_(capi.CE_MODE_NONE)
            eng.score_flags = 0      # a plain full-cache decode: no score work or launches
        # the CSR buffer the graph holds stays large enough; the warm-up steps
        # then size the decode workspace for it, so the capture allocates nothing
        eng._ensure_capacity(warmup + steps + 16)
        for _ in range(warmup):
            eng.step(q, out, sinks, scale)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        eng.join_scores()
        eng.new_score_events()
        with torch.cuda.graph(graph):
            eng.advance_device()
            eng.fill()
            for l in range(LAYERS):
                eng.decode_layer(l, q[l], out[l], sinks[l], scale)
            eng.join_scores()      # a capture ends with every forked stream joined
        eng.new_score_events()
        torch.cuda.synchronize()
        passes[scored] = dict(eng=eng, graph=graph, resident=[])

    def runner(ps):
        eng, graph = ps["eng"], ps["graph"]

        def fn(n):
            for _ in range(n):
                if eng.due():
                    eng.step(q, out, sinks, scale)
                else:
                    eng.advance_host()
                    graph.replay()
                ps["resident"].append(eng.resident_tokens(eng.active[0]))
            eng.join_scores()
        return fn

    barrier()
    torch.cuda.synchronize()
    ms_s, ms_u, pairs = paired_segments(runner(passes[True]), runner(passes[False]), steps, seg)
    barrier()
    ms = {True: max_over_ranks(ms_s), False: max_over_ranks(ms_u)}
    res = {}
    for scored in (True, False):
        ps = passes[scored]
        ps["eng"].check_errors()
        bounds = len(ps["eng"].rows[ps["eng"].active[0]].events)
        tok = statistics.mean(ps["resident"])
        nbytes = LAYERS * (tok * G * D * 2 * 2 + 2 * H * D * 2 + (-(-tok // PAGE)) * G * 8 * scored)
        res["scored" if scored else "no_score"] = {
            "tok_s": steps / (ms[scored] * 1e-3), "ms_per_step": ms[scored] / steps,
            "resident_tokens_mean": tok, "gbs": nbytes / (ms[scored] / steps * 1e-3) / 1e9,
            "boundaries": bounds}
    del passes
    torch.cuda.empty_cache()
    peak, kind = measured_peak_hbm()
    res["scored_over_no_score"] = res["scored"]["tok_s"] / res["no_score"]["tok_s"]
    res["hbm_frac_scored"] = res["scored"]["gbs"] / peak
    res["peak_kind"] = kind
    res["timing"] = f"alternating {seg}-step segments of the scored and unscored passes, {len(pairs)} pairs"
    return res


def continuous_microbench(world, rank, group, device, barrier, max_over_ranks, steps=512, warmup=8,
                          seed=77):
    """Config 3 as a continuous batch: up to 64 rows decode at once; each
    request leaves after a drawn number of new tokens (uniform 64-512) and
    the next arriving request (context, budget and policy drawn from the
    config-3 distribution) takes the freed row once the free units allow
    (it waits otherwise, as a scheduler's admission would).  Admissions
    (prompt units popped from the free stack, the prefill's last boundary
    for all of a step's arrivals in one batch) and retirements (units pushed
    back) run between steps inside the timed region; the arrivals' K/V pages
    keep what the units held (the prefill that would write them is outside
    this path) and their H2O scores are drawn lognormal.  The pool is sized
    to what the first batch can hold at once plus 8,192 units of slack, not
    to every token of every request served.  Value: decoded tokens / time."""
    import torch
    from cache_eviction_b200 import tp
    G, H, _ = _shard(rank, world)
    B = SEQS_PER_GPU * world
    specs = workload(B, seed=seed)
    arrivals = workload(8 * B, seed=seed + 1)
    rng = np.random.default_rng(seed + 2)
    units = pool_units_needed(specs, steps + warmup) + 8192
    from cache_eviction_b200.engine import RaggedDecodeEngine, synth_state
    eng = RaggedDecodeEngine(layers=LAYERS, q_heads=H, kv_heads=G, page_size=PAGE, pool_units=units,
                             max_rows=B, r2u_width=-(-(65536 + steps + warmup + 4096) // PAGE),
                             pos_cap=32768 // PAGE, device=device, head_offset=_shard_offset(rank, world),
                             global_kv_heads=G_TOTAL, process_group=group)
    synth_state(eng, specs, seed=seed + 3)
    scale = D ** -0.5
    gen = torch.Generator(device=device).manual_seed(seed + 4)
    q = torch.randn((LAYERS, B, H, D), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty((LAYERS, B, H, D), dtype=torch.bfloat16, device=device)
    sinks = [torch.randn(H, generator=gen, device=device) for _ in range(LAYERS)]
    left = {r: int(rng.integers(64, 513)) for r in range(B)}
    queue = list(arrivals)
    stats = dict(admitted=0, retired=0, waits=0, tokens=0, units_peak=0, served_token_units=0)

    def peak_units(r, rem):
        row = eng.rows[r]
        grown = -(-(row.n + rem) // PAGE) + 1
        if row.cfg is None:
            return grown
        b_u = row.cfg.budget // PAGE
        return min(grown, max(eng.resident_units(r), b_u) + 2048 // PAGE + 1)

    def admissions():
        free_rows = [r for r in range(B) if r not in eng.rows]
        if not free_rows or not queue:
            return
        reserve = sum(max(0, peak_units(r, left[r]) - eng.resident_units(r)) for r in eng.active)
        admitted = []
        for r in free_rows:
            if not queue:
                break
            sp = queue[0]
            need = -(-sp["ctx"] // PAGE)
            rem = int(rng.integers(64, 513))
            b_u = sp["cfg"].budget // PAGE if sp["cfg"] is not None else None
            after = -(-(sp["ctx"] + rem) // PAGE) + 1 if b_u is None else min(
                -(-(sp["ctx"] + rem) // PAGE) + 1, b_u + 2 * (2048 // PAGE) + 1)
            if eng.free_top - reserve < max(need, after):
                stats["waits"] += 1
                break
            queue.pop(0)

            def prompt(u, cfg=sp["cfg"]):
                if cfg is not None and cfg.score_mode:
                    eng.scores[:, :, u.long()] = torch.randn((LAYERS, G, u.numel()), generator=gen,
                                                             device=device).mul_(2.0).exp_()
            eng.admit(r, sp["cfg"], sp["ctx"], prompt=prompt, settle=False)
            left[r] = rem
            reserve += after
            admitted.append(r)
            stats["admitted"] += 1
            stats["served_token_units"] += -(-(sp["ctx"] + rem) // PAGE)
        eng.settle(admitted)

    def one_step():
        for r in list(eng.active):
            if left[r] == 0:
                eng.retire(r)
                stats["retired"] += 1
        admissions()
        eng.commit_rows()
        bs = len(eng.active)
        eng.step(q[:, :bs], out[:, :bs], sinks, scale)
        for r in eng.active:
            left[r] -= 1
        stats["tokens"] += bs
        stats["units_peak"] = max(stats["units_peak"], units - eng.free_top)

    for _ in range(warmup):
        one_step()
    for k in ("admitted", "retired", "waits", "tokens", "served_token_units"):
        stats[k] = 0
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        one_step()
    eng.join_scores()
    end.record()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    eng.check_errors()
    all_token = stats["served_token_units"] + sum(-(-(sp["ctx"] + steps + warmup) // PAGE) for sp in specs)
    res = {"tok_s": stats["tokens"] / (ms * 1e-3),
           "ms_per_step": ms / steps, "decoded_tokens": stats["tokens"], "admitted": stats["admitted"],
           "retired": stats["retired"], "admission_waits": stats["waits"],
           "boundary_rows": sum(len(eng.rows[r].events) for r in eng.active),
           "pool_units": units, "units_in_use_peak": stats["units_peak"],
           "units_if_every_token_kept": all_token,
           "what": "rows retire after 64-512 new tokens and arrivals take their rows when free units "
                   "allow; admissions, their prefill boundaries and retirements inside the timed region"}
    del eng
    torch.cuda.empty_cache()
    return res


def _shard_offset(rank, world):
    from cache_eviction_b200 import tp
    return _shard(rank, world)[2]


def model2_microbench(world, rank, device, max_len=16384, prompt_len=1024, seg=512, seed=2):
    """benchmark config 2: a gpt-oss-20b-shaped decoder with random bf16 weights
    (24 layers alternating a 128-token sliding window and full attention,
    hidden 2880, 32 experts top 4, vocabulary 201,088; cache_eviction_b200.oss20b),
    batch 1, a 1,024-token prompt of seeded uniform token ids, greedy decoding
    to 16,384 tokens.  Per-head H2O on the 12 full layers at budget 8192 = 512
    prefix + 1,024 recent + 6,656 scored, against the same decoder with H2O
    scoring off and the same boundaries (the full-cache rate at the same
    resident KV) and against a full cache that keeps every token; the three
    share the weights and are timed over their 15,360 generated tokens in
    alternating 512-step segments (each step one CUDA graph; the boundary
    steps run their boundary eagerly first).  One GPU: the model is not split
    across ranks."""
    import torch
    from cache_eviction_b200.oss20b import OssConfig, OssDecoder, OssWeights
    from cache_eviction_b200.policy import EvictionConfig
    if world > 1:
        return {"skipped": "config 2 runs on one GPU (the decoder is not sharded over ranks)"}
    cfg = OssConfig()
    t0 = time.perf_counter()
    W = OssWeights(cfg, device, seed=seed)
    torch.cuda.synchronize()
    init_s = time.perf_counter() - t0
    ev = EvictionConfig("head_sum_2048", 8192, 512, 1024, seed=seed)
    decs = {"scored": OssDecoder(W, ev, max_len, scored=True, device=device),
            "no_score_same_resident": OssDecoder(W, ev, max_len, scored=False, device=device),
            "full_cache": OssDecoder(W, None, max_len, scored=False, device=device)}
    gen = torch.Generator(device=device).manual_seed(seed + 1)
    prompt = torch.randint(0, cfg.vocab, (prompt_len,), generator=gen, device=device)
    for d in decs.values():
        d.prefill(prompt)
    torch.cuda.synchronize()
    steps = max_len - prompt_len

    def runner(d):
        def fn(n):
            for _ in range(n):
                d.step()
        return fn

    ms_a, ms_b, pairs = paired_segments(runner(decs["scored"]), runner(decs["no_score_same_resident"]), steps, seg)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    runner(decs["full_cache"])(steps)
    e1.record()
    torch.cuda.synchronize()
    ms = {"scored": ms_a, "no_score_same_resident": ms_b, "full_cache": e0.elapsed_time(e1)}
    out = {}
    for name, d in decs.items():
        eng = d.eng
        eng.check_errors()
        out[name] = {"tok_s": steps / (ms[name] * 1e-3), "ms_per_token": ms[name] / steps,
                     "tokens": d.n, "resident_tokens_end": eng.resident_tokens(0),
                     "boundaries": [e["boundary"] for e in eng.rows[0].events if e["status"] == 0]}
    out["scored_over_no_score"] = out["scored"]["tok_s"] / out["no_score_same_resident"]["tok_s"]
    out["scored_over_full_cache"] = out["scored"]["tok_s"] / out["full_cache"]["tok_s"]
    out["weights_gb"] = sum(t.numel() * 2 for t in [W.embed, W.lm_head] +
                            [v for lw in W.layers for v in lw.values() if v.dtype == torch.bfloat16]) / 1e9
    out["weight_init_s"] = init_s
    out["timing"] = (f"{steps} generated tokens per decoder; scored and unscored in alternating {seg}-step "
                     f"segments ({len(pairs)} pairs), the full cache after them")
    del decs, W
    torch.cuda.empty_cache()
    return out


PREFILL_CHUNK = 2048
PREFILL_PREFIXES = (0, 8192, 26624)   # resident tokens before a chunk; 26,624 + 2,048 = config 4's cache


def prefill_microbench(world, rank, device, reps=5, cpu=False, prefixes=PREFILL_PREFIXES):
    """benchmark config 4: one 2,048-token prefill chunk of one layer scored by
    ce_prefill_scores against a resident prefix of 0 / 8,192 / 26,624 tokens
    (16-token pages, this rank's KV heads, no eviction inside the chunk).
    Algorithmic work per call: two Q.K^T passes over the visible (query, key)
    pairs, 4 * 64 * H * pairs FLOP, and one exp2 per pair and query head in
    each pass.  Device time by CUDA events around the call (the GPU is kept
    busy while the host prepares it)."""
    import torch
    from cache_eviction_b200 import capi, kernels, tp
    G, H, _ = _shard(rank, world)
    out = {}
    gen = torch.Generator(device=device).manual_seed(77)
    nq = PREFILL_CHUNK
    q = torch.randn((nq, H, D), generator=gen, device=device).to(torch.bfloat16)
    sinks = torch.randn(H, generator=gen, device=device)
    for prefix in prefixes:
        ntok = prefix + nq
        units = ntok // PAGE
        kpool = torch.randn((units + 1, G, PAGE, D), generator=gen, device=device).to(torch.bfloat16)
        idx = (torch.randperm(units, generator=gen, device=device) + 1).int()
        scores = torch.zeros((G, units + 1), dtype=torch.float32, device=device)
        meta = [torch.tensor(v, dtype=torch.int32, device=device) for v in ([0, nq], [0, units], [ntok])]
        pairs = nq * prefix + nq * (nq + 1) // 2
        for mode in (capi.CE_MODE_SUM, capi.CE_MODE_MAX):
            mo = torch.tensor([mode], dtype=torch.int32, device=device)
            ts = []
            for it in range(reps + 1):
                a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda._sleep(SLEEP_CYCLES)
                a.record()
                kernels.prefill_scores(q, kpool, meta[0], meta[1], idx, meta[2], D ** -0.5, PAGE, nq, ntok,
                                       sinks=sinks, mode_of_row=mo, scores=scores, zero_new=True)
                e.record()
                torch.cuda.synchronize()
                if it:
                    ts.append(a.elapsed_time(e) * 1e3)
            us = statistics.median(ts)
            out[f"prefix{prefix}_{'sum' if mode == capi.CE_MODE_SUM else 'max'}"] = {
                "us": us, "tflops": 4 * D * H * pairs / (us * 1e-6) / 1e12,
                "gexp2_per_s": 2 * H * pairs / (us * 1e-6) / 1e9, "visible_pairs": pairs}
        del kpool, scores
        # Replay layer error of the same chunk (ce_replay_error): shadow K/V by
        # position, a quarter of each head's prefix evicted.  Tensor work per
        # visible pair and query head: Q.K^T twice plus four P.V products
        # (hi/lo parts of P_a and P_d), 12 * 64 FLOP; one exp2 in each pass.
        ks = torch.randn((ntok, G, D), generator=gen, device=device).to(torch.bfloat16)
        vs = torch.randn((ntok, G, D), generator=gen, device=device).to(torch.bfloat16)
        vis = torch.rand((G, ntok), generator=gen, device=device) < 0.75
        vis[:, prefix:] = True
        words = -(-ntok // 32)
        pad = torch.zeros((G, words * 32), dtype=torch.int64, device=device)
        pad[:, :ntok] = vis.to(torch.int64)
        bits = (pad.view(G, words, 32) << torch.arange(32, device=device)).sum(-1)
        bits = torch.where(bits >= 1 << 31, bits - (1 << 32), bits).to(torch.int32).contiguous()
        ts = []
        for it in range(reps + 1):
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda._sleep(SLEEP_CYCLES)
            a.record()
            kernels.replay_error(q, ks, vs, prefix, D ** -0.5, visible_bits=bits, sinks=sinks)
            e.record()
            torch.cuda.synchronize()
            if it:
                ts.append(a.elapsed_time(e) * 1e3)
        us = statistics.median(ts)
        out[f"prefix{prefix}_replay"] = {"us": us, "tflops": 12 * D * H * pairs / (us * 1e-6) / 1e12,
                                         "gexp2_per_s": 2 * H * pairs / (us * 1e-6) / 1e9,
                                         "visible_pairs": pairs}
        del ks, vs
    if cpu:
        from oracle import oracle
        import numpy as np
        rng = np.random.default_rng(3)
        nq_s, prefix = 8, PREFILL_PREFIXES[-1]
        ntok = prefix + nq_s
        units = -(-ntok // PAGE)
        kb = rng.integers(0, 1 << 16, (units + 1, G, PAGE, D), dtype=np.uint16) & 0xBFFF
        qb = rng.integers(0, 1 << 16, (nq_s, H, D), dtype=np.uint16) & 0xBFFF
        sc = np.zeros((G, units + 1), np.float32)
        t0 = time.perf_counter()
        oracle.prefill(qb, kb, np.array([0, nq_s]), np.array([0, units]), np.arange(1, units + 1),
                       np.array([ntok]), None, np.array([1]), D ** -0.5, PAGE, sc)
        dt = time.perf_counter() - t0
        pairs_s = nq_s * prefix + nq_s * (nq_s + 1) // 2
        pairs = nq * prefix + nq * (nq + 1) // 2
        out["cpu_baseline"] = {"us": dt * 1e6 * pairs / pairs_s, "cores": oracle.threads(),
                               "kind": "port",
                               "sample": f"oracle prefill scores of {nq_s} queries over {prefix} prefix "
                                         f"tokens, scaled to the {nq}-query chunk by visible pairs"}
    return out


def select_token_microbench(world, rank, device, reps=3, rows=32):
    """Config 5's page-size-1 stress variant of selection: ce_choose over
    32 rows x this rank's KV heads x 65,536 token columns (fp32 scores
    lognormal(0, 2); float64 uniforms for random), budgets 2K-32K tokens with
    prefix = recent = budget / 4.  Algorithmic bytes: positions + scores
    (+ uniforms) read once, kept indices written."""
    import torch
    from cache_eviction_b200 import kernels, tp
    G, _, _ = _shard(rank, world)
    R, N = rows, 65536
    gen = torch.Generator(device=device).manual_seed(56)
    pos = torch.arange(N, dtype=torch.int32, device=device).expand(R, G, N).contiguous()
    sc = torch.randn((R, G, N), generator=gen, device=device).mul_(2.0).exp_()
    uni = torch.rand((R, G, N), generator=gen, device=device, dtype=torch.float64)
    out = {}
    for pol in ("h2o_global_2048", "head_sum_2048", "random_2048"):
        for budget in BUDGETS:
            prm = kernels.row_params([dict(n=N, budget=budget, prefix=budget // 4, recent=budget // 4,
                                           cursor=None, policy=pol, seed=i) for i in range(R)], device)
            key = uni if pol == "random_2048" else sc
            ts = []
            for it in range(reps + 1):
                a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda._sleep(SLEEP_CYCLES)
                a.record()
                _, status, _ = kernels.choose(pos, key, prm, 1, G, max_n=N + 1, kept_stride=budget)
                e.record()
                torch.cuda.synchronize()
                if it:
                    ts.append(a.elapsed_time(e) * 1e3)
            assert bool((status == 0).all()), status
            us = statistics.median(ts)
            nbytes = R * G * N * (4 + key.element_size()) + R * G * budget * 4
            out[f"{pol}_{budget}"] = {"us": us, "gbs": nbytes / (us * 1e-6) / 1e9}
    return out


def evict_microbench(world, rank, device, reps=3, rows=32, page=PAGE):
    """benchmark config 5: one eviction step (select + compaction) over 32 rows x
    this rank's KV heads x 65,536-token contexts (4096 pages of 16 tokens, or
    with page=1 the reference's own token slots), fp32 scores lognormal(0, 2),
    P = R = B/4, for H2O global / H2O per-head / random at budgets 2K..32K
    tokens.  Device time of ce_boundary and (pages of 16) of ce_choose alone
    (CUDA events, state restored outside the timed window), moved units and
    algorithmic GB/s."""
    import torch
    from cache_eviction_b200 import kernels, tp
    G, _, off = _shard(rank, world)
    R, N = rows, 65536 // page
    units = R * N + 1
    gen = torch.Generator(device=device).manual_seed(55)
    kp = torch.randn((units, G, page, D), generator=gen, device=device).to(torch.bfloat16)
    vp = torch.randn((units, G, page, D), generator=gen, device=device).to(torch.bfloat16)
    kptr, vptr = kernels.layer_pointers([kp], device), kernels.layer_pointers([vp], device)
    scores0 = torch.randn((1, G, units), generator=gen, device=device).mul_(2.0).exp_()
    perm = torch.randperm(units - 1, generator=gen, device=device).int() + 1
    r2u0 = perm[:R * N].view(R, N).contiguous()
    rows = torch.arange(R, dtype=torch.int32, device=device)
    marks = torch.zeros(units, dtype=torch.int32, device=device)
    uni = torch.rand((R, 1, G, N), generator=gen, device=device, dtype=torch.float64)
    pos_fresh = torch.arange(N, dtype=torch.int32, device=device).expand(R, G, N).contiguous()
    out = {}
    epoch = 0
    for pol in ("h2o_global_2048", "head_sum_2048", "random_2048"):
        for budget in BUDGETS:
            b = budget // page
            params = [dict(n=N, budget=b, prefix=b // 4, recent=b // 4, cursor=None, policy=pol, seed=i)
                      for i in range(R)]
            prm = kernels.row_params(params, device)
            table = torch.zeros((R, N), dtype=torch.int32, device=device)
            frontier = torch.zeros(R, dtype=torch.int32, device=device)
            count = torch.zeros(R, dtype=torch.int32, device=device)
            pos = torch.zeros((R, 1, G, b), dtype=torch.int32, device=device)
            r2u, scores = r2u0.clone(), scores0.clone()
            times, sel_times = [], []
            for it in range(reps + 1):
                r2u.copy_(r2u0), scores.copy_(scores0), frontier.zero_(), count.zero_()
                epoch += 1
                a = torch.cuda.Event(enable_timing=True)
                e = torch.cuda.Event(enable_timing=True)
                # Keep the GPU busy while the host prepares the call, so the
                # events bracket device time only.
                torch.cuda._sleep(SLEEP_CYCLES)
                a.record()
                res, _ = kernels.boundary(table, r2u, frontier, count, pos, scores, kptr, vptr, G, page,
                                          rows, prm, N, N + 1, True, marks=marks, epoch=epoch,
                                          uniforms=uni if pol == "random_2048" else None,
                                          head_offset=off, hazard_bytes=1 << 30, max_width=b)
                e.record()
                if page == PAGE:
                    sc = scores0[0].gather(1, r2u0.view(1, -1).expand(G, -1).long()).view(G, R, N)
                    sc = sc.permute(1, 0, 2).contiguous()
                    a2 = torch.cuda.Event(enable_timing=True)
                    e2 = torch.cuda.Event(enable_timing=True)
                    torch.cuda._sleep(SLEEP_CYCLES)
                    a2.record()
                    kernels.choose(pos_fresh, uni.view(R, G, N) if pol == "random_2048" else sc, prm, 1, G,
                                   max_n=N + 1, kept_stride=b)
                    e2.record()
                torch.cuda.synchronize()
                if it:
                    times.append(a.elapsed_time(e) * 1e3)
                    if page == PAGE:
                        sel_times.append(a2.elapsed_time(e2) * 1e3)
            status = res[:, 0].cpu()
            assert bool((status == 0).all()), status
            p_u, mid = b // 4, b - 2 * (b // 4)
            mpos = pos[:, 0, :, p_u:p_u + mid]
            moved = int((mpos != (torch.arange(mid, device=device, dtype=torch.int32) + p_u)).sum())
            nbytes = R * G * N * 4 + (R * G * N * 8 if pol == "random_2048" else 0) + R * G * b * 4 \
                + moved * (2 * 2 * page * D * 2 + 8)
            us = statistics.median(times)
            out[f"{pol}_{budget}"] = {"evict_step_us": us,
                                      "select_us": statistics.median(sel_times) if sel_times else None,
                                      "moved_units": moved, "gbs": nbytes / (us * 1e-6) / 1e9}
    del kp, vp
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=512)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-oproj", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="CPU-baseline sample length (0 skips it)")
    ap.add_argument("--no-evict-bench", action="store_true",
                    help="skip the config-5 eviction-step leg")
    ap.add_argument("--seqs", type=int, default=SEQS_PER_GPU,
                    help="sequences per GPU (small cases for profiling)")
    ap.add_argument("--legs", default=None,
                    help="legs to run (default: every leg on one GPU; the config-3 headline, its "
                         "end-to-end pass and the paired unscored pass on several -- the other legs "
                         "are one-GPU shapes); without 'decode' only the listed microbenchmarks "
                         "run and one JSON line with their results is printed (profiling)")
    ap.add_argument("--evict-rows", type=int, default=32, help="rows of the config-5 leg")
    ap.add_argument("--score-overlap", action="store_true",
                    help="score each layer's pages on a second stream (engine overlap_scores)")
    ap.add_argument("--ordered-units", action="store_true",
                    help="profiling: consecutive units for each row instead of shuffled ones")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="profiling: run rank 0's shard of an N-GPU run on this one GPU, no collectives")
    ap.add_argument("--prefill-prefixes", default=",".join(map(str, PREFILL_PREFIXES)),
                    help="resident prefixes of the config-4 leg")
    args = ap.parse_args()
    if args.legs is None:
        several = int(os.environ.get("WORLD_SIZE", "1")) > 1
        args.legs = ("decode,e2e,noscore" if several else
                     "decode,e2e,noscore,cb3,model2,decode4,prefill4,evict5,select1,evict1")
    legs = set(args.legs.split(","))
    SHARD_OF[0] = args.shard_of
    ORDERED_UNITS[0] = args.ordered_units
    SCORE_OVERLAP[0] = args.score_overlap
    prefixes = tuple(int(x) for x in args.prefill_prefixes.split(","))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, world, rank)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    import torch
    import torch.distributed as dist
    from cache_eviction_b200 import capi, kernels, tp

    group, rank, world = tp.init_from_env("nccl")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
    capi.load()
    if "decode" not in legs:
        res = {}

        def barrier0():
            if world > 1:
                dist.barrier(device_ids=[device.index])

        def max0(x: float) -> float:
            if world == 1:
                return x
            t = torch.tensor([x], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        if "decode4" in legs:
            res["decode_config4"] = decode4_microbench(world, rank, group, device, barrier0, max0)
        if "cb3" in legs:
            res["continuous_config3"] = continuous_microbench(world, rank, group, device, barrier0, max0)
        if "model2" in legs:
            res["model_config2"] = model2_microbench(world, rank, device)
        if "prefill4" in legs:
            res["prefill_config4"] = prefill_microbench(world, rank, device, prefixes=prefixes)
        if "evict5" in legs:
            res["evict_config5"] = evict_microbench(world, rank, device, rows=args.evict_rows)
        if "select1" in legs:
            res["select_token_config5"] = select_token_microbench(world, rank, device, rows=args.evict_rows)
        if "evict1" in legs:
            res["evict_token_config5"] = evict_microbench(world, rank, device, rows=args.evict_rows, page=1)
        if rank == 0:
            print(json.dumps({"profile_legs": res}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0
    specs = workload(args.seqs * max(world, SHARD_OF[0]), first_boundary_step=args.warmup)
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else args.steps
    steps_total = args.warmup + max(args.steps, e2e_steps)
    G, H, off = _shard(rank, world)
    B = len(specs)
    scale = D ** -0.5

    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    q = torch.randn((LAYERS, B, H, D), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty((LAYERS, B, H, D), dtype=torch.bfloat16, device=device)
    sinks = [torch.randn(H, generator=gen, device=device) for _ in range(LAYERS)]
    w_o = [(torch.randn((H * D, HIDDEN), generator=gen, device=device) * 0.02).to(torch.bfloat16)
           for _ in range(LAYERS)] if not args.no_oproj else None
    hidden = torch.empty((B, HIDDEN), dtype=torch.bfloat16, device=device)

    def after_layer(l, o):
        if w_o is not None:
            tp.output_reduction(o, w_o[l], group, out=hidden)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[device.index])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ------------------------------------------------ device-resident pass
    eng = build_engine(specs, steps_total, world, rank, group, device)
    for _ in range(args.warmup):
        eng.step(q, out, sinks, scale, after_layer)
    barrier()
    torch.cuda.synchronize()
    ev = []   # (start, end, bytes) per fused decode launch
    proj_ev = []   # (start, after the output projection, after its all-reduce) per layer

    def after_layer_timed(l, o):
        if w_o is None:
            return
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        torch.matmul(o.reshape(o.shape[0], -1), w_o[l], out=hidden)
        e1.record()
        if group is not None and world > 1:
            dist.all_reduce(hidden, op=dist.ReduceOp.SUM, group=group)
        e2.record()
        proj_ev.append((e0, e1, e2))
    bound_before = len(eng.boundary_ms)
    events_before = sum(len(eng.rows[r].events) for r in eng.active)
    launches0 = kernels.LAUNCHES[0]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tokens_resident = []
    resident = ResidentCounter(eng)
    with ClockSampler(device.index) as clocks:
        start.record()
        for s in range(args.steps):
            eng.run_boundaries(eng.due())
            eng.advance()
            eng._ensure_capacity(0)
            eng.fill()
            res_tok, h2o_pages = resident()
            nbytes = res_tok * G * D * 2 * 2 + 2 * B * H * D * 2 + h2o_pages * G * 8
            tokens_resident.append(res_tok)
            for l in range(LAYERS):
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record()
                eng.decode_layer(l, q[l], out[l], sinks[l], scale)
                b.record()
                ev.append((a, b, nbytes))
                after_layer_timed(l, out[l])
        eng.join_scores()          # the last layers' page scores are inside the timed region
        end.record()
        torch.cuda.synchronize()
    barrier()
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    launches = kernels.LAUNCHES[0] - launches0
    eng.check_errors()
    dur = [a.elapsed_time(b) for a, b, _ in ev]
    avg_launch_ms = statistics.mean(dur)
    avg_bytes = statistics.mean(x for _, _, x in ev)
    achieved_gbs = avg_bytes / (avg_launch_ms * 1e-3) / 1e9
    layer_ms = {"attention": avg_launch_ms,
                "o_proj": statistics.mean(a.elapsed_time(b) for a, b, _ in proj_ev) if proj_ev else None,
                "all_reduce": statistics.mean(b.elapsed_time(c) for _, b, c in proj_ev) if proj_ev else None}
    if world > 1:
        layer_ms = {k: (max_over_ranks(v) if v is not None else None) for k, v in layer_ms.items()}
    boundary_ms = eng.boundary_ms[bound_before:]
    n_bound_rows = sum(len(eng.rows[r].events) for r in eng.active) - events_before
    value = B * args.steps / (elapsed_ms * 1e-3)
    clock_info = clocks.summary()
    del eng
    torch.cuda.empty_cache()

    # --------------------------------------------------------- e2e pass
    e2e_value, step_bytes = None, LAYERS * B * H * D * 2
    if e2e_steps > 0 and "e2e" in legs:
        e2e_value = run_e2e(args, specs, steps_total, world, rank, group, device, q, out, sinks,
                            scale, after_layer, barrier, max_over_ranks, e2e_steps)

    cb3 = None
    if "cb3" in legs:
        cb3 = continuous_microbench(world, rank, group, device, barrier, max_over_ranks)
    model2 = None
    if "model2" in legs:
        model2 = model2_microbench(world, rank, device)
    decode4 = None
    if "decode4" in legs:
        decode4 = decode4_microbench(world, rank, group, device, barrier, max_over_ranks)
    prefill4 = None
    if "prefill4" in legs:
        prefill4 = prefill_microbench(world, rank, device, cpu=(rank == 0 and args.cpu_seconds > 0),
                                      prefixes=prefixes)
    no_score = None
    if "noscore" in legs:
        no_score = run_no_score(args, specs, steps_total, world, rank, group, device, q, out, sinks,
                                scale, after_layer, barrier, max_over_ranks)

    evict5 = None
    if not args.no_evict_bench and "evict5" in legs:
        evict5 = evict_microbench(world, rank, device, rows=args.evict_rows)
        if world > 1:   # every rank runs its shard; report the slowest (same collectives on every rank)
            for k in evict5:
                evict5[k]["evict_step_us"] = max_over_ranks(evict5[k]["evict_step_us"])
    select1 = None
    if not args.no_evict_bench and "select1" in legs:
        select1 = select_token_microbench(world, rank, device, rows=args.evict_rows)
    evict1 = None
    if not args.no_evict_bench and "evict1" in legs:
        evict1 = evict_microbench(world, rank, device, rows=args.evict_rows, page=1)
        if world > 1:
            for k in evict1:
                evict1[k]["evict_step_us"] = max_over_ranks(evict1[k]["evict_step_us"])
    peak, peak_kind = measured_peak_hbm()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_block(world),
        "roofline": {"bound": "hbm", "kernel": "ce_decode_attn_score (attn_kernel + combine_kernel)",
                     "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                     "frac": achieved_gbs / peak, "peak_kind": peak_kind,
                     "bytes_per_launch": avg_bytes, "launch_ms": avg_launch_ms,
                     "traffic": TRAFFIC_BYTES_PER_RESIDENT_TOKEN * statistics.mean(tokens_resident)
                                * G / G_TOTAL,
                     "traffic_source": "ncu dram__bytes_read+write of an 8-sequence capture, "
                                       "scaled by resident tokens"},
        "clocks": clock_info,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": step_bytes,
                "d2h_bytes_per_step": step_bytes,
                "path": "pinned host q (all layers) -> device, engine.step via the C ABI, "
                        "attention outputs -> pinned host, every step; copies per layer on their "
                        "own streams, overlapped with the decode"},
        "gpu_launches": launches,
        "layer_ms": dict(layer_ms, what="per layer, by CUDA events in the timed steps (max over ranks): the "
                                        "fused decode launch, the row-parallel output projection, and its "
                                        "NCCL all-reduce across ranks"),
        "evict": {"boundary_batches": len(boundary_ms),
                  "boundary_ms_mean": statistics.mean(boundary_ms) if boundary_ms else None,
                  "boundary_rows": n_bound_rows},
        "resident_tokens_mean": statistics.mean(tokens_resident),
        "no_score_same_resident": None if no_score is None else {
                                   "value": no_score["value"], "unit": UNIT,
                                   "scored_value": no_score["scored_value"],
                                   "scored_over_no_score": no_score["scored_over_no_score"],
                                   "pairs": no_score["pairs"], "segment_steps": no_score["segment_steps"],
                                   "what": "scored and unscored engines (same rows, steps and boundaries, "
                                           "H2O scoring off in the second: full-cache decode at the same "
                                           "resident KV) timed in alternating segments"},
        "evict_config5": evict5,
        "select_token_config5": select1,
        "evict_token_config5": evict1,
        "continuous_config3": cb3,
        "model_config2": model2,
        "decode_config4": decode4,
        "prefill_config4": prefill4,
    }
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        from oracle import oracle
        cores = os.cpu_count() or 1
        oracle.set_threads(cores)
        per_step, info = cpu_steps(specs, 1, args.steps, budget_s=args.cpu_seconds)
        line["cpu_baseline"] = {"value": B / per_step, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": cpu_sample_text(info, B, args.steps)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
