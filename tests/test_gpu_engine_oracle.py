"""The ragged decode engine's own multi-step loop against the CPU oracle.

RaggedDecodeEngine.step (due boundaries, one token appended, CSR fill, the
fused decode of every layer) runs at 16-token pages while a host mirror of its
state (tables, req_to_unit rows, frontiers, counts, positions, scores and both
pools of every layer) is advanced by the oracle's restatement of the same
steps.  Every step checks:

  * the CSR page table against oracle.fill (runtime:136-152), bit for bit;
  * each layer's fp32 attention output against oracle.decode (relative L2
    error below 1e-3 per row) and the accumulated page scores of every layer
    against the mirror's (rtol 1e-3, atol 1e-6: the scores carry every step's
    additions since the last boundary, runtime:155-224);

and every boundary batch checks, bit for bit, the per-row results, freed
units, table, req_to_unit, frontier, count, positions, scores and both K/V
pools against oracle.boundary (runtime:415-507) run on the same scores and
the same uniforms ("bit-exact given identical scores and draws").  The test
writes each new token's K and V into its page before the layers run, as the
serving loop does.

Workloads: benchmark config 1 (one layer, 64 query / 8 KV heads, batch 1, a
4,096-token cache, per-head H2O at budget 2048 = 512 + 512 + 1024, 256 decode
steps), once from a never-evicted cache and once from a cache evicted at
4,096 whose next boundary works over kept plus new pages; with config 1 the
kept pages that a boundary taken at that step would choose are also checked
every step (ce_choose against oracle.choose on the engine's scores).  Then a
small config-3 mix: eight ragged rows over all five policies (per-head H2O sum
and max, H2O global, random with the engine's uniforms, reservoir, recent) and
one full-cache row on two layers, 40 steps crossing seven boundaries, two of
them in one batch.  Mirrors the reference's per-step causal checks
(code/tests/test_sglang_evict.py:48-78, 92-148; core.py:33-118).
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
H, G, D, P = 64, 8, 64, 16
SCALE = D ** -0.5


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi
    capi.load()


def _cfg(name, budget, seed):
    from cache_eviction_b200.policy import EvictionConfig, sweep_split
    p, r = sweep_split(budget, name)
    return EvictionConfig(name, budget, p, r, seed=seed)


def _bits(t):
    """bf16 device tensor -> uint16 host array of its bit patterns."""
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


class Mirror:
    """Host copy of the engine's eviction state, advanced by the oracle."""

    def __init__(self, eng):
        torch.cuda.synchronize()
        self.eng = eng
        self.state = {k: getattr(eng, k).cpu().numpy().copy()
                      for k in ("table", "r2u", "frontier", "count", "pos", "scores")}
        self.k = [_bits(t).copy() for t in eng.k]
        self.v = [_bits(t).copy() for t in eng.v]
        self.batches = 0

    # ---------------------------------------------------------- boundaries
    def boundary_from_engine(self):
        """Run the batch the engine just ran on the mirror and compare."""
        eng, lb = self.eng, self.eng.last_batch
        uni = None if lb["uniforms"] is None else lb["uniforms"].cpu().numpy()
        res_c, fr_c = oracle.boundary(self.state, self.k, self.v, lb["rows"], oracle.row_params(lb["params"]),
                                      lb["max_cols"], live=True, uniforms=uni)
        np.testing.assert_array_equal(lb["result"][:len(lb["rows"])], res_c)
        fr_g = lb["freed"].cpu().numpy()
        for i in range(len(lb["rows"])):
            nf = int(res_c[i, 3])
            np.testing.assert_array_equal(fr_g[i, :nf], fr_c[i, :nf], err_msg=f"freed of row {lb['rows'][i]}")
        self.compare_state(exact_scores=True)
        for l in range(eng.L):
            np.testing.assert_array_equal(_bits(eng.k[l]), self.k[l], err_msg=f"K pool of layer {l}")
            np.testing.assert_array_equal(_bits(eng.v[l]), self.v[l], err_msg=f"V pool of layer {l}")
        self.batches += 1
        return res_c

    def compare_state(self, exact_scores=False):
        eng = self.eng
        for key in ("table", "r2u", "frontier", "count", "pos"):
            np.testing.assert_array_equal(getattr(eng, key).cpu().numpy(), self.state[key], err_msg=key)
        got = eng.scores.cpu().numpy()
        if exact_scores:
            np.testing.assert_array_equal(got, self.state["scores"], err_msg="scores")
        else:
            np.testing.assert_allclose(got, self.state["scores"], rtol=1e-3, atol=1e-6, err_msg="scores")

    # ---------------------------------------------------------------- CSR
    def csr(self):
        eng = self.eng
        rows = np.array(eng.active, np.int64)
        lens = np.array([eng.rows[r].n for r in eng.active], np.int64)
        s = self.state
        indptr, indices, tokens = oracle.fill(s["table"], s["r2u"], s["frontier"], s["count"], rows, lens, page=P)
        bs = len(rows)
        np.testing.assert_array_equal(eng.kv_indptr[:bs + 1].cpu().numpy(), indptr)
        np.testing.assert_array_equal(eng.kv_indices[:indptr[-1]].cpu().numpy(), indices.astype(np.int32))
        np.testing.assert_array_equal(eng.kv_tokens[:bs].cpu().numpy(), tokens)
        return indptr, indices.astype(np.int32), tokens

    def take_new_pages(self):
        """The unit pool's choices for rows whose new token starts a page
        (ce_pool_alloc), copied from the device: the allocator is SGLang's
        side of the contract, the oracle's starts from its assignments."""
        eng = self.eng
        for r in eng.active:
            t = eng.rows[r].n - 1
            if t % P == 0:
                self.state["r2u"][r, t // P] = int(eng.r2u[r, t // P])

    def check_ownership(self):
        """Every unit is held at most once: by one row (its compacted table
        and tail) or by the free stack, and unit 0 (padding) by nobody."""
        eng = self.eng
        held = [eng.owned_units(r).cpu().numpy() for r in eng.active]
        free = eng.free_stack[:eng.free_top].cpu().numpy()
        assert int(eng.free_top_dev.item()) == eng.free_top
        allu = np.concatenate(held + [free])
        assert len(np.unique(allu)) == len(allu), "a unit is held twice"
        assert (allu > 0).all() and (allu < eng.units).all()
        return len(allu)

    def write_new_tokens(self, gen):
        """K and V of every row's newest token, into its page slot (GPU and mirror)."""
        eng = self.eng
        t = np.array([eng.rows[r].n - 1 for r in eng.active])
        units = self.state["r2u"][np.array(eng.active), t // P]
        slots = t % P
        u_t = torch.from_numpy(units.astype(np.int64)).to(DEV)
        s_t = torch.from_numpy(slots.astype(np.int64)).to(DEV)
        for l in range(eng.L):
            for pool, host in ((eng.k[l], self.k[l]), (eng.v[l], self.v[l])):
                new = torch.randn((len(units), G, D), generator=gen).to(torch.bfloat16)
                pool[u_t, :, s_t, :] = new.to(DEV)
                host[units, :, slots, :] = new.view(torch.int16).numpy().view(np.uint16)


def _kept_now_matches_oracle(eng, row):
    """ce_choose on the engine's current state of `row` (the pages a boundary
    taken now would keep, for every layer and head) against oracle.choose on
    the same positions and scores."""
    from cache_eviction_b200 import kernels
    r = eng.rows[row]
    cfg = r.cfg
    b, p, q = cfg.units(P)
    n_u = r.n // P
    cnt, fr = r.count, r.frontier
    N = cnt + n_u - fr
    if N <= b:
        return False
    pos = torch.empty((1, eng.L * G, N), dtype=torch.int32, device=DEV)
    pos[0, :, :cnt] = eng.pos[row, :, :, :cnt].reshape(eng.L * G, cnt)
    pos[0, :, cnt:] = torch.arange(fr, n_u, dtype=torch.int32, device=DEV)
    units = torch.cat([eng.table[row, :cnt], eng.r2u[row, fr:n_u]]).long()
    score = eng.scores[:, :, units].reshape(1, eng.L * G, N).contiguous()
    prm = [dict(n=n_u, budget=b, prefix=p, recent=q, cursor=None, policy=cfg.policy_id, seed=cfg.seed)]
    err = kernels.error_word(DEV)
    kept_g, st_g, _ = kernels.choose(pos, score, kernels.row_params(prm, DEV), eng.L, G, max_n=n_u + 1, err=err)
    kept_c, st_c, _ = oracle.choose(pos.cpu().numpy(), score.cpu().numpy(), oracle.row_params(prm), eng.L, G,
                                    score_is_f32=True)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert st_g.cpu().numpy().tolist() == st_c.tolist()
    np.testing.assert_array_equal(kept_g[0, :, :b].cpu().numpy(), kept_c[0, :, :b])
    return True


def _admit(eng, m, row, cfg, n, gen):
    """Admit a request into `row` on the engine (units from the free stack,
    random prompt K/V and lognormal page scores, then the prefill's last
    boundary) and on the mirror: the allocator's units, the prompt's contents
    and the scores the boundary ranks come from the device, the boundary
    itself from the oracle.  Returns whether a boundary batch ran."""
    def prompt(units):
        u = units.long()
        for l in range(eng.L):
            for pool in (eng.k[l], eng.v[l]):
                pool[u] = torch.randn((u.numel(), G, P, D), generator=gen, device=DEV).to(torch.bfloat16)
        eng.scores[:, :, u] = torch.randn((eng.L, G, u.numel()), generator=gen, device=DEV).mul_(2.0).exp_()
        torch.cuda.synchronize()
        un = units.cpu().numpy()
        m.state["r2u"][row, :len(un)] = un
        m.state["frontier"][row] = 0
        m.state["count"][row] = 0
        for l in range(eng.L):
            m.k[l][un] = _bits(eng.k[l][u])
            m.v[l][un] = _bits(eng.v[l][u])
        m.state["scores"][...] = eng.scores.cpu().numpy()

    before = eng.last_batch
    eng.admit(row, cfg, n, prompt=prompt)
    torch.cuda.synchronize()
    ran = eng.last_batch is not before
    if ran:
        m.boundary_from_engine()
    return ran


def _run(eng, steps, seed, check_kept_row=None, churn=None):
    """Drive engine.step for `steps` steps against the mirror; returns the
    boundary results seen (row, status) and the count of kept-set checks.
    churn: {step: [(row, spec)]} -- before that step, row retires and a new
    request (spec: ctx, cfg) is admitted into the same row slot."""
    gen_cpu = torch.Generator().manual_seed(seed)
    gen = torch.Generator(device=DEV).manual_seed(seed)
    L, B = eng.L, len(eng.active)
    sinks = [torch.randn(H, generator=gen, device=DEV) for _ in range(L)]
    sinks_h = [s.cpu().numpy() for s in sinks]
    out = torch.empty((L, B, H, D), dtype=torch.float32, device=DEV)
    m = Mirror(eng)
    m.compare_state(exact_scores=True)
    seen, kept_checks = [], 0
    gen_admit = torch.Generator(device=DEV).manual_seed(seed + 1)
    for step in range(steps):
        for row, spec in (churn or {}).get(step, []):
            eng.retire(row)
            m.state["frontier"][row] = 0
            m.state["count"][row] = 0
            _admit(eng, m, row, spec["cfg"], spec["ctx"], gen_admit)
            eng.commit_rows()
            m.check_ownership()
        due = eng.due()
        if due:
            # the boundary ranks the scores the GPU accumulated: give the
            # oracle those very scores (checked within tolerance every step)
            m.state["scores"][...] = eng.scores.cpu().numpy()
        batches0 = m.batches
        ctx = {}

        def before(l):
            if l:
                return
            torch.cuda.synchronize()
            # the step already allocated the new tokens' pages (after its
            # boundaries, whose columns end below them): take them first
            m.take_new_pages()
            if due:
                res = m.boundary_from_engine()
                seen.extend((r, int(res[i, 0])) for i, r in enumerate(eng.last_batch["rows"]))
            ctx["csr"] = m.csr()
            m.write_new_tokens(gen_cpu)

        q = torch.randn((L, B, H, D), generator=gen, device=DEV).to(torch.bfloat16)
        eng.step(q, out, sinks, SCALE, before_layer=before)
        torch.cuda.synchronize()
        assert m.batches == batches0 + (1 if due else 0)
        eng.check_errors()
        indptr, indices, tokens = ctx["csr"]
        modes = eng.mode.cpu().numpy()[np.array(eng.active)]
        qb = _bits(q)
        out_h = out.cpu().numpy()
        for l in range(L):
            o_c, _ = oracle.decode(qb[l], m.k[l], m.v[l], indptr, indices, tokens, sinks_h[l], modes, SCALE, P,
                                   scores=m.state["scores"][l], zero_new=True)
            num = np.linalg.norm((out_h[l] - o_c).reshape(B, -1), axis=1)
            den = np.linalg.norm(o_c.reshape(B, -1), axis=1)
            assert (num / den < 1e-3).all(), (step, l, (num / den).max())
        m.compare_state()
        assert m.check_ownership() == eng.units - 1     # no unit lost either
        if check_kept_row is not None:
            kept_checks += _kept_now_matches_oracle(eng, check_kept_row)
    return seen, kept_checks


def _engine(specs, steps, layers, pos_cap=512):
    from cache_eviction_b200.engine import RaggedDecodeEngine
    units = sum(-(-(sp["ctx"] + steps) // P) for sp in specs) + 64
    width = -(-(max(sp["ctx"] for sp in specs) + steps + 4096) // P)
    return RaggedDecodeEngine(layers=layers, q_heads=H, kv_heads=G, page_size=P, pool_units=units,
                              max_rows=len(specs), r2u_width=width, pos_cap=pos_cap, device=DEV)


def test_config1_fresh_cache_256_steps():
    """Config 1 from a 4,096-token cache never evicted (the prefill's boundary
    at 2,048 kept everything): the boundary at 4,096 is due on the first step,
    then 256 decode steps with every step's scores, outputs and would-be kept
    pages checked."""
    steps, ctx = 256, 4096
    cfg = _cfg("head_sum_2048", 2048, 11)
    eng = _engine([dict(ctx=ctx)], steps, layers=1)
    rng = np.random.default_rng(3)
    perm = (rng.permutation(eng.units - 1) + 1).astype(np.int32)
    units, free = perm[:ctx // P], perm[ctx // P:]
    eng.add_row(0, cfg, ctx, last_boundary=2048)
    eng.r2u[0, :ctx // P] = torch.from_numpy(units).to(DEV)
    eng.seed_free_units(free)
    gen = torch.Generator(device=DEV).manual_seed(12)
    idx = torch.from_numpy(units.astype(np.int64)).to(DEV)
    eng.scores[:, :, idx] = torch.randn((1, G, idx.numel()), generator=gen, device=DEV).mul_(2.0).exp_()
    for t in eng.k + eng.v:
        t.normal_(generator=gen)
    eng.commit_rows()
    seen, kept_checks = _run(eng, steps, seed=13, check_kept_row=0)
    assert seen == [(0, 0)]
    row = eng.rows[0]
    assert row.count == 128 and row.frontier == ctx // P and row.n == ctx + steps
    # every step once the row holds more pages than its budget (from 4,112 tokens)
    assert kept_checks == steps - 15


def test_config1_second_boundary_over_kept_and_new_pages():
    """Config 1 from a cache evicted at 4,096 (128 kept pages + 127 new ones
    and a partial page): the boundary at 6,144 ranks kept and new pages
    together; 256 steps."""
    from cache_eviction_b200.engine import synth_state
    steps = 256
    specs = [dict(ctx=6143, cfg=_cfg("head_sum_2048", 2048, 21))]
    eng = _engine(specs, steps, layers=1)
    synth_state(eng, specs, seed=22)
    seen, kept_checks = _run(eng, steps, seed=23, check_kept_row=0)
    assert seen == [(0, 0)]
    assert eng.rows[0].count == 128 and eng.rows[0].frontier == 6144 // P
    # the step before the boundary, then every step from 6,160 tokens
    assert kept_checks == 1 + steps - 16


def test_config3_mix_five_policies_two_layers():
    """Eight ragged rows covering every policy plus a full-cache row, two
    layers, 40 steps, seven boundaries (two rows due in the same batch)."""
    from cache_eviction_b200.engine import synth_state
    steps = 40
    specs = [dict(ctx=4090, cfg=_cfg("head_sum_2048", 2048, 1)),        # fresh; boundary at 4,096 (step 7)
             dict(ctx=6140, cfg=_cfg("h2o_global_2048", 2048, 2)),      # evicted at 4,096; 6,144 at step 5
             dict(ctx=8188, cfg=_cfg("head_sum_2048", 4096, 3)),        # evicted at 6,144; 8,192 at step 5
             dict(ctx=8180, cfg=_cfg("head_max_sum_2048", 2048, 4)),    # 8,192 at step 13
             dict(ctx=10230, cfg=_cfg("random_2048", 4096, 5)),         # 10,240 at step 11
             dict(ctx=4080, cfg=_cfg("prefix_sliding_2048", 2048, 6)),  # fresh; 4,096 at step 17
             dict(ctx=6120, cfg=_cfg("random_reservoir_2048", 2048, 7)),  # 6,144 at step 25
             dict(ctx=3000, cfg=None)]
    eng = _engine(specs, steps, layers=2)
    synth_state(eng, specs, seed=31)
    seen, _ = _run(eng, steps, seed=32)
    assert len(seen) == 7, seen
    assert all(status == 0 for _, status in seen), seen
    assert sorted(r for r, _ in seen) == [0, 1, 2, 3, 4, 5, 6]


def test_continuous_batch_reuses_units_of_retired_rows():
    """Continuous batching: mid-run, rows retire and new requests take their
    row slots; the prompts' units come from the free stack, which holds the
    retired rows' units and every boundary's leftovers, so freed units are
    reused.  Every step the engine matches the oracle (CSR, outputs,
    scores; every boundary bit for bit, the admissions' prefill boundaries
    included) and no unit is held twice or lost."""
    from cache_eviction_b200.engine import synth_state
    steps = 36
    specs = [dict(ctx=4090, cfg=_cfg("head_sum_2048", 2048, 1)),
             dict(ctx=6140, cfg=_cfg("h2o_global_2048", 2048, 2)),
             dict(ctx=5000, cfg=_cfg("random_2048", 2048, 3)),
             dict(ctx=3000, cfg=None),
             dict(ctx=8180, cfg=_cfg("head_max_sum_2048", 4096, 4))]
    churn = {3: [(3, dict(ctx=4200, cfg=_cfg("head_sum_2048", 2048, 9)))],      # full row out, H2O row in
             9: [(2, dict(ctx=2040, cfg=_cfg("prefix_sliding_2048", 1024, 10)))],  # boundary at 2,048 later
             20: [(0, dict(ctx=6500, cfg=_cfg("random_2048", 4096, 11))),
                  (1, dict(ctx=700, cfg=None))]}
    eng = _engine(specs + [dict(ctx=6500)], steps, layers=2)
    synth_state(eng, specs, seed=41)
    seen, _ = _run(eng, steps, seed=42, churn=churn)
    # the admitted prefix-sliding row crosses 2,048 at step 17; the others'
    # own boundaries fall at 4,096 (step 6), 6,144 (step 4) and 8,192 (step 12)
    assert sorted(r for r, _ in seen) == [0, 1, 2, 4], seen
    assert all(status == 0 for _, status in seen), seen
    assert sum(eng.rows[r].freed for r in eng.active) > 0
