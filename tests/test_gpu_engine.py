"""The ragged decode engine with each layer's H2O page scores deferred to a
second stream (ce_decode_attn_score with CE_SCORE_DEFER, then
ce_decode_scores from the same workspace) against the same engine scoring
inside the decode call: attention outputs every step, and scores, tables,
positions, req_to_unit rows, counts and frontiers at the end, bit for bit,
over steps that cross eviction boundaries of per-head H2O and H2O global rows.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
L, H, G, P = 2, 64, 8, 16
STEPS = 12


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi
    capi.load()


def _specs():
    from cache_eviction_b200.policy import EvictionConfig, sweep_split

    def cfg(name, budget, seed):
        p, r = sweep_split(budget, name)
        return EvictionConfig(name, budget, p, r, seed=seed)
    return [dict(ctx=4090, cfg=cfg("head_sum_2048", 2048, 1)),      # first boundary at 4,096
            dict(ctx=6140, cfg=cfg("h2o_global_2048", 2048, 2)),    # evicted; next at 6,144
            dict(ctx=5000, cfg=cfg("head_max_sum_2048", 2048, 3)),
            dict(ctx=9000, cfg=cfg("random_2048", 4096, 4)),
            dict(ctx=3000, cfg=None),
            dict(ctx=8190, cfg=cfg("head_sum_2048", 4096, 5))]       # boundary at 8,192


def _engine(overlap):
    from cache_eviction_b200.engine import RaggedDecodeEngine, synth_state
    specs = _specs()
    units = sum(-(-(sp["ctx"] + STEPS) // P) for sp in specs) + 64
    width = -(-(max(sp["ctx"] for sp in specs) + STEPS + 4096) // P)
    eng = RaggedDecodeEngine(layers=L, q_heads=H, kv_heads=G, page_size=P, pool_units=units,
                             max_rows=len(specs), r2u_width=width, pos_cap=512, device=DEV,
                             overlap_scores=overlap)
    synth_state(eng, specs, seed=5)
    torch.cuda.synchronize()
    return eng


def test_overlapped_scores_match_inline_scores():
    a, b = _engine(True), _engine(False)
    B = len(a.active)
    gen = torch.Generator(device=DEV).manual_seed(9)
    q = torch.randn((L, B, H, 64), generator=gen, device=DEV).to(torch.bfloat16)
    sinks = [torch.randn(H, generator=gen, device=DEV) for _ in range(L)]
    out_a = torch.empty((L, B, H, 64), dtype=torch.bfloat16, device=DEV)
    out_b = torch.empty_like(out_a)
    for _ in range(STEPS):
        a.step(q, out_a, sinks, 0.125)
        b.step(q, out_b, sinks, 0.125)
        a.join_scores()
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b)
    a.join_scores()
    a.check_errors()
    b.check_errors()
    events = [e for r in a.active for e in a.rows[r].events]
    assert sum(e["status"] == 0 for e in events) >= 2, events   # boundaries were crossed
    for key in ("scores", "table", "pos", "r2u", "count", "frontier"):
        assert torch.equal(getattr(a, key), getattr(b, key)), key
    assert a.scores.abs().sum() > 0


@pytest.mark.parametrize("page", [16, 1])
def test_deferred_scores_equal_inline_scores(page):
    """ce_decode_attn_score(CE_SCORE_DEFER) + ce_decode_scores against one
    ce_decode_attn_score call, over sum, max and unscored rows: outputs and
    scores bit for bit."""
    from cache_eviction_b200 import capi, kernels
    gen = torch.Generator(device=DEV).manual_seed(31 + page)
    lengths = [40, 300, 1025, 17, 2048 + 5]
    modes = torch.tensor([capi.CE_MODE_SUM, capi.CE_MODE_MAX, capi.CE_MODE_SUM, capi.CE_MODE_NONE,
                          capi.CE_MODE_MAX], dtype=torch.int32, device=DEV)
    pages = [-(-n // page) for n in lengths]
    units = sum(pages) + 8
    kp = torch.randn((units, G, page, 64), generator=gen, device=DEV).to(torch.bfloat16)
    vp = torch.randn((units, G, page, 64), generator=gen, device=DEV).to(torch.bfloat16)
    q = torch.randn((len(lengths), H, 64), generator=gen, device=DEV).to(torch.bfloat16)
    sinks = torch.randn(H, generator=gen, device=DEV)
    idx = (torch.randperm(units - 1, generator=gen, device=DEV)[:sum(pages)] + 1).int()
    indptr = torch.tensor([0] + list(torch.tensor(pages).cumsum(0)), dtype=torch.int32, device=DEV)
    tokens = torch.tensor(lengths, dtype=torch.int32, device=DEV)
    base = torch.rand((G, units), generator=gen, device=DEV)
    s_inline, s_defer = base.clone(), base.clone()
    err = kernels.error_word(DEV)
    o1 = kernels.decode_attn_score(q, kp, vp, indptr, idx, tokens, 0.125, page, sinks=sinks, mode_of_row=modes,
                                   scores=s_inline, out_f32=True, err=err)
    ws = torch.empty(kernels.decode_workspace_bytes(len(lengths), idx.numel(), H, G, page, 3),
                     dtype=torch.uint8, device=DEV)
    o2 = kernels.decode_attn_score(q, kp, vp, indptr, idx, tokens, 0.125, page, sinks=sinks, mode_of_row=modes,
                                   scores=s_defer, out_f32=True, err=err, workspace=ws,
                                   score_flags=3 | capi.CE_SCORE_DEFER)
    torch.cuda.synchronize()
    assert torch.equal(s_defer, base)          # nothing scored yet
    kernels.decode_scores(indptr, idx, tokens, units, page, H, G, len(lengths), modes, None, s_defer, ws, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(o1, o2)
    assert torch.equal(s_inline, s_defer)
    assert not torch.equal(s_inline, base)


def test_prepare_device_loads_kernels():
    """ce_prepare_device succeeds (and is idempotent) on the current device."""
    from cache_eviction_b200 import kernels
    kernels.prepare_device(DEV)
    kernels.prepare_device(DEV)
