"""ce_boundary at the config-5 shape (4,096 pages of 16 tokens per row, 8 KV
heads, budgets 2K-32K tokens, prefix = recent = budget / 4), checked through
properties that do not need the CPU oracle to move gigabytes of K/V:

* the kept positions of every (row, head) are the oracle's choice on the same
  keys (runtime:376-412), protected first then the middle set, each ascending;
* every (row, head, column) of the new table holds, bit for bit, the K and V
  slices of the position it claims (runtime:452-469);
* scores moved with their pages, and the freed units are exactly the row's
  other units (runtime:476-491).
The oracle pins the same kernels bit for bit at small sizes
(test_gpu_kernels.py); this runs them at full size on 8 rows.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
R, G, PAGE, D, N = 8, 8, 16, 64, 4096


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi
    capi.load()


@pytest.fixture(scope="module")
def pools():
    gen = torch.Generator(device=DEV).manual_seed(71)
    units = R * N + 1
    kp = torch.randn((units, G, PAGE, D), generator=gen, device=DEV).to(torch.bfloat16)
    vp = torch.randn((units, G, PAGE, D), generator=gen, device=DEV).to(torch.bfloat16)
    scores = torch.randn((1, G, units), generator=gen, device=DEV).mul_(2.0).exp_()
    r2u = (torch.randperm(units - 1, generator=gen, device=DEV)[:R * N].int() + 1).view(R, N).contiguous()
    uni = torch.rand((R, 1, G, N), generator=gen, device=DEV, dtype=torch.float64)
    return kp, vp, scores, r2u, uni


@pytest.mark.parametrize("policy", ["head_sum_2048", "h2o_global_2048", "random_2048"])
@pytest.mark.parametrize("budget_tokens", [2048, 8192, 32768])
def test_boundary_full_size_properties(pools, policy, budget_tokens):
    from cache_eviction_b200 import kernels
    kp0, vp0, scores0, r2u0, uni = pools
    kp, vp, scores, r2u = kp0.clone(), vp0.clone(), scores0.clone(), r2u0.clone()
    b = budget_tokens // PAGE
    p_, r_ = b // 4, b // 4
    params = [dict(n=N, budget=b, prefix=p_, recent=r_, cursor=None, policy=policy, seed=i) for i in range(R)]
    table = torch.zeros((R, N), dtype=torch.int32, device=DEV)
    frontier = torch.zeros(R, dtype=torch.int32, device=DEV)
    count = torch.zeros(R, dtype=torch.int32, device=DEV)
    pos = torch.zeros((R, 1, G, b), dtype=torch.int32, device=DEV)
    marks = torch.zeros(kp.shape[0], dtype=torch.int32, device=DEV)
    err = kernels.error_word(DEV)
    res, freed = kernels.boundary(table, r2u, frontier, count, pos, scores, kernels.layer_pointers([kp], DEV),
                                  kernels.layer_pointers([vp], DEV), G, PAGE,
                                  torch.arange(R, dtype=torch.int32, device=DEV), kernels.row_params(params, DEV),
                                  N, N + 1, True, marks=marks, epoch=1,
                                  uniforms=uni if policy == "random_2048" else None, err=err, max_width=b)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, hex(int(err.item()))
    res = res.cpu().numpy()
    assert (res[:, 0] == 0).all() and (res[:, 2] == b).all() and (res[:, 3] == N - b).all()

    # kept positions: the oracle's choice on the keys the boundary saw
    cols = np.broadcast_to(np.arange(N, dtype=np.int32), (R, G, N)).copy()
    if policy == "random_2048":
        key = uni.view(R, G, N).cpu().numpy()
    else:
        key = scores0[0][:, r2u0.long()].permute(1, 0, 2).contiguous().cpu().numpy()   # [R, G, N]
    kept_c, st_c, _ = oracle.choose(cols, key, oracle.row_params(params), 1, G,
                                    score_is_f32=policy != "random_2048")
    assert (st_c == 0).all()
    got = pos.cpu().numpy()[:, 0]                                     # [R, G, b]
    protected = np.concatenate([np.arange(p_), np.arange(N - r_, N)])
    for r in range(R):
        for g in range(G):
            kept = kept_c[r, g, :b]
            middle = np.setdiff1d(kept, protected)
            np.testing.assert_array_equal(got[r, g], np.concatenate([protected, middle]),
                                          err_msg=f"row {r} head {g}")

    # relocated K/V slices and scores, by gather on the device
    tab = table[:, :b].long()                                          # [R, b] new units
    src = torch.gather(r2u0.long(), 1, pos[:, 0].reshape(R, G * b).long()).view(R, G, b)   # original units
    heads = torch.arange(G, device=DEV).view(1, G, 1).expand(R, G, b)
    dst = tab.view(R, 1, b).expand(R, G, b)
    assert torch.equal(kp[dst, heads], kp0[src, heads])
    assert torch.equal(vp[dst, heads], vp0[src, heads])
    assert torch.equal(scores[0][heads, dst], scores0[0][heads, src])

    # freed units: every unit the row owned that the table does not hold
    fr = freed.cpu().numpy()
    owned = r2u0.cpu().numpy()
    tabn = tab.cpu().numpy()
    for r in range(R):
        want = np.setdiff1d(owned[r], tabn[r])
        np.testing.assert_array_equal(np.sort(fr[r, :N - b]), np.sort(want))
        assert len(np.unique(tabn[r])) == b and np.isin(tabn[r], owned[r]).all()
