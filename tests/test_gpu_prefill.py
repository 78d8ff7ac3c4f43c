"""GPU parity of the prefill / extend score kernel (ce_prefill_scores, the
reference's _prefill_scores, runtime:314-340), called through the C ABI,
against the reference's golden fixtures and the CPU oracle.

Tolerance: scores within 1e-3 relative (the north star's bound for fp32
scores), 1e-6 absolute for near-zero units; units of skipped entries must be
untouched bit for bit.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from golden import scenarios as sc
from helpers import prefill_inputs, prefill_want
from oracle import oracle

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
DEV = "cuda:0"
RTOL, ATOL = 1e-3, 1e-6


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi
    capi.load()


def K():
    from cache_eviction_b200 import kernels
    return kernels


def t16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(DEV).view(torch.bfloat16)


def ti(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(DEV)


def run(q_dev, kpool, qo_indptr, indptr, indices, tokens, sinks, modes, scale, page, scores0,
        zero_new=True, max_q=None, max_tokens=None):
    scores = torch.from_numpy(scores0.copy()).to(DEV)
    err = K().error_word(DEV)
    nq = np.diff(qo_indptr)
    K().prefill_scores(q_dev, t16(kpool), ti(qo_indptr), ti(indptr), ti(indices), ti(tokens), scale, page,
                       max_q=int(nq.max()) if max_q is None else max_q,
                       max_tokens=int(np.max(tokens)) if max_tokens is None else max_tokens,
                       sinks=None if sinks is None else torch.from_numpy(sinks).to(DEV),
                       mode_of_row=ti(modes), scores=scores, zero_new=zero_new, err=err)
    torch.cuda.synchronize()
    return scores.cpu().numpy(), int(err.item())


@pytest.mark.parametrize("page", [1, 16])
@pytest.mark.parametrize("mode", [1, 2])
def test_prefill_reference_golden(page, mode):
    z = np.load(GOLD / "prefill.npz")
    d, kpool, units, indptr, indices, tokens = prefill_inputs(page)
    init = np.random.default_rng(3).random((sc.G, kpool.shape[0])).astype(np.float32)
    got, err = run(t16(d["q"]), kpool, d["qo_indptr"], indptr, indices, tokens, sc.bits_to_f32(d["sinks"]),
                   np.full(len(tokens), mode, np.int32), d["scale"], page, init)
    assert err == 0
    want = prefill_want(z, mode, page, units, init.astype(np.float64))
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def ragged_case(G, page, seed):
    """Mixed entries: (prefix tokens, chunk queries, mode)."""
    entries = [(1000, 300, 1), (0, 1, 2), (517, 64, 0), (2000, 33, 2), (40, 200, 1), (255, 97, 1)]
    rng = np.random.default_rng(seed)
    H = 8 * G
    units_per = [-(-(p + n) // page) for p, n, _ in entries]
    pool_units = sum(units_per) + 7
    perm = rng.permutation(pool_units - 1) + 1
    lists, k = [], 0
    for u in units_per:
        lists.append(perm[k:k + u].astype(np.int32))
        k += u
    kpool = sc.bf16_bits(rng.standard_normal((pool_units, G, page, 64), dtype=np.float32))
    total_q = sum(n for _, n, _ in entries)
    # queries live inside a wider [total_q, 2H, 64] buffer: strided head and token steps
    qwide = sc.bf16_bits(rng.standard_normal((total_q, 2 * H, 64), dtype=np.float32))
    qo_indptr = np.concatenate([[0], np.cumsum([n for _, n, _ in entries])]).astype(np.int32)
    indptr = np.concatenate([[0], np.cumsum(units_per)]).astype(np.int32)
    tokens = np.array([p + n for p, n, _ in entries], np.int32)
    modes = np.array([m for _, _, m in entries], np.int32)
    sinks = rng.standard_normal(H).astype(np.float32)
    return dict(kpool=kpool, qwide=qwide, H=H, qo_indptr=qo_indptr, indptr=indptr,
                indices=np.concatenate(lists), tokens=tokens, modes=modes, sinks=sinks, lists=lists)


@pytest.mark.parametrize("G,page", [(8, 16), (8, 1), (2, 16), (1, 4)])
@pytest.mark.parametrize("with_sinks", [True, False])
def test_prefill_ragged_vs_oracle(G, page, with_sinks):
    c = ragged_case(G, page, seed=17 + G + page)
    H = c["H"]
    q_host = np.ascontiguousarray(c["qwide"][:, H:2 * H])        # the heads the kernel sees
    q_dev = t16(c["qwide"])[:, H:2 * H]                          # strided view
    sinks = c["sinks"] if with_sinks else None
    init = np.random.default_rng(5).random((G, c["kpool"].shape[0])).astype(np.float32)
    got, err = run(q_dev, c["kpool"], c["qo_indptr"], c["indptr"], c["indices"], c["tokens"], sinks,
                   c["modes"], 0.125, page, init)
    assert err == 0
    want = init.copy()
    oracle.prefill(q_host, c["kpool"], c["qo_indptr"], c["indptr"], c["indices"], c["tokens"], sinks,
                   c["modes"], 0.125, page, want, zero_new=True)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    skipped = c["lists"][2]                                      # mode 0 entry
    assert np.array_equal(got[:, skipped].view(np.uint32), init[:, skipped].view(np.uint32))


def test_prefill_accumulates_without_zero_new():
    c = ragged_case(8, 16, seed=3)
    init = np.random.default_rng(6).random((8, c["kpool"].shape[0])).astype(np.float32)
    q = np.ascontiguousarray(c["qwide"][:, :64])
    got, err = run(t16(q), c["kpool"], c["qo_indptr"], c["indptr"], c["indices"], c["tokens"], c["sinks"],
                   c["modes"], 0.125, 16, init, zero_new=False)
    assert err == 0
    want = init.copy()
    oracle.prefill(q, c["kpool"], c["qo_indptr"], c["indptr"], c["indices"], c["tokens"], c["sinks"],
                   c["modes"], 0.125, 16, want, zero_new=False)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def test_prefill_entry_beyond_bounds_is_flagged_and_skipped():
    from cache_eviction_b200 import capi
    c = ragged_case(8, 16, seed=4)
    init = np.zeros((8, c["kpool"].shape[0]), np.float32)
    q = np.ascontiguousarray(c["qwide"][:, :64])
    # max_q below the longest chunk (300 queries): that entry is skipped, the rest scored
    got, err = run(t16(q), c["kpool"], c["qo_indptr"], c["indptr"], c["indices"], c["tokens"], c["sinks"],
                   c["modes"], 0.125, 16, init, max_q=256)
    assert err & capi.CE_EW_SHAPE
    assert not got[:, c["lists"][0]].any()
    assert got[:, c["lists"][4]].all()


def test_prefill_full_size_mass_checksum():
    """Config-4 shape (26,624 resident prefix tokens + a 2,048-token chunk,
    16-token pages, no sinks): in SUM mode every query head's probabilities
    sum to 1, so each KV head's unit scores total 8 x 2048."""
    rng = np.random.default_rng(9)
    prefix, nq, G, page = 26624, 2048, 8, 16
    ntok = prefix + nq
    units = ntok // page
    kpool = torch.randn((units + 1, G, page, 64), device=DEV).to(torch.bfloat16)
    q = torch.randn((nq, 64, 64), device=DEV).to(torch.bfloat16)
    idx = torch.from_numpy((rng.permutation(units) + 1).astype(np.int32)).to(DEV)
    scores = torch.zeros((G, units + 1), dtype=torch.float32, device=DEV)
    err = K().error_word(DEV)
    K().prefill_scores(q, kpool, ti([0, nq]), ti([0, units]), idx, ti([ntok]), 0.125, page, nq, ntok,
                       mode_of_row=ti([1]), scores=scores, zero_new=True, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    tot = scores.double().sum(1).cpu().numpy()
    np.testing.assert_allclose(tot, 8.0 * nq, rtol=1e-4)
    # causality: the chunk's last page is seen only by queries at or after its tokens
    last = int(idx[-1])
    assert float(scores[:, last].min()) > 0
