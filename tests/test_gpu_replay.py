"""GPU parity of the replay layer-error kernel (ce_replay_error, the
reference's _replay_layer_difference, runtime:520-546) through the C ABI,
against the reference's golden errors and the CPU oracle.

Tolerance: errors within 1e-3 relative (the north star's bound for fp32
results; P is rounded to bf16 for the tensor cores, each term by at most
2^-9, which averages out over a query's 512 output values); masked outputs
within 1e-3 relative in norm per query.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from golden import scenarios as sc
from oracle import oracle

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
DEV = "cuda:0"


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


def bits_of(vis):
    """[G, T] bool -> [G, ceil(T/32)] int32 bit words (bit t of word t/32)."""
    G, T = vis.shape
    W = (T + 31) // 32
    padded = np.zeros((G, W * 32), bool)
    padded[:, :T] = vis
    words = (padded.reshape(G, W, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)).sum(-1)
    return torch.from_numpy(words.astype(np.uint32).view(np.int32)).to(DEV)


def run(q_dev, kbits, vbits, start, scale, vis=None, sinks=None, out=False):
    err = K().error_word(DEV)
    o = torch.full(tuple(q_dev.shape), float("nan"), dtype=torch.float32, device=DEV) if out else None
    e = K().replay_error(q_dev, t16(kbits), t16(vbits), start, scale,
                         visible_bits=None if vis is None else bits_of(vis),
                         sinks=None if sinks is None else torch.from_numpy(sinks).to(DEV), out_masked=o, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, hex(int(err.item()))
    return e.cpu().numpy(), (None if o is None else o.cpu().numpy())


@pytest.mark.parametrize("chunk", range(len(sc.REPLAY_CHUNKS)))
def test_replay_reference_golden(chunk):
    z = np.load(GOLD / "replay.npz")
    d = sc.replay_setup()
    lo, hi, evicted = sc.REPLAY_CHUNKS[chunk]
    vis = sc.replay_visible(d["pos"], sc.REPLAY_FRONTIER, hi) if evicted else None
    got, _ = run(t16(d["q"][lo:hi]), d["keys"], d["values"], lo, d["scale"], vis, d["sinks"])
    want = z[f"chunk{chunk}"]
    if not evicted:
        assert not got.any()      # nothing evicted: b == a exactly
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=1e-6)


def _case(rng, G, start, count, keep_frac, rows_extra=37):
    H = 8 * G
    n = start + count + rows_extra
    k = sc.bf16_bits(rng.standard_normal((n, G, 64), dtype=np.float32) * 1.5)
    v = sc.bf16_bits(rng.standard_normal((n, G, 64), dtype=np.float32))
    q = sc.bf16_bits(rng.standard_normal((count, 2 * H, 64), dtype=np.float32) * 1.5)
    vis = rng.random((G, start + count)) < keep_frac
    vis[:, start:] = True     # the chunk itself stays visible, as after a boundary
    return H, k, v, q, vis


@pytest.mark.parametrize("G,start,count,keep", [(8, 0, 1, 0.5), (2, 333, 70, 0.6), (1, 1000, 129, 0.3),
                                                (8, 4096, 16, 0.97), (4, 2048, 200, 0.995)])
@pytest.mark.parametrize("with_sinks", [True, False])
def test_replay_vs_oracle(G, start, count, keep, with_sinks):
    rng = np.random.default_rng(G * 1000 + start + count)
    H, k, v, q, vis = _case(rng, G, start, count, keep)
    sinks = rng.standard_normal(H).astype(np.float32) if with_sinks else None
    # queries are heads H..2H-1 of a wider buffer: strided token steps
    q_dev = t16(q)[:, H:2 * H]
    got, out = run(q_dev, k, v, start, 0.125, vis, sinks, out=True)
    want, want_out = oracle.replay_error(np.ascontiguousarray(q[:, H:2 * H]), k, v, start, 0.125, vis, sinks,
                                         want_out=True)
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=1e-6)
    dn = np.linalg.norm((out - want_out).reshape(count, -1), axis=1)
    nn = np.linalg.norm(want_out.reshape(count, -1), axis=1)
    assert (dn <= 1e-3 * nn + 1e-6).all(), (dn / nn).max()


def test_replay_all_visible_is_exactly_zero():
    rng = np.random.default_rng(5)
    H, k, v, q, vis = _case(rng, 8, 2500, 64, 1.0)
    vis[:] = True
    got, out = run(t16(np.ascontiguousarray(q[:, :H])), k, v, 2500, 0.125, vis, None, out=True)
    assert not got.any()
    got2, out2 = run(t16(np.ascontiguousarray(q[:, :H])), k, v, 2500, 0.125, None, None, out=True)
    assert not got2.any()
    np.testing.assert_array_equal(out, out2)


def test_replay_full_size_chunk_matches_oracle_sample():
    """Config-4 shape: a 2,048-query chunk after a 26,624-token resident
    prefix, 8 KV heads, a quarter of the prefix evicted per head; the oracle
    checks every 97th query (it is O(queries x keys x heads) in float64)."""
    rng = np.random.default_rng(11)
    G, start, count = 8, 26624, 2048
    H = 8 * G
    n = start + count
    k = torch.randn((n, G, 64), device=DEV).mul_(1.5).to(torch.bfloat16)
    v = torch.randn((n, G, 64), device=DEV).to(torch.bfloat16)
    q = torch.randn((count, H, 64), device=DEV).mul_(1.5).to(torch.bfloat16)
    vis = rng.random((G, n)) < 0.75
    vis[:, start:] = True
    err = K().error_word(DEV)
    e = K().replay_error(q, k, v, start, 0.125, visible_bits=bits_of(vis), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = e.cpu().numpy()
    assert np.isfinite(got).all() and (got > 0).all()
    kb = k.view(torch.int16).cpu().numpy().view(np.uint16)
    vb = v.view(torch.int16).cpu().numpy().view(np.uint16)
    qb = q.view(torch.int16).cpu().numpy().view(np.uint16)
    for i in range(0, count, 97):
        want = oracle.replay_error(qb[i:i + 1], kb, vb, start + i, 0.125, vis[:, :start + i + 1])
        np.testing.assert_allclose(got[i], want[0], rtol=1e-3)
