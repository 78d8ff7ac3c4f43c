"""ce_decode_attn_score_static: decode for callers that cannot allocate.

Some callers cannot call cudaMalloc when they run a decode step -- an engine
that gave all of HBM to its KV pool at start-up, a host that forbids device
allocations after initialisation, a global-mode CUDA graph capture -- so they
cannot hand the fused decode kernel a workspace either.  The static entry point
uses a fixed scratch array inside libce_b200.so instead.  This test calls it
through the C ABI twice in a row (the second call reuses the array the first
one left behind) and checks both results against the workspace entry point on
the same inputs, and that a batch too large for the array is refused.

The file name makes pytest collect it last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _case(dev):
    rng = np.random.default_rng(42)
    G, H, D, P = 8, 64, 64, 16
    lengths = [1, 16, 17, 300, 1025, 4000, 77]
    modes = [1, 2, 0, 1, 2, 1, 0]
    pages = [-(-n // P) for n in lengths]
    units = sum(pages) + 5
    kp = torch.randn((units, G, P, D), device=dev).to(torch.bfloat16)
    vp = torch.randn((units, G, P, D), device=dev).to(torch.bfloat16)
    q = torch.randn((len(lengths), H, D), device=dev).to(torch.bfloat16)
    sinks = torch.randn(H, device=dev)
    indices = torch.from_numpy((rng.permutation(units - 1) + 1)[:sum(pages)].astype(np.int32)).to(dev)
    indptr = torch.from_numpy(np.concatenate([[0], np.cumsum(pages)]).astype(np.int32)).to(dev)
    tokens = torch.tensor(lengths, dtype=torch.int32, device=dev)
    mode = torch.tensor(modes, dtype=torch.int32, device=dev)
    scores0 = torch.rand((G, units), device=dev)
    return dict(kp=kp, vp=vp, q=q, sinks=sinks, indices=indices, indptr=indptr, tokens=tokens,
                mode=mode, scores0=scores0, H=H, G=G, P=P, units=units)


def _static_call(lib, c, scores, out, lse, err, indices=None, capacity=None):
    q = c["q"]
    idx = c["indices"] if indices is None else indices
    cap = idx.numel() if capacity is None else capacity
    return lib.ce_decode_attn_score_static(
        _ptr(q), q.stride(0), q.stride(1), _ptr(c["kp"]), _ptr(c["vp"]), c["units"],
        _ptr(c["indptr"]), _ptr(idx), _ptr(c["tokens"]), cap, _ptr(c["sinks"]), _ptr(c["mode"]),
        None, 0.125, q.shape[0], c["H"], c["G"], 64, c["P"], _ptr(scores), scores.stride(0), 1,
        _ptr(out), 1, out.stride(0), out.stride(1), _ptr(lse), 3, _ptr(err),
        C.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_static_scratch_matches_workspace_entry_on_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi, kernels
    lib = capi.load()
    dev = torch.device("cuda:0")
    c = _case(dev)
    bs = c["q"].shape[0]

    # the existing entry point, with a caller workspace
    s_ref = c["scores0"].clone()
    lse_ref = torch.zeros((bs, c["H"]), device=dev)
    err_ref = torch.zeros(1, dtype=torch.int32, device=dev)
    o_ref = kernels.decode_attn_score(c["q"], c["kp"], c["vp"], c["indptr"], c["indices"], c["tokens"],
                                      0.125, c["P"], sinks=c["sinks"], mode_of_row=c["mode"],
                                      scores=s_ref, zero_new=True, out_f32=True, lse=lse_ref,
                                      err=err_ref)
    torch.cuda.synchronize()
    assert int(err_ref.item()) == 0

    for _ in range(2):  # the second call starts from the first call's leftovers
        s = c["scores0"].clone()
        out = torch.full((bs, c["H"], 64), float("nan"), device=dev)
        lse = torch.zeros((bs, c["H"]), device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        assert _static_call(lib, c, s, out, lse, err) == capi.CE_OK
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        for i in range(bs):
            rel = float((out[i] - o_ref[i]).norm() / o_ref[i].norm())
            assert rel < 1e-3, (i, rel)
        torch.testing.assert_close(s, s_ref, rtol=1e-3, atol=1e-6)
        torch.testing.assert_close(lse, lse_ref, rtol=1e-5, atol=1e-5)


def test_static_scratch_refuses_batches_beyond_its_maximum():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi
    lib = capi.load()
    dev = torch.device("cuda:0")
    c = _case(dev)
    # a real index buffer of 600K entries: its score side data alone (256 B each)
    # exceeds the static array, so the call is refused before any launch
    big = torch.zeros(600_000, dtype=torch.int32, device=dev)
    big[:c["indices"].numel()] = c["indices"]
    need = lib.ce_decode_workspace_bytes(c["q"].shape[0], big.numel(), c["H"], c["G"], c["P"], 3)
    assert need > capi.CE_DECODE_STATIC_SCRATCH_BYTES
    s = c["scores0"].clone()
    out = torch.zeros((c["q"].shape[0], c["H"], 64), device=dev)
    lse = torch.zeros((c["q"].shape[0], c["H"]), device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    st = _static_call(lib, c, s, out, lse, err, indices=big)
    assert st == capi.CE_ERR_WORKSPACE
    assert "static maximum" in lib.ce_last_error().decode()
    torch.cuda.synchronize()
    assert torch.equal(s, c["scores0"])
