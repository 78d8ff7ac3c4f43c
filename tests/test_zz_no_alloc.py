"""ce_decode_attn_score_static: decode for callers that cannot allocate.

Some callers cannot call cudaMalloc when they run a decode step -- an engine
that gave all of HBM to its KV pool at start-up, a host that forbids device
allocations after initialisation, a global-mode CUDA graph capture -- so they
cannot hand the fused decode kernel a workspace either.  The static entry point
uses a fixed scratch array inside libce_b200.so instead.

These tests call it through the C ABI: a set-up call (bs == 0), then a call on
a different batch that leaves other values in every region of the array, then
two calls in a row on the compared batch, each checked against the workspace
entry point on the same inputs -- at 16-token pages with fp32 output and at
page size 1 (8 KV heads) with bf16 output.  Device free memory must not change
after the set-up call.  A batch too large for the array is refused.

The file name makes pytest collect it last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
G, H, D = 8, 64, 64


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _case(dev, page, lengths, modes, seed):
    gen = torch.Generator(device=dev).manual_seed(seed)
    rng = np.random.default_rng(seed)
    pages = [-(-n // page) for n in lengths]
    units = sum(pages) + 5
    kp = torch.randn((units, G, page, D), generator=gen, device=dev).to(torch.bfloat16)
    vp = torch.randn((units, G, page, D), generator=gen, device=dev).to(torch.bfloat16)
    q = torch.randn((len(lengths), H, D), generator=gen, device=dev).to(torch.bfloat16)
    sinks = torch.randn(H, generator=gen, device=dev)
    indices = torch.from_numpy((rng.permutation(units - 1) + 1)[:sum(pages)].astype(np.int32)).to(dev)
    indptr = torch.from_numpy(np.concatenate([[0], np.cumsum(pages)]).astype(np.int32)).to(dev)
    tokens = torch.tensor(lengths, dtype=torch.int32, device=dev)
    mode = torch.tensor(modes, dtype=torch.int32, device=dev)
    scores0 = torch.rand((G, units), generator=gen, device=dev)
    return dict(kp=kp, vp=vp, q=q, sinks=sinks, indices=indices, indptr=indptr, tokens=tokens,
                mode=mode, scores0=scores0, P=page, units=units)


def _static_call(lib, c, scores, out, lse, err, indices=None, bs=None):
    q = c["q"]
    idx = c["indices"] if indices is None else indices
    return lib.ce_decode_attn_score_static(
        _ptr(q), q.stride(0), q.stride(1), _ptr(c["kp"]), _ptr(c["vp"]), c["units"],
        _ptr(c["indptr"]), _ptr(idx), _ptr(c["tokens"]), idx.numel(), _ptr(c["sinks"]), _ptr(c["mode"]),
        None, 0.125, q.shape[0] if bs is None else bs, H, G, D, c["P"], _ptr(scores), scores.stride(0), 1,
        _ptr(out), 1 if out.dtype == torch.float32 else 0, out.stride(0), out.stride(1), _ptr(lse), 3,
        _ptr(err), C.c_void_p(torch.cuda.current_stream().cuda_stream))


CASES = {
    # page, output dtype, compared batch (lengths, modes), the other batch run first
    "page16_f32": (16, torch.float32, ([1, 16, 17, 300, 1025, 4000, 77], [1, 2, 0, 1, 2, 1, 0]),
                   ([5000, 33, 2048, 9], [2, 1, 1, 2])),
    "page1_bf16": (1, torch.bfloat16, ([1, 2, 300, 1025, 3000, 77], [1, 2, 1, 0, 2, 1]),
                   ([4100, 64, 700], [2, 2, 1])),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_static_scratch_matches_workspace_entry_on_two_calls(name):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi, kernels
    lib = capi.load()
    dev = torch.device("cuda:0")
    page, odt, (lengths, modes), (o_lengths, o_modes) = CASES[name]
    c = _case(dev, page, lengths, modes, seed=42 + page)
    other = _case(dev, page, o_lengths, o_modes, seed=7 + page)
    bs = c["q"].shape[0]

    # the existing entry point, with a caller workspace
    s_ref = c["scores0"].clone()
    lse_ref = torch.zeros((bs, H), device=dev)
    err_ref = torch.zeros(1, dtype=torch.int32, device=dev)
    o_ref = kernels.decode_attn_score(c["q"], c["kp"], c["vp"], c["indptr"], c["indices"], c["tokens"],
                                      0.125, page, sinks=c["sinks"], mode_of_row=c["mode"],
                                      scores=s_ref, zero_new=True, out_f32=odt == torch.float32,
                                      lse=lse_ref, err=err_ref)
    torch.cuda.synchronize()
    assert int(err_ref.item()) == 0

    # every buffer of the static calls exists before the set-up call
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    s_other = other["scores0"].clone()
    o_other = torch.empty((other["q"].shape[0], H, D), dtype=odt, device=dev)
    lse_other = torch.zeros((other["q"].shape[0], H), device=dev)
    runs = [(c["scores0"].clone(), torch.full((bs, H, D), float("nan"), dtype=odt, device=dev),
             torch.zeros((bs, H), device=dev)) for _ in range(2)]
    torch.cuda.synchronize()

    assert _static_call(lib, c, runs[0][0], runs[0][1], runs[0][2], err, bs=0) == capi.CE_OK  # set-up only
    torch.cuda.synchronize()
    free_after_setup = torch.cuda.mem_get_info(dev)[0]
    # another batch first: other lengths, modes and size leave other values in
    # the prefix, normaliser, record and per-page regions of the array
    assert _static_call(lib, other, s_other, o_other, lse_other, err) == capi.CE_OK
    for s, out, lse in runs:   # the compared batch twice in a row
        assert _static_call(lib, c, s, out, lse, err) == capi.CE_OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free_after_setup   # no device memory taken
    assert int(err.item()) == 0
    tol = 1e-3 if odt == torch.float32 else 5e-3
    for s, out, lse in runs:
        for i in range(bs):
            rel = float((out[i].float() - o_ref[i].float()).norm() / o_ref[i].float().norm())
            assert rel < tol, (i, rel)
        torch.testing.assert_close(s, s_ref, rtol=1e-3, atol=1e-6)
        torch.testing.assert_close(lse, lse_ref, rtol=1e-5, atol=1e-5)


def test_static_scratch_refuses_batches_beyond_its_maximum():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi
    lib = capi.load()
    dev = torch.device("cuda:0")
    c = _case(dev, 16, [1, 16, 17, 300, 1025, 4000, 77], [1, 2, 0, 1, 2, 1, 0], seed=42)
    # a real index buffer of 600K entries: its score side data alone (256 B each)
    # exceeds the static array, so the call is refused before any launch
    big = torch.zeros(600_000, dtype=torch.int32, device=dev)
    big[:c["indices"].numel()] = c["indices"]
    need = lib.ce_decode_workspace_bytes(c["q"].shape[0], big.numel(), H, G, 16, 3)
    assert need > capi.CE_DECODE_STATIC_SCRATCH_BYTES
    s = c["scores0"].clone()
    out = torch.zeros((c["q"].shape[0], H, D), device=dev)
    lse = torch.zeros((c["q"].shape[0], H), device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    st = _static_call(lib, c, s, out, lse, err, indices=big)
    assert st == capi.CE_ERR_WORKSPACE
    assert "static maximum" in lib.ce_last_error().decode()
    torch.cuda.synchronize()
    assert torch.equal(s, c["scores0"])
