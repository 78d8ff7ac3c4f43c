"""Failure detection on the GPU without a fault: the bounded device waits that
every pipelined kernel uses (mbarrier phases fed by TMA and the tensor cores)
give up after their limit, flag CE_EW_TIMEOUT and return, and a warp waiting
on the same phase leaves through the CTA's abort flag.  The failure is an
mbarrier nothing arrives on; the context stays usable afterwards."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi
    capi.load()


def _run(complete, limit_ns):
    from cache_eviction_b200 import capi, kernels
    lib = capi.load()
    err = kernels.error_word(DEV)
    status = torch.full((3,), -1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    st = lib.ce_selftest_wait(complete, limit_ns, kernels._p(err), kernels._p(status),
                              kernels._stream(torch.device(DEV)))
    capi.check(st, "ce_selftest_wait")
    torch.cuda.synchronize()
    return int(err.item()), status.tolist(), time.perf_counter() - t0


def test_wait_that_never_completes_gives_up_and_flags_timeout():
    from cache_eviction_b200 import capi
    err, status, dt = _run(0, 20_000_000)          # 20 ms
    assert err & capi.CE_EW_TIMEOUT
    assert status == [1, 1, 1]
    assert 0.02 <= dt < 1.5                         # gave up at its limit, not the 2 s default
    # the context is still usable: a completed wait right after
    err, status, _ = _run(1, 20_000_000)
    assert err == 0 and status == [0, 0, 1]


def test_selftest_rejects_unbounded_limits():
    from cache_eviction_b200 import capi, kernels
    lib = capi.load()
    status = torch.zeros(3, dtype=torch.int32, device=DEV)
    for bad in (0, 500, 3_000_000_000):
        assert lib.ce_selftest_wait(0, bad, None, kernels._p(status), None) == capi.CE_ERR_ARG
