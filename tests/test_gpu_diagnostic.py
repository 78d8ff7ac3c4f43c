"""The regret diagnostic (runtime:549-613) on the GPU kernels against the
reference's own outputs: per-token head_sum / head_max tables, each spec's
resident mask after its boundary, and the per-query lost mass (the
reference test's tolerance, test_sglang_evict.py:218-220)."""
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from golden import scenarios as sc

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
DEV = "cuda:0"


@pytest.fixture(autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")


def t16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(DEV).view(torch.bfloat16)


def test_diagnostic_matches_reference():
    from cache_eviction_b200 import kernels
    from cache_eviction_b200 import runtime as ge
    z = np.load(GOLD / "diagnostic.npz")
    d = sc.diagnostic_setup()
    keys, q = t16(d["keys"]), t16(d["q"])
    sinks = torch.from_numpy(d["sinks"]).to(DEV)
    st = SimpleNamespace(first_full=1, full_layers=[1], page_size=1, err=kernels.error_word(DEV))
    layer = SimpleNamespace(layer_id=1, tp_q_head_num=sc.DIAG_H, tp_k_head_num=sc.DIAG_G, scaling=d["scale"])
    req = SimpleNamespace(rid="r", session=None, origin_input_ids=[0] * sc.DIAG_LEN)
    e = ge._diagnostic_entry(req, {"seed": d["seed"], "policies": d["policies"]}, DEV, 1, sc.DIAG_G)
    assert e["specs"] == [tuple(s) for s in sc.DIAG_SPECS]
    for lo, hi in sc.DIAG_CHUNKS:
        ge._diagnose(st, e, 0, layer, q[lo:hi], keys, sinks, torch.arange(1, hi + 1, device=DEV), lo)
    torch.cuda.synchronize()
    assert int(st.err.item()) == 0
    np.testing.assert_allclose(e["score_sum"].cpu().numpy(), z["score_sum"], rtol=1e-3, atol=1e-5)
    np.testing.assert_allclose(e["score_max"].cpu().numpy(), z["score_max"], rtol=1e-3, atol=1e-5)
    # each spec's resident positions after its boundary, from its kept positions
    end = z["resident"].shape[-1]
    resident = np.stack([np.stack([ge._diagnostic_resident(e, j, 0, end).cpu().numpy()])
                         for j in range(len(e["specs"]))])
    np.testing.assert_array_equal(resident, z["resident"])
    assert float(z["lost"].sum()) > 0
    np.testing.assert_allclose(e["lost"].cpu().numpy(), z["lost"], rtol=1e-3, atol=1e-5)
    assert e["layers_seen"] == {1}
