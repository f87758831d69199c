"""The router oracle (oracle/route.py) against the reference's own moe_route (model.py:798-808), executed on its
inputs by tests/golden/make_route_golden.py: same expert order (ties included) and the same fp32 weights."""
import os

import ml_dtypes
import numpy as np
import pytest

from oracle import route

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "route.npz")


@pytest.mark.parametrize("norm", [1, 0])
@pytest.mark.parametrize("case", ["", "_tie"])
def test_route_matches_reference(norm, case):
    f = np.load(GOLDEN)
    x = f["x"].view(ml_dtypes.bfloat16).astype(np.float32)
    W = f["W"].view(ml_dtypes.bfloat16).astype(np.float32)
    idx, w = route.moe_route(x, W, f["b" + case], int(f["k"]), bool(norm), float(f["scaling"]))
    assert np.array_equal(idx, f[f"idx{case}_{norm}"])
    np.testing.assert_allclose(w, f[f"w{case}_{norm}"], rtol=1e-6, atol=0)


def test_tie_order_is_lower_index_first():
    f = np.load(GOLDEN)
    assert list(f["idx_tie_1"][3][:3]) == [7, 9, 40]   # x row 3 is zero: equal choices 0.5 + 5.0
