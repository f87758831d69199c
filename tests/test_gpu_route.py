"""Fused router (cbmoe_route through cbmoe.moe_route) against the reference's moe_route (model.py:798-808): its own
outputs on the fixture inputs (tests/golden/route.npz) and the oracle (oracle/route.py) on config-sized inputs.
The kernel's fp32 sums run in another order than the reference's dot, so an expert may change place only with
another whose choice value is within 1e-5; the weights agree to 1e-5 relative. Needs a B200 (-m gpu)."""
import os

import ml_dtypes
import numpy as np
import pytest
import torch

from oracle import route

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "route.npz")


@pytest.fixture(scope="module")
def cbmoe():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cbmoe as c
    c.lib()
    return c


def _check(x, W, b, idx, w, want_idx, want_w):
    choice = route.choice_values(x, W, b)
    for n in range(idx.shape[0]):
        for j in range(idx.shape[1]):
            if idx[n, j] != want_idx[n, j]:
                assert abs(choice[n, idx[n, j]] - choice[n, want_idx[n, j]]) < 1e-5, (n, j, idx[n], want_idx[n])
            else:
                np.testing.assert_allclose(w[n, j], want_w[n, j], rtol=1e-5, atol=1e-7)


def _run(cbmoe, x_bf16, W_bf16, b, k, norm, scaling):
    xt = torch.from_numpy(x_bf16.view(np.uint16).copy()).cuda().view(torch.bfloat16)
    Wt = torch.from_numpy(W_bf16.view(np.uint16).copy()).cuda().view(torch.bfloat16)
    idx, w = cbmoe.moe_route(xt, Wt, torch.from_numpy(b).cuda(), k, norm, scaling)
    return idx.cpu().numpy(), w.cpu().numpy()


@pytest.mark.parametrize("norm", [1, 0])
@pytest.mark.parametrize("case", ["", "_tie"])
def test_route_reference_fixture(cbmoe, norm, case):
    f = np.load(GOLDEN)
    x, W = f["x"].view(ml_dtypes.bfloat16), f["W"].view(ml_dtypes.bfloat16)
    b = f["b" + case]
    idx, w = _run(cbmoe, x, W, b, int(f["k"]), bool(norm), float(f["scaling"]))
    _check(x.astype(np.float32), W.astype(np.float32), b, idx, w, f[f"idx{case}_{norm}"], f[f"w{case}_{norm}"])
    assert list(idx[3][:3]) == list(f[f"idx{case}_{norm}"][3][:3])     # exact ties: the lower index first


@pytest.mark.parametrize("N", [1, 8, 37, 300])
@pytest.mark.parametrize("norm", [True, False])
def test_route_config_sizes(cbmoe, N, norm):
    rng = np.random.default_rng(N + 2 * norm)
    D, E, k = 5120, 160, 8
    x = rng.standard_normal((N, D)).astype(ml_dtypes.bfloat16)
    W = (rng.standard_normal((D, E)) * 0.02).astype(ml_dtypes.bfloat16)
    b = (rng.standard_normal(E) * 0.05).astype(np.float32)
    idx, w = _run(cbmoe, x, W, b, k, norm, 2.5)
    want_idx, want_w = route.moe_route(x.astype(np.float32), W.astype(np.float32), b, k, norm, 2.5)
    _check(x.astype(np.float32), W.astype(np.float32), b, idx, w, want_idx, want_w)
    assert (idx >= 0).all() and (idx < E).all()
    assert all(len(set(r)) == k for r in idx.tolist())


def test_route_rejects_bad_arguments(cbmoe):
    from cbmoe._lib import stream_handle
    L = cbmoe.lib()
    assert L.cbmoe_route(None, 1, 64, None, None, 300, 8, 1, 1.0, None, None, stream_handle()) != 0   # E > 256
    assert L.cbmoe_route(None, 1, 64, None, None, 16, 17, 1, 1.0, None, None, stream_handle()) != 0   # k > E
    assert L.cbmoe_route(None, 0, 64, None, None, 16, 8, 1, 1.0, None, None, stream_handle()) == 0    # nothing to do
