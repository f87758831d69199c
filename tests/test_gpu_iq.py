"""IQ-format dequant on the GPU (cbmoe_iq_dequant through cbmoe.iq.dequant_rows) against the reference: the three
real GLM-5.3-Flash tensor slices of the reference's tests with the reference's own fp32 output
(tests/golden/iq_samples.npz), and random blocks against the oracle (oracle/iq.py, itself pinned to the reference
and gguf-py in test_iq_oracle.py). Bar: bit-exact fp32. Needs a B200 (-m gpu)."""
import os

import numpy as np
import pytest
import torch

from oracle import iq as oiq

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "iq_samples.npz")
QTYPES = list(oiq.BLOCK_BYTES)


@pytest.fixture(scope="module")
def cbmoe():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cbmoe as c
    c.lib()
    c.device_errors(clear=True)
    return c


@pytest.mark.parametrize("qt", QTYPES)
def test_reference_samples_bit_exact(cbmoe, qt):
    f = np.load(GOLDEN)
    raw = torch.from_numpy(f[f"{qt}_raw"].copy()).cuda()
    got = cbmoe.iq.dequant_rows(raw, qt, int(f[f"{qt}_ne0"])).cpu().numpy()
    want = f[f"{qt}_ref"]
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert cbmoe.device_errors(clear=True) == 0


@pytest.mark.parametrize("qt", QTYPES)
@pytest.mark.parametrize("n_blocks", [1, 7, 8, 1000, 20011])
def test_random_blocks_bit_exact(cbmoe, qt, n_blocks):
    rng = np.random.default_rng(n_blocks * 3 + len(qt))
    blk = oiq.random_blocks(rng, n_blocks, qt)
    if n_blocks >= 8:   # zero, negative and subnormal block scales
        blk[:3, 0:2] = np.frombuffer(np.array([0.0, -0.02, 6.0e-5], np.float16).tobytes(), np.uint8).reshape(3, 2)
    want = oiq.DEQUANT[qt](blk, oiq.tables()[qt])
    got = cbmoe.iq.dequant_rows(torch.from_numpy(blk.reshape(-1)).cuda(), qt, 256).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert cbmoe.device_errors(clear=True) == 0


def test_rejects_bad_arguments(cbmoe):
    L = cbmoe.lib()
    assert L.cbmoe_iq_block_bytes(12) == 0                        # Q4_K: not an IQ type here
    out = torch.empty(256, dtype=torch.float32, device="cuda")
    raw = torch.zeros(82, dtype=torch.uint8, device="cuda")
    tab = cbmoe.iq.table("IQ2_S", raw.device)
    from cbmoe._lib import ptr, stream_handle
    assert L.cbmoe_iq_dequant(12, ptr(raw), 1, ptr(tab), ptr(out), stream_handle()) != 0
    assert L.cbmoe_iq_dequant(22, ptr(raw), -1, ptr(tab), ptr(out), stream_handle()) != 0
    assert L.cbmoe_iq_dequant(22, ptr(raw), 0, None, None, stream_handle()) == 0   # nothing to do
