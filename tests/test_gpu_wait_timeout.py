"""Bounded waits (needs a B200: -m gpu). A kernel waits on a barrier phase that nothing completes; the wait must
give up after its limit, report CBMOE_DEVERR_TIMEOUT through cbmoe_device_errors, and leave the context usable
(a matvec right after still matches the oracle). No fault, trap or hang is involved: the waiting CTA returns on
its own."""
import time

import numpy as np
import pytest
import torch

from helpers import t_bf16, t_u32
from oracle import cb3, gen, moe

pytestmark = pytest.mark.gpu
DEVERR_TIMEOUT = 1


@pytest.fixture(scope="module")
def cbmoe():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cbmoe as m
    m.lib()
    m.device_errors(clear=True)
    return m


def test_wait_gives_up_and_context_survives(cbmoe):
    from cbmoe._lib import check, lib, stream_handle
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    check(lib().cbmoe_selftest_wait_timeout(100_000_000, flag.data_ptr(), stream_handle()),
          "cbmoe_selftest_wait_timeout")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(flag.item()) == 1                       # the wait gave up
    assert 0.09 < elapsed < 5.0, elapsed               # after about its limit, not never
    assert cbmoe.device_errors(clear=True) & DEVERR_TIMEOUT
    assert cbmoe.device_errors(clear=True) == 0        # cleared

    c = gen.config0(seed=5)                            # the context still runs kernels correctly
    x = gen.activations(np.random.default_rng(5), 3, 2048)
    idx_k, cb_k = cbmoe.ops.pack_cb3(t_u32(c["idx"][None]), t_bf16(c["cb"][None]))
    y = cbmoe.ops.cb3_matvec(idx_k, cb_k, 1024, 2048, t_bf16(x)).cpu().numpy()
    want = cb3.matvec(c["idx"], c["cb"], x.astype(np.float32))
    assert moe.max_rel_err(y, want) < 1e-3
    assert cbmoe.device_errors(clear=True) == 0


def test_wait_limit_is_validated(cbmoe):
    from cbmoe._lib import lib, stream_handle
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib().cbmoe_selftest_wait_timeout(0, flag.data_ptr(), stream_handle()) == -1
    assert lib().cbmoe_selftest_wait_timeout(100, None, stream_handle()) == -1
