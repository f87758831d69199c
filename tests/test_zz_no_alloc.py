"""cbmoe_experts_apply_noalloc against cbmoe_experts_apply and the CPU oracle, through the C ABI (needs a B200:
-m gpu).

The no-alloc entry point exists for callers that cannot allocate device memory for a workspace (an engine whose
allocator owns all device memory, a plugin host that forbids allocation during execute, host code that must not
block on cudaMalloc). It keeps its scratch in a fixed 48 MiB device array inside the library. This file is
collected last on purpose, so a run that stops at the first failure has run every other test before it; it also
passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import shared_to_gpu, t_bf16, table_to_gpu
from oracle import gen, moe

pytestmark = pytest.mark.gpu

TOL = 1e-2          # the layer bar every GPU test uses (max |got - want| / max |want|)


def _call_noalloc(cbmoe, p, x, idx, w, limit):
    from cbmoe._lib import lib, ptr, stream_handle
    from cbmoe.resident import _experts_struct
    N, k = idx.shape
    ex = _experts_struct(p)
    y = torch.empty((N, p["H"]), dtype=torch.float32, device="cuda")
    rc = lib().cbmoe_experts_apply_noalloc(ctypes.byref(ex), ptr(x), N, ptr(idx), ptr(w), k, float(limit), ptr(y),
                                           stream_handle())
    return rc, y


def test_noalloc_matches_workspace_entry_point_twice():
    assert torch.cuda.is_available()
    import cbmoe
    E, H, I, k = 16, 512, 256, 4
    rng = np.random.default_rng(77)
    L = gen.moe_layer(rng, E, H, I)
    p = cbmoe.pack_layer(table_to_gpu(L["gate"]), table_to_gpu(L["up"]), table_to_gpu(L["down"]),
                         shared_to_gpu(L["shared"]))
    fetch = cbmoe.ResidentFetch(path="decode")
    for N in (8, 3):                                   # two calls in a row; the second reuses the array's leftovers
        x_np = gen.activations(rng, N, H)
        x = t_bf16(x_np)
        idx_np, w_np = gen.routing(rng, N, E, k)
        idx, w = torch.from_numpy(idx_np).cuda(), torch.from_numpy(w_np).cuda()
        want = fetch.apply(p, x, idx, w, 0, gen.LIMIT)
        rc, got = _call_noalloc(cbmoe, p, x, idx, w, gen.LIMIT)
        assert rc == 0, cbmoe.lib().cbmoe_status_string(rc)
        torch.cuda.synchronize()
        assert moe.max_rel_err(got.cpu().numpy(), want.cpu().numpy()) < TOL
        # and against the CPU oracle directly, on the same bf16 activations
        ref = moe.decode_apply(x_np.astype(np.float32), idx_np, w_np, L["gate"], L["up"], L["down"], gen.LIMIT)
        assert moe.max_rel_err(got.cpu().numpy(), ref) < TOL
    assert cbmoe.device_errors(clear=True) == 0


def test_noalloc_rejects_requests_beyond_the_array():
    import cbmoe
    E, H, I = 160, 5120, 1536
    p = {"E": E, "H": H, "I": I, "gate_up_q": (torch.empty(16, dtype=torch.uint8, device="cuda"),) * 2,
         "down_q": (torch.empty(16, dtype=torch.uint8, device="cuda"),) * 2}
    N, k = 512, 8                                      # needs ~120 MB of scratch: more than the 48 MiB array
    x = torch.zeros((N, H), dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros((N, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((N, k), dtype=torch.float32, device="cuda")
    rc, _ = _call_noalloc(cbmoe, p, x, idx, w, gen.LIMIT)
    assert rc == -3                                    # CBMOE_ERR_WORKSPACE, returned before any launch
