"""The C-ABI library loads without a GPU and exports every function include/*.h declares; host-side argument
checks reject bad calls before touching the device. No GPU: nothing here launches a kernel."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DECL = re.compile(r"^\s*(?:const\s+)?(?:long\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(cbmoe_[A-Za-z0-9_]+)\s*\(", re.M)


def declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        names |= set(DECL.findall(open(h).read()))
    return sorted(names)


@pytest.fixture(scope="module")
def L():
    import cbmoe
    return cbmoe.lib()


def test_header_declares_the_layer_api():
    names = declared()
    for n in ("cbmoe_experts_apply", "cbmoe_moe_layer", "cbmoe_route_plan", "cbmoe_cb3k_repack", "cbmoe_w8k_repack",
              "cbmoe_cb3_matvec", "cbmoe_w8_linear"):
        assert n in names


def test_every_declared_symbol_is_exported(L):
    missing = [n for n in declared() if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_every_symbol():
    from cbmoe._lib import SIGNATURES
    assert sorted(SIGNATURES) == declared()


def test_host_side_checks_without_gpu(L):
    from cbmoe._lib import Experts
    assert L.cbmoe_version() >= 1
    assert L.cbmoe_status_string(-1) == b"invalid argument"
    # bad shapes never reach a kernel
    assert L.cbmoe_cb3k_idx_bytes(160, 1536, 5120, 2) == 160 * 1536 * 5120 * 2 * 3 // 8
    assert L.cbmoe_cb3k_cb_bytes(160, 1536, 2) == 160 * 1536 * 2 * 16
    assert L.cbmoe_w8k_bytes(1536, 5120, 2) == 1536 * 5120 * 2
    assert L.cbmoe_cb3k_repack(None, None, None, None, 1, 1, 100, 256, None, None, None) == -1   # rows % 64
    assert L.cbmoe_cb3k_repack(None, None, None, None, 1, 1, 64, 100, None, None, None) == -1    # K % 256
    ex = Experts(0, 5120, 1536, None, None, None, None)
    assert L.cbmoe_experts_apply(ctypes.byref(ex), None, 8, None, None, 8, 10.0, 0, None, None, 0, None) == -1
    ex = Experts(160, 5120, 1536, 16, 16, 16, 16)
    assert L.cbmoe_experts_apply(ctypes.byref(ex), None, 8, None, None, 8, 10.0, 0, None, None, 0, None) == -1
    assert L.cbmoe_experts_apply(ctypes.byref(ex), 16, 8, 16, 16, 8, 10.0, 0, 16, None, 0, None) == -3   # workspace


def test_plan_layout_sizes(L):
    off = (ctypes.c_int64 * 14)()
    assert L.cbmoe_plan_layout(4096, 8, 160, 128, 32, off) == 0
    S, E, tm = 4096 * 8, 160, 128
    G = -(-S // tm) + E
    assert off[7] - off[6] >= G and off[8] - off[7] >= G * tm and off[10] - off[9] >= S
    assert L.cbmoe_plan_layout(8, 8, 2048, 1, 8, off) == -1      # more experts than the plan kernel supports


def test_iq_and_route_host_side(L):
    """The IQ-format and router entry points answer shape queries and reject bad calls without a GPU."""
    from cbmoe._lib import IqExperts
    assert (L.cbmoe_iq_block_bytes(22), L.cbmoe_iq_block_bytes(21), L.cbmoe_iq_block_bytes(23)) == (82, 110, 136)
    assert L.cbmoe_iq_block_bytes(12) == 0                                    # Q4_K: not an IQ type here
    e, w = ctypes.c_int(), ctypes.c_int()
    for t, shape in ((22, (1024, 8)), (21, (512, 4)), (23, (16, 1))):
        assert L.cbmoe_iq_table_shape(t, ctypes.byref(e), ctypes.byref(w)) == 0 and (e.value, w.value) == shape
    assert L.cbmoe_iq_table_shape(12, ctypes.byref(e), ctypes.byref(w)) == -4   # unsupported
    assert L.cbmoe_iq_dequant(12, None, 1, None, None, None) == -4
    assert L.cbmoe_iq_dequant(22, None, -1, None, None, None) == -1
    assert L.cbmoe_iq_dequant(22, None, 0, None, None, None) == 0             # nothing to do
    ex = IqExperts(160, 5120, 1536, 22, 22, 21, 16, 16, 16, 16, 16, 16)
    assert L.cbmoe_iq_workspace_bytes(ctypes.byref(ex), 8, 8) > 0
    bad = IqExperts(160, 5000, 1536, 22, 22, 21, 16, 16, 16, 16, 16, 16)      # H not a multiple of 256
    assert L.cbmoe_iq_workspace_bytes(ctypes.byref(bad), 8, 8) == 0
    assert L.cbmoe_iq_experts_apply(ctypes.byref(bad), 16, 8, 16, 16, 8, 10.0, 16, None, 0, None) == -1
    assert L.cbmoe_iq_experts_apply(ctypes.byref(ex), 16, 8, 16, 16, 8, 10.0, 16, None, 0, None) == -3   # workspace
    assert L.cbmoe_route(None, 1, 64, None, None, 300, 8, 1, 1.0, None, None, None) == -1   # E > 256
    assert L.cbmoe_route(None, 1, 64, None, None, 16, 17, 1, 1.0, None, None, None) == -1   # k > E
    assert L.cbmoe_route(None, 0, 64, None, None, 16, 8, 1, 1.0, None, None, None) == 0     # nothing to do


def test_workspace_queries_without_gpu(L):
    """Workspace sizes of every path are host arithmetic: positive, growing with the batch, and the tcgen05 decode
    path (which adds the gathered token rows) larger than the mma.sync one at the same shape."""
    from cbmoe._lib import Experts
    ex = Experts(160, 5120, 1536, 16, 16, 16, 16)
    dec = [L.cbmoe_workspace_bytes(ctypes.byref(ex), n, 8, 1) for n in (1, 8, 64)]
    assert all(v > 0 for v in dec) and dec[0] <= dec[1] <= dec[2]
    assert L.cbmoe_workspace_bytes(ctypes.byref(ex), 8, 8, 3) == 0                 # not a path
    ex8 = Experts(160, 5120, 1536, 16, 16, 16, 16, 16, 16)                          # with CB8 tables
    assert L.cbmoe_workspace_bytes(ctypes.byref(ex8), 8, 8, 1) > 0
    assert L.cbmoe_cb8_matvec_workspace_bytes(1, 2048) >= 2048 * 2 + 4
    assert L.cbmoe_cb8_matvec_workspace_bytes(1, 100) == 0                          # K % 256 != 0
    assert L.cbmoe_cb8_bytes(160, 1536, 2) == 160 * 1536 * 2 * 20
    assert L.cbmoe_workspace_bytes(ctypes.byref(ex), 4096, 8, 2) > dec[2]          # grouped, config 3
    assert L.cbmoe_ep_workspace_bytes(ctypes.byref(Experts(20, 5120, 1536, 16, 16, 16, 16)), 32, 8, 8, 64, 0) > 0
