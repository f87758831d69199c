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
SAMPLED = ["IQ2_S", "IQ3_S", "IQ4_XS"]


@pytest.fixture(scope="module")
def cbmoe():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cbmoe as c
    c.lib()
    c.device_errors(clear=True)
    return c


@pytest.mark.parametrize("qt", SAMPLED)
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
        off = oiq.D_OFFSET[qt]
        blk[:3, off:off + 2] = np.frombuffer(np.array([0.0, -0.02, 6.0e-5], np.float16).tobytes(),
                                             np.uint8).reshape(3, 2)
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


# ---------------------------------------------------------------------------------- routed experts on IQ tables
@pytest.mark.parametrize("types", [("IQ2_S", "IQ2_S", "IQ3_S"), ("IQ4_XS", "IQ4_XS", "IQ4_XS"),
                                   ("IQ3_S", "IQ2_S", "IQ4_XS"), ("Q2_K", "Q2_K", "Q3_K")])
@pytest.mark.parametrize("N,k,E", [(1, 8, 16), (8, 8, 24), (37, 4, 8)])
def test_iq_experts_apply(cbmoe, types, N, k, E):
    """ResidentFetch.apply over raw GGUF IQ tables (per-matrix formats, as the reference's qtypes) against the
    oracle's fp64 composition of the same dequantized experts. Bar: max rel err 2e-3 (fp32 sums and SwiGLU)."""
    from oracle import gen, moe
    H, I = 512, 256
    rng = np.random.default_rng(N * 101 + E + len("".join(types)))
    qtypes = dict(zip(("gate_q", "up_q", "down_q"), types))
    shapes = {"gate_q": (I, H), "up_q": (I, H), "down_q": (H, I)}
    raw = {key: oiq.random_blocks(rng, E * rows * (K // 256), qtypes[key]) for key, (rows, K) in shapes.items()}
    dev = {key: torch.from_numpy(b.reshape(-1)).cuda() for key, b in raw.items()}
    p = cbmoe.iq.pack_layer(dev["gate_q"], dev["up_q"], dev["down_q"], qtypes, E, H, I)
    x = gen.activations(rng, N, H)
    idx, w = gen.routing(rng, N, E, k)
    fetch = cbmoe.ResidentFetch(qtypes={3: qtypes})
    y = fetch.apply(p, torch.from_numpy(x.view(np.uint16).copy()).cuda().view(torch.bfloat16),
                    torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda(), 3, gen.LIMIT)
    tabs = oiq.tables()
    W = {key: oiq.experts_dense(raw[key], qtypes[key], E, rows, K, tabs) for key, (rows, K) in shapes.items()}
    want = oiq.decode_apply(x.astype(np.float32), idx, w, W["gate_q"], W["up_q"], W["down_q"], gen.LIMIT)
    assert y.shape == (N, H)
    assert moe.max_rel_err(y.cpu().numpy(), want) < 2e-3
    assert cbmoe.device_errors(clear=True) == 0


@pytest.mark.parametrize("types", [("IQ2_S", "IQ2_S", "IQ3_S"), ("IQ3_S", "IQ2_S", "IQ2_S"),
                                   ("IQ2_S", "IQ4_XS", "IQ3_S")])
@pytest.mark.parametrize("N,k,E", [(1, 8, 16), (8, 8, 24), (37, 4, 8), (64, 8, 8)])
def test_iq_int8_layout_against_fp32_kernels(cbmoe, types, N, k, E):
    """The IQ2_S / IQ3_S matrices on the int8 tensor-core layout (exact transcode, X8 activations) against the same
    layer on the fp32 kernels and against the oracle; passes of 1-8 tokens (N = 64, E = 8: 64 slots per expert)."""
    from oracle import gen, moe
    H, I = 512, 256
    rng = np.random.default_rng(N * 7 + E + len("".join(types)))
    qtypes = dict(zip(("gate_q", "up_q", "down_q"), types))
    shapes = {"gate_q": (I, H), "up_q": (I, H), "down_q": (H, I)}
    raw = {key: oiq.random_blocks(rng, E * rows * (K // 256), qtypes[key]) for key, (rows, K) in shapes.items()}
    dev = {key: torch.from_numpy(b.reshape(-1)).cuda() for key, b in raw.items()}
    p8 = cbmoe.iq.pack_layer(dev["gate_q"], dev["up_q"], dev["down_q"], qtypes, E, H, I)
    p32 = cbmoe.iq.pack_layer(dev["gate_q"], dev["up_q"], dev["down_q"], qtypes, E, H, I, int8=False)
    for key in shapes:
        assert (p8["int8"][key] is not None) == (qtypes[key] in ("IQ2_S", "IQ3_S"))
    x = gen.activations(rng, N, H)
    idx, w = gen.routing(rng, N, E, k)
    xt = torch.from_numpy(x.view(np.uint16).copy()).cuda().view(torch.bfloat16)
    it, wt = torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda()
    y8 = cbmoe.iq.apply(p8, xt, it, wt, gen.LIMIT)
    y32 = cbmoe.iq.apply(p32, xt, it, wt, gen.LIMIT)
    tabs = oiq.tables()
    W = {key: oiq.experts_dense(raw[key], qtypes[key], E, rows, K, tabs) for key, (rows, K) in shapes.items()}
    want = oiq.decode_apply(x.astype(np.float32), idx, w, W["gate_q"], W["up_q"], W["down_q"], gen.LIMIT)
    assert moe.max_rel_err(y8.cpu().numpy(), want) < 2e-3
    assert moe.max_rel_err(y8.cpu().numpy(), y32.cpu().numpy()) < 2e-3
    assert cbmoe.device_errors(clear=True) == 0


def test_iq8_build_rejects_bad_arguments(cbmoe):
    L = cbmoe.lib()
    from cbmoe._lib import ptr, stream_handle
    assert L.cbmoe_iq8_bytes(23, 2, 64, 256) == 0                   # IQ4_XS: no int8 layout
    assert L.cbmoe_iq8_bytes(22, 2, 48, 256) == 0                   # rows not a multiple of 64
    n = L.cbmoe_iq8_bytes(22, 2, 64, 256)
    assert n > 0
    raw = torch.zeros(2 * 64 * 82, dtype=torch.uint8, device="cuda")
    out = torch.empty(n, dtype=torch.uint8, device="cuda")
    tab = cbmoe.iq.table("IQ2_S", raw.device)
    assert L.cbmoe_iq8_build(23, ptr(raw), ptr(tab), 2, 64, 256, ptr(out), stream_handle()) == -4
    assert L.cbmoe_iq8_build(22, ptr(raw), ptr(tab), 2, 48, 256, ptr(out), stream_handle()) == -1
    bad = tab.clone()
    bad[5] = 7.0                                                      # not a value the 3-bit code holds
    assert L.cbmoe_iq8_build(22, ptr(raw), ptr(bad), 2, 64, 256, ptr(out), stream_handle()) == -4
    assert L.cbmoe_iq8_build(22, ptr(raw), ptr(tab), 2, 64, 256, ptr(out), stream_handle()) == 0


def test_iq_qtypes_mismatch_raises(cbmoe):
    E, H, I = 2, 256, 256
    qtypes = {"gate_q": "IQ3_S", "up_q": "IQ3_S", "down_q": "IQ3_S"}
    rng = np.random.default_rng(3)
    t = {key: torch.from_numpy(oiq.random_blocks(rng, E * 256, "IQ3_S").reshape(-1)).cuda() for key in qtypes}
    p = cbmoe.iq.pack_layer(t["gate_q"], t["up_q"], t["down_q"], qtypes, E, H, I)
    x = torch.zeros((1, H), dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros((1, 2), dtype=torch.int32, device="cuda")
    w = torch.ones((1, 2), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        cbmoe.ResidentFetch(qtypes={0: {"gate_q": "IQ2_S"}}).apply(p, x, idx, w, 0, 10.0)
