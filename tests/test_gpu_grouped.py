"""Parity of the grouped (prefill) tensor-core path with the CPU oracle, through the C ABI (needs a B200: -m gpu).

The grouped path rounds h (the SwiGLU output) and the per-slot down outputs to bf16, as the reference's ragged
kernels do (pallas_moe.py:622-755, out_dtype bf16); its combine is fp32 ("gather" mode). Bars: against the
oracle's restatement of that path (moe.ragged_apply, combine="gather") and against the fp64 ideal, max |got -
want| / max |want| <= 1e-2; the dense int8 GEMM (fp32 out, fp32 accumulation) <= 1e-3.
"""
import os

import numpy as np
import pytest
import torch

from helpers import shared_to_gpu, t_bf16, table_to_gpu
from oracle import cb3, gen, moe, q8

pytestmark = pytest.mark.gpu
LAYER_TOL = 1e-2
MATVEC_TOL = 1e-3


@pytest.fixture(scope="module")
def cbmoe():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cbmoe as m
    m.lib()
    m.device_errors(clear=True)
    return m


def _pack(cbmoe, L, shared=True):
    return cbmoe.pack_layer(table_to_gpu(L["gate"]), table_to_gpu(L["up"]), table_to_gpu(L["down"]),
                            shared_to_gpu(L["shared"]) if shared else None)


@pytest.mark.parametrize("N,k,E,zipf", [(300, 4, 8, None), (700, 8, 16, None), (1500, 2, 4, 1.1), (40, 2, 6, None)])
def test_grouped_apply_matches_oracle(cbmoe, N, k, E, zipf):
    H, I = 512, 256
    rng = np.random.default_rng(N + E)
    L = gen.moe_layer(rng, E, H, I)
    x = gen.activations(rng, N, H)
    idx, w = gen.routing(rng, N, E, k, zipf=zipf)
    p = _pack(cbmoe, L, shared=False)
    y = cbmoe.ResidentFetch(path="grouped").apply(p, t_bf16(x), torch.from_numpy(idx).cuda(),
                                                   torch.from_numpy(w).cuda(), 0, gen.LIMIT)
    xf = x.astype(np.float32)
    got = y.cpu().numpy()
    ragged = moe.ragged_apply(xf, idx, w, L["gate"], L["up"], L["down"], gen.LIMIT, tm=1, combine="gather")
    assert moe.max_rel_err(got, ragged) < LAYER_TOL
    ideal = moe.decode_apply(xf, idx, w, L["gate"], L["up"], L["down"], gen.LIMIT)
    assert moe.max_rel_err(got, ideal) < LAYER_TOL
    assert cbmoe.device_errors(clear=True) == 0


def test_grouped_matches_decode_path(cbmoe):
    """Same layer, same tokens: the grouped and the decode kernels agree within the bf16 rounding of h and y."""
    E, H, I, N, k = 12, 512, 256, 160, 8
    rng = np.random.default_rng(3)
    L = gen.moe_layer(rng, E, H, I)
    x = t_bf16(gen.activations(rng, N, H))
    idx_np, w_np = gen.routing(rng, N, E, k)
    idx, w = torch.from_numpy(idx_np).cuda(), torch.from_numpy(w_np).cuda()
    p = _pack(cbmoe, L, shared=False)
    yg = cbmoe.ResidentFetch(path="grouped").apply(p, x, idx, w, 0, gen.LIMIT)
    yd = cbmoe.ResidentFetch(path="decode").apply(p, x, idx, w, 0, gen.LIMIT)
    assert moe.max_rel_err(yg.cpu().numpy(), yd.cpu().numpy()) < LAYER_TOL


@pytest.mark.parametrize("axis", [1, 0])
def test_grouped_moe_layer_with_shared_expert(cbmoe, axis):
    E, H, I, N, k = 8, 512, 256, 520, 4
    rng = np.random.default_rng(40 + axis)
    L = gen.moe_layer(rng, E, H, I, shared_axis=axis)
    x = gen.activations(rng, N, H)
    idx, w = gen.routing(rng, N, E, k)
    p = _pack(cbmoe, L)
    out = cbmoe.ResidentFetch(path="grouped").layer(p, t_bf16(x), torch.from_numpy(idx).cuda(),
                                                     torch.from_numpy(w).cuda(), gen.LIMIT)
    want = moe.moe_layer(x.astype(np.float32), idx, w, L["gate"], L["up"], L["down"], L["shared"], gen.LIMIT)
    assert moe.max_rel_err(out.float().cpu().numpy(), want) < LAYER_TOL
    assert cbmoe.device_errors(clear=True) == 0


@pytest.mark.parametrize("axis", [1, 0])
@pytest.mark.parametrize("N,K,rows", [(65, 512, 256), (300, 768, 384), (1000, 256, 128)])
def test_w8_linear_tensor_core_path(cbmoe, axis, N, K, rows):
    rng = np.random.default_rng(N + K + axis)
    q, s = gen.q8_leaf(rng, K, rows, axis)
    x = gen.activations(rng, N, K)
    qk = cbmoe.ops.pack_w8(torch.from_numpy(q).cuda())
    y = cbmoe.ops.w8_linear(qk, torch.from_numpy(s.reshape(-1)).cuda(), axis, rows, K, t_bf16(x)).cpu().numpy()
    assert moe.max_rel_err(y, q8.matmul(x.astype(np.float32), q, s)) < MATVEC_TOL
    assert cbmoe.device_errors(clear=True) == 0


def test_ragged_composition_reference_fixture(cbmoe):
    """The reference's own `_apply_ragged_kernel` composition (executed on a NumPy stand-in) vs the grouped path."""
    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "ragged_compose_gather.npz"))
    tabs = [(f[f"{kk}_idx"], f[f"{kk}_cb"].view(cb3.BF16)) for kk in ("gate", "up", "down")]
    p = cbmoe.pack_layer(*[table_to_gpu(t) for t in tabs])
    x = f["x"].astype(cb3.BF16)
    y = cbmoe.ResidentFetch(path="grouped").apply(p, t_bf16(x), torch.from_numpy(f["idx"]).cuda(),
                                                   torch.from_numpy(f["w"]).cuda(), 0, float(f["limit"]))
    assert moe.max_rel_err(y.cpu().numpy(), f["y"]) < LAYER_TOL


@pytest.mark.parametrize("axis", [1, 0])
@pytest.mark.parametrize("K,rows", [(5120, 12288), (12288, 5120)])
def test_w8_linear_config3_projections_full_size(cbmoe, axis, K, rows):
    """The config-3 dense projections at full size: QKV [5120 -> 96 x 128 = 12288] and O [12288 -> 5120] with 4096
    tokens through the tcgen05 path, per-output-channel and per-input-row scales; a sample of 96 token rows (the
    first, the last and spread ones) against quant8's dequant + fp64 product."""
    T = 4096
    rng = np.random.default_rng(K + axis)
    q, s = gen.q8_leaf(rng, K, rows, axis)
    x = gen.activations(rng, T, K)
    qk = cbmoe.ops.pack_w8(torch.from_numpy(q).cuda())
    y = cbmoe.ops.w8_linear(qk, torch.from_numpy(s.reshape(-1)).cuda(), axis, rows, K, t_bf16(x)).cpu().numpy()
    sample = np.unique(np.concatenate([np.arange(16), np.arange(T - 16, T), rng.choice(T, 64, replace=False)]))
    want = q8.matmul(x[sample].astype(np.float32), q, s)
    assert moe.max_rel_err(y[sample], want) < MATVEC_TOL
    assert np.isfinite(y).all()
    assert cbmoe.device_errors(clear=True) == 0
