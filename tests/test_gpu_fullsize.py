"""Parity at the benchmark's full layer size (needs a B200: -m gpu): E = 160 CB3 experts, hidden 5120,
intermediate 1536, top-8, int8 shared expert, limit 10, through the library against the C oracle
(oracle/cbmoe_cpu.c, fp32, checked against the NumPy oracle in test_oracle.py) on the same seeded inputs:
config 1 (8 tokens, decode), config 2 (64 tokens with Zipf(1.1)-skewed routing, decode and grouped), the decode
ones on both decode kernels (int8-digit CB8 tables, and the bf16 kernels when the layer carries no CB8 tables), and
config 3 (4096 tokens on the grouped tensor-core path, checked on a sample of token rows; the layer is
independent per token). Bar: max |got - want| / max |want| <= 1e-2 (bf16 out, fp32 accumulation)."""
import numpy as np
import pytest
import torch

from helpers import shared_to_gpu, t_bf16, table_to_gpu
from oracle import cpu, gen, moe

pytestmark = pytest.mark.gpu
E, H, I, K = 160, 5120, 1536, 8
TOL = 1e-2


@pytest.fixture(scope="module")
def setup():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cbmoe
    cbmoe.lib()
    cbmoe.device_errors(clear=True)
    cpu.build()
    rng = np.random.default_rng(2024)
    L = gen.moe_layer(rng, E, H, I, words=True)
    p = cbmoe.pack_layer(table_to_gpu(L["gate"]), table_to_gpu(L["up"]), table_to_gpu(L["down"]),
                         shared_to_gpu(L["shared"]))
    torch.cuda.synchronize()
    return cbmoe, L, p, rng


def _want(L, x, idx, w):
    return cpu.moe_layer(x.astype(np.float32), idx, w, L["gate"], L["up"], L["down"], L["shared"], gen.LIMIT)


def _run(cbmoe, p, x, idx, w, path):
    if path == "decode_bf16":   # the same tables without the CB8 ones: the bf16 decode kernels
        p = {kk: v for kk, v in p.items() if kk not in ("gate_up_cb8", "down_cb8")}
        path = "decode"
    out = cbmoe.ResidentFetch(path=path).layer(p, t_bf16(x), torch.from_numpy(idx).cuda(),
                                               torch.from_numpy(w).cuda(), gen.LIMIT)
    return out.float().cpu().numpy()


@pytest.mark.parametrize("path", ["decode", "decode_bf16"])
def test_config1_decode_layer(setup, path):
    cbmoe, L, p, _ = setup
    rng = np.random.default_rng(8)
    x = gen.activations(rng, 8, H)
    idx, w = gen.routing(rng, 8, E, K)
    got = _run(cbmoe, p, x, idx, w, path)
    assert moe.max_rel_err(got, _want(L, x, idx, w)) < TOL
    assert cbmoe.device_errors(clear=True) == 0


@pytest.mark.parametrize("path", ["decode", "grouped", "decode_bf16"])
def test_config2_skewed_batch(setup, path):
    cbmoe, L, p, _ = setup
    rng = np.random.default_rng(64)
    x = gen.activations(rng, 64, H)
    idx, w = gen.routing(rng, 64, E, K, zipf=1.1)
    counts = np.bincount(idx.reshape(-1), minlength=E)
    assert counts.max() > 3 * counts.mean() and (counts == 0).sum() > 0   # hot experts and idle ones
    got = _run(cbmoe, p, x, idx, w, path)
    assert moe.max_rel_err(got, _want(L, x, idx, w)) < TOL
    assert cbmoe.device_errors(clear=True) == 0


def test_config3_prefill_rows(setup):
    """Config 3 on the grouped path, checked on 272 token rows: for every expert, the first and the last token routed
    to it (so every expert's first and last 128-row block is covered), the first and last 8 tokens, and spread ones
    up to 272."""
    cbmoe, L, p, _ = setup
    rng = np.random.default_rng(4096)
    x = gen.activations(rng, 4096, H)
    idx, w = gen.routing(rng, 4096, E, K)
    got = _run(cbmoe, p, x, idx, w, "grouped")
    ends = []
    for e in range(E):
        toks = np.nonzero((idx == e).any(axis=1))[0]
        if toks.size:
            ends += [toks[0], toks[-1]]
    rows = np.unique(np.concatenate([np.arange(8), np.arange(4088, 4096), np.array(ends, np.int64)]))
    rest = np.setdiff1d(np.arange(4096), rows)
    rows = np.union1d(rows, rng.choice(rest, 272 - rows.size, replace=False))
    assert rows.size == 272, rows.size
    want = _want(L, x[rows], idx[rows], w[rows])
    assert moe.max_rel_err(got[rows], want) < TOL
    assert np.isfinite(got).all()
    assert cbmoe.device_errors(clear=True) == 0
