"""Parity of the CUDA decode path with the CPU oracle, through the C ABI (needs a B200: -m gpu).

Tolerances: dequantized weights and the routing plan are compared bit for bit; layer outputs use the benchmark's
bar, max |got - want| / max |want| <= 1e-2 (bf16 output, fp32 accumulation); single-matrix products, whose only
rounding is the fp32 accumulation, are held to 1e-3.
"""
import os

import numpy as np
import pytest
import torch

from helpers import bf16_bits_of, shared_to_gpu, t_bf16, table_to_gpu, t_u32
from oracle import cb3, gen, moe, q8, split8

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


def _no_device_errors(cbmoe):
    assert cbmoe.device_errors(clear=True) == 0


# ------------------------------------------------------------------------------------------------ layouts
@pytest.mark.parametrize("nmat,E,rows,K", [(1, 1, 64, 256), (1, 3, 128, 512), (2, 2, 192, 768), (1, 1, 1024, 2048)])
def test_cb3k_dequant_bit_exact(cbmoe, nmat, E, rows, K):
    rng = np.random.default_rng(100 + rows)
    tabs = [gen.cb3_table(rng, E, rows, K) for _ in range(nmat)]
    g = [table_to_gpu(t) for t in tabs]
    idx_k, cb_k = cbmoe.ops.pack_cb3(g[0][0], g[0][1], *(g[1] if nmat == 2 else (None, None)))
    assert idx_k.numel() == E * rows * K * nmat * 3 // 8 and cb_k.numel() == E * rows * nmat * 16
    out = bf16_bits_of(cbmoe.ops.dequant_cb3k(idx_k, cb_k, nmat, E, rows, K))
    for m in range(nmat):
        want = cb3.bf16_bits(cb3.dequant(tabs[m][0], tabs[m][1], K))
        assert np.array_equal(out[m], want)
    _no_device_errors(cbmoe)


@pytest.mark.parametrize("axis", [0, 1])
@pytest.mark.parametrize("nmat", [1, 2])
def test_w8k_dequant_bit_exact(cbmoe, axis, nmat):
    rng = np.random.default_rng(7 + axis)
    K, rows = 512, 128
    leaves = [gen.q8_leaf(rng, K, rows, axis) for _ in range(nmat)]
    qs = [torch.from_numpy(q).cuda() for q, _ in leaves]
    ss = [torch.from_numpy(s.reshape(-1)).cuda() for _, s in leaves]
    qk = cbmoe.ops.pack_w8(qs[0], qs[1] if nmat == 2 else None)
    out = bf16_bits_of(cbmoe.ops.dequant_w8k(qk, ss[0], ss[1] if nmat == 2 else None, axis, nmat, rows, K))
    for m in range(nmat):
        want = q8.dequant(*leaves[m]).T.view(np.uint16)          # [in, out] -> [out, in]
        assert np.array_equal(out[m], want)


def _wide_codebooks(rng, E, rows):
    """Codebooks with the edge cases of the CB8 split: all-zero rows, rows with tiny and huge entries beside
    ordinary ones, entries far below their row's largest, negative-only rows, subnormal bf16 values."""
    cb = cb3.make_codebooks(rng, (E, rows)).astype(np.float32)
    flat = cb.reshape(-1, 8)
    n = flat.shape[0]
    flat[0::17] = 0.0
    flat[1::17, 3] = 3e-7                                         # 2^-22-ish beside entries ~0.02
    flat[2::17] *= 1e4                                            # large rows
    flat[3::17] = -np.abs(flat[3::17])
    flat[4::17, :4] = 1e-39                                       # bf16 subnormals
    flat[5::17] *= 1e-30
    flat[6::17, 0] = -2.5e-3
    flat[7::17] = np.linspace(-0.75, 0.6, 8)                      # largest magnitude in [0.5, 1)
    flat[8::17] = 1.0
    return flat.reshape(E, rows, 8).astype(cb3.BF16)


@pytest.mark.parametrize("nmat,E,rows", [(1, 2, 64), (2, 3, 128), (1, 1, 1024)])
def test_cb8_tables_bit_exact(cbmoe, nmat, E, rows):
    """The CB8 tables built on the GPU (int8 hi / uint8 lo bytes + row factors) equal the oracle's, byte for byte."""
    rng = np.random.default_rng(300 + rows)
    K = 256
    tabs = [(cb3.pack(cb3.make_indices(rng, (E, rows, K))), _wide_codebooks(rng, E, rows)) for _ in range(nmat)]
    g = [table_to_gpu(t) for t in tabs]
    _, cb_k = cbmoe.ops.pack_cb3(g[0][0], g[0][1], *(g[1] if nmat == 2 else (None, None)))
    got = cbmoe.ops.build_cb8(cb_k, nmat, E, rows).cpu().numpy()
    want = split8.cb8_table([t[1] for t in tabs])
    assert got.shape == want.shape
    assert np.array_equal(got, want)
    _no_device_errors(cbmoe)


# ------------------------------------------------------------------------------------------------ routing plan
def _check_plan(got, want, T, k):
    for key in ("blk_expert", "tok_row"):
        assert np.array_equal(got[key].cpu().numpy(), want[key]), key
    assert int(got["n_blocks"].item()) == int(want["n_blocks"][0])
    assert np.array_equal(got["row_slot"].cpu().numpy(), want["row_slot"].reshape(T, k))
    assert np.array_equal(got["w_row"].cpu().numpy().view(np.uint32), want["w_row"].astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("case", range(6))
def test_route_plan_matches_reference_fixture(cbmoe, case):
    f = np.load(os.path.join(os.path.dirname(__file__), "golden", f"plan_{case}.npz"))
    idx, w = f["idx"], f["w"]
    T, k = idx.shape
    got = cbmoe.ops.route_plan(torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda(), int(f["E"]), int(f["tm"]))
    _check_plan(got, {kk: f[kk] for kk in ("blk_expert", "n_blocks", "tok_row", "w_row", "row_slot")}, T, k)


@pytest.mark.parametrize("T,k,E,tm,pt", [(8, 8, 160, 1, 8), (64, 8, 160, 1, 32), (4096, 8, 160, 128, 32),
                                          (3, 2, 5, 4, 8), (0, 8, 160, 1, 8), (700, 6, 1024, 16, 16)])
def test_route_plan_matches_oracle(cbmoe, T, k, E, tm, pt):
    rng = np.random.default_rng(T + E)
    if T:
        idx, w = gen.routing(rng, T, E, k, zipf=1.1 if T == 64 else None)
    else:
        idx, w = np.zeros((0, k), np.int32), np.zeros((0, k), np.float32)
    got = cbmoe.ops.route_plan(torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda(), E, tm, pt)
    want = moe.ragged_plan(idx, w, E, tm)
    _check_plan(got, want, T, k)
    counts = np.bincount(idx.reshape(-1), minlength=E)
    assert np.array_equal(got["counts"].cpu().numpy(), counts)
    act = np.nonzero(counts)[0]
    assert int(got["n_act"].item()) == len(act)
    assert np.array_equal(got["act"].cpu().numpy()[:len(act)], act)
    # pass lists: each active expert's rows cut into pieces of at most pt rows, in expert order
    pe, pr, pc = (got[n].cpu().numpy() for n in ("pass_expert", "pass_row0", "pass_cnt"))
    n_pass = int(got["n_pass"].item())
    padded = -(-counts // tm) * tm
    rs = np.cumsum(padded) - padded
    want_p = [(e, rs[e] + j * pt, min(pt, counts[e] - j * pt)) for e in act for j in range(-(-counts[e] // pt))]
    assert n_pass == len(want_p)
    assert [tuple(v) for v in zip(pe[:n_pass], pr[:n_pass], pc[:n_pass])] == want_p


# ------------------------------------------------------------------------------------------------ matvecs
@pytest.mark.parametrize("N", [1, 5, 13, 40])
def test_cb3_matvec_config0_shape(cbmoe, N):
    c = gen.config0(seed=N)
    x = gen.activations(np.random.default_rng(N), N, 2048)
    idx_k, cb_k = cbmoe.ops.pack_cb3(t_u32(c["idx"][None]), t_bf16(c["cb"][None]))
    y = cbmoe.ops.cb3_matvec(idx_k, cb_k, 1024, 2048, t_bf16(x)).cpu().numpy()
    want = cb3.matvec(c["idx"], c["cb"], x.astype(np.float32))
    assert moe.max_rel_err(y, want) < MATVEC_TOL
    _no_device_errors(cbmoe)


@pytest.mark.parametrize("N", [1, 4, 5, 13, 40])
def test_cb8_matvec_config0_shape(cbmoe, N):
    """The int8 decode kernel on the config-0 matrix; its workspace holds the split activations, which must equal
    the oracle's X8 rows byte for byte."""
    c = gen.config0(seed=N)
    rng = np.random.default_rng(N)
    x = gen.activations(rng, N, 2048)
    if N == 5:
        x[1] = 0.0                                            # an all-zero token
        x[2] *= 1e3                                           # a large one
        x[3] = np.clip(x[3], -0.9, 0.9)                       # and one whose largest magnitude is in [0.5, 1)
    x = x.astype(cb3.BF16)
    idx_k, cb_k = cbmoe.ops.pack_cb3(t_u32(c["idx"][None]), t_bf16(c["cb"][None]))
    cb8 = cbmoe.ops.build_cb8(cb_k, 1, 1, 1024)
    ws = torch.empty(cbmoe.lib().cbmoe_cb8_matvec_workspace_bytes(N, 2048), dtype=torch.uint8, device="cuda")
    y = cbmoe.ops.cb8_matvec(idx_k, cb8, 1024, 2048, t_bf16(x), ws=ws).cpu().numpy()
    want = cb3.matvec(c["idx"], c["cb"], x.astype(np.float32))
    assert moe.max_rel_err(y, want) < MATVEC_TOL
    x8, xs = split8.split_x(x)
    w = ws.cpu().numpy()
    assert np.array_equal(w[:x8.size].reshape(x8.shape), x8)
    off = -(-x8.size // 256) * 256
    assert np.array_equal(w[off:off + 4 * N].view(np.float32), xs)
    _no_device_errors(cbmoe)


@pytest.mark.parametrize("axis", [0, 1])
@pytest.mark.parametrize("N", [1, 9, 33])
def test_w8_linear(cbmoe, axis, N):
    rng = np.random.default_rng(N * 3 + axis)
    K, rows = 768, 320
    q, s = gen.q8_leaf(rng, K, rows, axis)
    x = gen.activations(rng, N, K)
    qk = cbmoe.ops.pack_w8(torch.from_numpy(q).cuda())
    y = cbmoe.ops.w8_linear(qk, torch.from_numpy(s.reshape(-1)).cuda(), axis, rows, K, t_bf16(x)).cpu().numpy()
    assert moe.max_rel_err(y, q8.matmul(x.astype(np.float32), q, s)) < MATVEC_TOL


# ------------------------------------------------------------------------------------------------ layer
def _layer(seed, E, H, I, axis=1):
    rng = np.random.default_rng(seed)
    L = gen.moe_layer(rng, E, H, I, shared_axis=axis)
    return rng, L


def _pack(cbmoe, L, tables="int8"):
    return cbmoe.pack_layer(table_to_gpu(L["gate"]), table_to_gpu(L["up"]), table_to_gpu(L["down"]),
                            shared_to_gpu(L["shared"]), decode_tables=tables)


@pytest.mark.parametrize("tables", ["int8", "bf16"])
@pytest.mark.parametrize("N,k,E,zipf", [(1, 8, 16, None), (3, 4, 16, None), (8, 8, 24, None), (20, 6, 16, 1.1),
                                        (64, 8, 32, 1.1), (40, 2, 4, None)])
def test_experts_apply_decode(cbmoe, N, k, E, zipf, tables):
    H, I = 512, 256
    rng, L = _layer(N * 31 + E, E, H, I)
    x = gen.activations(rng, N, H)
    idx, w = gen.routing(rng, N, E, k, zipf=zipf)
    p = _pack(cbmoe, L, tables)
    fetch = cbmoe.ResidentFetch(path="decode")
    y = fetch.apply(p, t_bf16(x), torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda(), 0, gen.LIMIT)
    want = moe.decode_apply(x.astype(np.float32), idx, w, L["gate"], L["up"], L["down"], gen.LIMIT)
    assert moe.max_rel_err(y.cpu().numpy(), want) < LAYER_TOL
    _no_device_errors(cbmoe)


@pytest.mark.parametrize("tables", ["int8", "bf16"])
@pytest.mark.parametrize("axis", [1, 0])
@pytest.mark.parametrize("N", [1, 8, 24])
def test_moe_layer_decode(cbmoe, N, axis, tables):
    E, H, I, k = 16, 512, 256, 8
    rng, L = _layer(N + 7 * axis, E, H, I, axis)
    x = gen.activations(rng, N, H)
    idx, w = gen.routing(rng, N, E, k)
    p = _pack(cbmoe, L, tables)
    out = cbmoe.moe_dense(p, t_bf16(x), torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda(), gen.LIMIT,
                          cbmoe.ResidentFetch(path="decode"))
    want = moe.moe_layer(x.astype(np.float32), idx, w, L["gate"], L["up"], L["down"], L["shared"], gen.LIMIT)
    assert out.dtype == torch.bfloat16
    assert moe.max_rel_err(out.float().cpu().numpy(), want) < LAYER_TOL
    _no_device_errors(cbmoe)


@pytest.mark.parametrize("tables", ["int8", "bf16"])
def test_decode_composition_reference_fixture(cbmoe, tables):
    """The reference's own `_apply_kernel` composition (executed on a NumPy stand-in) vs the CUDA path."""
    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "decode_compose.npz"))
    tabs = [(f[f"{kk}_idx"], f[f"{kk}_cb"].view(cb3.BF16)) for kk in ("gate", "up", "down")]
    p = cbmoe.pack_layer(*[table_to_gpu(t) for t in tabs], decode_tables=tables)
    x = f["x"].astype(cb3.BF16)                      # the kernels take bf16 activations
    y = cbmoe.ResidentFetch(path="decode").apply(p, t_bf16(x), torch.from_numpy(f["idx"]).cuda(),
                                                 torch.from_numpy(f["w"]).cuda(), 0, float(f["limit"]))
    want = moe.decode_apply(x.astype(np.float32), f["idx"], f["w"], *tabs, float(f["limit"]))
    assert moe.max_rel_err(y.cpu().numpy(), want) < 1e-4
    # the fixture itself was computed from fp32 activations: same result within the bf16 input rounding
    assert moe.max_rel_err(y.cpu().numpy(), f["y"]) < LAYER_TOL


def test_apply_is_linear_in_routing_weights(cbmoe):
    E, H, I, N, k = 12, 512, 256, 8, 4
    rng, L = _layer(5, E, H, I)
    x, (idx, w) = gen.activations(rng, N, H), gen.routing(rng, N, E, k)
    p = _pack(cbmoe, L)
    f = cbmoe.ResidentFetch(path="decode")
    xi, ii = t_bf16(x), torch.from_numpy(idx).cuda()
    y1 = f.apply(p, xi, ii, torch.from_numpy(w).cuda(), 0, gen.LIMIT)
    y2 = f.apply(p, xi, ii, torch.from_numpy(2 * w).cuda(), 0, gen.LIMIT)
    assert torch.equal(y2, 2 * y1)


def test_out_of_range_expert_is_reported_not_fatal(cbmoe):
    E, H, I, N, k = 8, 256, 256, 4, 2
    rng, L = _layer(9, E, H, I)
    x = gen.activations(rng, N, H)
    idx = np.array([[0, 1], [2, 3], [4, E + 5], [6, 7]], np.int32)      # one id past E
    w = np.full((N, k), 0.5, np.float32)
    p = _pack(cbmoe, L)
    y = cbmoe.ResidentFetch(path="decode").apply(p, t_bf16(x), torch.from_numpy(idx).cuda(),
                                                  torch.from_numpy(w).cuda(), 0, gen.LIMIT)
    assert cbmoe.device_errors(clear=True) == 2                        # CBMOE_DEVERR_INDEX
    idx_ok = idx.copy()
    w_ok = w.copy()
    idx_ok[2, 1], w_ok[2, 1] = 0, 0.0                                    # the bad slot contributes nothing
    want = moe.decode_apply(x.astype(np.float32), idx_ok, w_ok, L["gate"], L["up"], L["down"], gen.LIMIT)
    assert moe.max_rel_err(y.cpu().numpy(), want) < LAYER_TOL


def test_empty_batch(cbmoe):
    E, H, I = 4, 256, 256
    _, L = _layer(1, E, H, I)
    p = _pack(cbmoe, L)
    x = torch.zeros((0, H), dtype=torch.bfloat16, device="cuda")
    y = cbmoe.ResidentFetch(path="decode").apply(p, x, torch.zeros((0, 8), dtype=torch.int32, device="cuda"),
                                                  torch.zeros((0, 8), device="cuda"), 0, gen.LIMIT)
    assert y.shape == (0, H)


def test_w8_logits_reference_fixture(cbmoe):
    """The int8 lm_head kernel against the reference's `Engine._logits_local` (int8 columns, executed by
    tests/golden/make_golden.py): within one bf16 unit in the last place (the sums run in another order)."""
    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "logits_q8.npz"))
    q, s = f["q"], f["s"].reshape(-1)
    D, V = q.shape
    qk = cbmoe.ops.pack_w8(torch.from_numpy(q).cuda())
    h = torch.from_numpy(f["h"].view(np.int16).copy()).cuda().view(torch.bfloat16)
    got = cbmoe.ops.w8_logits(qk, torch.from_numpy(s).cuda(), V, D, h).float().cpu().numpy()
    want = f["z"].view(cb3.BF16).astype(np.float32)
    assert np.all(np.abs(got - want) <= _logit_tol(want))
    assert np.mean(got == want) > 0.9
    _no_device_errors(cbmoe)


def _logit_tol(want):
    """One bf16 unit in the last place of each logit, plus 2^-12 of its row's largest: a logit that nearly cancels
    carries the summation order's rounding (the reference sums in f32, the kernel exactly in int32) at the scale of
    its terms, not of its own value."""
    return np.abs(want) * 2.0 ** -7 + np.abs(want).max(axis=-1, keepdims=True) * 2.0 ** -12


@pytest.mark.parametrize("B", [1, 8, 13])
def test_w8_logits_lm_head_shape(cbmoe, B):
    """[B, 5120] x [5120, V/8] (V = 151552: one GPU's vocab columns of an 8-way split) against the oracle's
    bf16(f32(h @ q) * s): within one bf16 unit in the last place."""
    D, V = 5120, 151552 // 8
    rng = np.random.default_rng(B)
    q, s = gen.q8_leaf(rng, D, V, 1)
    h = gen.activations(rng, B, D)
    qk = cbmoe.ops.pack_w8(torch.from_numpy(q).cuda())
    got = cbmoe.ops.w8_logits(qk, torch.from_numpy(s.reshape(-1)).cuda(), V, D, t_bf16(h)).float().cpu().numpy()
    want = q8.logits_colscale(h, q, s).astype(np.float32)
    assert np.all(np.abs(got - want) <= _logit_tol(want))
    _no_device_errors(cbmoe)
