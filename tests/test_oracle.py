"""The CPU oracle against the golden fixtures made by executing the reference's own functions, and the CB3 spec's
known-answer vectors. No GPU."""
import os

import numpy as np
import pytest

from oracle import cb3, gen, moe, q8


# ------------------------------------------------------------------------------------------ CB3 known answers
def _pack_by_int(q):
    """Independent packer: one Python big integer per row, index j at bit 3j."""
    K = len(q)
    stream = 0
    for j, v in enumerate(q):
        stream |= int(v) << (3 * j)
    return [(stream >> (32 * m)) & 0xFFFFFFFF for m in range(K * 3 // 32)]


def test_cb3_known_answers():
    q = np.zeros(32, np.uint8)
    q[0] = 1
    assert cb3.pack(q).tolist() == [1, 0, 0]
    q = np.zeros(32, np.uint8)
    q[10] = 7                                   # bits 30, 31 of word 0 and bit 0 of word 1
    assert cb3.pack(q).tolist() == [0xC0000000, 1, 0]
    q = np.zeros(32, np.uint8)
    q[21] = 5                                   # bits 63, 64, 65: bit 63 (=1) in word 1, bit 65 (=1) in word 2
    assert cb3.pack(q).tolist() == [0, 0x80000000, 2]
    q = np.arange(32, dtype=np.uint8) % 8
    assert cb3.pack(q).tolist() == _pack_by_int(q)
    assert cb3.words_per_row(2048) == 192 and cb3.words_per_row(5120) == 480 and cb3.words_per_row(1536) == 144


@pytest.mark.parametrize("K", [32, 64, 96, 2048])
def test_cb3_pack_roundtrip(K):
    rng = np.random.default_rng(K)
    q = cb3.make_indices(rng, (3, 5, K))
    w = cb3.pack(q)
    assert w.dtype == np.uint32 and w.shape == (3, 5, K * 3 // 32)
    assert np.array_equal(cb3.unpack(w, K), q)
    for r in range(5):
        assert w[1, r].tolist() == _pack_by_int(q[1, r])


def test_cb3_dequant_exact():
    rng = np.random.default_rng(3)
    R, K = 7, 96
    q = cb3.make_indices(rng, (R, K))
    cb = cb3.make_codebooks(rng, (R,))
    assert np.all(np.diff(cb.astype(np.float32), axis=-1) >= 0)
    d = cb3.dequant(cb3.pack(q), cb, K)
    want = np.array([[cb[r, q[r, j]] for j in range(K)] for r in range(R)], dtype=cb3.BF16)
    assert np.array_equal(cb3.bf16_bits(d), cb3.bf16_bits(want))


def test_config0_matvec_matches_dense():
    c = gen.config0(seed=0)
    y = cb3.matvec(c["idx"], c["cb"], c["x"].astype(np.float32))
    W = cb3.dequant(c["idx"], c["cb"], 2048).astype(np.float64)
    assert y.shape == (1, 1024)
    np.testing.assert_allclose(y, c["x"].astype(np.float64) @ W.T, rtol=1e-12, atol=1e-12)


# ------------------------------------------------------------------------------------------ reference fixtures
@pytest.mark.parametrize("case", range(6))
def test_ragged_plan_matches_reference(golden_dir, case):
    f = np.load(os.path.join(golden_dir, f"plan_{case}.npz"))
    p = moe.ragged_plan(f["idx"], f["w"], int(f["E"]), int(f["tm"]))
    for key in ("blk_expert", "n_blocks", "tok_row", "row_slot"):
        assert np.array_equal(p[key], f[key]), key
    assert np.array_equal(p["w_row"].view(np.uint32), f["w_row"].astype(np.float32).view(np.uint32))


def test_swiglu_matches_reference(golden_dir):
    f = np.load(os.path.join(golden_dir, "swiglu.npz"))
    for L in (10, 7):
        got = moe.swiglu_clamped(f["g"].astype(np.float64), f["u"].astype(np.float64), float(L))
        np.testing.assert_allclose(got, f[f"out_{L}"], rtol=2e-6, atol=1e-6)


def test_quant8_matches_reference(golden_dir):
    f = np.load(os.path.join(golden_dir, "quant8.npz"))
    for axis in (0, 1):
        q, s = q8.quantize_array(f["w"], axis)
        assert np.array_equal(q, f[f"q{axis}"])
        assert np.array_equal(s.view(np.uint32), f[f"s{axis}"].view(np.uint32))
        assert np.array_equal(q8.dequant(q, s).view(np.uint16), f[f"deq{axis}"])


def _tables(f):
    return tuple((f[f"{k}_idx"], f[f"{k}_cb"].view(cb3.BF16)) for k in ("gate", "up", "down"))


def test_decode_composition_matches_reference(golden_dir):
    f = np.load(os.path.join(golden_dir, "decode_compose.npz"))
    g, u, d = _tables(f)
    got = moe.decode_apply(f["x"], f["idx"], f["w"], g, u, d, float(f["limit"]))
    assert moe.max_rel_err(got, f["y"]) < 1e-5


@pytest.mark.parametrize("combine", ["matmul", "gather"])
def test_ragged_composition_matches_reference(golden_dir, combine):
    f = np.load(os.path.join(golden_dir, f"ragged_compose_{combine}.npz"))
    g, u, d = _tables(f)
    got = moe.ragged_apply(f["x"], f["idx"], f["w"], g, u, d, float(f["limit"]), tm=int(f["tm"]), combine=combine)
    assert moe.max_rel_err(got, f["y"]) < 5e-3
    ideal = moe.decode_apply(f["x"].astype(np.float32).astype(cb3.BF16), f["idx"], f["w"], g, u, d, float(f["limit"]))
    assert moe.max_rel_err(got, ideal) < 1e-2


def test_routing_generators():
    rng = np.random.default_rng(0)
    idx, w = gen.routing(rng, 64, 160, 8)
    assert idx.shape == (64, 8) and np.all([len(set(r)) == 8 for r in idx])
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)
    idx_z, _ = gen.routing(np.random.default_rng(1), 64, 160, 8, zipf=1.1)
    counts = np.bincount(idx_z.reshape(-1), minlength=160)
    assert counts.max() >= 32 and (counts == 0).sum() >= 40          # skewed: hot experts and many idle ones


# ------------------------------------------------------------------------------------------ C oracle
def test_c_oracle_matches_numpy_oracle():
    from oracle import cpu
    rng = np.random.default_rng(21)
    E, H, I, N, k = 6, 256, 128, 3, 2
    L = gen.moe_layer(rng, E, H, I)
    x = gen.activations(rng, N, H).astype(np.float32)
    idx, w = gen.routing(rng, N, E, k)
    got = cpu.moe_layer(x, idx, w, L["gate"], L["up"], L["down"], L["shared"], gen.LIMIT)
    want = moe.moe_layer(x, idx, w, L["gate"], L["up"], L["down"], L["shared"], gen.LIMIT)
    assert moe.max_rel_err(got, want) < 1e-5
    y = cpu.cb3_matvec(L["down"][0][1], L["down"][1][1], x[:, :I] if False else rng.standard_normal((2, I)).astype(np.float32))
    assert y.shape == (2, H)


def test_logits_colscale_matches_reference_fixture():
    """oracle q8.logits_colscale against the reference's own `Engine._logits_local` with int8 columns (executed on the
    NumPy stand-in by tests/golden/make_golden.py): bf16(f32(h @ q) * s). The reference sums in float32 and the
    oracle in float64, so the bf16 logits agree to within one bf16 unit in the last place."""
    import ml_dtypes
    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "logits_q8.npz"))
    h = f["h"].view(ml_dtypes.bfloat16)
    got = q8.logits_colscale(h, f["q"], f["s"]).astype(np.float32)
    want = f["z"].view(ml_dtypes.bfloat16).astype(np.float32)
    tol = np.abs(want) * 2.0 ** -7 + np.abs(want).max(axis=-1, keepdims=True) * 2.0 ** -12
    assert np.all(np.abs(got - want) <= tol)
    assert np.mean(got == want) > 0.95
