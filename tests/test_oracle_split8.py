"""The byte-digit splits of the CB8 decode path, on the CPU (oracle/split8.py): the stated exactness and error
bounds, the digit ranges the int8 MMAs need, and the edge cases (zero rows, subnormal and huge entries)."""
import numpy as np

from oracle import cb3, split8


def _codebooks(rng):
    cb = cb3.make_codebooks(rng, (6, 64)).astype(np.float32).reshape(-1, 8)
    cb[0] = 0.0
    cb[1, 2] = 3e-7
    cb[2] *= 1e4
    cb[3] = -np.abs(cb[3])
    cb[4, :4] = 1e-39
    cb[5] *= 1e-30
    cb[6] = np.linspace(-0.75, 0.6, 8)                             # largest magnitude in [0.5, 1)
    cb[7] = 1.0
    return cb.astype(cb3.BF16)


def test_cb8_rows_exact_within_2_7_and_bounded_below():
    cb = _codebooks(np.random.default_rng(0))
    hi, lo, f, T = split8.cb8_rows(cb)
    v = cb.astype(np.float64)
    mx = np.abs(v).max(axis=-1, keepdims=True)
    assert np.array_equal(T, hi.astype(np.int32) * 256 + lo.astype(np.int32))
    assert np.abs(T).max() < 2 ** 15
    err = np.abs(T * f[:, None].astype(np.float64) - v)
    near = np.abs(v) >= mx / 2 ** 7
    assert np.all(err[near] == 0)
    assert np.all(err <= mx * 2.0 ** -15 + 1e-300)


def test_split_x_digits_and_bounds():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((4, 512)).astype(np.float32)
    x[1] = 0.0
    x[2] *= 1e-3
    x[3, :5] = [1e-30, -2.5, 1e-8, 0.0, 7.0]
    x[2] = np.clip(x[2] * 1e3, -0.7, 0.7)                         # largest magnitude in [0.5, 1)
    xb = x.astype(cb3.BF16)
    x8, s = split8.split_x(xb)
    d = x8.reshape(4, 2, 4, 2, 64).view(np.int8)
    assert d[:, :, :, 1].max() <= 64 and d[:, :, :, 1].min() >= -64          # high digit: |X| < 2^14
    back = split8.x8_values(x8, s)
    xv = xb.astype(np.float64)
    mx = np.abs(xv).max(axis=1, keepdims=True)
    err = np.abs(back - xv)
    assert np.all(err[np.abs(xv) >= mx / 2 ** 6] == 0)
    assert np.all(err <= mx * 2.0 ** -14)
    assert np.all(back[1] == 0)


def test_h8_digits_reconstruct_the_fp32_value():
    rng = np.random.default_rng(2)
    for scale in (1e-20, 1e-3, 0.2, 0.3, 1.0, 37.0, 1e10):
        h = (rng.standard_normal(64) * scale).astype(np.float32)
        h[5] = 0.0
        d, f = split8.h8_digits(h)
        assert np.abs(d[:3].astype(np.int32)).max() <= 128 and np.abs(d[3].astype(np.int32)).max() <= 33
        v = (d.astype(np.float64) * (256.0 ** np.arange(4))[:, None]).sum(0) * np.float64(f)
        mx = np.abs(h.astype(np.float64)).max()
        near = np.abs(h) >= mx / 2 ** 5
        assert np.all(v[near] == h[near].astype(np.float64))
        assert np.all(np.abs(v - h) <= mx * 2.0 ** -29)
    d, f = split8.h8_digits(np.zeros(64, np.float32))
    assert not d.any()


def test_cb8_table_layout_roundtrip():
    rng = np.random.default_rng(3)
    cbs = [cb3.make_codebooks(rng, (2, 128)) for _ in range(2)]
    t = split8.cb8_table(cbs).reshape(2, 2, 2 * 64 * 20)
    for m in range(2):
        hi, lo, f, _ = split8.cb8_rows(cbs[m])
        for e in range(2):
            for r in range(128):
                rb, w, r16 = r // 64, (r % 64) // 16, r % 16
                base = (w * 2 + m) * 16 + r16
                blk = t[e, rb]
                assert np.array_equal(blk[base * 16:base * 16 + 8], hi[e, r].view(np.uint8))
                assert np.array_equal(blk[base * 16 + 8:base * 16 + 16], lo[e, r])
                assert blk[2 * 1024 + base * 4:2 * 1024 + base * 4 + 4].view(np.float32)[0] == f[e, r]
