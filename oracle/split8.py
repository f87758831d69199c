"""Byte-digit splits of the CB8 decode path: the CPU restatement the GPU tables and activations are checked against,
bit for bit (test infrastructure, see oracle/__init__.py; nothing in the product imports it).

The decode kernels multiply int8 digits on the tensor cores with exact int32 sums instead of bf16 values (no
counterpart in the reference, whose decode kernel dequantizes to f32, pallas_moe.py:238-307; the result is the same
f32 contraction up to the fixed-point rounding stated below):
  * codebooks (CB8): per row, the 8 bf16 entries v as T = rint(v 2^s), s = 15 - e where max|v| = f 2^e,
    f in [0.5, 1), so max|T| in [2^14, 2^15); hi = T >> 8 (int8), lo = T & 255 (uint8); row factor 2^-s.
    T = v 2^s exactly for entries within 2^7 of the row's largest, else to within 2^-15 of it.
  * activations (X8): per row of x (bf16), X = rint(x 2^t), t = 14 - e (max|X| in [2^13, 2^14)); digits
    d1 = (X + 128) >> 8, d0 = X - 256 d1 (both int8); x = 2^-t (256 d1 + d0), exactly within 2^6 of the row's
    largest, else to within 2^-14 of it.
  * the SwiGLU output (H8): per (slot, 64-input chunk), V = rint(h 2^u), u = 29 - e of the chunk's largest |h|;
    4 balanced base-256 digits (the last one takes what remains); h = 2^-u sum_p 256^p d_p.
rint = round half to even (numpy.rint, CUDA __float2int_rn).
"""
import numpy as np

from . import cb3

STAGE_K = 256


def shift_for(m, top):
    """top - e where m = f 2^e, f in [0.5, 1) (frexp's exponent): m 2^shift in [2^(top-1), 2^top); 0 where m is
    zero or not finite."""
    m = np.asarray(m, np.float32)
    ok = (m > 0) & np.isfinite(m) & (m < 3e38)
    _, e = np.frexp(np.where(ok, m, np.float32(1.0)))
    return np.where(ok, top - e, 0).astype(np.int32)


def cb8_rows(cb):
    """bf16 codebooks [..., 8] -> (hi int8 [..., 8], lo uint8 [..., 8], factor f32 [...], T int32 [..., 8])."""
    v = np.asarray(cb, cb3.BF16).astype(np.float32)
    sh = shift_for(np.abs(v).max(axis=-1), 15)
    T = np.rint(np.ldexp(v.astype(np.float64), sh[..., None])).astype(np.int32)
    assert np.abs(T).max(initial=0) < 2 ** 15
    return (T >> 8).astype(np.int8), (T & 255).astype(np.uint8), np.ldexp(np.float32(1.0), -sh).astype(np.float32), T


def cb8_table(cbs):
    """Codebooks of nmat matrices ([E, rows, 8] bf16 each: gate, up or the only one) -> uint8 CB8 bytes in the
    kernels' layout: per (expert, 64-row block), tables [warp 4][matrix][row 16][hi 8 | lo 8], then row factors
    [warp 4][matrix][row 16] f32."""
    nmat = len(cbs)
    E, rows, _ = cbs[0].shape
    RB = rows // 64
    out = np.zeros((E, RB, nmat * 64 * 20), np.uint8)
    for m, cb in enumerate(cbs):
        hi, lo, f, _ = cb8_rows(cb)
        hi = hi.view(np.uint8).reshape(E, RB, 4, 16, 8)
        lo = lo.reshape(E, RB, 4, 16, 8)
        f = f.reshape(E, RB, 4, 16)
        for w in range(4):
            base = (w * nmat + m) * 16
            out[:, :, base * 16:(base + 16) * 16] = np.concatenate([hi[:, :, w], lo[:, :, w]], -1).reshape(E, RB, 256)
            off = nmat * 1024 + base * 4
            out[:, :, off:off + 64] = np.ascontiguousarray(f[:, :, w]).view(np.uint8).reshape(E, RB, 64)
    return out.reshape(-1)


def cb8_values(cb):
    """The codebook values the CB8 tables stand for: T * factor, float64 [..., 8]."""
    _, _, f, T = cb8_rows(cb)
    return T.astype(np.float64) * f[..., None].astype(np.float64)


def split_x(x):
    """x bf16 [N, K] -> (X8 bytes uint8 [N, K/256, 512]: per 256-input stage [chunk 4][digit 2][64], factor f32 [N])."""
    xf = np.asarray(x, cb3.BF16).astype(np.float32)
    N, K = xf.shape
    t = shift_for(np.abs(xf).max(axis=1), 14)
    X = np.rint(np.ldexp(xf.astype(np.float64), t[:, None])).astype(np.int32)
    d1 = (X + 128) >> 8
    d0 = X - 256 * d1
    assert np.abs(d1).max(initial=0) <= 127 and np.abs(d0).max(initial=0) <= 128
    KS = K // STAGE_K
    both = np.stack([d0.reshape(N, KS, 4, 64), d1.reshape(N, KS, 4, 64)], axis=3).astype(np.int8)
    return both.view(np.uint8).reshape(N, KS, 512), np.ldexp(np.float32(1.0), -t).astype(np.float32)


def x8_values(x8, scale):
    """X8 bytes [N, KS, 512] + factors [N] -> the float64 values they stand for, [N, KS*256]."""
    N, KS, _ = x8.shape
    d = np.asarray(x8, np.uint8).view(np.int8).reshape(N, KS, 4, 2, 64).astype(np.float64)
    val = d[:, :, :, 0] + 256.0 * d[:, :, :, 1]
    return val.reshape(N, KS * 256) * np.asarray(scale, np.float64)[:, None]


def h8_digits(h_chunk):
    """One (slot, 64-input chunk) of the SwiGLU output, f32 [64] -> (digits int8 [4, 64], factor f32)."""
    h = np.asarray(h_chunk, np.float32)
    u = int(shift_for(np.abs(h).max(), 29))
    V = np.rint(np.ldexp(h.astype(np.float64), u)).astype(np.int64)
    digs = []
    for q in range(4):
        d = ((V & 255) ^ 128) - 128 if q < 3 else V
        digs.append(d)
        V = (V - d) >> 8
    return np.stack(digs).astype(np.int8), np.float32(np.ldexp(1.0, -u))
