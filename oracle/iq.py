"""The reference's GGUF expert formats (llama.cpp IQ2_S / IQ3_S / IQ4_XS, and Q2_K / Q3_K of its MTP layer):
CPU restatement (test infrastructure, see oracle/__init__.py).

The reference's GLM-5.3-Flash tables use llama.cpp's codebook ("IQ") quantizations; its dequant is
launcher/glm53-flash/engine/glm53/iqquant.py (dequant_iq2_s :108-121, dequant_iq3_s :124-134, dequant_iq4_xs
:137-146), restating the published ggml algorithm (dequantize_row_iq2_s / iq3_s / iq4_xs). The third-party
arithmetic boundary is gguf-py (Python package `gguf`, 0.19.0 in this image; unpinned by the reference,
G/tools/verify_local.sh:18), whose grid tables this module loads at run time (nothing is retyped here).

Block = 256 weights with an f16 scale d in bytes 0-1:
  IQ2_S  82 B: qs[32] (low 8 bits of a 10-bit grid index, one per group of 8 weights) | signs[32] (bit k of byte
         g = sign of weight 8g + k) | qh[8] (bits 2(g%4)..+1 of byte g/4 = high index bits of group g) |
         scales[8] (nibble g/2 of the 16: low nibble first; one per 16 weights).
         w = d * (0.5 + s) * 0.25 * grid2[idx][k] * (+-1); grid2: 1024 entries x 8 values in {8, 25, 43}.
  IQ3_S  110 B: qs[64] (low 8 bits of a 9-bit index, one per group of 4) | qh[8] (bit g%8 of byte g/8 = high bit) |
         signs[32] (bit k of byte b = sign of weight 8b + k) | scales[4] (8 nibbles, one per 32 weights).
         w = d * (1 + 2 s) * grid3[idx][k] * (+-1); grid3: 512 entries x 4 values in {1, 3, .., 15}.
  IQ4_XS 136 B: scales_h u16 (bits 2i..2i+1 = high bits of sub-block i's scale) | scales_l[4] (nibble i, low
         first) | qs[128]: sub-block i (32 weights) = bytes 16i..16i+15, weights 0-15 the low nibbles, 16-31 the
         high ones. w = d * (scale_i - 32) * kvalues[nibble]; kvalues: the 16 IQ4_NL levels.
All arithmetic in fp32 in this order, matching gguf-py and the reference bit for bit (tests/test_iq_oracle.py).
"""
import numpy as np

QK = 256
BLOCK_BYTES = {"IQ2_S": 82, "IQ3_S": 110, "IQ4_XS": 136, "Q2_K": 84, "Q3_K": 110}
GGML_TYPE = {"Q2_K": 10, "Q3_K": 11, "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23}   # ggml_type numbers
D_OFFSET = {"IQ2_S": 0, "IQ3_S": 0, "IQ4_XS": 0, "Q2_K": 80, "Q3_K": 108}        # byte of the f16 block scale


def tables():
    """{qtype: fp32 lookup table}: IQ2_S [1024, 8], IQ3_S [512, 4], IQ4_XS [16] (from gguf-py)."""
    import gguf.quants as gq
    out = {}
    for qt in ("IQ2_S", "IQ3_S"):
        cls = getattr(gq, qt)
        cls.init_grid()
        out[qt] = np.asarray(cls.grid, np.float32).reshape(cls.grid_shape)
    out["IQ4_XS"] = np.asarray(gq.IQ4_NL.kvalues, np.float32)
    out["Q2_K"] = out["Q3_K"] = None                                          # no lookup table
    return out


def _d(blk):
    return np.ascontiguousarray(blk[:, 0:2]).view(np.float16).astype(np.float32)[:, 0]


def _signs(b):
    """uint8 [nb, n] -> fp32 [nb, n, 8]: -1 where bit k of the byte is set, else +1."""
    bits = (b[..., None] >> np.arange(8, dtype=np.uint8)) & 1
    return np.where(bits == 1, np.float32(-1.0), np.float32(1.0))


def dequant_iq2_s(blk, grid):
    nb = blk.shape[0]
    d = _d(blk)
    qs = blk[:, 2:34].astype(np.int32)
    qh = blk[:, 66:74]
    sc = blk[:, 74:82]
    hi = ((qh[:, :, None] >> np.array([0, 2, 4, 6], np.uint8)) & 3).reshape(nb, 32).astype(np.int32)
    idx = qs | (hi << 8)                                                     # [nb, 32] groups of 8
    s = np.stack([sc & 15, sc >> 4], -1).reshape(nb, 16).astype(np.float32)
    db = d[:, None] * (np.float32(0.5) + s) * np.float32(0.25)               # [nb, 16] one per 2 groups
    db = np.repeat(db, 2, axis=1)[:, :, None]                                # [nb, 32, 1]
    return (db * grid[idx] * _signs(blk[:, 34:66])).reshape(nb, QK)


def dequant_iq3_s(blk, grid):
    nb = blk.shape[0]
    d = _d(blk)
    qs = blk[:, 2:66].astype(np.int32)
    qh = ((blk[:, 66:74, None] >> np.arange(8, dtype=np.uint8)) & 1).reshape(nb, 64).astype(np.int32)
    idx = qs | (qh << 8)                                                     # [nb, 64] groups of 4
    sc = blk[:, 106:110]
    s = np.stack([sc & 15, sc >> 4], -1).reshape(nb, 8).astype(np.int32)
    db = d[:, None] * (1 + 2 * s).astype(np.float32)                         # [nb, 8] one per 8 groups
    db = np.repeat(db, 8, axis=1)[:, :, None]                                # [nb, 64, 1]
    sg = _signs(blk[:, 74:106]).reshape(nb, 64, 4)                           # bits of byte b: groups 2b, 2b+1
    return (db * grid[idx] * sg).reshape(nb, QK)


def dequant_iq4_xs(blk, kvalues):
    nb = blk.shape[0]
    d = _d(blk)
    sh = np.ascontiguousarray(blk[:, 2:4]).view(np.uint16)[:, 0].astype(np.int32)
    sl = blk[:, 4:8]
    lo = np.stack([sl & 15, sl >> 4], -1).reshape(nb, 8).astype(np.int32)
    hi = (sh[:, None] >> (2 * np.arange(8))) & 3
    dl = d[:, None] * ((lo | (hi << 4)) - 32).astype(np.float32)             # [nb, 8] per 32 weights
    q = blk[:, 8:136].reshape(nb, 8, 16)
    nib = np.concatenate([q & 15, q >> 4], -1).astype(np.int32)              # [nb, 8, 32]
    return (dl[:, :, None] * kvalues[nib]).reshape(nb, QK)


def dequant_q2_k(blk, _table=None):
    """Q2_K (84 B: scales[16] | qs[64] | d f16 | dmin f16), the reference's MTP-layer experts (iqquant.py:200-212).
    Weight 128n + 32s + l = (qs[32n + l] >> 2s) & 3, scale byte 8n + 2s + l // 16 (low nibble x d, high nibble x
    dmin): w = (d * sc) * q - dmin * m, each product and the difference rounded to fp32."""
    nb = blk.shape[0]
    sc = blk[:, 0:16]
    d = np.ascontiguousarray(blk[:, 80:82]).view(np.float16).astype(np.float32)[:, 0]
    dmin = np.ascontiguousarray(blk[:, 82:84]).view(np.float16).astype(np.float32)[:, 0]
    dl = (d[:, None] * (sc & 15).astype(np.float32))[:, :, None]            # [nb, 16, 1]
    ml = (dmin[:, None] * (sc >> 4).astype(np.float32))[:, :, None]
    q = (blk[:, 16:80].reshape(nb, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3
    q = q.reshape(nb, 16, 16).astype(np.float32)
    return (dl * q - ml).reshape(nb, QK)


def q3k_scales(sc):
    """The 16 six-bit scales of a Q3_K block's 12 bytes: scale m = (low nibble m // 8 of byte m % 8) | (2 bits
    2 (m // 4) of byte 8 + m % 4) << 4."""
    nb = sc.shape[0]
    lo = (sc[:, 0:8].reshape(nb, 1, 8) >> np.array([0, 4], np.uint8).reshape(1, 2, 1)).reshape(nb, 16) & 15
    hi = (sc[:, 8:12].reshape(nb, 1, 4) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 4, 1)).reshape(nb, 16) & 3
    return (lo | (hi << 4)).astype(np.int32)


def dequant_q3_k(blk, _table=None):
    """Q3_K (110 B: hmask[32] | qs[64] | scales[12] | d f16), iqquant.py:215-226. Weight 128n + 32s + l:
    q = ((qs[32 + 32n + l] >> 2s) & 3) - 4 unless bit 4n + s of hmask[l] is set; w = (d * (scale - 32)) * q."""
    nb = blk.shape[0]
    d = np.ascontiguousarray(blk[:, 108:110]).view(np.float16).astype(np.float32)[:, 0]
    dl = (d[:, None] * (q3k_scales(blk[:, 96:108]) - 32).astype(np.float32))[:, :, None]   # [nb, 16, 1]
    ql = (blk[:, 32:96].reshape(nb, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3
    qh = (blk[:, 0:32].reshape(nb, 1, 32) >> np.arange(8, dtype=np.uint8).reshape(1, 8, 1)) & 1
    q = ql.reshape(nb, 16, 16).astype(np.int32) - 4 * (1 - qh.reshape(nb, 16, 16).astype(np.int32))
    return (dl * q.astype(np.float32)).reshape(nb, QK)


DEQUANT = {"IQ2_S": dequant_iq2_s, "IQ3_S": dequant_iq3_s, "IQ4_XS": dequant_iq4_xs, "Q2_K": dequant_q2_k,
           "Q3_K": dequant_q3_k}


def dequant_rows(raw, qtype, ne0, tabs=None):
    """raw uint8 bytes of a row-major tensor with ne0 weights per row -> fp32 [rows, ne0]."""
    tabs = tabs or tables()
    blk = np.asarray(raw, np.uint8).reshape(-1, BLOCK_BYTES[qtype])
    return DEQUANT[qtype](blk, tabs[qtype]).reshape(-1, ne0)


def random_blocks(rng, n, qtype, dmin=1e-3, dmax=2e-2):
    """n random blocks (uint8 [n, block bytes]) with a positive f16 block scale in [dmin, dmax] (Q2_K: also its
    f16 min scale, a tenth of that)."""
    bb, off = BLOCK_BYTES[qtype], D_OFFSET[qtype]
    b = rng.integers(0, 256, (n, bb), dtype=np.uint8)
    b[:, off:off + 2] = np.frombuffer(rng.uniform(dmin, dmax, n).astype(np.float16).tobytes(), np.uint8).reshape(n, 2)
    if qtype == "Q2_K":
        b[:, 82:84] = np.frombuffer(rng.uniform(dmin / 10, dmax / 10, n).astype(np.float16).tobytes(),
                                    np.uint8).reshape(n, 2)
    return b


def experts_dense(raw, qtype, E, rows, K, tabs=None):
    """Raw GGUF expert table ([E][rows][K/256][block bytes] bytes) -> fp32 [E, rows, K]."""
    return dequant_rows(raw, qtype, K, tabs).reshape(E, rows, K)


def decode_apply(x, idx, w, Wg, Wu, Wd, limit):
    """resident.py:110-120 over dense fp32 experts (Wg, Wu [E, I, H], Wd [E, H, I]), in float64: per (token, slot)
    g = Wg x, u = Wu x, h = swiglu_clamped(g, u), y += w * (Wd h). -> [N, H]."""
    from oracle import moe
    x = np.asarray(x, np.float64)
    out = np.zeros((x.shape[0], Wd.shape[1]), np.float64)
    for n in range(x.shape[0]):
        for j in range(idx.shape[1]):
            e = int(idx[n, j])
            h = moe.swiglu_clamped(Wg[e].astype(np.float64) @ x[n], Wu[e].astype(np.float64) @ x[n], limit)
            out[n] += float(w[n, j]) * (Wd[e].astype(np.float64) @ h)
    return out
