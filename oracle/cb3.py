"""CB3 expert format: the CPU restatement used as the parity checker (test infrastructure, see oracle/__init__.py).

CB3 is the 3-bit codebook format named by the benchmark configs. The reference repository has no implementation of
it (its experts are GGUF IQ2_S/IQ3_S/IQ4_XS); the dequant semantics follow the reference's planar dequant +
f32 contraction (launcher/glm53-flash/engine/glm53/pallas_moe.py:310-323, `moe_matvec_ref`).

Spec, for one matrix W [R, K] (R output rows, K inputs, K a multiple of 32):
  * cb [R, 8] bf16: row r's codebook. Benchmark inputs draw the 8 entries from N(0, 0.02), round them to bf16
    (round-to-nearest-even) and sort them ascending.
  * q [R, K] in [0, 8): index of W[r, j] in row r's codebook.
  * packing: the row's indices form one little-endian bit stream, index j in bits 3j .. 3j+2 (bit 3j = least
    significant bit of the index); word m of the row holds stream bits 32m .. 32m+31, bit 0 = stream bit 32m.
    A row has K*3/32 uint32 words (192 for K=2048, 480 for K=5120, 144 for K=1536).
  * dequant: W[r, j] = cb[r, q[r, j]] exactly (bf16 bit patterns equal).
An expert table is idx [E, R, K*3/32] uint32 + cb [E, R, 8] bf16.
"""
import numpy as np
import ml_dtypes

BF16 = ml_dtypes.bfloat16
N_CODES = 8
BITS = 3


def words_per_row(K: int) -> int:
    assert K % 32 == 0, K
    return K * BITS // 32


def pack(q: np.ndarray) -> np.ndarray:
    """q uint8 [..., K] (values < 8) -> uint32 [..., K*3/32], little-endian bit stream per row."""
    q = np.asarray(q, np.uint8)
    K = q.shape[-1]
    assert np.all(q < N_CODES)
    bits = ((q[..., None] >> np.arange(BITS, dtype=np.uint8)) & 1).astype(np.uint8)   # [..., K, 3], LSB first
    stream = bits.reshape(q.shape[:-1] + (K * BITS,))
    by = np.packbits(stream, axis=-1, bitorder="little")                                 # [..., 3K/8]
    return np.ascontiguousarray(by).view("<u4").reshape(q.shape[:-1] + (words_per_row(K),))


def unpack(words: np.ndarray, K: int) -> np.ndarray:
    """uint32 [..., K*3/32] -> uint8 [..., K] indices."""
    w = np.ascontiguousarray(np.asarray(words, "<u4"))
    assert w.shape[-1] == words_per_row(K), (w.shape, K)
    by = w.view(np.uint8).reshape(w.shape[:-1] + (w.shape[-1] * 4,))
    stream = np.unpackbits(by, axis=-1, bitorder="little").reshape(w.shape[:-1] + (K, BITS))
    return (stream[..., 0] | (stream[..., 1] << 1) | (stream[..., 2] << 2)).astype(np.uint8)


def make_codebooks(rng: np.random.Generator, shape, std: float = 0.02) -> np.ndarray:
    """bf16 [*shape, 8]: N(0, std) entries rounded to bf16, sorted ascending along the last axis."""
    v = rng.standard_normal(tuple(shape) + (N_CODES,)).astype(np.float32) * np.float32(std)
    return np.sort(v.astype(BF16).astype(np.float32), axis=-1).astype(BF16)


def make_indices(rng: np.random.Generator, shape) -> np.ndarray:
    """uint8 [*shape] uniform in [0, 8)."""
    return rng.integers(0, N_CODES, size=tuple(shape), dtype=np.uint8)


def dequant(words: np.ndarray, cb: np.ndarray, K: int) -> np.ndarray:
    """Exact dequant: words [..., R, K*3/32], cb bf16 [..., R, 8] -> bf16 [..., R, K] with W[r, j] = cb[r, q[r, j]]."""
    q = unpack(words, K)
    cb = np.asarray(cb, BF16)
    return np.take_along_axis(cb, q.astype(np.int64), axis=-1)


def matvec(words: np.ndarray, cb: np.ndarray, x: np.ndarray) -> np.ndarray:
    """`moe_matvec_ref` for one CB3 matrix: gather + exact dequant + f64 contraction. words [R, K*3/32],
    cb [R, 8], x [..., K] -> [..., R] float64."""
    K = np.asarray(x).shape[-1]
    W = dequant(words, cb, K).astype(np.float64)
    return np.asarray(x, np.float64) @ W.T


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """bf16 array -> uint16 bit patterns (for bit-exact comparisons)."""
    return np.ascontiguousarray(np.asarray(a, BF16)).view(np.uint16)
