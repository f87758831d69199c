"""int8 weight-only storage: CPU restatement (test infrastructure, see oracle/__init__.py).

Follows launcher/glm53-flash/engine/glm53/quant8.py:
  * quantize_array (quant8.py:26-32): w [in, out] -> q int8, s fp32. axis=1: per-output-column scales s [1, out]
    (max over the input axis); axis=0: per-input-row scales s [in, 1]. s = max(amax, 1e-12) / 127,
    q = clip(round_half_even(w / s), -127, 127).
  * dequant_tree (quant8.py:91-99): W = bf16(f32(q) * s), product in f32, rounded to bf16 (nearest-even).
The benchmark configs name per-output-channel scales (axis=1); axis=0 is what the reference uses for row-parallel
leaves (quant8.py:5-6) and is supported too.
"""
import numpy as np
import ml_dtypes

BF16 = ml_dtypes.bfloat16


def quantize_array(w: np.ndarray, axis: int):
    """w [in, out] -> (q int8 [in, out], s f32 [1, out] (axis=1) or [in, 1] (axis=0))."""
    w32 = np.asarray(w).astype(np.float32)
    amax = np.max(np.abs(w32), axis=1 - axis, keepdims=True)
    s = (np.maximum(amax, np.float32(1e-12)) / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.round(w32 / s), -127, 127).astype(np.int8)
    return q, s


def dequant(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """bf16(f32(q) * s), broadcasting s ([1, out] or [in, 1])."""
    return (np.asarray(q).astype(np.float32) * np.asarray(s, np.float32)).astype(BF16)


def matmul(x: np.ndarray, q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """x [..., in] @ dequant(q, s) [in, out] in float64 -> [..., out]."""
    return np.asarray(x, np.float64) @ dequant(q, s).astype(np.float64)


def logits_colscale(h, q, s):
    """The int8 lm_head of engine.py:345-351 (`_logits_local`): bf16(f32(h @ bf16(q)) * s), the per-column scale
    s [1, V] applied after the dot; h bf16 [..., D], q int8 [D, V]. The dot in float64 (exact at these sizes), the
    scaling and the rounding in float32, as the reference scales its f32 result and casts it to bf16."""
    z = (np.asarray(h, BF16).astype(np.float64) @ np.asarray(q).astype(np.float64)).astype(np.float32)
    return (z * np.asarray(s, np.float32)).astype(BF16)

