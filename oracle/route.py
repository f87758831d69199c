"""MoE router: CPU restatement (test infrastructure, see oracle/__init__.py).

Follows launcher/glm53-flash/engine/glm53/model.py:798-808 (`moe_route`, n_group == 1):
  logits = f32(x) @ f32(W) [N, E];  scores = sigmoid(logits);  choice = scores + bias;
  idx = top_k(choice, k) (largest first, the lower expert index first among equal choices);
  w = scores[idx] (the raw scores, not the biased choice); if norm_topk: w /= (sum_k w + 1e-20);  w *= scaling.
Pinned by tests/golden/route.npz (the reference's function executed by tests/golden/make_route_golden.py).
"""
import numpy as np


def moe_route(x, W, bias, k, norm_topk=True, scaling=1.0):
    """x [N, D], W [D, E], bias [E] -> (idx int32 [N, k], w f32 [N, k]); fp32 arithmetic."""
    logits = np.asarray(x, np.float32) @ np.asarray(W, np.float32)
    scores = (1.0 / (1.0 + np.exp(-logits))).astype(np.float32)
    choice = scores + np.asarray(bias, np.float32)
    idx = np.argsort(-choice, axis=-1, kind="stable")[:, :k]
    w = np.take_along_axis(scores, idx, -1)
    if norm_topk:
        w = w / (w.sum(-1, keepdims=True) + np.float32(1e-20))
    return idx.astype(np.int32), (w * np.float32(scaling)).astype(np.float32)


def choice_values(x, W, bias):
    """The top-k criterion, for judging near-ties: scores + bias [N, E] in float64."""
    logits = np.asarray(x, np.float64) @ np.asarray(W, np.float64)
    return 1.0 / (1.0 + np.exp(-logits)) + np.asarray(bias, np.float64)
