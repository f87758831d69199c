"""Seeded synthetic inputs with the benchmark configs' shapes and distributions (test infrastructure).

The configs (benchmark definition, not the reference's own model):
  0  one CB3 matrix [1024, 2048], x [1, 2048] ~ N(0, 1) in bf16
  1  MoE decode layer: hidden 5120, 160 routed experts + 1 shared, intermediate 1536, top-8, 8 tokens
  2  as 1 with 64 tokens and a Zipf(1.1) per-expert logit bias (skewed expert load)
  3  as 1 in prefill: 4096 tokens, uniform routing; plus int8 QKV [5120 -> 12288] and O [12288 -> 5120]
  4  4 layers of the config-1 shape, 256 tokens, uniform routing, experts sharded over 1/2/4/8 GPUs
Routing is "top-8 softmax gating": the k largest logits per token (ties -> lower expert id), softmax over those k.
The Zipf bias of config 2: experts get a random rank r (a seeded permutation of 1..E), p_r = r^-1.1 / sum, and the
logit bias log(E * p_r), so an expert's selection odds scale with its Zipf weight.
SwiGLU limit: 10.0 unless a test says otherwise.
"""
import numpy as np

from . import cb3, q8

H, I, E, TOPK = 5120, 1536, 160, 8
LIMIT = 10.0


def softmax_topk(logits, k):
    """logits [N, E] -> (idx int32 [N, k], w f32 [N, k]): top-k by value (stable: ties to the lower id), softmax
    over the selected logits."""
    logits = np.asarray(logits, np.float32)
    idx = np.argsort(-logits, axis=1, kind="stable")[:, :k].astype(np.int32)
    sel = np.take_along_axis(logits, idx, axis=1).astype(np.float64)
    ex = np.exp(sel - sel.max(axis=1, keepdims=True))
    return idx, (ex / ex.sum(axis=1, keepdims=True)).astype(np.float32)


def zipf_bias(rng, n_experts, s=1.1):
    ranks = rng.permutation(n_experts) + 1
    p = ranks.astype(np.float64) ** -s
    p /= p.sum()
    return np.log(n_experts * p).astype(np.float32)


def routing(rng, n_tokens, n_experts=E, k=TOPK, zipf=None):
    logits = rng.standard_normal((n_tokens, n_experts)).astype(np.float32)
    if zipf is not None:
        logits = logits + zipf_bias(rng, n_experts, zipf)[None, :]
    return softmax_topk(logits, k)


def activations(rng, n, d):
    """bf16 [n, d] from N(0, 1)."""
    return rng.standard_normal((n, d)).astype(np.float32).astype(cb3.BF16)


def cb3_table(rng, n_experts, rows, K):
    """(idx uint32 [E, rows, K*3/32], cb bf16 [E, rows, 8]) with uniform indices and sorted N(0, 0.02) codebooks."""
    q = cb3.make_indices(rng, (n_experts, rows, K))
    return cb3.pack(q), cb3.make_codebooks(rng, (n_experts, rows))


def cb3_table_words(rng, n_experts, rows, K):
    """The same distribution as cb3_table, drawn as random words: every bit of a CB3 bit stream is an independent
    fair bit, so uniform uint32 words are uniform 3-bit indices. Fast enough for full-size layers."""
    words = rng.integers(0, 2 ** 32, size=(n_experts, rows, cb3.words_per_row(K)), dtype=np.uint32)
    return words, cb3.make_codebooks(rng, (n_experts, rows))


def q8_leaf(rng, n_in, n_out, axis=1, std=0.02):
    """int8 leaf (q [in, out], s) quantized from an N(0, std) matrix as quant8.quantize_array does."""
    w = rng.standard_normal((n_in, n_out)).astype(np.float32) * np.float32(std)
    return q8.quantize_array(w, axis)


def moe_layer(rng, n_experts=E, hidden=H, inter=I, shared_axis=1, words=False):
    """Routed CB3 tables and int8 shared expert for one layer: dict(gate, up, down, shared=(gate, up, down)).
    words=True draws the index bits as random words (cb3_table_words) instead of packing drawn indices."""
    table = cb3_table_words if words else cb3_table
    gate = table(rng, n_experts, inter, hidden)
    up = table(rng, n_experts, inter, hidden)
    down = table(rng, n_experts, hidden, inter)
    shared = (q8_leaf(rng, hidden, inter, shared_axis), q8_leaf(rng, hidden, inter, shared_axis),
              q8_leaf(rng, inter, hidden, shared_axis))
    return {"gate": gate, "up": up, "down": down, "shared": shared}


def config0(seed=0):
    rng = np.random.default_rng(seed)
    idx, cb = cb3_table(rng, 1, 1024, 2048)
    return {"idx": idx[0], "cb": cb[0], "x": activations(rng, 1, 2048)}
