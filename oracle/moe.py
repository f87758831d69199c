"""MoE expert-layer semantics: CPU restatement used as the parity checker (test infrastructure, see oracle/__init__.py).

Reference functions restated (paths relative to launcher/glm53-flash/engine/glm53/):
  swiglu_clamped     model.py:119-122
  decode_apply       resident.py:110-120 (`ResidentFetch._apply_kernel`): per (token, slot) gate/up matvec ->
                     swiglu_clamped -> down matvec -> sum over the k slots weighted by w
  ragged_plan        pallas_moe.py:564-592 (expert sort of the T*k slots into `tm`-row blocks)
  ragged_apply       resident.py:144-165 + pallas_moe.py:622-755 (grouped GEMM path, bf16 rounding points kept)
  shared_mlp         model.py:125-127 (`mlp_partial`) with int8 leaves dequantized as quant8.py:91-99
  moe_layer          model.py:840-856 (`moe_dense` after the router: routed partial + shared expert)

Expert tables are CB3 (oracle/cb3.py): gate/up [E, I, H] (rows = intermediate, inputs = hidden) and down [E, H, I],
each given as (idx_words, codebooks). Shared-expert leaves are (q int8 [in, out], s fp32) as in quant8.py.
"""
import numpy as np

from . import cb3, q8


def silu(x):
    return x / (1.0 + np.exp(-x))


def swiglu_clamped(gate, up, limit):
    """model.py:119-122: silu(min(gate, limit)) * clip(up, -limit, limit)."""
    gate = np.minimum(gate, limit)
    up = np.clip(up, -limit, limit)
    return silu(gate) * up


def dense_experts(tbl, K):
    """CB3 table (idx [E, R, K*3/32], cb [E, R, 8]) -> float64 [E, R, K] exact dequant."""
    idx, cb = tbl
    return cb3.dequant(idx, cb, K).astype(np.float64)


def decode_apply(x, idx, w, gate, up, down, limit):
    """resident.py:110-120. x [N, H]; idx int [N, k]; w [N, k]; gate/up/down CB3 tables -> f64 [N, H].
    Each (token, slot) pair runs its expert's gate/up matvec, swiglu_clamped, the down matvec, and the k slot
    outputs are summed with the routing weights (einsum "nkd,nk->nd")."""
    x = np.asarray(x, np.float64)
    N, H = x.shape
    k = idx.shape[1]
    I = gate[0].shape[1]
    Wg, Wu, Wd = dense_experts(gate, H), dense_experts(up, H), dense_experts(down, I)
    out = np.zeros((N, H), np.float64)
    for n in range(N):
        for j in range(k):
            e = int(idx[n, j])
            h = swiglu_clamped(Wg[e] @ x[n], Wu[e] @ x[n], limit)
            out[n] += float(w[n, j]) * (Wd[e] @ h)
    return out


def ragged_plan(idx, w, E, tm):
    """pallas_moe.py:564-592. idx int [T, k], w f32 [T, k] -> dict(blk_expert int32 [G], n_blocks int32 [1],
    tok_row int32 [Rp] (-1 = padding), w_row f32 [Rp], row_slot int32 [T, k]); G = ceil(T*k / tm) + E, Rp = G*tm.
    Slots are sorted by expert with a stable sort; each expert's rows start on a block boundary."""
    idx = np.asarray(idx)
    T, k = idx.shape
    S = T * k
    G = -(-S // tm) + E
    Rp = G * tm
    flat = idx.reshape(-1).astype(np.int32)
    order = np.argsort(flat, kind="stable")
    se = flat[order]
    counts = np.bincount(flat, minlength=E).astype(np.int32)[:E]
    padded = -(-counts // tm) * tm
    pstart = np.cumsum(padded) - padded
    ustart = np.cumsum(counts) - counts
    row_sorted = (pstart[se] + (np.arange(S) - ustart[se])).astype(np.int32)
    tok_row = np.full((Rp,), -1, np.int32)
    tok_row[row_sorted] = (order // k).astype(np.int32)
    w_row = np.zeros((Rp,), np.float32)
    w_row[row_sorted] = np.asarray(w, np.float32).reshape(-1)[order]
    row_slot = np.zeros((S,), np.int32)
    row_slot[order] = row_sorted
    nb = padded // tm
    bstart = np.cumsum(nb) - nb
    n_blocks = int(np.sum(nb))
    g = np.arange(G)
    be = np.sum(g[:, None] >= (bstart + nb)[None, :], axis=1)
    be = np.minimum(be, E - 1)
    last = be[max(n_blocks - 1, 0)]
    be = np.where(g < n_blocks, be, last).astype(np.int32)
    return {"blk_expert": be, "n_blocks": np.array([n_blocks], np.int32), "tok_row": tok_row, "w_row": w_row,
            "row_slot": row_slot.reshape(T, k)}


def _bf16(a):
    return np.asarray(a, np.float32).astype(cb3.BF16).astype(np.float64)


def ragged_apply(x, idx, w, gate, up, down, limit, tm=32, combine="matmul"):
    """resident.py:144-165 with the grouped kernels' numerics (pallas_moe.py:622-755): activations and dequantized
    weights in bf16, f32 accumulation, h rounded to bf16, the down output rounded to bf16, and the combine either a
    bf16 [T, Rp] weight matrix times y ("matmul") or a row gather + f32 einsum ("gather"). -> f64 [T, H]."""
    x = np.asarray(x, np.float32)
    T, H = x.shape
    E = gate[0].shape[0]
    I = gate[0].shape[1]
    plan = ragged_plan(idx, w, E, tm)
    tok = plan["tok_row"]
    Wg, Wu, Wd = dense_experts(gate, H), dense_experts(up, H), dense_experts(down, I)
    xs = np.where((tok >= 0)[:, None], _bf16(x)[np.maximum(tok, 0)], 0.0)
    Rp = tok.shape[0]
    h = np.zeros((Rp, I))
    y = np.zeros((Rp, H))
    for g in range(int(plan["n_blocks"][0])):
        e = int(plan["blk_expert"][g])
        rows = slice(g * tm, (g + 1) * tm)
        h[rows] = _bf16(swiglu_clamped(xs[rows] @ Wg[e].T, xs[rows] @ Wu[e].T, limit))
        y[rows] = _bf16(h[rows] @ Wd[e].T)
    if combine == "matmul":
        wc = (tok[None, :] == np.arange(T)[:, None]) * plan["w_row"][None, :]
        return _bf16(wc) @ y
    ys = y[plan["row_slot"].reshape(-1)].reshape(T, idx.shape[1], H)
    return np.einsum("tkd,tk->td", ys, np.asarray(w, np.float64))


def shared_mlp(x, gate, up, down, limit):
    """model.py:125-127 with int8 leaves (q [in, out], s): swiglu_clamped(x @ G, x @ U) @ D, G/U/D = bf16(q * s).
    Computed in float64 from the exactly dequantized bf16 weights -> [N, H]."""
    x = np.asarray(x, np.float64)
    g = q8.matmul(x, *gate)
    u = q8.matmul(x, *up)
    return q8.matmul(swiglu_clamped(g, u, limit), *down)


def moe_layer(x, idx, w, gate, up, down, shared, limit):
    """model.py:840-856 below the router: routed experts (decode composition) + shared expert -> f64 [N, H]."""
    return decode_apply(x, idx, w, gate, up, down, limit) + shared_mlp(x, *shared, limit)


def max_rel_err(got, want):
    """max |got - want| / max |want|: the tolerance measure used by every parity test."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = np.max(np.abs(want))
    return float(np.max(np.abs(got - want)) / (den if den > 0 else 1.0))
