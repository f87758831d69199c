"""Tensor-level wrappers of the C ABI: load-time repacks, the routing plan, and the single-matrix ops.

Every function takes and returns torch tensors on the current CUDA device and enqueues on the current stream.
bf16 tensors cross the ABI as raw bit patterns; int/float tensors as-is.
"""
import ctypes

import torch

from ._lib import check, lib, ptr, require_cuda, stream_handle

PLAN_FIELDS = ("counts", "row_start", "act", "n_act", "n_blocks", "n_pass", "blk_expert", "tok_row", "w_row",
               "row_slot", "pass_expert", "pass_row0", "pass_cnt")


def _contig(t, dtype):
    assert t.dtype == dtype, (t.dtype, dtype)
    return t.contiguous()


def pack_cb3(idx0, cb0, idx1=None, cb1=None):
    """CB3 tables idx uint32-as-int32 [E, rows, K*3/32], cb bf16 [E, rows, 8] (one matrix, or gate + up) ->
    (idx_k uint8, cb_k uint8) in the kernel layout. Replaces pack_chip_planes (resident.py:48-60)."""
    require_cuda(idx0, cb0, idx1, cb1)
    nmat = 1 if idx1 is None else 2
    E, rows, wpr = idx0.shape
    K = wpr * 32 // 3
    idx0, cb0 = _contig(idx0, torch.int32), _contig(cb0, torch.bfloat16)
    if nmat == 2:
        idx1, cb1 = _contig(idx1, torch.int32), _contig(cb1, torch.bfloat16)
        assert idx1.shape == idx0.shape and cb1.shape == cb0.shape
    L = lib()
    idx_k = torch.empty(L.cbmoe_cb3k_idx_bytes(E, rows, K, nmat), dtype=torch.uint8, device=idx0.device)
    cb_k = torch.empty(L.cbmoe_cb3k_cb_bytes(E, rows, nmat), dtype=torch.uint8, device=idx0.device)
    check(L.cbmoe_cb3k_repack(ptr(idx0), ptr(cb0), ptr(idx1), ptr(cb1), nmat, E, rows, K, ptr(idx_k), ptr(cb_k),
                              stream_handle()), "cbmoe_cb3k_repack")
    return idx_k, cb_k


def build_cb8(cb_k, nmat, E, rows):
    """CB3K codebooks -> CB8 tables (uint8: int8 hi / uint8 lo bytes + row factors) for the int8-digit decode kernels."""
    require_cuda(cb_k)
    out = torch.empty(lib().cbmoe_cb8_bytes(E, rows, nmat), dtype=torch.uint8, device=cb_k.device)
    check(lib().cbmoe_cb8_build(ptr(cb_k), nmat, E, rows, ptr(out), stream_handle()), "cbmoe_cb8_build")
    return out


def cb8_matvec(idx_k, cb8, rows, K, x, ws=None):
    """One matrix (expert 0 of a CB3K table) times x bf16 [N, K] -> fp32 [N, rows] on the int8-digit decode kernel.
    `ws`: the workspace (uint8, at least cbmoe_cb8_matvec_workspace_bytes); allocated when not given."""
    require_cuda(idx_k, cb8, x)
    N = x.shape[0]
    xb = x.to(torch.bfloat16).contiguous()
    y = torch.empty((N, rows), dtype=torch.float32, device=x.device)
    if ws is None:
        ws = torch.empty(max(1, lib().cbmoe_cb8_matvec_workspace_bytes(N, K)), dtype=torch.uint8, device=x.device)
    check(lib().cbmoe_cb8_matvec(ptr(idx_k), ptr(cb8), rows, K, ptr(xb), N, ptr(y), ptr(ws), ws.numel(),
                                 stream_handle()), "cbmoe_cb8_matvec")
    return y


def dequant_cb3k(idx_k, cb_k, nmat, E, rows, K):
    """Kernel-layout table -> bf16 [nmat, E, rows, K] through the kernels' register dequant."""
    require_cuda(idx_k, cb_k)
    out = torch.empty((nmat, E, rows, K), dtype=torch.bfloat16, device=idx_k.device)
    check(lib().cbmoe_cb3k_dequant(ptr(idx_k), ptr(cb_k), nmat, E, rows, K, ptr(out), stream_handle()),
          "cbmoe_cb3k_dequant")
    return out


def pack_w8(q0, q1=None):
    """int8 leaves q [K_in, rows_out] (quant8 "[in, out]"; one, or gate + up) -> W8K uint8."""
    require_cuda(q0, q1)
    nmat = 1 if q1 is None else 2
    K, rows = q0.shape
    q0 = _contig(q0, torch.int8)
    q1 = None if q1 is None else _contig(q1, torch.int8)
    out = torch.empty(lib().cbmoe_w8k_bytes(rows, K, nmat), dtype=torch.uint8, device=q0.device)
    check(lib().cbmoe_w8k_repack(ptr(q0), ptr(q1), nmat, K, rows, ptr(out), stream_handle()), "cbmoe_w8k_repack")
    return out


def dequant_w8k(qk, s0, s1, scale_axis, nmat, rows, K):
    require_cuda(qk, s0, s1)
    out = torch.empty((nmat, rows, K), dtype=torch.bfloat16, device=qk.device)
    check(lib().cbmoe_w8k_dequant(ptr(qk), ptr(s0.contiguous()), ptr(None if s1 is None else s1.contiguous()),
                                  scale_axis, nmat, rows, K, ptr(out), stream_handle()), "cbmoe_w8k_dequant")
    return out


def plan_layout(T, k, E, tm, pass_tokens):
    off = (ctypes.c_int64 * 14)()
    check(lib().cbmoe_plan_layout(T, k, E, tm, pass_tokens, off), "cbmoe_plan_layout")
    return list(off)


def route_plan(idx, w, E, tm, pass_tokens=8):
    """pallas_moe.ragged_plan (pallas_moe.py:564-592) on the GPU -> dict of int32/fp32 tensors (views of one
    buffer): blk_expert, n_blocks, tok_row, w_row, row_slot [T, k], and the decode lists."""
    require_cuda(idx, w)
    T, k = idx.shape
    off = plan_layout(T, k, E, tm, pass_tokens)
    buf = torch.empty(off[13], dtype=torch.int32, device=idx.device)
    check(lib().cbmoe_route_plan(ptr(_contig(idx, torch.int32)), ptr(_contig(w, torch.float32)), T, k, E, tm,
                                 pass_tokens, ptr(buf), off[13] * 4, stream_handle()), "cbmoe_route_plan")
    out = {}
    for i, name in enumerate(PLAN_FIELDS):
        v = buf[off[i]:off[i + 1]] if i < 12 else buf[off[i]:off[13]]
        out[name] = v
    for name, n in (("counts", E), ("row_start", E), ("act", E)):
        out[name] = out[name][:n]
    out["n_act"], out["n_blocks"], out["n_pass"] = out["n_act"][:1], out["n_blocks"][:1], out["n_pass"][:1]
    S = T * k
    G = -(-S // tm) + E
    P = -(-S // pass_tokens) + E
    out["blk_expert"] = out["blk_expert"][:G]
    out["tok_row"] = out["tok_row"][:G * tm]
    out["w_row"] = out["w_row"][:G * tm].view(torch.float32)
    out["row_slot"] = out["row_slot"][:S].view(T, k)
    for name in ("pass_expert", "pass_row0", "pass_cnt"):
        out[name] = out[name][:P]
    return out


def cb3_matvec(idx_k, cb_k, rows, K, x):
    """One CB3K matrix times x bf16 [N, K] -> fp32 [N, rows] (moe_matvec with every slot on one expert)."""
    require_cuda(idx_k, cb_k, x)
    x = _contig(x, torch.bfloat16)
    N = x.shape[0]
    y = torch.empty((N, rows), dtype=torch.float32, device=x.device)
    check(lib().cbmoe_cb3_matvec(ptr(idx_k), ptr(cb_k), rows, K, ptr(x), N, ptr(y), None, 0, stream_handle()),
          "cbmoe_cb3_matvec")
    return y


def w8_linear(qk, s, scale_axis, rows, K, x):
    """x bf16 [N, K] @ bf16(q * s) -> fp32 [N, rows] (quant8.dequant_tree + dot)."""
    require_cuda(qk, s, x)
    x = _contig(x, torch.bfloat16)
    N = x.shape[0]
    y = torch.empty((N, rows), dtype=torch.float32, device=x.device)
    check(lib().cbmoe_w8_linear(ptr(qk), ptr(_contig(s, torch.float32)), scale_axis, rows, K, ptr(x), N, ptr(y),
                                None, 0, stream_handle()), "cbmoe_w8_linear")
    return y


def w8_logits(qk, s, rows, K, x, ws=None):
    """The int8 lm_head (engine.py:345-351): x bf16 [N, K] times int8 columns (W8K, per-column scales s [rows])
    -> bf16 [N, rows] = bf16(f32(x @ q) * s), the scale after the dot."""
    require_cuda(qk, s, x)
    N = x.shape[0]
    xb = x.to(torch.bfloat16).contiguous()
    out = torch.empty((N, rows), dtype=torch.bfloat16, device=x.device)
    if ws is None:
        ws = torch.empty(max(1, lib().cbmoe_cb8_matvec_workspace_bytes(N, K)), dtype=torch.uint8, device=x.device)
    check(lib().cbmoe_w8_logits(ptr(qk), ptr(s.float().contiguous()), rows, K, ptr(xb), N, ptr(out), ptr(ws),
                                ws.numel(), stream_handle()), "cbmoe_w8_logits")
    return out

