"""The reference's GGUF expert formats on the GPU (llama.cpp IQ2_S 82 B, IQ3_S 110 B, IQ4_XS 136 B per 256 weights:
the GLM-5.3-Flash tables; Q2_K 84 B and Q3_K 110 B: its MTP layer):
  * dequant_rows: the counterpart of iqquant.dequant_rows (engine/glm53/iqquant.py:230-235) through
    cbmoe_iq_dequant, bit for bit the reference's fp32 values;
  * pack_layer / apply: routed experts from the GGUF tables (ResidentFetch.apply with IQ qtypes,
    resident.py:100-120), through cbmoe_iq_experts_apply: IQ2_S and IQ3_S matrices on the int8 tensor cores from
    an exact load-time transcode (cbmoe_iq8_build), the other formats in fp32 from the raw blocks like the
    reference's kernel.
The lookup tables are gguf-py's grids (the reference loads the same ones, iq_grids_data.py), uploaded once per
device.
"""
import ctypes

import numpy as np
import torch

from ._lib import IqExperts, check, lib, ptr, require_cuda, stream_handle

GGML_TYPE = {"Q2_K": 10, "Q3_K": 11, "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23}
NO_TABLE = ("Q2_K", "Q3_K")   # the K-quants of the reference's MTP layer need no lookup table
QK_K = 256
_tables = {}


def block_bytes(qtype):
    return int(lib().cbmoe_iq_block_bytes(GGML_TYPE[qtype]))


def _host_table(qtype):
    import gguf.quants as gq
    if qtype == "IQ4_XS":
        return np.asarray(gq.IQ4_NL.kvalues, np.float32)
    cls = getattr(gq, qtype)
    cls.init_grid()
    return np.asarray(cls.grid, np.float32).reshape(cls.grid_shape)


def table(qtype, device):
    """The format's fp32 lookup table on `device` (gguf-py's grid / IQ4_NL levels), shape checked by the library;
    None for the K-quants."""
    if qtype in NO_TABLE:
        return None
    key = (qtype, torch.device(device))
    t = _tables.get(key)
    if t is None:
        host = _host_table(qtype)
        entries, width = ctypes.c_int(), ctypes.c_int()
        check(lib().cbmoe_iq_table_shape(GGML_TYPE[qtype], ctypes.byref(entries), ctypes.byref(width)),
              "cbmoe_iq_table_shape")
        assert host.size == entries.value * width.value, (qtype, host.shape, entries.value, width.value)
        t = torch.from_numpy(host.reshape(-1).copy()).to(device)
        _tables[key] = t
    return t


def dequant_rows(raw, qtype, ne0):
    """raw uint8 [nbytes] (GPU) of a row-major GGUF tensor with ne0 weights per row -> fp32 [rows, ne0]."""
    require_cuda(raw)
    assert raw.dtype == torch.uint8 and raw.dim() == 1, (raw.dtype, raw.shape)
    bb = block_bytes(qtype)
    assert ne0 % QK_K == 0 and raw.numel() % (bb * (ne0 // QK_K)) == 0, (raw.numel(), bb, ne0)
    n_blocks = raw.numel() // bb
    raw = raw.contiguous()
    out = torch.empty((n_blocks * QK_K,), dtype=torch.float32, device=raw.device)
    check(lib().cbmoe_iq_dequant(GGML_TYPE[qtype], ptr(raw), n_blocks, ptr(table(qtype, raw.device)), ptr(out),
                                 stream_handle()), "cbmoe_iq_dequant")
    return out.view(-1, ne0)


INT8_TYPES = ("IQ2_S", "IQ3_S")   # formats with an int8 tensor-core layout (cbmoe_iq8_build)
ERR_UNSUPPORTED = -4              # CBMOE_ERR_UNSUPPORTED


def build_int8(raw, qtype, E, rows, K):
    """The int8 tensor-core layout of one matrix (an exact transcode of its raw GGUF blocks), or None when the format
    has none or its lookup table holds a grid value the layout cannot code."""
    if qtype not in INT8_TYPES:
        return None
    nbytes = lib().cbmoe_iq8_bytes(GGML_TYPE[qtype], E, rows, K)
    if nbytes == 0:
        return None
    out = torch.empty(nbytes, dtype=torch.uint8, device=raw.device)
    rc = lib().cbmoe_iq8_build(GGML_TYPE[qtype], ptr(raw), ptr(table(qtype, raw.device)), E, rows, K, ptr(out),
                               stream_handle())
    if rc == ERR_UNSUPPORTED:   # a grid value the layout cannot code: this matrix stays on the fp32 kernel
        return None
    check(rc, "cbmoe_iq8_build")
    return out


def pack_layer(gate, up, down, qtypes, E, H, I, int8=True):
    """Raw GGUF expert tables of one layer on the GPU (uint8, each [E][rows][K/256][block bytes] flattened: gate and
    up I rows over H inputs, down H rows over I inputs) with their formats, qtypes = {"gate_q": "IQ2_S", "up_q":
    ..., "down_q": ...} (the reference's per-layer qtypes) -> the table dict ResidentFetch.apply takes. int8: also
    build the int8 tensor-core layout of the IQ2_S / IQ3_S matrices (those then run on the int8 kernels)."""
    require_cuda(gate, up, down)
    assert H % QK_K == 0 and I % QK_K == 0, (H, I)
    mats = {"gate_q": (gate, I, H), "up_q": (up, I, H), "down_q": (down, H, I)}
    for key, (t, rows, K) in mats.items():
        qt = qtypes[key]
        assert qt in GGML_TYPE, qt
        assert t.dtype == torch.uint8 and t.numel() == E * rows * (K // QK_K) * block_bytes(qt), \
            (key, qt, t.numel(), E, rows, K)
    p = {"format": "IQ", "E": E, "H": H, "I": I, "qtypes": dict(qtypes),
         "gate_q": gate.contiguous().view(-1), "up_q": up.contiguous().view(-1), "down_q": down.contiguous().view(-1),
         "tables": {key: table(qtypes[key], gate.device) for key in mats}}
    p["int8"] = {key: (build_int8(p[key], qtypes[key], E, rows, K) if int8 else None)
                 for key, (_, rows, K) in mats.items()}
    return p


def experts_struct(p):
    q, t = p["qtypes"], p["tables"]
    tp = {k: (None if v is None else v.data_ptr()) for k, v in t.items()}
    i8 = {k: (None if v is None else v.data_ptr()) for k, v in p.get("int8", {}).items()}
    return IqExperts(p["E"], p["H"], p["I"], GGML_TYPE[q["gate_q"]], GGML_TYPE[q["up_q"]], GGML_TYPE[q["down_q"]],
                     p["gate_q"].data_ptr(), p["up_q"].data_ptr(), p["down_q"].data_ptr(),
                     tp["gate_q"], tp["up_q"], tp["down_q"], i8.get("gate_q"), i8.get("up_q"), i8.get("down_q"))


_ws = {}


def apply(p, x, idx, w, limit):
    """x bf16 [N, H]; idx int32 [N, k]; w fp32 [N, k] -> fp32 [N, H] routed partial (resident.py:110-120)."""
    N, k = idx.shape
    ex = experts_struct(p)
    y = torch.empty((N, p["H"]), dtype=torch.float32, device=x.device)
    if N == 0:
        return y
    nbytes = lib().cbmoe_iq_workspace_bytes(ex, N, k)
    key = (x.device, nbytes)
    ws = _ws.get(key)
    if ws is None:
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
        _ws.clear()
        _ws[key] = ws
    check(lib().cbmoe_iq_experts_apply(ex, ptr(x), N, ptr(idx), ptr(w), k, float(limit), ptr(y), ptr(ws),
                                       ws.numel(), stream_handle()), "cbmoe_iq_experts_apply")
    return y
